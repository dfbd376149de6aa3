// TEST INFRASTRUCTURE ONLY — scheduler/generation differential shim (filled in below).
