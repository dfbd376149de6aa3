"""Block-table structure check (reference src/core/block_table.cpp:12-130):
the per-thread-bitmap duplicate detection gives the same verdict as comparing
every pair of handles, on random tables built to collide. Compiled from the
library's own source with the host C++ compiler; CPU only."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_duplicate_check_matches_pairwise_definition(tmp_path):
    exe = tmp_path / "block_table_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(ROOT / "kim-kvcache_b200" / "csrc" / "host"),
                    str(ROOT / "tests" / "native" / "block_table_check.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe), "100000"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "mismatches 0" in out.stdout
