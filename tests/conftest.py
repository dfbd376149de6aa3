"""Shared test fixtures.

* `kk`       — the product bindings module (kim-kvcache_b200/__init__.py),
               with lib/libkk_b200.so built in-tree if missing.
* `ref_lib`  — the reference oracle twin (oracle/_ref/libkimkv_ref.so, built
               from the reference's own sources by oracle/Makefile when the
               reference tree is present). Test infrastructure only.
* `oracle_lib` — the plain-C restatement oracle (oracle/_build/libkk_oracle.so).
"""
from __future__ import annotations

import ctypes as C
import importlib.util
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def load_kk():
    spec = importlib.util.spec_from_file_location(
        "kim_kvcache_b200", ROOT / "kim-kvcache_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["kim_kvcache_b200"] = mod
    spec.loader.exec_module(mod)
    if not mod.LIB_PATH.exists():
        subprocess.run([sys.executable, str(ROOT / "kim-kvcache_b200" / "build.py")], check=True)
    return mod


@pytest.fixture(scope="session")
def kk():
    return load_kk()


@pytest.fixture(scope="session")
def kk_lib(kk):
    return kk.load_library()


@pytest.fixture(scope="session")
def ref_lib():
    import kk_oracle_py
    path = kk_oracle_py.REF_LIB
    if not path.exists():
        kk_oracle_py.build_ref()
    if not path.exists():
        pytest.skip("reference oracle library not built: no reference tree here (set "
                    "KK_REFERENCE_DIR, or BASELINE.json reference_path, to build it)")
    return C.CDLL(str(path))


@pytest.fixture(scope="session")
def oracle_lib():
    import kk_oracle_py
    return kk_oracle_py.load()
