"""Builds libkk_b200.so in-tree: the host token-loop runtime (C++17), the
sm_100a CUDA kernels and their C ABI, in one shared library.

Usage: python kim-kvcache_b200/build.py [--force] [-j N] [--trace]

--trace builds the same library with phase tracing compiled in (-DKK_TRACE,
objects in _build_trace/): every CTA of the projection and attention kernels
records %globaltimer stamps of its phases, read back by
`python bench.py --trace OUT`. Rebuild without --trace for measurements.

--define NAME[=VALUE] (repeatable) compiles the CUDA sources with an extra
preprocessor definition, objects in their own _build_<defines>/ folder:
the tuning variants the kernels expose (KK_GEMM_STAGES[_N64], KK_PLAN_SEGMENT_COST,
KK_ATTN_MIN_PART_COST, KK_XNORM_WARPS[_QKV], KK_MBAR_SPIN, ...), for A/B timing against
the default build.

Objects go to kim-kvcache_b200/_build/, the library to
kim-kvcache_b200/lib/libkk_b200.so (both git-ignored; the .so travels to the
GPU box with the working tree). Recompiles a source when it or any header
under csrc/ or include/ is newer than its object.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "lib" / "libkk_b200.so"

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
CUDA_HOME = Path(NVCC).resolve().parent.parent
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}"]
CXXFLAGS = COMMON + ["-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra", "-ffp-contract=off"]
NVCCFLAGS = COMMON + ARCH + ["-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                            "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def sources() -> list[Path]:
    out = []
    for sub in ("host", "capi", "cuda"):
        d = CSRC / sub
        if d.exists():
            out += sorted(d.glob("*.cpp")) + sorted(d.glob("*.cu"))
    return out


def newest_header() -> float:
    stamps = [p.stat().st_mtime for d in (CSRC, ROOT / "include")
              for p in d.rglob("*") if p.suffix in (".h", ".cuh", ".inc")]
    return max(stamps, default=0.0)


def compile_one(src: Path, force: bool, hdr_time: float, extra: list[str],
                obj_dir: Path = OBJ) -> tuple[Path, str]:
    obj = obj_dir / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
            and obj.stat().st_mtime >= hdr_time):
        return obj, ""
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCCFLAGS, *extra, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXXFLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return obj, (res.stdout + res.stderr).strip()


def build(force: bool = False, jobs: int | None = None, verbose: bool = False,
          ptxas_info: bool = False, trace: bool = False, defines: list[str] | None = None) -> Path:
    defines = sorted(defines or [])
    obj_dir = PKG / "_build_trace" if trace else OBJ
    if defines:
        obj_dir = obj_dir.parent / (obj_dir.name + "_" + "_".join(d.replace("=", "-") for d in defines))
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    hdr_time = newest_header()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    if trace:
        extra.append("-DKK_TRACE")
    extra += [f"-D{d}" for d in defines]
    srcs = sources()
    jobs = jobs or min(8, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as pool:
        results = list(pool.map(lambda s: compile_one(s, force, hdr_time, extra, obj_dir), srcs))
    objs = [r[0] for r in results]
    for (obj, log) in results:
        if log and (verbose or ptxas_info):
            print(f"[{obj.name}]\n{log}")
    lib_time = LIB.stat().st_mtime if LIB.exists() else 0.0
    # The library is relinked whenever it was last linked from the other
    # object set (plain vs trace), recorded beside it.
    stamp = LIB.parent / ".variant"
    variant = ("trace" if trace else "plain") + "".join(f" -D{d}" for d in defines)
    switched = not stamp.exists() or stamp.read_text() != variant
    if force or switched or not LIB.exists() or any(o.stat().st_mtime > lib_time for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        stamp.write_text(variant)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--trace", action="store_true")
    ap.add_argument("--define", action="append", default=[], metavar="NAME[=VALUE]",
                    help="extra preprocessor definition for the CUDA sources (tuning variants)")
    a = ap.parse_args()
    try:
        print(build(a.force, a.j, a.v, a.ptxas_info, a.trace, a.define))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
