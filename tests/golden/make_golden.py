"""Regenerates the golden fixtures in this directory from the reference itself.

Run from the repository root where the reference tree is present (its CPU
sources are compiled into oracle/_ref/libkimkv_ref.so by oracle/Makefile):

    python tests/golden/make_golden.py

Every fixture holds the *reference's* outputs on seeded inputs, so
tests/test_golden.py can check the product host runtime and the CPU oracle
against the reference on a machine without the reference tree:

* codec.json      - float->half over a seeded 20k sample plus boundary
                    classes, and half->float over all 65,536 halves (as
                    SHA-256 digests of the output arrays, plus spot values);
* attention.json  - referenceAttention outputs (FP32 bit patterns) on the
                    seeded cases of tests/test_oracle_pinned.py;
* manager_*.json.gz - every call and return value of KvCacheManager op
                    streams (random, promotion-heavy, prefill/promote/decode)
                    recorded on the reference;
* scheduler.json  - the reference scheduler's admissions, per-iteration
                    counters, terminals and model-batch log per scenario.
"""
from __future__ import annotations

import ctypes as C
import gzip
import hashlib
import json
import struct
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "tests"))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT))

import conftest  # noqa: E402

MANAGER_STREAMS = [("random", s, 300) for s in range(4)] + [("promotion", s, 250) for s in range(3)] \
    + [("prefill_decode", 0, 0)]


def jsonable(v):
    if isinstance(v, (tuple, list)):
        return [jsonable(x) for x in v]
    if isinstance(v, (np.integer,)):
        return int(v)
    return v


class Recorder:
    """Forwards every call to the reference manager and records it."""

    def __init__(self, mgr):
        self.mgr, self.log = mgr, []

    def __getattr__(self, name):
        fn = getattr(self.mgr, name)

        def call(*args):
            r = fn(*args)
            self.log.append([name, jsonable(args), jsonable(r)])
            return r
        return call


def codec_fixture(ref):
    import random
    ref.kref_float_to_half.restype = C.c_uint16
    ref.kref_float_to_half.argtypes = [C.c_float]
    ref.kref_half_to_float.restype = C.c_float
    ref.kref_half_to_float.argtypes = [C.c_uint16]
    from test_golden import codec_samples
    samples = codec_samples()
    f2h = np.array([ref.kref_float_to_half(struct.unpack("<f", struct.pack("<I", b))[0]) for b in samples],
                   np.uint16)
    h2f = np.array([struct.unpack("<I", struct.pack("<f", ref.kref_half_to_float(h)))[0]
                    for h in range(1 << 16)], np.uint32)
    # NaN payloads are not part of the contract: digests cover the non-NaN outputs.
    return {"f2h_sha256": hashlib.sha256(f2h.tobytes()).hexdigest(), "f2h_count": len(samples),
            "f2h_first": f2h[:64].tolist(),
            "h2f_sha256_non_nan": hashlib.sha256(h2f[~np.isnan(h2f.view(np.float32))].tobytes()).hexdigest(),
            "h2f_spot": {str(h): int(h2f[h]) for h in (0, 1, 0x3C00, 0x7BFF, 0x8001, 0x0400, 0x03FF, 0xFBFF)}}


def attention_fixture(ref):
    import test_oracle_pinned as top
    out = {}
    for layers, heads, dim, tokens in [(1, 1, 64, 1), (2, 4, 64, 17), (1, 2, 8, 513), (3, 1, 64, 100)]:
        rng = np.random.default_rng(tokens + dim)
        kv = (rng.standard_normal(layers * 2 * tokens * heads * dim) / 8).astype(np.float16).view(np.uint16)
        q = (rng.standard_normal(layers * heads * dim) / 8).astype(np.float32)
        r = top.ref_attention(ref, kv, tokens, q, layers, heads, dim)
        out[f"{layers}x{heads}x{dim}x{tokens}"] = r.view(np.uint32).tolist()
    # GQA paged attention (4 KV heads, 32 query heads) over a mixed
    # extent/micro table: the reference's referenceAttention per query head on
    # the gathered pages, rounded to FP16.
    case = paged_case()
    ref_out = []
    for qh in range(case["q_heads"]):
        h = qh // (case["q_heads"] // case["kv_heads"])
        pools = case["pools"]
        k = np.concatenate([pools[e[3]][e[0], case["layer"], 0, :e[2], h] for e in case["table"]])
        v = np.concatenate([pools[e[3]][e[0], case["layer"], 1, :e[2], h] for e in case["table"]])
        qf = case["q"][qh * 64:(qh + 1) * 64].view(np.float16).astype(np.float32)
        r = top.ref_attention(ref, np.concatenate([k.reshape(-1), v.reshape(-1)]), case["tokens"], qf, 1, 1, 64)
        ref_out += r.astype(np.float16).view(np.uint16).tolist()
    out["paged_gqa"] = ref_out
    return out


def paged_case():
    """Seeded pools, table and query of the paged GQA golden case."""
    rng = np.random.default_rng(3)
    layers, kv_heads, q_heads = 2, 4, 32
    micro = (rng.standard_normal((20, layers, 2, 8, kv_heads, 64)) / 8).astype(np.float16).view(np.uint16)
    extent = (rng.standard_normal((4, layers, 2, 64, kv_heads, 64)) / 8).astype(np.float16).view(np.uint16)
    table = [(2, 0, 64, 1), (0, 64, 64, 1), (7, 128, 8, 0), (13, 136, 8, 0), (3, 144, 5, 0)]
    q = (rng.standard_normal(q_heads * 64) / 8).astype(np.float16).view(np.uint16)
    return {"pools": (micro, extent), "layers": layers, "kv_heads": kv_heads, "q_heads": q_heads,
            "table": table, "tokens": sum(e[2] for e in table), "q": q, "layer": 1}


def manager_fixture(kk, kk_lib, ref, kind, seed, steps):
    import test_manager_parity as tmp
    if kind == "random":
        micro, extent = [(48, 6), (24, 2), (200, 16), (9, 1)][seed % 4]
    elif kind == "promotion":
        micro, extent = 400, [4, 12, 40][seed % 3]
    else:
        micro, extent = 4096, 128
    pair = tmp.Pair(kk, kk_lib, ref, micro, extent)
    rec = Recorder(pair.b)
    pair.b = rec
    if kind == "random":
        tmp.run_stream(pair, seed, steps)
    elif kind == "promotion":
        tmp.run_promotion_stream(pair, seed, steps)
    else:
        tmp.prefill_promote_decode(pair)
    return {"kind": kind, "seed": seed, "steps": steps, "micro": micro, "extent": extent, "calls": rec.log}


def scheduler_fixture(kk, kk_lib, ref):
    import test_scheduler_parity as tsp
    out = []
    for name, args, kw in tsp.SCENARIOS:
        fns = tsp.bind_scheduler(kk, ref, "kref_")
        res = tsp.run_scenario(kk, fns, *args, **kw)
        out.append({"name": name, "result": jsonable(res)})
    return out


def main():
    if not (ROOT / "oracle" / "_ref" / "libkimkv_ref.so").exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "ref"], check=True)
    kk = conftest.load_kk()
    kk_lib = kk.load_library()
    ref = C.CDLL(str(ROOT / "oracle" / "_ref" / "libkimkv_ref.so"))
    (HERE / "codec.json").write_text(json.dumps(codec_fixture(ref), indent=1))
    (HERE / "attention.json").write_text(json.dumps(attention_fixture(ref)))
    for kind, seed, steps in MANAGER_STREAMS:
        data = manager_fixture(kk, kk_lib, ref, kind, seed, steps)
        with gzip.open(HERE / f"manager_{kind}_{seed}.json.gz", "wt") as f:
            json.dump(data, f, separators=(",", ":"))
    (HERE / "scheduler.json").write_text(json.dumps(scheduler_fixture(kk, kk_lib, ref), separators=(",", ":")))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
