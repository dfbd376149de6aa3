"""The product host runtime and the CPU oracle against golden fixtures recorded
from the reference itself (tests/golden/, written by
tests/golden/make_golden.py where the reference tree is present). These run
anywhere, with no reference build: FP16 codec, contiguous attention, KvCacheManager
op streams (every return value, table, page record and snapshot) and the
iteration scheduler (admissions, counters, terminals, model-batch log)."""
import ctypes as C
import gzip
import hashlib
import json
import random
import struct
from pathlib import Path

import numpy as np
import pytest

import kk_oracle_py as ko

GOLDEN = Path(__file__).resolve().parent / "golden"


def codec_samples():
    """The seeded float32 bit patterns whose FP16 rounding is pinned."""
    rng = random.Random(7)
    samples = [rng.getrandbits(32) for _ in range(20000)]
    for e in range(90, 150):
        for m in (0x1000, 0x0fff, 0x1001, 0x3000, 0x7fffff, 0x2000, 0):
            samples += [(e << 23) | m, (1 << 31) | (e << 23) | m]
    samples += [0x7f800000, 0xff800000, 0x7fc00000, 0x7f800001, 0x477ff000, 0x477fefff, 0x33000000,
                0x33000001, 0x387fc000]
    return samples


def load(name):
    path = GOLDEN / name
    if not path.exists():
        pytest.skip(f"golden fixture {name} missing")
    if name.endswith(".gz"):
        with gzip.open(path, "rt") as f:
            return json.load(f)
    return json.loads(path.read_text())


def tup(v):
    return tuple(tup(x) for x in v) if isinstance(v, (list, tuple)) else v


@pytest.fixture(scope="module")
def o():
    return ko.load()


def test_codec_matches_golden(o, kk_lib):
    g = load("codec.json")
    kk_lib.kkrt_float_to_half.restype = C.c_uint16
    kk_lib.kkrt_float_to_half.argtypes = [C.c_float]
    kk_lib.kkrt_half_to_float.restype = C.c_float
    kk_lib.kkrt_half_to_float.argtypes = [C.c_uint16]
    samples = codec_samples()
    assert len(samples) == g["f2h_count"]
    floats = [struct.unpack("<f", struct.pack("<I", b))[0] for b in samples]
    for f2h in (o.kko_f2h, kk_lib.kkrt_float_to_half):
        got = np.array([f2h(f) for f in floats], np.uint16)
        assert got[:64].tolist() == g["f2h_first"]
        assert hashlib.sha256(got.tobytes()).hexdigest() == g["f2h_sha256"]
    for h2f in (o.kko_h2f, kk_lib.kkrt_half_to_float):
        table = np.array([struct.unpack("<I", struct.pack("<f", h2f(h)))[0] for h in range(1 << 16)], np.uint32)
        assert hashlib.sha256(table[~np.isnan(table.view(np.float32))].tobytes()).hexdigest() == \
            g["h2f_sha256_non_nan"]
        for h, bits in g["h2f_spot"].items():
            assert int(table[int(h)]) == bits


def test_oracle_paged_gqa_attention_matches_golden(o):
    import sys
    sys.path.insert(0, str(GOLDEN))
    from make_golden import paged_case
    g = load("attention.json")
    c = paged_case()
    micro, extent = c["pools"]
    out = ko.paged_attention(micro, extent, c["layers"], c["kv_heads"], 64, c["layer"], c["q_heads"],
                             c["table"], c["q"])
    assert out.tolist() == g["paged_gqa"]


def test_oracle_attention_matches_golden(o):
    g = {k: v for k, v in load("attention.json").items() if k != "paged_gqa"}
    for key, bits in g.items():
        layers, heads, dim, tokens = map(int, key.split("x"))
        rng = np.random.default_rng(tokens + dim)
        kv = (rng.standard_normal(layers * 2 * tokens * heads * dim) / 8).astype(np.float16).view(np.uint16)
        q = (rng.standard_normal(layers * heads * dim) / 8).astype(np.float32)
        mine = ko.reference_attention(kv, tokens, q, layers, heads, dim)
        assert mine.view(np.uint32).tolist() == bits, key


class Replay:
    """Returns the reference's recorded results, checking the call sequence."""

    def __init__(self, calls):
        self.calls, self.i = calls, 0

    def __getattr__(self, name):
        def call(*args):
            rec_name, rec_args, rec_result = self.calls[self.i]
            self.i += 1
            assert rec_name == name and tup(rec_args) == tup(args), (self.i, name, args, rec_name, rec_args)
            return tup(rec_result)
        return call


class TupleResults:
    """The product manager with results in the tuple form of the recording."""

    def __init__(self, mgr):
        self.mgr = mgr

    def __getattr__(self, attr):
        fn = getattr(self.mgr, attr)
        return lambda *args: tup(fn(*args))


@pytest.mark.parametrize("name", sorted(p.name for p in GOLDEN.glob("manager_*.json.gz")) or ["none"])
def test_manager_streams_match_golden(kk, kk_lib, name):
    import test_manager_parity as tmp
    g = load(name)
    pair = tmp.Pair.__new__(tmp.Pair)
    pair.a = TupleResults(kk.Manager(kk_lib, "kkrt_", g["micro"], g["extent"]))
    pair.b = Replay(g["calls"])
    pair.handles = set()
    if g["kind"] == "random":
        tmp.run_stream(pair, g["seed"], g["steps"])
    elif g["kind"] == "promotion":
        tmp.run_promotion_stream(pair, g["seed"], g["steps"])
    else:
        tmp.prefill_promote_decode(pair)
    assert pair.b.i == len(g["calls"]), "the product made fewer calls than the reference"


def test_scheduler_scenarios_match_golden(kk, kk_lib):
    import test_scheduler_parity as tsp
    g = load("scheduler.json")
    assert [e["name"] for e in g] == [s[0] for s in tsp.SCENARIOS]
    for (name, args, kw), rec in zip(tsp.SCENARIOS, g):
        fns = tsp.bind_scheduler(kk, kk_lib, "kkrt_")
        res = tsp.run_scenario(kk, fns, *args, **kw)
        assert tup(res) == tup(rec["result"]), name
