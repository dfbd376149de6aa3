"""Pins the CPU oracle (oracle/kk_oracle.c) and the product's host arithmetic
to the reference itself and to the reference tests' known answers:

* FP16 codec: known answers of tests/reference/kv_reference_test.cpp:24-43,
  then bit-exact against the reference codec (oracle/_ref) on every class of
  input (normals, subnormals, ties, overflow, NaN/Inf) — for the oracle and
  for the product runtime's codec;
* attention: the 2-token known answer of kv_reference_test.cpp:45-95, then
  bit-exact against the reference's referenceAttention on random cases;
* paged GQA attention: the oracle's gather + per-head attention equals the
  reference's referenceAttention run on the same gathered data;
* weight manifest: the product loader returns the reference's error codes on
  valid and corrupted manifests; its SHA-256 equals hashlib's and the
  reference's.
"""
import ctypes as C
import hashlib
import math
import random
import struct

import numpy as np
import pytest

import kk_oracle_py as ko


@pytest.fixture(scope="module")
def o():
    return ko.load()


def bits(f: float) -> int:
    return struct.unpack("<I", struct.pack("<f", f))[0]


def from_bits(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


def test_codec_known_answers(o, kk_lib):
    for f in (o.kko_f2h, kk_lib.kkrt_float_to_half):
        f.restype = C.c_uint16
        f.argtypes = [C.c_float]
    for f2h in (o.kko_f2h, kk_lib.kkrt_float_to_half):
        assert f2h(0.0) == 0x0000 and f2h(-0.0) == 0x8000 and f2h(1.0) == 0x3C00
        assert f2h(-2.0) == 0xC000 and f2h(65504.0) == 0x7BFF
    assert o.kko_h2f(0x3C00) == 1.0 and o.kko_h2f(0xC000) == -2.0 and o.kko_h2f(0x7BFF) == 65504.0
    assert math.isinf(o.kko_h2f(0x7C00)) and math.isnan(o.kko_h2f(0x7E00))


def test_codec_matches_reference_bit_exact(o, kk_lib, ref_lib):
    ref_lib.kref_float_to_half.restype = C.c_uint16
    ref_lib.kref_float_to_half.argtypes = [C.c_float]
    ref_lib.kref_half_to_float.restype = C.c_float
    ref_lib.kref_half_to_float.argtypes = [C.c_uint16]
    kk_lib.kkrt_half_to_float.restype = C.c_float
    kk_lib.kkrt_half_to_float.argtypes = [C.c_uint16]
    rng = random.Random(7)
    samples = [rng.getrandbits(32) for _ in range(20000)]
    # ties and near-ties at every exponent, subnormal range, overflow boundary, specials
    for e in range(90, 150):
        for m in (0x1000, 0x0fff, 0x1001, 0x3000, 0x7fffff, 0x2000, 0):
            samples += [(e << 23) | m, (1 << 31) | (e << 23) | m]
    samples += [0x7f800000, 0xff800000, 0x7fc00000, 0x7f800001, 0x477ff000, 0x477fefff, 0x33000000,
                0x33000001, 0x387fc000]
    for b in samples:
        f = from_bits(b)
        r = ref_lib.kref_float_to_half(f)
        assert o.kko_f2h(f) == r, hex(b)
        assert kk_lib.kkrt_float_to_half(f) == r, hex(b)
    for h in range(0, 1 << 16):
        r = ref_lib.kref_half_to_float(h)
        mine = o.kko_h2f(h)
        assert (math.isnan(r) and math.isnan(mine)) or bits(r) == bits(mine), hex(h)
        prod = kk_lib.kkrt_half_to_float(h)
        assert (math.isnan(r) and math.isnan(prod)) or bits(r) == bits(prod), hex(h)


def test_attention_known_answer(o):
    # layout {1 layer, 1 head, dim 2}, 2 tokens: K = [(0,0), (1,0)], V = [(1,2), (3,4)], q = (1,0)
    f2h = o.kko_f2h
    kv = np.array([f2h(0), f2h(0), f2h(1), f2h(0), f2h(1), f2h(2), f2h(3), f2h(4)], dtype=np.uint16)
    out = ko.reference_attention(kv, 2, np.array([1.0, 0.0], np.float32), 1, 1, 2)
    w = math.exp(1.0 / math.sqrt(2.0))
    assert abs(out[0] - (1 + 3 * w) / (1 + w)) < 1e-6
    assert abs(out[1] - (2 + 4 * w) / (1 + w)) < 1e-6
    assert ko.reference_attention(kv, 0, np.array([1.0, 0.0], np.float32), 1, 1, 2) is None


def ref_attention(ref_lib, kv, tokens, q, layers, heads, dim):
    f = ref_lib.kref_reference_attention
    f.restype = C.c_int
    f.argtypes = [C.c_uint32] * 3 + [C.POINTER(C.c_uint16), C.c_uint32, C.POINTER(C.c_float),
                                     C.POINTER(C.c_float)]
    out = np.zeros(layers * heads * dim, np.float32)
    kv = np.ascontiguousarray(kv, np.uint16)
    q = np.ascontiguousarray(q, np.float32)
    assert f(layers, heads, dim, ko.ptr(kv, C.c_uint16), tokens, ko.ptr(q, C.c_float),
             ko.ptr(out, C.c_float))
    return out


@pytest.mark.parametrize("layers,heads,dim,tokens", [(1, 1, 64, 1), (2, 4, 64, 17), (1, 2, 8, 513),
                                                     (3, 1, 64, 100)])
def test_attention_matches_reference_bit_exact(o, ref_lib, layers, heads, dim, tokens):
    rng = np.random.default_rng(tokens + dim)
    kv = (rng.standard_normal(layers * 2 * tokens * heads * dim) / 8).astype(np.float16).view(np.uint16)
    q = (rng.standard_normal(layers * heads * dim) / 8).astype(np.float32)
    mine = ko.reference_attention(kv, tokens, q, layers, heads, dim)
    ref = ref_attention(ref_lib, kv, tokens, q, layers, heads, dim)
    assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))


def test_paged_attention_oracle_equals_reference_on_gathered_pages(o, ref_lib):
    rng = np.random.default_rng(3)
    layers, kv_heads, dim, q_heads = 2, 4, 64, 32
    micro = (rng.standard_normal((20, layers, 2, 8, kv_heads, dim)) / 8).astype(np.float16).view(np.uint16)
    extent = (rng.standard_normal((4, layers, 2, 64, kv_heads, dim)) / 8).astype(np.float16).view(np.uint16)
    table = [(2, 0, 64, 1), (0, 64, 64, 1), (7, 128, 8, 0), (13, 136, 8, 0), (3, 144, 5, 0)]
    T = sum(e[2] for e in table)
    q = (rng.standard_normal(q_heads * dim) / 8).astype(np.float16).view(np.uint16)
    layer = 1
    out = ko.paged_attention(micro, extent, layers, kv_heads, dim, layer, q_heads, table, q)
    group = q_heads // kv_heads
    for qh in range(q_heads):
        h = qh // group
        k = np.concatenate([(micro if e[3] == 0 else extent)[e[0], layer, 0, :e[2], h] for e in table])
        v = np.concatenate([(micro if e[3] == 0 else extent)[e[0], layer, 1, :e[2], h] for e in table])
        kv = np.concatenate([k.reshape(-1), v.reshape(-1)])
        qf = q[qh * dim:(qh + 1) * dim].view(np.float16).astype(np.float32)
        ref = ref_attention(ref_lib, kv, T, qf, 1, 1, dim)
        expect = ref.astype(np.float16).view(np.uint16)  # RNE rounding of the FP32 result
        assert np.array_equal(out[qh * dim:(qh + 1) * dim], expect)


def test_manifest_loader_matches_reference_errors(kk, kk_lib, ref_lib, tmp_path):
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location(
        "kk_synth", Path(kk.__file__).parent / "synthetic.py")
    synth = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(synth)
    cfg = dict(hidden=128, intermediate=256, layers=2, q_heads=2, kv_heads=1, head_dim=64,
               vocab=300, max_positions=64, eps=1e-5, theta=10000.0)
    manifest, data, _ = synth.write_archive(tmp_path / "good", cfg, seed=1)
    ref_check = ref_lib.kref_manifest_check
    ref_check.restype = C.c_int
    ref_check.argtypes = [C.c_char_p, C.c_char_p]
    mine = kk_lib.kkrt_manifest_check
    mine.restype = C.c_int
    mine.argtypes = [C.c_char_p, C.c_char_p]
    text = open(manifest).read()

    def variant(name, new_text, new_data=None):
        d = tmp_path / name
        d.mkdir()
        (d / "model.manifest").write_text(new_text)
        dp = d / "model.weights"
        dp.write_bytes(open(data, "rb").read() if new_data is None else new_data)
        return str(d / "model.manifest"), str(dp)

    lines = text.splitlines()
    tensor_line = next(i for i, l in enumerate(lines) if l.startswith("tensor="))
    cases = {
        "ok": (text, None),
        "version": (text.replace("version=1", "version=2"), None),
        "dtype": (text.replace("dtype=fp16", "dtype=bf16"), None),
        "dup_key": (text + "hidden_size=128\n", None),
        "bad_line": (text + "garbage\n", None),
        "missing_field": ("\n".join(l for l in lines if not l.startswith("rope_theta")) + "\n", None),
        "count": (text.replace(f"tensor_count={len(lines) - tensor_line}", "tensor_count=3"), None),
        "shape": (text.replace("|128,128|", "|128,64|", 1), None),
        "dup_tensor": ("\n".join(lines + [lines[tensor_line]]).replace(
            f"tensor_count={len(lines) - tensor_line}", f"tensor_count={len(lines) - tensor_line + 1}") + "\n", None),
        "missing_tensor": ("\n".join(lines[:-1]).replace(
            f"tensor_count={len(lines) - tensor_line}", f"tensor_count={len(lines) - tensor_line - 1}") + "\n", None),
        "checksum": (text, b"\x01" + open(data, "rb").read()[1:]),
        "short": (text, open(data, "rb").read()[:-2]),
        "config": (text.replace("kv_head_count=1", "kv_head_count=3"), None),
    }
    for name, (t, d) in cases.items():
        m, dp = variant(name, t, d)
        got = mine(m.encode(), dp.encode())
        want = ref_check(m.encode(), dp.encode())
        assert got == want, f"{name}: product {got} reference {want}"
        if name == "ok":
            assert got == 0
    # SHA-256 of a byte range: product == hashlib == reference
    raw = open(data, "rb").read()
    buf = C.create_string_buffer(65)
    for off, n in [(0, 1), (3, 1000), (0, len(raw)), (100, 55)]:
        assert kk_lib.kkrt_sha256_range(data.encode(), C.c_uint64(off), C.c_uint64(n), buf) == 0
        ours = buf.value.decode()
        assert ref_lib.kref_sha256_range(data.encode(), C.c_uint64(off), C.c_uint64(n), buf) == 0
        assert ours == buf.value.decode() == hashlib.sha256(raw[off:off + n]).hexdigest()


# ---- the model oracle against the reference's own ReferenceModel ------------------
#
# ReferenceModel (tests/cuda/cuda_model_runner_test.cpp:213-420 of the
# reference) is test-local C++; oracle/ref_model_shim.cpp compiles that test
# file in place into oracle/_ref and exposes it. kk_oracle.c must reproduce
# it bit for bit: same rounding points, same summation order, same libm calls.

MODEL_SMALL = dict(hidden=512, intermediate=1024, layers=3, q_heads=8, kv_heads=2, head_dim=64,
                   vocab=1000, max_positions=512, eps=1e-5, theta=10000.0)


def _synth():
    import importlib.util
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    spec = importlib.util.spec_from_file_location("kk_synth", root / "kim-kvcache_b200" / "synthetic.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _synthetic_weights(cfg, seed, std):
    synth = _synth()
    rng = np.random.default_rng(seed)
    return [synth.make_tensor(n, s, rng, std) for n, s in synth.tensor_list(cfg)]


def _run_both(ref, oracle, tokens):
    """Feeds the same positions to the reference model and the oracle; both
    logits (FP32 bit patterns) and the final normalised hidden states (FP16
    bits) must be identical."""
    for pos, tok in enumerate(tokens):
        rl, rh = ref.forward(tok, pos)
        _, ol, oh = oracle.forward([7], [tok], [pos])
        assert np.array_equal(rl.view(np.uint32), ol[0].view(np.uint32)), \
            f"position {pos}: max |diff| {np.max(np.abs(rl - ol[0]))}"
        assert np.array_equal(rh, oh[0]), f"position {pos}: final hidden differs"


def test_model_oracle_equals_reference_model_on_the_contract_archive(ref_lib):
    """The reference test's own contract archive and weights (TestArchive,
    :55-211): every logit and final hidden value bit-exact over a prompt, and
    the greedy generation equal to the reference's referenceGeneration."""
    ref = ko.RefModel()
    cfg = dict(ref.cfg)
    oracle = ko.Model(cfg, ref.tensors(), threads=2)
    oracle.create(7)
    prompt = [1, 3, 7, 11, 2, 15, 4, 9, 0, 13]
    _run_both(ref, oracle, prompt)
    gen = ko.RefModel()
    want = gen.generate(prompt[:4], 12)
    oracle.create(8)
    tok = None
    for pos, t in enumerate(prompt[:4]):
        g, _, _ = oracle.forward([8], [t], [pos], want_hidden=False)
        tok = int(g[0])
    got = []
    for i in range(12):
        got.append(tok)
        if i < 11:
            g, _, _ = oracle.forward([8], [tok], [4 + i], want_hidden=False)
            tok = int(g[0])
    assert got == want
    gen.close()
    ref.close()
    oracle.close()


def test_model_oracle_equals_reference_model_small_config(ref_lib):
    """A 3-layer GQA config (hidden 512, 8 query / 2 KV heads, head_dim 64,
    vocab 1000) with seeded N(0, 0.05) FP16 weights, 9 positions."""
    w = _synthetic_weights(MODEL_SMALL, 31, 0.05)
    ref = ko.RefModel(MODEL_SMALL, w)
    oracle = ko.Model(MODEL_SMALL, w, threads=4)
    oracle.create(7)
    _run_both(ref, oracle, [1, 999, 5, 17, 400, 3, 3, 250, 77])
    ref.close()
    oracle.close()


def test_reference_lanes_on_given_kv_match_the_oracle(ref_lib):
    """The reference arm's form of the reference model: several
    ReferenceModel lanes over one archive, each fed a seeded past K/V and run
    concurrently; every greedy token equals the oracle's on the same K/V and
    a lone lane's run on one thread."""
    w = _synthetic_weights(MODEL_SMALL, 44, 0.05)
    ref = ko.RefModel(MODEL_SMALL, w)
    oracle = ko.Model(MODEL_SMALL, w, threads=4)
    L, row = MODEL_SMALL["layers"], MODEL_SMALL["kv_heads"] * MODEL_SMALL["head_dim"]
    rng = np.random.default_rng(9)
    contexts = [1, 9, 40, 77]
    lanes = []
    for i, ctx in enumerate(contexts):
        k = (rng.standard_normal((ctx, L, row)) / 8).astype(np.float16).view(np.uint16)
        v = (rng.standard_normal((ctx, L, row)) / 8).astype(np.float16).view(np.uint16)
        lane = ref.lane_create()
        ref.lane_append_kv(lane, k, v)
        assert ref.lane_length(lane) == ctx
        lanes.append(lane)
        oracle.create(100 + i)
        oracle.append_kv(100 + i, k, v)
        if i == len(contexts) - 1:
            single = ko.RefModel(MODEL_SMALL, w)
            single_lane = single.lane_create()
            single.lane_append_kv(single_lane, k, v)
    toks, pos = [5, 17, 999, 3], list(contexts)
    for _ in range(3):
        got = ref.forward_lanes(lanes, toks, pos, threads=3)
        want, _, _ = oracle.forward([100 + i for i in range(len(contexts))], toks, pos, want_logits=False,
                                    want_hidden=False)
        assert got == [int(x) for x in want]
        one = single.forward_lanes([single_lane], [toks[-1]], [pos[-1]], threads=1)
        assert one == [got[-1]]
        toks, pos = got, [p + 1 for p in pos]
    single.close()
    ref.close()
    oracle.close()


@pytest.mark.slow
def test_model_oracle_equals_reference_model_tinyllama_shape(ref_lib):
    """BASELINE config 2's shape (TinyLlama-1.1B: 22 layers, hidden 2048, 32
    query / 4 KV heads, vocab 32000, N(0, 0.02) weights), batch 1, 3 positions."""
    synth = _synth()
    cfg = {k: v for k, v in synth.TINYLLAMA.items() if k not in ("bos", "eos")}
    w = _synthetic_weights(cfg, 5, 0.02)
    ref = ko.RefModel(cfg, w)
    oracle = ko.Model(cfg, w, threads=8)
    del w
    oracle.create(7)
    _run_both(ref, oracle, [2207, 31999, 3])
    ref.close()
    oracle.close()


def test_config1_step_tables_and_attention_match_the_reference(kk, kk_lib, ref_lib):
    """BASELINE config 1 on the CPU side, at a 512-page pool: the seeded
    permutation layout built through the product KvCacheManager and through
    the reference's gives identical reserved tables (partial-tail COW pages
    included), and the oracle's paged GQA attention over the reserved tables
    equals the reference's own config-1 host step (reserveToken, K/V store,
    COW copy, gather, referenceAttention per query head) bit for bit.
    (512 pages: a lane's context is appended as micro pages before its full
    runs are promoted.)"""
    synth = _synth()
    pages = 512
    data = synth.c1_data(11, pool_pages=pages)
    mgrs = [kk.Manager(kk_lib, "kkrt_", pages, pages), kk.Manager(ref_lib, "kref_", pages, pages)]
    for m in mgrs:
        def promote(rid, begin, m=m):
            err, pid, _, _ = m.prepare_promotion(rid, begin)
            return err if err else m.commit_promotion(pid)
        synth.c1_layout(m.create, m.append, m.seal, promote, m.release, 11, pool_pages=pages)
    B = len(synth.C1_CONTEXTS)
    micro, extent = data["micro"].copy(), data["extent"].copy()
    for i, ctx in enumerate(synth.C1_CONTEXTS):
        got = [m.reserve(i + 1, ctx) for m in mgrs]
        assert got[0][0] == 0 and got[0][2:] == got[1][2:], f"lane {i}: tables differ"
        _, rid, before, reserved = got[1]
        for old in before[1]:
            for new in reserved[1]:
                if new[0] == old[0] and (new[3], new[4]) != (old[3], old[4]):
                    micro[new[3], :, :, :old[1]] = micro[old[3], :, :, :old[1]]
        for e in reserved[1]:
            if e[0] <= ctx < e[0] + e[1]:
                pool = micro if e[2] == 0 else extent
                pool[e[3], 0, 0, ctx - e[0]] = data["k"][i].reshape(4, 64)
                pool[e[3], 0, 1, ctx - e[0]] = data["v"][i].reshape(4, 64)
        table = [(e[3], e[0], e[1], e[2]) for e in reserved[1]]
        data.setdefault("oracle", []).append(ko.paged_attention(micro, extent, 1, 4, 64, 0, 32, table,
                                                                data["q"][i]))
        for m, g in zip(mgrs, got):
            assert m.rollback(g[1]) == 0
    assert mgrs[0].snapshot() == mgrs[1].snapshot()
    f = ref_lib.kref_c1_step
    u16p = C.POINTER(C.c_uint16)
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(C.c_uint64), C.POINTER(C.c_uint32), u16p, u16p,
                  C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, u16p, u16p, u16p, u16p,
                  C.c_int, C.c_uint32]
    out = np.zeros((B, 32 * 64), np.uint16)
    rm, rx = data["micro"].copy(), data["extent"].copy()
    p = lambda a: a.ctypes.data_as(u16p)
    assert f(mgrs[1].h, B, (C.c_uint64 * B)(*range(1, B + 1)), (C.c_uint32 * B)(*synth.C1_CONTEXTS), p(rm),
             p(rx), 1, 0, 4, 64, 32, p(data["k"]), p(data["v"]), p(data["q"]), p(out), 0, 3) == 1
    for i in range(B):
        assert np.array_equal(out[i], data["oracle"][i]), f"lane {i}"
    for m in mgrs:
        assert m.invariants()
        m.close()
