"""End-to-end parity of the fused sm_100a decode step (runner + CUDA KV
backend, through the C ABI) against the CPU oracle, the restatement of the
reference's FP16-rounding decoder (tests/cuda/cuda_model_runner_test.cpp
:213-457). Tolerances: hidden states and logits within
2e-2 absolute; greedy tokens identical wherever the oracle's top-2 logit gap
exceeds 2e-2; page tables and commit bookkeeping exact."""
import ctypes as C
import importlib.util
import random
from pathlib import Path

import numpy as np
import pytest
import torch

import kk_oracle_py as ko

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

ROOT = Path(__file__).resolve().parent.parent
TOL = 2e-2
SMALL = dict(hidden=512, intermediate=1024, layers=3, q_heads=8, kv_heads=2, head_dim=64, vocab=1000,
             max_positions=512, eps=1e-5, theta=10000.0, bos=1, eos=2)


def synth():
    spec = importlib.util.spec_from_file_location("kk_synth", ROOT / "kim-kvcache_b200" / "synthetic.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


class Stack:
    """Backend + runner + oracle for one model config."""

    def __init__(self, kk, tmp, cfg, seed=1, std=0.05, batch=8, graphs=1, micro=256, extent=16):
        self.kk, self.cfg = kk, cfg
        self.R = kk.runtime()
        man, data, w = synth().write_archive(tmp, cfg, seed=seed, std=std, keep_weights=True)
        self.stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        self.backend = self.R["backend_create"](cfg["layers"], cfg["kv_heads"], cfg["head_dim"],
                                                cfg["q_heads"], cfg["q_heads"] * cfg["max_positions"] * 4,
                                                micro, extent)
        st, det = C.c_int(0), C.create_string_buffer(256)
        self.runner = self.R["runner_create"](man.encode(), data.encode(), self.backend, self.stream,
                                              batch, graphs, 1, C.byref(st), det, 256)
        assert self.runner, det.value.decode()
        self.oracle = ko.Model(cfg, w, threads=8)

    def close(self):
        self.R["runner_destroy"](self.runner)
        self.R["backend_destroy"](self.backend)
        self.oracle.close()

    def create(self, rid):
        assert self.R["backend_create_request"](self.backend, rid) == 0
        self.oracle.create(rid)

    def batch(self, ids, toks, pos):
        n = len(ids)
        out, ok = (C.c_uint32 * n)(), (C.c_uint8 * n)()
        assert self.R["runner_forward_batch"](self.runner, n, (C.c_uint64 * n)(*ids),
                                              (C.c_uint32 * n)(*toks), (C.c_uint32 * n)(*pos), out, ok)
        if not all(ok[i] for i in range(n)):
            buf = C.create_string_buffer(512)
            self.R["runner_last_error"](self.runner, buf, 512)
            print("fused step failure:", buf.value.decode())
        return [out[i] for i in range(n)], [ok[i] for i in range(n)]

    def snapshot(self):
        s = self.kk.BackendSnapshot()
        self.R["backend_snapshot"](self.backend, C.byref(s))
        return s


def assert_greedy(got, want, logits):
    for g, w, row in zip(got, want, logits):
        top = np.sort(row)[-2:]
        if top[1] - top[0] > TOL:
            assert g == w, f"greedy {g} != oracle {w} (gap {top[1] - top[0]:.4f})"


@pytest.mark.parametrize("graphs", [0, 1])
def test_forward_token_logits_and_hidden_match_oracle(kk, tmp_path, graphs):
    s = Stack(kk, tmp_path, SMALL, graphs=graphs)
    s.create(41)
    cfg = SMALL
    for pos, tok in enumerate([1, 7, 999, 3, 500]):
        logits = np.zeros(cfg["vocab"], np.float32)
        emb = np.zeros(cfg["hidden"], np.uint16)
        fin = np.zeros(cfg["hidden"], np.uint16)
        layers = (C.c_uint32 * 2)(0, 2)
        lh = np.zeros((2, cfg["hidden"]), np.uint16)
        out = C.c_uint32(0)
        rc = s.R["runner_forward_token"](s.runner, 41, tok, pos, C.byref(out), ko.ptr(logits, C.c_float),
                                         ko.ptr(emb, C.c_uint16), ko.ptr(fin, C.c_uint16), layers, 2,
                                         ko.ptr(lh, C.c_uint16))
        assert rc == 0
        want, ref_logits, ref_hidden = s.oracle.forward([41], [tok], [pos])
        assert np.max(np.abs(logits - ref_logits[0])) < TOL
        fh = fin.view(np.float16).astype(np.float32)
        rh = ref_hidden[0].view(np.float16).astype(np.float32)
        assert np.max(np.abs(fh - rh)) < TOL
        assert_greedy([out.value], want, ref_logits)
    snap = s.snapshot()
    assert snap.committed_token_count == 5 and snap.active_transaction_count == 0
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()


def test_batched_decode_with_fork_and_partial_tail_cow(kk, tmp_path):
    s = Stack(kk, tmp_path, SMALL)
    rng = random.Random(3)
    prompts = {1: [rng.randrange(3, 1000) for _ in range(13)], 2: [rng.randrange(3, 1000) for _ in range(6)],
               3: [rng.randrange(3, 1000) for _ in range(21)]}
    for rid in prompts:
        s.create(rid)
    pos, nxt = {r: 0 for r in prompts}, {}

    def step(ids):
        toks = [prompts[r][pos[r]] if pos[r] < len(prompts[r]) else nxt[r] for r in ids]
        ps = [pos[r] for r in ids]
        got, ok = s.batch(ids, toks, ps)
        want, logits, _ = s.oracle.forward(ids, toks, ps, want_hidden=False)
        assert all(ok)
        assert_greedy(got, want, logits)
        for i, r in enumerate(ids):
            nxt[r] = int(want[i])
            pos[r] += 1

    for _ in range(11):
        step([1, 2, 3])
    # fork request 1 at 11 tokens (a partial 3-token tail page): both sides
    # continue, each next write copies the shared tail first
    assert s.R["backend_fork"](s.backend, 1, 9) == 0
    s.oracle.fork(1, 9)
    prompts[9], pos[9], nxt[9] = prompts[1], pos[1], nxt[1]
    for _ in range(14):
        step([1, 2, 3, 9])
    tbl = (kk.KkEntry * 64)()
    t = kk.KkTableOut(C.cast(tbl, C.POINTER(kk.KkEntry)), 64, 0, 0)
    assert s.R["backend_block_table"](s.backend, 9, C.byref(t)) == 1
    assert sum(tbl[i].valid_tokens for i in range(t.count)) == pos[9]
    assert s.R["backend_check_invariants"](s.backend) == 1
    for rid in (1, 2, 3, 9):
        assert s.R["backend_release"](s.backend, rid) == 0
    assert s.snapshot().allocated_micro_pages == 0
    s.close()


def test_scheduler_end_to_end_matches_oracle_generation(kk, tmp_path):
    s = Stack(kk, tmp_path, SMALL, batch=4)
    rng = random.Random(8)
    reqs = {rid: [rng.randrange(3, 1000) for _ in range(rng.randint(3, 40))] for rid in (1, 2, 3, 4, 5)}
    sched = kk.Scheduler(s.R, s.backend, s.runner, 8, 16, 10 ** 6, 8)
    for rid, prompt in reqs.items():
        assert sched.submit(rid, prompt, 12) == 0
    terms = {t["request_id"]: t for t in sched.drain()}
    sched.close()
    for rid, prompt in reqs.items():
        s.oracle.create(100 + rid)
        tok = None
        for p, t in enumerate(prompt):
            g, lg, _ = s.oracle.forward([100 + rid], [t], [p], want_hidden=False)
            tok = int(g[0])
        out = []
        gaps_ok = True
        for i in range(12):
            out.append(tok)
            if tok == SMALL["eos"] or i == 11:
                break
            g, lg, _ = s.oracle.forward([100 + rid], [tok], [len(prompt) + i], want_hidden=False)
            top = np.sort(lg[0])[-2:]
            gaps_ok = gaps_ok and top[1] - top[0] > TOL
            tok = int(g[0])
        got = terms[rid]["tokens"]
        if gaps_ok:
            assert got == out, f"request {rid}: {got} vs oracle {out}"
        assert terms[rid]["error"] == 0
    assert s.snapshot().request_count == 0
    s.close()


def _oracle_generation(s, seq, prompt, max_new, eos):
    """The oracle fed one position at a time (the reference's scheduler
    path): greedy outputs, and whether every top-2 gap exceeded the
    tolerance (only then must the tokens match exactly)."""
    s.oracle.create(seq)
    for p_, t in enumerate(prompt):
        g, lg, _ = s.oracle.forward([seq], [t], [p_], want_hidden=False)
    tok, out, gaps_ok = int(g[0]), [], True
    top = np.sort(lg[0])[-2:]
    gaps_ok = top[1] - top[0] > TOL
    for i in range(max_new):
        out.append(tok)
        if tok == eos or i == max_new - 1:
            break
        g, lg, _ = s.oracle.forward([seq], [tok], [len(prompt) + i], want_hidden=False)
        top = np.sort(lg[0])[-2:]
        gaps_ok = gaps_ok and top[1] - top[0] > TOL
        tok = int(g[0])
    return out, gaps_ok


@pytest.mark.parametrize("fused", [True, False], ids=["fused_prefill", "waves"])
def test_scheduler_forked_prefix_requests_match_oracle(kk, tmp_path, fused):
    """BASELINE config 3's structure at a small shape: two requests share a
    prompt prefix of 40 + k tokens (k = 3: the shared tail page is partial),
    built once and forked in the backend, then submitted with that prefix
    already in the KV cache (kv_prefix_tokens); two more requests are fresh.
    The scheduler runs chunked prefill (chunk 16) mixed with decode, as fused
    multi-position prefill calls or as the reference's one-position waves.
    Each request's greedy output must equal the oracle fed its whole prompt
    one position at a time, the forked pair's first writes copying the shared
    partial tail."""
    s = Stack(kk, tmp_path, SMALL, batch=16)
    rng = random.Random(33)
    P = 40 + 3
    prefix = [rng.randrange(3, 1000) for _ in range(P)]
    assert s.R["backend_create_request"](s.backend, 1) == 0
    got, err = _prefill(s, 1, prefix, 0)
    assert got is not None, err
    assert s.R["backend_fork"](s.backend, 1, 2) == 0
    prompts = {1: prefix + [rng.randrange(3, 1000) for _ in range(21)],
               2: prefix + [rng.randrange(3, 1000) for _ in range(5)],
               3: [rng.randrange(3, 1000) for _ in range(19)],
               4: [rng.randrange(3, 1000) for _ in range(70)]}
    sched = kk.Scheduler(s.R, s.backend, s.runner, 8, 64, 10 ** 6, 16, fused_prefill=fused)
    for rid, prompt in prompts.items():
        assert sched.submit(rid, prompt, 10, kv_prefix=P if rid in (1, 2) else 0) == 0
    terms = {t["request_id"]: t for t in sched.drain()}
    sched.close()
    for rid, prompt in prompts.items():
        want, gaps_ok = _oracle_generation(s, 100 + rid, prompt, 10, SMALL["eos"])
        assert terms[rid]["error"] == 0, terms[rid]
        if gaps_ok:
            assert terms[rid]["tokens"] == want, (rid, terms[rid]["tokens"], want)
    assert s.snapshot().request_count == 0
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()


def test_injected_failures_roll_back_one_lane(kk, tmp_path):
    s = Stack(kk, tmp_path, SMALL)
    for rid in (1, 2):
        s.create(rid)
    got, ok = s.batch([1, 2], [5, 6], [0, 0])
    assert ok == [1, 1]
    assert s.R["backend_inject_failure"](s.backend, 0) == 1          # submission
    got, ok = s.batch([1, 2], [7, 8], [1, 1])
    assert sorted(ok) == [0, 1]
    failed = [1, 2][ok.index(0)]
    assert s.R["backend_inject_failure"](s.backend, 1) == 1          # completion
    pos = {1: 2 if failed != 1 else 1, 2: 2 if failed != 2 else 1}
    got, ok = s.batch([1, 2], [9, 9], [pos[1], pos[2]])
    assert sorted(ok) == [0, 1]
    assert s.snapshot().active_transaction_count == 0
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()


EXECUTION_FAILED = 9  # EngineKvError::ExecutionFailed


def _last_error(s):
    buf = C.create_string_buffer(512)
    s.R["runner_last_error"](s.runner, buf, 512)
    return buf.value.decode()


@pytest.mark.parametrize("graphs", [0, 1])
def test_device_wait_timeout_fails_the_step_and_rolls_back(kk, tmp_path, graphs):
    """A device-detected error fails the fused step at commit: the test hook
    makes CTA 0 of every attention launch drop a stage with a 1 ms wait limit,
    so a bounded wait runs out and the step's error word is set. Every lane
    reports failure, every reservation rolls back (committed lengths,
    tables and invariants unchanged, no transaction left open), and the same
    positions decode correctly once the hook is cleared (reference: a
    completion failure surfaces as ExecutionFailed and rolls the transaction
    back, src/cuda/engine/transaction.cpp:84-120)."""
    s = Stack(kk, tmp_path, SMALL, batch=4, graphs=graphs)
    K = kk.kernels()
    ids = [1, 2, 3]
    for rid in ids:
        s.create(rid)
    toks, pos = [5, 6, 7], [0, 0, 0]
    for _ in range(9):   # a few tokens of context, a micro page filled and sealed
        got, ok = s.batch(ids, toks, pos)
        want, logits, _ = s.oracle.forward(ids, toks, pos, want_hidden=False)
        assert ok == [1, 1, 1]
        assert_greedy(got, want, logits)
        toks, pos = [int(w) for w in want], [p_ + 1 for p_ in pos]
    snap0 = s.snapshot()
    assert K["debug_attention_fault"](0, 1_000_000) == 0
    try:
        got, ok = s.batch(ids, toks, pos)
    finally:
        assert K["debug_attention_fault"](0xFFFFFFFF, 0) == 0
    assert ok == [0, 0, 0]
    assert "bounded device wait" in _last_error(s)
    snap = s.snapshot()
    assert snap.committed_token_count == snap0.committed_token_count == 27
    assert snap.active_transaction_count == 0
    assert snap.allocated_micro_pages == snap0.allocated_micro_pages
    assert s.R["backend_check_invariants"](s.backend) == 1
    # the module-global words of the public entry points saw nothing
    assert K["device_status"](s.stream) == 0
    got, ok = s.batch(ids, toks, pos)
    want, logits, _ = s.oracle.forward(ids, toks, pos, want_hidden=False)
    assert ok == [1, 1, 1]
    assert_greedy(got, want, logits)
    assert s.snapshot().committed_token_count == 30
    s.close()


def test_per_layer_commit_fails_on_device_error(kk):
    """The per-layer transaction SPI: a bounded wait that runs out inside
    attendLayer fails the transaction at commit with ExecutionFailed and
    rolls it back; a transaction on the same stream after the error commits."""
    R, K = kk.runtime(), kk.kernels()
    L, hkv, D, hq = 2, 4, 64, 32
    backend = R["backend_create"](L, hkv, D, hq, hq * 512 * 4, 64, 4)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert R["backend_create_request"](backend, 1) == 0
    assert R["backend_append"](backend, 1, 70) == 0
    g = torch.Generator().manual_seed(9)
    q = (torch.randn(hq * D, generator=g) / 8).half().cuda()
    out = torch.zeros_like(q)
    ws = torch.zeros(hq * 512 * 4, dtype=torch.uint8, device="cuda")

    def token(length, fault):
        st = C.c_int(0)
        t = R["txn_reserve"](backend, 1, length, stream, C.byref(st))
        assert t and st.value == 0
        for layer in range(L):
            k = (torch.randn(hkv * D, generator=g) / 8).half().cuda()
            v = (torch.randn(hkv * D, generator=g) / 8).half().cuda()
            assert R["txn_write_layer"](t, layer, k.data_ptr(), v.data_ptr()) == 0
            if fault:
                assert K["debug_attention_fault"](0, 1_000_000) == 0
            try:
                assert R["txn_attend_layer"](t, layer, q.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                             ws.numel(), 0.125) == 0
                torch.cuda.synchronize()
            finally:
                assert K["debug_attention_fault"](0xFFFFFFFF, 0) == 0
        rc = R["txn_commit"](t)
        R["txn_destroy"](t)
        return rc

    assert token(70, fault=True) == EXECUTION_FAILED
    snap = kk.BackendSnapshot()
    R["backend_snapshot"](backend, C.byref(snap))
    assert snap.committed_token_count == 70 and snap.active_transaction_count == 0
    assert R["backend_check_invariants"](backend) == 1
    assert token(70, fault=False) == 0
    R["backend_snapshot"](backend, C.byref(snap))
    assert snap.committed_token_count == 71 and snap.active_transaction_count == 0
    assert R["backend_check_invariants"](backend) == 1
    R["backend_destroy"](backend)


class _DevArray:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<u2", "data": (ptr, False),
                                         "version": 3}


def dev_view(ptr, n):
    """Zero-copy uint16 view of device memory owned by the library."""
    return torch.as_tensor(_DevArray(ptr, n), device="cuda")


def test_per_layer_spi_write_attend_matches_oracle(kk, tmp_path):
    """The reference-facing per-layer transaction SPI (writeLayer / attendLayer /
    attendLayerBatch, reference tests/cuda/cuda_engine_kv_backend_test.cpp:258-345)
    on this backend, against the oracle's paged GQA attention over the
    reserved table (prefix + the token just written)."""
    R = kk.runtime()
    L, hkv, D, hq = 2, 4, 64, 32
    micro_cap, extent_cap = 128, 8
    backend = R["backend_create"](L, hkv, D, hq, hq * 512 * 4, micro_cap, extent_cap)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    pools = kk.KvPools()
    assert R["backend_pools"](backend, C.byref(pools))
    row = hkv * D
    micro = dev_view(pools.micro, micro_cap * L * 2 * 8 * row)
    extent = dev_view(pools.extent, extent_cap * L * 2 * 64 * row)
    K = kk.kernels()
    K["fill_fp16"](C.c_void_p(pools.micro), micro.numel(), 5, 0.3, stream)
    K["fill_fp16"](C.c_void_p(pools.extent), extent.numel(), 6, 0.3, stream)
    g = torch.Generator().manual_seed(2)
    lengths = {1: 0, 2: 70, 3: 131}
    for rid, n in lengths.items():
        assert R["backend_create_request"](backend, rid) == 0
        if n:
            assert R["backend_append"](backend, rid, n) == 0
    R["backend_seal"](backend, 3)
    assert R["backend_promote"](backend, 3, 0, stream) == 0
    assert R["backend_promote"](backend, 3, 64, stream) == 0
    assert R["backend_fork"](backend, 2, 4) == 0   # shared partial tail -> COW on next write
    lengths[4] = 70
    ids = [1, 2, 3, 4]
    for step in range(3):
        txns, st = [], C.c_int(0)
        for rid in ids:
            t = R["txn_reserve"](backend, rid, lengths[rid], stream, C.byref(st))
            assert t and st.value == 0
            txns.append(t)
        tables = []
        for t in txns:
            buf = (kk.KkEntry * 64)()
            tt = kk.KkTableOut(C.cast(buf, C.POINTER(kk.KkEntry)), 64, 0, 0)
            assert R["txn_reserved_table"](t, C.byref(tt)) == 1
            tables.append([(buf[j].slot, buf[j].logical_token_begin, buf[j].valid_tokens, buf[j].kind)
                           for j in range(tt.count)])
        q = (torch.randn(len(ids), hq * D, generator=g) / 8).half().cuda()
        out = torch.zeros_like(q)
        ws = torch.zeros(hq * 512 * 4, dtype=torch.uint8, device="cuda")
        for layer in range(L):
            for t in txns:
                k = (torch.randn(row, generator=g) / 8).half().cuda()
                v = (torch.randn(row, generator=g) / 8).half().cuda()
                assert R["txn_write_layer"](t, layer, k.data_ptr(), v.data_ptr()) == 0
            if step % 2 == 0:
                statuses = (C.c_int * len(ids))()
                R["txn_attend_batch"]((C.c_void_p * len(ids))(*txns), len(ids), layer, q.data_ptr(),
                                      out.data_ptr(), hq * D * 2, ws.data_ptr(), ws.numel(), 0.125,
                                      statuses)
                assert list(statuses) == [0] * len(ids)
            else:
                for i, t in enumerate(txns):
                    assert R["txn_attend_layer"](t, layer, q[i].data_ptr(), out[i].data_ptr(),
                                                 ws.data_ptr(), ws.numel(), 0.125) == 0
            torch.cuda.synchronize()
            hm, he = micro.cpu().numpy(), extent.cpu().numpy()
            for i in range(len(ids)):
                ref = ko.paged_attention(hm, he, L, hkv, D, layer, hq, tables[i],
                                         q[i].cpu().view(torch.int16).numpy().view(np.uint16))
                got = out[i].cpu().float().numpy()
                assert np.max(np.abs(got - ref.view(np.float16).astype(np.float32))) < TOL
        for t in txns:
            assert R["txn_commit"](t) == 0
            R["txn_destroy"](t)
        for rid in lengths:
            lengths[rid] += 1
    assert R["backend_check_invariants"](backend) == 1
    snap = kk.BackendSnapshot()
    R["backend_snapshot"](backend, C.byref(snap))
    assert snap.batched_attention_submissions == 2 * L
    R["backend_destroy"](backend)


def test_backend_gather_returns_committed_kv(kk):
    """kkrt_backend_gather: the committed KV of a request (extent body after
    promotion + micro tail) as one contiguous tensor."""
    R = kk.runtime()
    L, hkv, D = 2, 4, 64
    backend = R["backend_create"](L, hkv, D, 32, 1 << 20, 64, 8)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert R["backend_create_request"](backend, 7) == 0
    assert R["backend_append"](backend, 7, 150) == 0
    R["backend_seal"](backend, 7)
    assert R["backend_promote"](backend, 7, 0, stream) == 0
    assert R["backend_promote"](backend, 7, 64, stream) == 0
    pools = kk.KvPools()
    assert R["backend_pools"](backend, C.byref(pools))
    K = kk.kernels()
    for ptr, cap, tokens in [(pools.micro, pools.micro_capacity, 8), (pools.extent, pools.extent_capacity, 64)]:
        assert K["fill_fp16"](C.c_void_p(ptr), cap * L * 2 * tokens * hkv * D, 17 + tokens, 0.5, stream) == 0
    out = torch.zeros(L, 2, 150, hkv, D, dtype=torch.half, device="cuda")
    assert R["backend_gather"](backend, 7, out.data_ptr(), stream) == 0
    buf = (kk.KkEntry * 64)()
    t = kk.KkTableOut(C.cast(buf, C.POINTER(kk.KkEntry)), 64, 0, 0)
    assert R["backend_block_table"](backend, 7, C.byref(t))
    entries = [buf[i] for i in range(t.count)]
    assert [e.kind for e in entries][:2] == [1, 1]
    micro = dev_view(pools.micro, pools.micro_capacity * L * 2 * 8 * hkv * D).view(torch.half).view(
        pools.micro_capacity, L, 2, 8, hkv, D)
    extent = dev_view(pools.extent, pools.extent_capacity * L * 2 * 64 * hkv * D).view(torch.half).view(
        pools.extent_capacity, L, 2, 64, hkv, D)
    for e in entries:
        src = (micro if e.kind == 0 else extent)[e.slot, :, :, :e.valid_tokens]
        assert torch.equal(out[:, :, e.logical_token_begin:e.logical_token_begin + e.valid_tokens], src)
    R["backend_destroy"](backend)


def test_auto_promotion_folds_full_runs_and_keeps_outputs(kk, tmp_path):
    """With auto-promotion on, every 64-aligned run of 8 sealed micro pages
    becomes one extent page as generation crosses it; greedy tokens and
    logits still follow the oracle, and the pool accounting stays valid."""
    cfg = dict(SMALL, max_positions=256)
    s = Stack(kk, tmp_path, cfg, batch=4, micro=128, extent=8)
    assert s.R["runner_set_auto_promote"](s.runner, 1) == 1
    ids = [1, 2, 3]
    for rid in ids:
        s.create(rid)
    pos = {1: 0, 2: 0, 3: 0}
    tok = {1: 5, 2: 9, 3: 77}
    start = {1: 0, 2: 20, 3: 60}   # lanes cross 64-token boundaries at different steps
    for rid in ids:
        for p in range(start[rid]):
            g, ok = s.batch([rid], [tok[rid]], [p])
            w, _, _ = s.oracle.forward([rid], [tok[rid]], [p], want_hidden=False)
            assert ok == [1]
            tok[rid] = int(w[0])
        pos[rid] = start[rid]
    for step in range(140):
        toks = [tok[r] for r in ids]
        ps = [pos[r] for r in ids]
        got, ok = s.batch(ids, toks, ps)
        want, logits, _ = s.oracle.forward(ids, toks, ps, want_hidden=False)
        assert ok == [1, 1, 1]
        assert_greedy(got, want, logits)
        for i, r in enumerate(ids):
            tok[r] = int(want[i])
            pos[r] += 1
    buf = (kk.KkEntry * 512)()
    for r in ids:
        t = kk.KkTableOut(C.cast(buf, C.POINTER(kk.KkEntry)), 512, 0, 0)
        assert s.R["backend_block_table"](s.backend, r, C.byref(t))
        kinds = [buf[i].kind for i in range(t.count)]
        extents = sum(1 for k in kinds if k == 1)
        assert extents == pos[r] // 64, (r, pos[r], kinds)
        assert all(k == 1 for k in kinds[:extents]) and all(k == 0 for k in kinds[extents:])
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()


@pytest.mark.slow
def test_tinyllama_shape_greedy_decode_config2(kk, tmp_path):
    """TinyLlama-1.1B shape, batch 1, 6 seeded prompt ids
    uniform in [3, 32000), 32 new tokens; greedy tokens vs the oracle."""
    cfg = dict(synth().TINYLLAMA)
    s = Stack(kk, tmp_path, cfg, seed=2, std=0.02, batch=1, micro=64, extent=4)
    rng = random.Random(0x4B564341434845)
    prompt = [rng.randrange(3, 32000) for _ in range(6)]
    s.create(1)
    tok, got, want_all = None, [], []
    for p in range(6 + 31):
        t = prompt[p] if p < 6 else tok
        g, ok = s.batch([1], [t], [p])
        w, logits, _ = s.oracle.forward([1], [t], [p], want_hidden=False)
        assert ok == [1]
        if p >= 5:
            got.append(g[0])
            want_all.append((int(w[0]), logits[0]))
        tok = int(w[0])
    mism = [(i, a, b) for i, (a, (b, lg)) in enumerate(zip(got, want_all))
            if a != b and np.diff(np.sort(lg)[-2:])[0] > TOL]
    assert not mism, mism
    s.close()


def _prefill(s, rid, toks, first):
    n = len(toks)
    out = C.c_uint32(0)
    ok = s.R["runner_prefill"](s.runner, rid, (C.c_uint32 * n)(*toks), n, first, C.byref(out))
    if not ok:
        buf = C.create_string_buffer(512)
        s.R["runner_last_error"](s.runner, buf, 512)
        return None, buf.value.decode()
    return out.value, ""


def _oracle_prompt(s, rid, toks, first):
    """The oracle fed one position at a time, as the reference's scheduler
    feeds a prompt; returns the greedy token and logits after the last one."""
    for i, t in enumerate(toks):
        want, logits, _ = s.oracle.forward([rid], [t], [first + i], want_hidden=False)
    return int(want[0]), logits


@pytest.mark.parametrize("batch,lengths", [(8, [150]), (16, [13, 37, 1, 64, 9]), (32, [200]), (64, [300, 77])])
def test_fused_prefill_matches_per_position_oracle(kk, tmp_path, batch, lengths):
    """kkrt_runner_prefill: the prompt runs as chunks of up to max_batch_size
    consecutive positions of one request, each attending causally to tokens
    [0, p]. The greedy token after every prefill call and the decode tokens
    that follow match the oracle fed one position at a time; the page table
    covers exactly the prompt."""
    s = Stack(kk, tmp_path, SMALL, batch=batch)
    rng = random.Random(batch + sum(lengths))
    s.create(5)
    pos = 0
    for n in lengths:
        toks = [rng.randrange(3, 1000) for _ in range(n)]
        got, err = _prefill(s, 5, toks, pos)
        assert got is not None, err
        want, logits = _oracle_prompt(s, 5, toks, pos)
        assert_greedy([got], [want], logits)
        pos += n
        tok = want
    for _ in range(12):
        g, ok = s.batch([5], [tok], [pos])
        w, logits, _ = s.oracle.forward([5], [tok], [pos], want_hidden=False)
        assert ok == [1]
        assert_greedy(g, w, logits)
        tok, pos = int(w[0]), pos + 1
    tbl = (kk.KkEntry * 128)()
    t = kk.KkTableOut(C.cast(tbl, C.POINTER(kk.KkEntry)), 128, 0, 0)
    assert s.R["backend_block_table"](s.backend, 5, C.byref(t)) == 1
    assert sum(tbl[i].valid_tokens for i in range(t.count)) == pos
    assert s.snapshot().committed_token_count == pos
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()


def test_fused_prefill_after_fork_copies_the_shared_tail(kk, tmp_path):
    """A child forked at 11 tokens shares a 3-token partial tail; the child's
    prefill appends through partial-tail copy-on-write, and both the parent's
    decode and the child's prefill continue to follow the oracle."""
    s = Stack(kk, tmp_path, SMALL, batch=16)
    rng = random.Random(17)
    s.create(1)
    head = [rng.randrange(3, 1000) for _ in range(11)]
    got, err = _prefill(s, 1, head, 0)
    assert got is not None, err
    want, _ = _oracle_prompt(s, 1, head, 0)
    assert s.R["backend_fork"](s.backend, 1, 2) == 0
    s.oracle.fork(1, 2)
    tail = [rng.randrange(3, 1000) for _ in range(29)]
    got2, err = _prefill(s, 2, tail, 11)
    assert got2 is not None, err
    want2, logits2 = _oracle_prompt(s, 2, tail, 11)
    assert_greedy([got2], [want2], logits2)
    # the parent still sees its own (unmodified) tail
    g, ok = s.batch([1, 2], [want, want2], [11, 40])
    w, logits, _ = s.oracle.forward([1, 2], [want, want2], [11, 40], want_hidden=False)
    assert ok == [1, 1]
    assert_greedy(g, w, logits)
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()


def test_fused_prefill_auto_promotes_and_rejects_bad_calls(kk, tmp_path):
    cfg = dict(SMALL, max_positions=256)
    s = Stack(kk, tmp_path, cfg, batch=32, micro=128, extent=8)
    assert s.R["runner_set_auto_promote"](s.runner, 1) == 1
    rng = random.Random(23)
    s.create(7)
    toks = [rng.randrange(3, 1000) for _ in range(150)]
    got, err = _prefill(s, 7, toks, 0)
    assert got is not None, err
    want, logits = _oracle_prompt(s, 7, toks, 0)
    assert_greedy([got], [want], logits)
    buf = (kk.KkEntry * 64)()
    t = kk.KkTableOut(C.cast(buf, C.POINTER(kk.KkEntry)), 64, 0, 0)
    assert s.R["backend_block_table"](s.backend, 7, C.byref(t)) == 1
    assert [buf[i].kind for i in range(t.count)][:2] == [1, 1]
    assert sum(1 for i in range(t.count) if buf[i].kind == 1) == 2
    # wrong first position, unknown request, out-of-range token: rejected, state intact
    assert _prefill(s, 7, [5], 149)[0] is None
    assert _prefill(s, 99, [5], 0)[0] is None
    assert _prefill(s, 7, [cfg["vocab"]], 150)[0] is None
    assert s.snapshot().committed_token_count == 150
    g, ok = s.batch([7], [want], [150])
    w, logits, _ = s.oracle.forward([7], [want], [150], want_hidden=False)
    assert ok == [1]
    assert_greedy(g, w, logits)
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()
