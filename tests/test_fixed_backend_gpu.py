"""Fixed-page CUDA backend (Fixed-8/16/32/64; reference
createFixedCudaEngineKvBackend, src/cuda/engine/backend.cpp:579-598, with
FixedPageManager metadata, src/fixed/*.cpp) behind the same SPI as the two-pool
backend, through the C ABI:

* the paged attention kernels over pages of every fixed size against the
  plain PyTorch FP32 reference (tolerance as for the two-pool pages);
* KV write and copy into fixed pages: exact;
* the fused decode step (fork, partial-tail copy-on-write), fused prefill
  and the gather against the CPU oracle: greedy tokens identical wherever
  the oracle's top-2 logit gap exceeds 2e-2, tables and gathered KV exact.
"""
import ctypes as C
import importlib.util
import random
from pathlib import Path

import numpy as np
import pytest
import torch

import kk_oracle_py as ko
from gpu_util import attention_ref, p, to_device_bytes

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

ROOT = Path(__file__).resolve().parent.parent
TOL = 2e-2
SMALL = dict(hidden=512, intermediate=1024, layers=3, q_heads=8, kv_heads=2, head_dim=64, vocab=1000,
             max_positions=512, eps=1e-5, theta=10000.0, bos=1, eos=2)
SIZES = [8, 16, 32, 64]


class _DevArray:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<u2", "data": (ptr, False),
                                         "version": 3}


def dev_view(ptr, n):
    """Zero-copy uint16 view of device memory owned by the library."""
    return torch.as_tensor(_DevArray(ptr, n), device="cuda")


def sync_ok(K):
    torch.cuda.synchronize()
    assert K["device_status"](None) == 0


def fixed_pools(kk, layers, kv_heads, head_dim, tokens, pages, seed):
    g = torch.Generator().manual_seed(seed)
    pool = (torch.randn(pages, layers, 2, tokens, kv_heads, head_dim, generator=g) / 8).half().cuda()
    pools = kk.KvPools(p(pool), 0, pages, 0, layers, kv_heads, head_dim, tokens)
    return pools, pool


def fixed_tables(contexts, tokens, pages, rng):
    slots = list(range(pages))
    rng.shuffle(slots)
    tables = []
    for ctx in contexts:
        entries, t = [], 0
        while t < ctx:
            n = min(tokens, ctx - t)
            entries.append((slots.pop(), t, n))
            t += n
        tables.append(entries)
    return tables


@pytest.mark.parametrize("tokens", [16, 32, 64])
@pytest.mark.parametrize("hkv,hq", [(4, 32), (1, 16), (8, 64), (2, 8)])
@pytest.mark.parametrize("variant,plan", [(1, "lane"), (2, "lane"), (2, "balanced")],
                         ids=["direct-lane", "tma-lane", "tma-balanced"])
def test_fixed_pages_attention_matches_torch(kk, tokens, hkv, hq, variant, plan):
    """Pages of a fixed-page pool (kk_kv_pools::micro_page_tokens = 16/32/64):
    the TMA kernel loads them in chunks like extent pages (per-head boxes when
    a page is shorter than a stage), the direct kernel row by row."""
    K = kk.kernels()
    assert K["attention_set_variant"](variant) == 0
    try:
        contexts = [1, tokens - 1, tokens, tokens + 1, 5 * tokens + 3, 700]
        layers, D = 2, 64
        pages = sum((c + tokens - 1) // tokens for c in contexts) + 4
        pools, pool = fixed_pools(kk, layers, hkv, D, tokens, pages, seed=tokens + hkv)
        tables = fixed_tables(contexts, tokens, pages, random.Random(tokens * 7 + hkv))
        flat = [e for tbl in tables for e in tbl]
        descs = (kk.PageDesc * len(flat))(*[kk.PageDesc(s, b, v, 0, 0, 0) for s, b, v in flat])
        B = len(contexts)
        lanes = (kk.AttnLane * B)()
        off = 0
        for b, tbl in enumerate(tables):
            lanes[b].desc_offset, lanes[b].desc_count = off, len(tbl)
            lanes[b].token_count, lanes[b].query_row = sum(e[2] for e in tbl), b
            off += len(tbl)
        items = (kk.AttnItem * 4096)()
        if plan == "balanced":
            n_items = K["attention_plan_balanced"](descs, lanes, B, 5, items, 4096)
        else:
            n_items = K["attention_plan"](descs, lanes, B, 96, items, 4096)
        assert 0 < n_items <= 4096
        q = (torch.randn(B, hq * D) / 8).half().cuda()
        out = torch.zeros(B, hq * D, dtype=torch.half, device="cuda")
        ws_bytes = K["attention_workspace_bytes"](B, n_items, hq, D)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
        d_descs, d_lanes, d_items = to_device_bytes(descs), to_device_bytes(lanes), to_device_bytes(items)
        for layer in range(layers):
            rc = K["paged_decode_attention"](C.byref(pools), layer, hq, p(d_descs), p(d_lanes), B, p(d_items),
                                             n_items, p(q), hq * D, p(out), hq * D, 0.125, p(ws), ws_bytes, None)
            assert rc == 0
            sync_ok(K)
            for b, tbl in enumerate(tables):
                k = torch.cat([pool[s, layer, 0, :v].float() for s, _, v in tbl])
                v = torch.cat([pool[s, layer, 1, :v].float() for s, _, v in tbl])
                ref = attention_ref(q[b].view(hq, D), k, v, 0.125)
                torch.testing.assert_close(out[b].view(hq, D).float(), ref, atol=2e-3, rtol=2e-2)
    finally:
        K["attention_set_variant"](0)


@pytest.mark.parametrize("tokens", [16, 64])
def test_fixed_pages_reject_bad_page_size_and_overfull_descriptors(kk, tokens):
    K = kk.kernels()
    pools, pool = fixed_pools(kk, 1, 4, 64, tokens, 4, seed=1)
    bad = kk.KvPools(pools.micro, 0, 4, 0, 1, 4, 64, 24)   # 24-token pages are not supported
    slots = (kk.KvSlot * 1)(kk.KvSlot(0, 0, 0, 1))
    kv = torch.zeros(2, 256, dtype=torch.half, device="cuda")
    d_slots = to_device_bytes(slots)
    assert K["kv_write"](C.byref(bad), 0, 1, p(d_slots), 1, p(kv[0]), p(kv[1]), 0, 0, None) == kk.KK_EINVAL
    # a write past the page's capacity is reported, not performed
    over = (kk.KvSlot * 1)(kk.KvSlot(1, tokens, 0, 1))
    before = pool.clone()
    assert K["kv_write"](C.byref(pools), 0, 1, p(to_device_bytes(over)), 1, p(kv[0]), p(kv[1]), 0, 0, None) == 0
    torch.cuda.synchronize()
    assert K["device_status"](None) != 0
    assert torch.equal(pool, before)


@pytest.mark.parametrize("tokens", SIZES)
def test_fixed_pages_write_and_copy_are_exact(kk, tokens):
    K = kk.kernels()
    L, hkv, D = 3, 4, 64
    pools, pool = fixed_pools(kk, L, hkv, D, tokens, 6, seed=tokens)
    row = hkv * D
    key = torch.randn(L, row).half().cuda()
    val = torch.randn(L, row).half().cuda()
    slots = (kk.KvSlot * 1)(kk.KvSlot(2, tokens - 1, 0, 1))
    assert K["kv_write"](C.byref(pools), 0, L, p(to_device_bytes(slots)), 1, p(key), p(val), 0, row, None) == 0
    sync_ok(K)
    for layer in range(L):
        assert torch.equal(pool[2, layer, 0, tokens - 1].reshape(-1), key[layer])
        assert torch.equal(pool[2, layer, 1, tokens - 1].reshape(-1), val[layer])
    n = max(tokens // 2, 1)
    copies = (kk.KvCopy * 1)(kk.KvCopy(2, 5, n, 0, 0))
    assert K["kv_copy_tokens"](C.byref(pools), 0, L, p(to_device_bytes(copies)), 1, None) == 0
    sync_ok(K)
    assert torch.equal(pool[5, :, :, :n], pool[2, :, :, :n])


# ---------------------------------------------------------------------------
# backend + runner against the oracle

def synth():
    spec = importlib.util.spec_from_file_location("kk_synth", ROOT / "kim-kvcache_b200" / "synthetic.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


class FixedStack:
    """Fixed-page backend + runner + oracle for one model config."""

    def __init__(self, kk, tmp, cfg, tokens, pages=160, batch=8):
        self.kk, self.cfg = kk, cfg
        self.R = kk.runtime()
        man, data, w = synth().write_archive(tmp, cfg, seed=3, std=0.05, keep_weights=True)
        self.stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        self.backend = self.R["fixed_backend_create"](cfg["layers"], cfg["kv_heads"], cfg["head_dim"],
                                                      cfg["q_heads"], cfg["q_heads"] * cfg["max_positions"] * 4,
                                                      tokens, pages)
        assert self.backend
        assert self.R["backend_kind"](self.backend) == 1
        st, det = C.c_int(0), C.create_string_buffer(256)
        self.runner = self.R["runner_create"](man.encode(), data.encode(), self.backend, self.stream,
                                              batch, 1, 1, C.byref(st), det, 256)
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
        return [out[i] for i in range(n)], [ok[i] for i in range(n)]

    def table(self, rid):
        buf = (self.kk.KkEntry * 256)()
        t = self.kk.KkTableOut(C.cast(buf, C.POINTER(self.kk.KkEntry)), 256, 0, 0)
        assert self.R["backend_block_table"](self.backend, rid, C.byref(t)) == 1
        return [buf[i] for i in range(t.count)]

    def snapshot(self):
        s = self.kk.BackendSnapshot()
        self.R["backend_snapshot"](self.backend, C.byref(s))
        return s


def assert_greedy(got, want, logits):
    for g, w, row in zip(got, want, logits):
        top = np.sort(row)[-2:]
        if top[1] - top[0] > TOL:
            assert g == w, f"greedy {g} != oracle {w} (gap {top[1] - top[0]:.4f})"


@pytest.mark.parametrize("tokens", SIZES)
def test_fixed_backend_decode_with_fork_and_partial_tail_cow(kk, tmp_path, tokens):
    s = FixedStack(kk, tmp_path, SMALL, tokens)
    rng = random.Random(tokens)
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
    # fork request 1 at 11 tokens: a partial tail page for every page size,
    # so both sides copy the shared tail before their next write
    assert s.R["backend_fork"](s.backend, 1, 9) == 0
    s.oracle.fork(1, 9)
    prompts[9], pos[9], nxt[9] = prompts[1], pos[1], nxt[1]
    for _ in range(2 * tokens + 3):
        step([1, 2, 3, 9])
    for rid in (1, 9):
        entries = s.table(rid)
        assert sum(e.valid_tokens for e in entries) == pos[rid]
        assert all(e.kind == 0 and e.valid_tokens <= tokens for e in entries)
        assert all(e.valid_tokens == tokens for e in entries[:-1])
    # pages that were full at the fork stay shared; the partial tail was
    # copied by each side before its first write
    shared = 11 // tokens
    t1, t9 = s.table(1), s.table(9)
    assert all(t1[i].slot == t9[i].slot for i in range(shared))
    assert t1[shared].slot != t9[shared].slot
    snap = s.snapshot()
    assert snap.committed_token_count == sum(pos.values()) and snap.active_transaction_count == 0
    assert s.R["backend_check_invariants"](s.backend) == 1
    for rid in (1, 2, 3, 9):
        assert s.R["backend_release"](s.backend, rid) == 0
    assert s.snapshot().allocated_micro_pages == 0
    s.close()


@pytest.mark.parametrize("tokens", [16, 64])
def test_fixed_backend_prefill_then_decode_matches_oracle(kk, tmp_path, tokens):
    s = FixedStack(kk, tmp_path, SMALL, tokens, batch=16)
    rng = random.Random(40 + tokens)
    s.create(5)
    pos, tok = 0, None
    for n in (37, 5):
        toks = [rng.randrange(3, 1000) for _ in range(n)]
        out = C.c_uint32(0)
        assert s.R["runner_prefill"](s.runner, 5, (C.c_uint32 * n)(*toks), n, pos, C.byref(out)) == 1
        want = logits = None
        for i, t in enumerate(toks):
            want, logits, _ = s.oracle.forward([5], [t], [pos + i], want_hidden=False)
        assert_greedy([out.value], want, logits)
        pos += n
        tok = int(want[0])
    for _ in range(8):
        g, ok = s.batch([5], [tok], [pos])
        w, logits, _ = s.oracle.forward([5], [tok], [pos], want_hidden=False)
        assert ok == [1]
        assert_greedy(g, w, logits)
        tok, pos = int(w[0]), pos + 1
    assert sum(e.valid_tokens for e in s.table(5)) == pos
    assert s.R["backend_check_invariants"](s.backend) == 1
    s.close()


@pytest.mark.parametrize("tokens", SIZES)
def test_fixed_backend_gather_returns_committed_kv(kk, tokens):
    R = kk.runtime()
    K = kk.kernels()
    L, hkv, D, pages = 2, 4, 64, 32
    backend = R["fixed_backend_create"](L, hkv, D, 32, 1 << 20, tokens, pages)
    assert backend and R["backend_kind"](backend) == 1
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert R["backend_create_request"](backend, 7) == 0
    assert R["backend_append"](backend, 7, 150) == 0
    assert R["backend_promote"](backend, 7, 0, stream) != 0      # no promotion on fixed pages
    pools = kk.KvPools()
    assert R["backend_pools"](backend, C.byref(pools))
    assert pools.micro_page_tokens == tokens and pools.extent_capacity == 0
    n = pools.micro_capacity * L * 2 * tokens * hkv * D
    assert K["fill_fp16"](C.c_void_p(pools.micro), n, 23 + tokens, 0.5, stream) == 0
    out = torch.zeros(L, 2, 150, hkv, D, dtype=torch.half, device="cuda")
    assert R["backend_gather"](backend, 7, out.data_ptr(), stream) == 0
    buf = (kk.KkEntry * 64)()
    t = kk.KkTableOut(C.cast(buf, C.POINTER(kk.KkEntry)), 64, 0, 0)
    assert R["backend_block_table"](backend, 7, C.byref(t))
    pool = dev_view(pools.micro, n).view(torch.half).view(pools.micro_capacity, L, 2, tokens, hkv, D)
    for i in range(t.count):
        e = buf[i]
        src = pool[e.slot, :, :, :e.valid_tokens]
        assert torch.equal(out[:, :, e.logical_token_begin:e.logical_token_begin + e.valid_tokens], src)
    R["backend_destroy"](backend)
