"""GPU numerics of the sm_100a kernels through the C ABI (include/kk_kernels.h),
each against a plain PyTorch FP32 reference of the same op. Tolerances are
written per test; integer / byte work (KV writes, copies, argmax) is exact."""
import ctypes as C
import random

import numpy as np
import pytest
import torch

from gpu_util import (attention_ref, build_tables, descs_and_lanes, gather_kv, make_pools, p,
                      rope_ref, to_device_bytes)

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


@pytest.fixture(scope="module")
def K(kk):
    return kk.kernels()


@pytest.fixture
def attn_variant(K):
    """Selects the attention kernel for one test and restores AUTO after it."""
    yield lambda v: K["attention_set_variant"](v) == 0 or pytest.fail("variant rejected")
    K["attention_set_variant"](0)


def sync_ok(K):
    torch.cuda.synchronize()
    assert K["device_status"](None) == 0


@pytest.fixture(params=[0, 1], ids=["rowmajor", "packed"])
def wlayout(request):
    return request.param


_PACKED = {}


def packed_weight(kk, K, w):
    """kk_gemm_pack_weight output for w (cached per tensor for the test's lifetime)."""
    key = (w.data_ptr(), tuple(w.shape))
    if key not in _PACKED or _PACKED[key][0] is not w:
        buf = torch.empty(K["gemm_packed_bytes"](*w.shape) // 2, dtype=torch.half, device="cuda")
        assert K["gemm_pack_weight"](p(w), w.shape[0], w.shape[1], p(buf), None) == 0
        _PACKED.clear()
        _PACKED[key] = (w, buf)
    return _PACKED[key][1]


def gemm(kk, K, w, x, epi, out=None, out_stride=0, split=0, layout=0, **extra):
    d = kk.GemmDesc()
    d.weight, d.M, d.K = p(w), w.shape[0], w.shape[1]
    if layout == kk.W_PACKED:
        d.weight, d.weight_layout = p(packed_weight(kk, K, w)), layout
    d.x, d.N, d.x_stride, d.x_rows = p(x), extra.pop("N", x.shape[0]), x.shape[1], x.shape[0]
    d.epilogue, d.out, d.out_stride, d.split_k = epi, p(out), out_stride, split
    for k_, v in extra.items():
        setattr(d, k_, v)
    rc = K["gemm"](C.byref(d), None)
    assert rc == 0, f"kk_gemm returned {rc}"


@pytest.mark.parametrize("M,Kd,N,split", [
    (128, 64, 16, 1), (256, 2048, 32, 0), (300, 1000, 7, 3), (2560, 2048, 32, 0),
    (2048, 5632, 64, 0), (640, 512, 1, 2), (11264, 2048, 33, 0), (100, 256, 64, 4),
    (11264, 2048, 64, 0), (384, 640, 62, 3)])
def test_gemm_store_f32_matches_torch(kk, K, M, Kd, N, split, wlayout):
    g = torch.Generator().manual_seed(M * 7 + Kd + N)
    w = (torch.randn(M, Kd, generator=g) * 0.05).half().cuda()
    x = torch.randn(N, Kd, generator=g).half().cuda()
    out = torch.full((N, M), float("nan"), device="cuda")
    gemm(kk, K, w, x, kk.EPI_STORE_F32, out, M, split, layout=wlayout)
    sync_ok(K)
    ref = (x.float() @ w.float().T)
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=1e-3)  # FP32 accumulation


def test_gemm_store_f16_and_residual(kk, K, wlayout):
    g = torch.Generator().manual_seed(3)
    M, Kd, N = 512, 768, 24
    w = (torch.randn(M, Kd, generator=g) * 0.05).half().cuda()
    x = torch.randn(N, Kd, generator=g).half().cuda()
    acc = (x.float() @ w.float().T)
    out = torch.zeros(N, M, dtype=torch.half, device="cuda")
    gemm(kk, K, w, x, kk.EPI_STORE_F16, out, M, layout=wlayout)
    h = torch.randn(N, M, generator=g).half().cuda()
    h2 = h.clone()
    gemm(kk, K, w, x, kk.EPI_RESIDUAL, h2, M, layout=wlayout)
    sync_ok(K)
    # rounding point: half(acc), then an FP16 add; allow one FP16 ulp of slack
    torch.testing.assert_close(out.float(), acc.half().float(), atol=2e-3, rtol=2e-3)
    torch.testing.assert_close(h2.float(), (h.float() + acc.half().float()).half().float(),
                               atol=4e-3, rtol=2e-3)


def test_gemm_silu_pairs(kk, K, wlayout):
    g = torch.Generator().manual_seed(5)
    inter, Kd, N = 384, 512, 9
    wg = (torch.randn(inter, Kd, generator=g) * 0.05).half()
    wu = (torch.randn(inter, Kd, generator=g) * 0.05).half()
    w = torch.stack([wg, wu], dim=1).reshape(2 * inter, Kd).cuda()  # row 2i gate, 2i+1 up
    x = torch.randn(N, Kd, generator=g).half().cuda()
    out = torch.zeros(N, inter, dtype=torch.half, device="cuda")
    gemm(kk, K, w, x, kk.EPI_SILU_PAIRS, out, inter, layout=wlayout)
    sync_ok(K)
    gate = (x.float() @ wg.cuda().float().T).half().float()
    up = (x.float() @ wu.cuda().float().T).half().float()
    ref = (gate / (1 + torch.exp(-gate)) * up).half()
    torch.testing.assert_close(out.float(), ref.float(), atol=5e-3, rtol=5e-3)


def test_gemm_qkv_rope_writes_q_and_pages(kk, K, wlayout):
    layers, hkv, hq, D, hidden = 3, 2, 8, 64, 256
    pools, micro, extent = make_pools(kk, layers, hkv, D, 16, 4, seed=1)
    g = torch.Generator().manual_seed(9)
    M = (hq + 2 * hkv) * D
    w = (torch.randn(M, hidden, generator=g) * 0.05).half().cuda()
    N = 5
    x = torch.randn(16, hidden, generator=g).half().cuda()
    positions = torch.tensor([0, 7, 100, 513, 2047], dtype=torch.int32).cuda()
    slots = (kk.KvSlot * N)(*[kk.KvSlot(s, t, kd, 1) for s, t, kd in
                              [(3, 0, 0), (5, 7, 0), (1, 36, 1), (9, 2, 0), (2, 63, 1)]])
    slots_dev = to_device_bytes(slots)
    q_out = torch.zeros(N, hq * D, dtype=torch.half, device="cuda")
    layer = 1
    before_micro, before_extent = micro.clone(), extent.clone()
    gemm(kk, K, w, x, kk.EPI_QKV_ROPE, q_out, hq * D, N=N, positions=p(positions),
         slots=p(slots_dev), pools=pools, layer=layer, q_rows=hq * D, kv_rows=hkv * D,
         head_dim=D, rope_theta=10000.0, layout=wlayout)
    sync_ok(K)
    acc = (x[:N].float() @ w.float().T).half()  # [N, M] rounded projection outputs
    q_ref = rope_ref(acc[:, :hq * D].reshape(N, hq, D), positions, 10000.0).reshape(N, -1)
    k_ref = rope_ref(acc[:, hq * D:(hq + hkv) * D].reshape(N, hkv, D), positions, 10000.0)
    v_ref = acc[:, (hq + hkv) * D:].reshape(N, hkv, D)
    torch.testing.assert_close(q_out.float(), q_ref.float(), atol=4e-3, rtol=4e-3)
    for n in range(N):
        s = slots[n]
        pool = micro if s.kind == 0 else extent
        torch.testing.assert_close(pool[s.slot, layer, 0, s.page_token].float(), k_ref[n].float(),
                                   atol=4e-3, rtol=4e-3)
        # V is the rounded projection itself; FP32 summation order may move it by one ulp
        torch.testing.assert_close(pool[s.slot, layer, 1, s.page_token].float(), v_ref[n].float(),
                                   atol=2e-3, rtol=2e-3)
    # nothing else in the pools changed
    mask_m = torch.ones_like(micro, dtype=torch.bool)
    mask_e = torch.ones_like(extent, dtype=torch.bool)
    for n in range(N):
        s = slots[n]
        (mask_m if s.kind == 0 else mask_e)[s.slot, layer, :, s.page_token] = False
    assert torch.equal(micro[mask_m], before_micro[mask_m])
    assert torch.equal(extent[mask_e], before_extent[mask_e])


@pytest.mark.parametrize("V,N", [(32000, 4), (1000, 33), (130, 1)])
def test_gemm_argmax_matches_numpy(kk, K, V, N, wlayout):
    g = torch.Generator().manual_seed(V + N)
    Kd = 256
    w = (torch.randn(V, Kd, generator=g) * 0.05).half().cuda()
    x = torch.randn(64, Kd, generator=g).half().cuda()
    if V == 130:
        w[7] = w[100]  # exact tie between rows 7 and 100 -> lowest index wins
        w[100, 0] = w[7, 0]
    tokens = torch.zeros(N, dtype=torch.int32, device="cuda")
    ws = torch.zeros(K["argmax_workspace_bytes"](V, N), dtype=torch.uint8, device="cuda")
    logits = torch.zeros(N, V, device="cuda")
    for _ in range(2):  # the completion counter must reset itself between launches
        gemm(kk, K, w, x, kk.EPI_ARGMAX, logits, V, N=N, tokens=p(tokens), argmax_workspace=p(ws),
             layout=wlayout)
        sync_ok(K)
        ref = np.argmax(logits.cpu().numpy(), axis=1)
        assert tokens.cpu().numpy().tolist() == ref.tolist()
    torch.testing.assert_close(logits, x[:N].float() @ w.float().T, atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("M,Kd,N,epi", [(2560, 2048, 32, "f32"), (11264, 2048, 7, "silu"),
                                         (32000, 2048, 4, "argmax"), (300, 512, 33, "f32")])
def test_gemm_fused_rmsnorm_matches_torch(kk, K, M, Kd, N, epi):
    """norm_input + norm_weight = the reference's FP16 RMSNorm of x (weight g,
    rounded to FP16 as rmsNormBatchKernel stores it) followed by the
    projection, in one kernel: the kernel normalises its X tiles in shared
    memory before the tensor cores read them."""
    g = torch.Generator().manual_seed(M + N)
    w = (torch.randn(M, Kd, generator=g) * 0.05).half().cuda()
    gw = (1.0 + 0.1 * torch.randn(Kd, generator=g)).half().cuda()
    x = (torch.randn(64, Kd, generator=g) * 3).half().cuda()
    packed = packed_weight(kk, K, w)
    eps = 1e-5
    xf = x[:N].float()
    normed = (xf * (1.0 / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * gw.float()).half().float()
    ref = normed @ w.float().T
    d = kk.GemmDesc()
    d.weight, d.weight_layout, d.M, d.K = p(packed), kk.W_PACKED, M, Kd
    d.x, d.N, d.x_stride, d.x_rows = p(x), N, Kd, 64
    d.norm_input, d.norm_stride, d.norm_eps, d.norm_weight = p(x), Kd, eps, p(gw)
    if epi == "f32":
        out = torch.zeros(N, M, device="cuda")
        d.epilogue, d.out, d.out_stride = kk.EPI_STORE_F32, p(out), M
        assert K["gemm"](C.byref(d), None) == 0
        sync_ok(K)
        torch.testing.assert_close(out, ref, atol=3e-2, rtol=2e-2)
    elif epi == "silu":
        out = torch.zeros(N, M // 2, dtype=torch.half, device="cuda")
        d.epilogue, d.out, d.out_stride = kk.EPI_SILU_PAIRS, p(out), M // 2
        assert K["gemm"](C.byref(d), None) == 0
        sync_ok(K)
        gate, up = ref[:, 0::2].half().float(), ref[:, 1::2].half().float()
        torch.testing.assert_close(out.float(), (gate / (1 + torch.exp(-gate)) * up), atol=3e-2, rtol=2e-2)
    else:
        tokens = torch.zeros(N, dtype=torch.int32, device="cuda")
        ws = torch.zeros(K["argmax_workspace_bytes"](M, N), dtype=torch.uint8, device="cuda")
        logits = torch.zeros(N, M, device="cuda")
        d.epilogue, d.out, d.out_stride = kk.EPI_ARGMAX, p(logits), M
        d.tokens, d.argmax_workspace = p(tokens), p(ws)
        assert K["gemm"](C.byref(d), None) == 0
        sync_ok(K)
        torch.testing.assert_close(logits, ref, atol=3e-2, rtol=2e-2)
        assert tokens.cpu().tolist() == logits.argmax(-1).int().cpu().tolist()


@pytest.mark.parametrize("M,Kd", [(128, 64), (300, 1000), (32000, 256), (2560, 2048)])
def test_gemm_pack_weight_layout_is_exact(kk, K, M, Kd):
    """Tile (t, b) holds rows t*128.., columns b*64.. with 16-byte chunk c of row r
    at r*128 + ((c ^ (r % 8)) * 16); padding is zero."""
    g = torch.Generator().manual_seed(M + Kd)
    w = torch.randn(M, Kd, generator=g).half().cuda()
    packed = packed_weight(kk, K, w).view(torch.int16).cpu()
    tiles, kb = (M + 127) // 128, (Kd + 63) // 64
    assert packed.numel() == tiles * kb * 128 * 64
    wp = torch.zeros(tiles * 128, kb * 64, dtype=torch.int16)
    wp[:M, :Kd] = w.view(torch.int16).cpu()
    ref = wp.view(tiles, 128, kb, 8, 8).permute(0, 2, 1, 3, 4).contiguous()  # [t, b, r, c, 8]
    r = torch.arange(128)[:, None]
    c = torch.arange(8)[None, :]
    swz = torch.empty_like(ref)
    swz[:, :, r, c ^ (r % 8)] = ref[:, :, r, c]
    assert torch.equal(packed.view(tiles, kb, 128, 8, 8), swz)


@pytest.mark.parametrize("contexts,target", [
    ([17, 100, 513, 2000], 256), ([1, 8, 9, 64, 65], 64), ([4096, 1024, 3000], 512),
    ([33], 8)])
@pytest.mark.parametrize("hkv,hq", [(4, 32), (2, 8), (1, 16), (8, 64)])
@pytest.mark.parametrize("variant", [1, 2], ids=["direct", "tma"])
def test_paged_attention_matches_torch(kk, K, attn_variant, contexts, target, hkv, hq, variant,
                                       poison=False):
    attn_variant(variant)
    layers, D = 2, 64
    rng = random.Random(sum(contexts) + hq)
    micro_cap = sum((c % 64 + 7) // 8 for c in contexts) + 16
    extent_cap = sum(c // 64 for c in contexts) + 4
    pools, micro, extent = make_pools(kk, layers, hkv, D, micro_cap, extent_cap, seed=len(contexts))
    tables = build_tables(contexts, micro_cap, extent_cap, rng)
    if poison:
        # Bytes past a page's valid tokens must never reach the output.
        for tbl in tables:
            for slot, _, valid, kind in tbl:
                (micro if kind == 0 else extent)[slot, :, :, valid:] = float("nan")
    descs, lanes = descs_and_lanes(kk, tables)
    max_items = 4096
    items = (kk.AttnItem * max_items)()
    n_items = K["attention_plan"](descs, lanes, len(tables), target, items, max_items)
    B = len(contexts)
    q = (torch.randn(B, hq * D) / 8).half().cuda()
    out = torch.zeros(B, hq * D, dtype=torch.half, device="cuda")
    ws_bytes = K["attention_workspace_bytes"](B, n_items, hq, D)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    d_descs, d_lanes, d_items = to_device_bytes(descs), to_device_bytes(lanes), to_device_bytes(items)
    scale = 1.0 / 8.0
    for layer in range(layers):
        rc = K["paged_decode_attention"](C.byref(pools), layer, hq, p(d_descs), p(d_lanes), B,
                                         p(d_items), n_items, p(q), hq * D, p(out), hq * D,
                                         scale, p(ws), ws_bytes, None)
        assert rc == 0
        sync_ok(K)
        for b, tbl in enumerate(tables):
            k, v = gather_kv(micro, extent, tbl, layer)
            ref = attention_ref(q[b].view(hq, D), k, v, scale)
            torch.testing.assert_close(out[b].view(hq, D).float(), ref, atol=2e-3, rtol=2e-2)


@pytest.mark.parametrize("contexts,parts", [
    ([17, 100, 513, 2000], 3), ([1, 8, 9, 64, 65, 0, 300], 4), ([4096, 1024, 3000], 148),
    ([33], 1), ([2000] * 8, 5), ([0, 70, 0, 0, 129], 2)])
@pytest.mark.parametrize("hkv,hq", [(4, 32), (2, 8), (1, 16), (8, 64)])
def test_paged_attention_balanced_plan_matches_torch(kk, K, attn_variant, contexts, parts, hkv, hq):
    """Token-balanced items that span lanes (TMA kernel): every non-empty lane
    matches the FP32 reference, whether it is whole inside one item or split."""
    attn_variant(kk.ATTN_TMA)
    layers, D = 2, 64
    rng = random.Random(sum(contexts) + parts)
    micro_cap = sum((c % 64 + 7) // 8 for c in contexts) + 16
    extent_cap = sum(c // 64 for c in contexts) + 4
    pools, micro, extent = make_pools(kk, layers, hkv, D, micro_cap, extent_cap, seed=parts)
    tables = build_tables(contexts, micro_cap, extent_cap, rng)
    descs, lanes = descs_and_lanes(kk, tables)
    items = (kk.AttnItem * 4096)()
    B = len(contexts)
    n_items = K["attention_plan_balanced"](descs, lanes, B, parts, items, 4096)
    assert 0 < n_items <= parts
    q = (torch.randn(B, hq * D) / 8).half().cuda()
    out = torch.zeros(B, hq * D, dtype=torch.half, device="cuda")
    ws_bytes = K["attention_workspace_bytes"](B, n_items, hq, D)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    d_descs, d_lanes, d_items = to_device_bytes(descs), to_device_bytes(lanes), to_device_bytes(items)
    for layer in range(layers):
        for _ in range(2):  # completion counters must reset themselves
            rc = K["paged_decode_attention"](C.byref(pools), layer, hq, p(d_descs), p(d_lanes), B,
                                             p(d_items), n_items, p(q), hq * D, p(out), hq * D,
                                             0.125, p(ws), ws_bytes, None)
            assert rc == 0
            sync_ok(K)
            for b, tbl in enumerate(tables):
                if not tbl:
                    continue
                k, v = gather_kv(micro, extent, tbl, layer)
                ref = attention_ref(q[b].view(hq, D), k, v, 0.125)
                torch.testing.assert_close(out[b].view(hq, D).float(), ref, atol=2e-3, rtol=2e-2)


def test_direct_kernel_rejects_multi_lane_items(kk, K, attn_variant):
    attn_variant(kk.ATTN_DIRECT)
    pools, micro, extent = make_pools(kk, 1, 4, 64, 8, 2, seed=5)
    tables = [[(0, 0, 8, 0)], [(1, 0, 8, 0)]]
    descs, lanes = descs_and_lanes(kk, tables)
    items = (kk.AttnItem * 4)()
    n_items = K["attention_plan_balanced"](descs, lanes, 2, 1, items, 4)
    assert n_items == 1 and items[0].desc_end == 2
    q = (torch.randn(2, 32 * 64) / 8).half().cuda()
    out = torch.zeros(2, 32 * 64, dtype=torch.half, device="cuda")
    ws = torch.zeros(K["attention_workspace_bytes"](2, n_items, 32, 64), dtype=torch.uint8,
                     device="cuda")
    d_descs, d_lanes, d_items = to_device_bytes(descs), to_device_bytes(lanes), to_device_bytes(items)
    rc = K["paged_decode_attention"](C.byref(pools), 0, 32, p(d_descs), p(d_lanes), 2, p(d_items),
                                     n_items, p(q), 32 * 64, p(out), 32 * 64, 0.125, p(ws),
                                     ws.numel(), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert K["device_status"](None) == 3  # kErrBadArgument, then cleared
    assert K["device_status"](None) == 0
    assert torch.count_nonzero(out) == 0


@pytest.mark.parametrize("variant", [1, 2], ids=["direct", "tma"])
def test_paged_attention_ignores_page_tails(kk, K, attn_variant, variant):
    test_paged_attention_matches_torch(kk, K, attn_variant, [5, 70, 130, 1001], 64, 4, 32, variant,
                                       poison=True)


@pytest.mark.parametrize("variant", [1, 2], ids=["direct", "tma"])
def test_paged_attention_reports_bad_descriptor(kk, K, attn_variant, variant):
    """A descriptor outside its pool is never dereferenced; the launch reports it."""
    attn_variant(variant)
    pools, micro, extent = make_pools(kk, 1, 4, 64, 8, 2, seed=3)
    tables = [[(1, 0, 64, 1), (7, 64, 5, 0)], [(9, 0, 8, 0), (0, 8, 3, 0)]]  # slot 9 > micro_cap
    descs, lanes = descs_and_lanes(kk, tables)
    items = (kk.AttnItem * 8)()
    n_items = K["attention_plan"](descs, lanes, 2, 256, items, 8)
    q = (torch.randn(2, 32 * 64) / 8).half().cuda()
    out = torch.zeros(2, 32 * 64, dtype=torch.half, device="cuda")
    ws = torch.zeros(K["attention_workspace_bytes"](2, n_items, 32, 64), dtype=torch.uint8,
                     device="cuda")
    d_descs, d_lanes, d_items = to_device_bytes(descs), to_device_bytes(lanes), to_device_bytes(items)
    rc = K["paged_decode_attention"](C.byref(pools), 0, 32, p(d_descs), p(d_lanes), 2, p(d_items),
                                     n_items, p(q), 32 * 64, p(out), 32 * 64, 0.125, p(ws),
                                     ws.numel(), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert K["device_status"](None) == 2  # kErrBadDescriptor, then cleared
    assert K["device_status"](None) == 0
    k, v = gather_kv(micro, extent, tables[0], 0)
    ref = attention_ref(q[0].view(32, 64), k, v, 0.125)
    torch.testing.assert_close(out[0].view(32, 64).float(), ref, atol=2e-3, rtol=2e-2)
    # lane 1's output is unspecified (its table is corrupt); the other lanes are unaffected


def test_paged_attention_wait_timeout_is_reported_not_hung(kk, K):
    """A bounded wait that runs out: the test hook makes CTA 0 of the TMA
    kernel drop its first stage (no copy, no arrival) and lowers the wait
    limit to 1 ms. The launch ends on its own, reports kErrWaitTimeout (1),
    and the next launch with the hook cleared is correct again."""
    pools, micro, extent = make_pools(kk, 1, 4, 64, 64, 8, seed=21)
    tables = build_tables([300, 17, 140], 64, 8, random.Random(4))
    descs, lanes = descs_and_lanes(kk, tables)
    items = (kk.AttnItem * 64)()
    n_items = K["attention_plan_balanced"](descs, lanes, 3, 8, items, 64)
    q = (torch.randn(3, 32 * 64) / 8).half().cuda()
    out = torch.zeros(3, 32 * 64, dtype=torch.half, device="cuda")
    ws = torch.zeros(K["attention_workspace_bytes"](3, n_items, 32, 64), dtype=torch.uint8,
                     device="cuda")
    d_descs, d_lanes, d_items = to_device_bytes(descs), to_device_bytes(lanes), to_device_bytes(items)

    def run():
        rc = K["paged_decode_attention"](C.byref(pools), 0, 32, p(d_descs), p(d_lanes), 3, p(d_items),
                                         n_items, p(q), 32 * 64, p(out), 32 * 64, 0.125, p(ws),
                                         ws.numel(), None)
        assert rc == 0
        torch.cuda.synchronize()

    assert K["debug_attention_fault"](0, 1_000_000) == 0
    try:
        run()
    finally:
        assert K["debug_attention_fault"](0xFFFFFFFF, 0) == 0
    assert K["device_status"](None) == 1  # kErrWaitTimeout, then cleared
    ws.zero_()                            # completion counters left mid-count by the aborted CTA
    run()
    assert K["device_status"](None) == 0
    for b, tbl in enumerate(tables):
        k, v = gather_kv(micro, extent, tbl, 0)
        ref = attention_ref(q[b].view(32, 64), k, v, 0.125)
        torch.testing.assert_close(out[b].view(32, 64).float(), ref, atol=2e-3, rtol=2e-2)


def test_attention_variant_switch_rejects_unknown(kk, K, attn_variant):
    assert K["attention_set_variant"](7) == kk.KK_EINVAL
    assert K["attention_set_variant"](-1) == kk.KK_EINVAL


def test_kv_write_and_copy_are_exact(kk, K):
    layers, hkv, D = 4, 4, 64
    pools, micro, extent = make_pools(kk, layers, hkv, D, 12, 3, seed=11)
    B = 3
    key = torch.randn(B, layers, hkv * D).half().cuda()
    val = torch.randn(B, layers, hkv * D).half().cuda()
    slots = (kk.KvSlot * B)(kk.KvSlot(2, 5, 0, 1), kk.KvSlot(1, 40, 1, 1), kk.KvSlot(7, 0, 0, 0))
    d_slots = to_device_bytes(slots)
    m0, e0 = micro.clone(), extent.clone()
    rc = K["kv_write"](C.byref(pools), 1, 2, p(d_slots), B, p(key[:, 1]), p(val[:, 1]),
                       layers * hkv * D, hkv * D, None)
    assert rc == 0
    sync_ok(K)
    for li, layer in enumerate([1, 2]):
        assert torch.equal(micro[2, layer, 0, 5].flatten(), key[0, layer])
        assert torch.equal(micro[2, layer, 1, 5].flatten(), val[0, layer])
        assert torch.equal(extent[1, layer, 0, 40].flatten(), key[1, layer])
        assert torch.equal(extent[1, layer, 1, 40].flatten(), val[1, layer])
    assert torch.equal(micro[7], m0[7])  # inactive lane untouched
    assert torch.equal(micro[2, 0], m0[2, 0]) and torch.equal(micro[2, 3], m0[2, 3])
    copies = (kk.KvCopy * 2)(kk.KvCopy(2, 9, 6, 0, 0), kk.KvCopy(1, 2, 8, 1, 1))
    d_copies = to_device_bytes(copies)
    m1, e1 = micro.clone(), extent.clone()
    assert K["kv_copy_tokens"](C.byref(pools), 0, layers, p(d_copies), 2, None) == 0
    sync_ok(K)
    assert torch.equal(micro[9, :, :, :6], m1[2, :, :, :6])
    assert torch.equal(micro[9, :, :, 6:], m1[9, :, :, 6:])
    assert torch.equal(extent[2, :, :, :8], e1[1, :, :, :8])
    assert torch.equal(extent[2, :, :, 8:], e1[2, :, :, 8:])


def test_kv_gather_and_scatter_are_exact(kk, K):
    """K6: pages -> contiguous [layer][K|V][token][head][dim] and back."""
    layers, hkv, D = 3, 4, 64
    contexts = [17, 100, 513, 2000]
    micro_cap = sum((c % 64 + 7) // 8 for c in contexts) + 8
    extent_cap = sum(c // 64 for c in contexts) + 2
    pools, micro, extent = make_pools(kk, layers, hkv, D, micro_cap, extent_cap, seed=21)
    tables = build_tables(contexts, micro_cap, extent_cap, random.Random(5))
    for tbl, T in zip(tables, contexts):
        descs, _ = descs_and_lanes(kk, [tbl])
        d_descs = to_device_bytes(descs)
        out = torch.full((layers, 2, T, hkv, D), float("nan"), dtype=torch.half, device="cuda")
        assert K["kv_gather"](C.byref(pools), p(d_descs), len(tbl), T, p(out), None) == 0
        sync_ok(K)
        for layer in range(layers):
            k, v = gather_kv(micro, extent, tbl, layer)
            assert torch.equal(out[layer, 0].float(), k) and torch.equal(out[layer, 1].float(), v)
        # scatter a window of new values back and check exactly those tokens changed
        first, count = T // 3, min(70, T - T // 3)
        new = torch.randn(layers, 2, count, hkv, D, generator=torch.Generator().manual_seed(T)).half().cuda()
        m0, e0 = micro.clone(), extent.clone()
        assert K["kv_scatter"](C.byref(pools), p(d_descs), len(tbl), first, count, p(new), None) == 0
        sync_ok(K)
        out2 = torch.empty_like(out)
        assert K["kv_gather"](C.byref(pools), p(d_descs), len(tbl), T, p(out2), None) == 0
        sync_ok(K)
        expect = out.clone()
        expect[:, :, first:first + count] = new
        assert torch.equal(out2, expect)
        changed = (micro != m0).sum() + (extent != e0).sum()
        assert int(changed) <= new.numel()
    bad = (kk.PageDesc * 1)(kk.PageDesc(micro_cap + 3, 0, 8, 0, 0, 0))
    out = torch.zeros(layers, 2, 8, hkv, D, dtype=torch.half, device="cuda")
    d_bad = to_device_bytes(bad)
    assert K["kv_gather"](C.byref(pools), p(d_bad), 1, 8, p(out), None) == 0
    torch.cuda.synchronize()
    assert K["device_status"](None) == 2
    assert int(out.count_nonzero()) == 0


def test_kv_promote_is_exact(kk, K):
    """8 micro pages -> 1 extent, every layer, K and V: extent token 8k+t is
    micro page k's token t; other extents and the micro pages are untouched."""
    layers, hkv, D = 3, 4, 64
    pools, micro, extent = make_pools(kk, layers, hkv, D, 16, 3, seed=13)
    m0, e0 = micro.clone(), extent.clone()
    slots = (C.c_uint32 * 8)(*[11, 3, 0, 7, 15, 2, 9, 4])
    assert K["kv_promote"](C.byref(pools), slots, 1, None) == 0
    sync_ok(K)
    for k, sl in enumerate(slots):
        assert torch.equal(extent[1, :, :, 8 * k:8 * k + 8], m0[sl])
    assert torch.equal(extent[0], e0[0]) and torch.equal(extent[2], e0[2])
    assert torch.equal(micro, m0)
    bad = (C.c_uint32 * 8)(*[11, 3, 0, 7, 15, 2, 9, 16])  # slot 16 is outside the pool
    assert K["kv_promote"](C.byref(pools), bad, 1, None) == kk.KK_EINVAL
    assert K["kv_promote"](C.byref(pools), slots, 3, None) == kk.KK_EINVAL


def test_rmsnorm_embedding_rope_silu_residual(kk, K):
    g = torch.Generator().manual_seed(21)
    rows, cols, V = 6, 2048, 100
    embed = torch.randn(V, cols, generator=g).half().cuda()
    weight = (1 + 0.1 * torch.randn(cols, generator=g)).half().cuda()
    tokens = torch.tensor([3, 99, 0, 3, 50, 7], dtype=torch.int32).cuda()
    hidden = torch.zeros(rows, cols, dtype=torch.half, device="cuda")
    y = torch.zeros_like(hidden)
    assert K["embed_rmsnorm"](p(embed), p(tokens), p(weight), p(hidden), p(y), rows, cols, 1e-5, None) == 0
    y2 = torch.zeros_like(hidden)
    assert K["rmsnorm"](p(hidden), p(weight), p(y2), rows, cols, 1e-5, None) == 0
    sync_ok(K)
    x = embed[tokens.long()].float()
    ref = (x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-5) * weight.float()).half()
    assert torch.equal(hidden, embed[tokens.long()])
    torch.testing.assert_close(y.float(), ref.float(), atol=2e-3, rtol=2e-3)
    assert torch.equal(y, y2)
    hq, hkv, D = 4, 2, 64
    q = torch.randn(rows, hq * D, generator=g).half().cuda()
    k = torch.randn(rows, hkv * D, generator=g).half().cuda()
    pos = torch.tensor([0, 1, 17, 400, 2047, 4000], dtype=torch.int32).cuda()
    q_ref = rope_ref(q.view(rows, hq, D), pos, 10000.0).view(rows, -1)
    k_ref = rope_ref(k.view(rows, hkv, D), pos, 10000.0).view(rows, -1)
    assert K["rope"](p(q), hq * D, p(k), hkv * D, p(pos), rows, hq, hkv, D, 10000.0, None) == 0
    gate = torch.randn(rows, 512, generator=g).half().cuda()
    up = torch.randn(rows, 512, generator=g).half().cuda()
    act = torch.zeros_like(gate)
    assert K["silu_mul"](p(gate), p(up), p(act), rows, 512, None) == 0
    h = torch.randn(rows, 512, generator=g).half().cuda()
    h0 = h.clone()
    assert K["residual_add"](p(h), p(up), rows * 512, None) == 0
    sync_ok(K)
    torch.testing.assert_close(q.float(), q_ref.float(), atol=4e-3, rtol=4e-3)
    torch.testing.assert_close(k.float(), k_ref.float(), atol=4e-3, rtol=4e-3)
    gf = gate.float()
    torch.testing.assert_close(act.float(), (gf / (1 + torch.exp(-gf)) * up.float()).half().float(),
                               atol=4e-3, rtol=4e-3)
    torch.testing.assert_close(h.float(), (h0 + up).float(), atol=4e-3, rtol=1e-3)


def test_invalid_arguments_are_rejected_without_launch(kk, K):
    d = kk.GemmDesc()
    assert K["gemm"](C.byref(d), None) == kk.KK_EINVAL
    pools = kk.KvPools(0, 0, 0, 0, 1, 4, 64, 0)
    assert K["paged_decode_attention"](C.byref(pools), 0, 32, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0.125,
                                       0, 0, None) == kk.KK_EINVAL
