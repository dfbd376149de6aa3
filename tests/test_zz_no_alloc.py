"""kk_paged_decode_attention_noalloc: the attention entry point that takes no
workspace (its scratch is a fixed device array inside the library) must give
the same results as kk_paged_decode_attention with a caller workspace, call
after call, and must reject work lists that need more scratch than it has.

Collected last (file name), so it also runs after every other GPU test has
used the library in the same process."""
import ctypes as C
import random

import pytest
import torch

from gpu_util import attention_ref, build_tables, descs_and_lanes, gather_kv, make_pools, p, to_device_bytes

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _case(kk, K, contexts, hkv, hq, parts, seed):
    layers, D = 2, 64
    rng = random.Random(seed)
    micro_cap = sum((c % 64 + 7) // 8 for c in contexts) + 16
    extent_cap = sum(c // 64 for c in contexts) + 4
    pools, micro, extent = make_pools(kk, layers, hkv, D, micro_cap, extent_cap, seed=seed)
    tables = build_tables(contexts, micro_cap, extent_cap, rng)
    descs, lanes = descs_and_lanes(kk, tables)
    items = (kk.AttnItem * 4096)()
    B = len(contexts)
    n_items = K["attention_plan_balanced"](descs, lanes, B, parts, items, 4096)
    q = (torch.randn(B, hq * D, generator=torch.Generator().manual_seed(seed)) / 8).half().cuda()
    dev = [to_device_bytes(descs), to_device_bytes(lanes), to_device_bytes(items)]
    return pools, micro, extent, tables, dev, n_items, q


@pytest.mark.parametrize("contexts,hkv,hq,parts", [
    ([17, 100, 513, 2000], 4, 32, 7),          # lanes split across items: counters and partials
    ([4096, 1024, 3000, 8, 65], 4, 32, 148),
    ([300, 700], 2, 8, 3),
    ([129, 64, 1], 1, 16, 2),
])
def test_noalloc_matches_workspace_entry_point_twice(kk, K_noalloc, contexts, hkv, hq, parts):
    K = K_noalloc
    pools, micro, extent, tables, (d_descs, d_lanes, d_items), n_items, q = _case(
        kk, K, contexts, hkv, hq, parts, seed=sum(contexts) + parts)
    B, D = len(contexts), 64
    ws_bytes = K["attention_workspace_bytes"](B, n_items, hq, D)
    assert ws_bytes <= kk.ATTN_SCRATCH_BYTES
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    ref_out = torch.zeros(B, hq * D, dtype=torch.half, device="cuda")
    out = torch.zeros(B, hq * D, dtype=torch.half, device="cuda")
    for layer in range(2):
        rc = K["paged_decode_attention"](C.byref(pools), layer, hq, p(d_descs), p(d_lanes), B,
                                         p(d_items), n_items, p(q), hq * D, p(ref_out), hq * D,
                                         0.125, p(ws), ws_bytes, None)
        assert rc == 0
        for call in range(2):  # two calls in a row through the static scratch
            out.zero_()
            rc = K["paged_decode_attention_noalloc"](C.byref(pools), layer, hq, p(d_descs),
                                                     p(d_lanes), B, p(d_items), n_items, p(q),
                                                     hq * D, p(out), hq * D, 0.125, None)
            assert rc == 0
            torch.cuda.synchronize()
            assert K["device_status"](None) == 0
            torch.testing.assert_close(out.float(), ref_out.float(), atol=1e-3, rtol=1e-3)
        for b, tbl in enumerate(tables):
            k, v = gather_kv(micro, extent, tbl, layer)
            ref = attention_ref(q[b].view(hq, D), k, v, 0.125)
            torch.testing.assert_close(out[b].view(hq, D).float(), ref, atol=2e-3, rtol=2e-2)


def test_noalloc_rejects_work_lists_beyond_its_scratch(kk, K_noalloc):
    K = K_noalloc
    pools, micro, extent, tables, (d_descs, d_lanes, d_items), n_items, q = _case(
        kk, K, [64] * 4, 4, 32, 4, seed=5)
    hq, D = 64, 64
    big_items = 1200  # 2 partial slots x 1200 items x 64 heads x 256 B > 4 MiB
    assert K["attention_workspace_bytes"](4, big_items, hq, D) > kk.ATTN_SCRATCH_BYTES
    out = torch.full((4, hq * D), 7.0, dtype=torch.half, device="cuda")
    rc = K["paged_decode_attention_noalloc"](C.byref(pools), 0, hq, p(d_descs), p(d_lanes), 4,
                                             p(d_items), big_items, p(q), hq * D, p(out), hq * D,
                                             0.125, None)
    assert rc == kk.KK_ENOSCRATCH
    torch.cuda.synchronize()
    assert K["device_status"](None) == 0
    assert bool((out == 7.0).all()), "a rejected call launches nothing"


@pytest.fixture(scope="module")
def K_noalloc(kk):
    return kk.kernels()
