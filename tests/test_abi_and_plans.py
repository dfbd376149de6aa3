"""CPU checks of the C ABI: every function declared in include/*.h is exported
by lib/libkk_b200.so, and the host-side attention planners
(kk_attention_plan, kk_attention_plan_balanced) produce work lists that
cover every page descriptor exactly once, in order, with consistent per-lane
item ranges. No kernel is launched."""
import ctypes as C
import random
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        for m in re.finditer(r"^(?:KK_KAPI|KK_API)\s+[\w\s\*]+?\b(\w+)\s*\(", text, re.M):
            names.append((header.name, m.group(1)))
    return names


def test_every_declared_function_is_exported(kk_lib):
    decl = declared_functions()
    assert len(decl) > 60
    missing = [f"{h}:{n}" for h, n in decl if not hasattr(kk_lib, n)]
    assert not missing, missing


def test_bindings_cover_the_kernel_header(kk):
    names = {n for h, n in declared_functions() if h == "kk_kernels.h"}
    bound = {"kk_" + k for k in kk.KERNEL_SIGNATURES}
    assert names <= bound, sorted(names - bound)


def make_tables(kk, contexts, seed):
    rng = random.Random(seed)
    descs, lanes = [], (kk.AttnLane * len(contexts))()
    slot = 0
    for b, ctx in enumerate(contexts):
        lanes[b].desc_offset, lanes[b].query_row, lanes[b].token_count = len(descs), b, ctx
        t = 0
        while t + 64 <= ctx and rng.random() < 0.9:
            descs.append(kk.PageDesc(slot, t, 64, 1, 0, 0))
            slot += 1
            t += 64
        while t < ctx:
            n = min(8, ctx - t)
            descs.append(kk.PageDesc(slot, t, n, 0, 0, 0))
            slot += 1
            t += n
        lanes[b].desc_count = len(descs) - lanes[b].desc_offset
    arr = (kk.PageDesc * max(len(descs), 1))(*descs)
    return arr, lanes, len(descs)


def item_span(it, e, descs):
    """Tokens [first, last) of descriptor e that item `it` covers."""
    valid = descs[e].valid_tokens
    first = (it.reserved >> 8) & 0xFF if e == it.desc_begin else 0
    limit = (it.reserved >> 16) & 0xFF
    last = limit if e == it.desc_end - 1 and limit else valid
    return first, last


def check_cover(kk, descs, lanes, items, n_items, multi_lane):
    """Items tile the descriptor array in order, token for token: an item
    starts where the previous one ended, on the same descriptor only when
    that descriptor (a full extent) is cut at its half. Lane ranges match."""
    nl = len(lanes)
    pos = (0, 0)   # (descriptor, token) where the next item must start
    touched = {b: [] for b in range(nl)}
    for i in range(n_items):
        it = items[i]
        flags = it.reserved & 0xFF
        assert flags == (kk.ATTN_ITEM_MULTI_LANE if multi_lane else 0)
        assert it.desc_end > it.desc_begin
        first, _ = item_span(it, it.desc_begin, descs)
        if first:
            assert pos == (it.desc_begin, first) and descs[it.desc_begin].kind == 1, (i, pos)
        else:
            assert pos == (it.desc_begin, 0), (i, pos)
        b = it.lane
        for e in range(it.desc_begin, it.desc_end):
            while lanes[b].desc_offset + lanes[b].desc_count <= e:
                b += 1
                assert multi_lane, "per-lane items never cross a lane"
            assert lanes[b].desc_offset <= e
            f, l = item_span(it, e, descs)
            assert f < l or descs[e].valid_tokens == 0
            if l != descs[e].valid_tokens:
                assert e == it.desc_end - 1 and descs[e].kind == 1 and descs[e].valid_tokens == 64 and l == 32
            if not touched[b] or touched[b][-1] != i:
                touched[b].append(i)
        last_e = it.desc_end - 1
        _, l = item_span(it, last_e, descs)
        pos = (last_e, l) if l != descs[last_e].valid_tokens else (it.desc_end, 0)
    assert pos == (sum(lanes[b].desc_count for b in range(nl)), 0)
    for b in range(nl):
        got = list(range(lanes[b].item_offset, lanes[b].item_offset + lanes[b].item_count))
        assert got == touched[b], (b, got, touched[b])
        # the lane's first item begins in an earlier lane exactly when flagged
        shared = bool(got) and items[got[0]].lane != b
        assert lanes[b].first_item_shared == int(shared), b


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("parts", [1, 3, 7, 148, 5000])
def test_balanced_plan_covers_and_balances(kk, seed, parts):
    K = kk.kernels()
    rng = random.Random(seed)
    contexts = [rng.choice([0, 1, 7, 8, 9, 63, 64, 65, rng.randint(1, 4096)]) for _ in range(rng.randint(1, 40))]
    descs, lanes, nd = make_tables(kk, contexts, seed)
    items = (kk.AttnItem * 8192)()
    n = K["attention_plan_balanced"](descs, lanes, len(contexts), parts, items, 8192)
    total = sum(contexts)
    if total == 0:
        assert n == 0
        return
    check_cover(kk, descs, lanes, items, n, multi_lane=True)
    # Cost model: every token plus SEG per lane segment start. Each cut is the
    # page boundary nearest to k * total_cost / parts, off by at most half a
    # page plus one segment charge.
    SEG = 144
    starts = {lanes[b].desc_offset for b in range(len(contexts)) if lanes[b].desc_count}
    total_cost = total + SEG * len(starts)
    per = total_cost / parts
    def span_cost(i, e):
        f, l = item_span(items[i], e, descs)
        seg = SEG if e in starts and f == 0 else 0
        return (l - f) + seg
    costs = [sum(span_cost(i, e) for e in range(items[i].desc_begin, items[i].desc_end)) for i in range(n)]
    assert n <= parts
    # A cut lands within half a unit (a micro page, or half of a full extent)
    # of its target, plus a segment charge.
    assert max(costs) <= per + 2 * (16 + SEG) + 8
    if per >= 128:
        assert n == parts
        assert min(costs) >= per - 2 * (16 + SEG) - 8


def test_balanced_plan_counts_items_beyond_capacity(kk):
    K = kk.kernels()
    descs, lanes, nd = make_tables(kk, [640, 640], 1)
    full = (kk.AttnItem * 64)()
    n_full = K["attention_plan_balanced"](descs, lanes, 2, 20, full, 64)
    items = (kk.AttnItem * 2)()
    n = K["attention_plan_balanced"](descs, lanes, 2, 20, items, 2)
    assert n == n_full and n > 2   # counted, not written
    for i in range(2):
        assert (items[i].lane, items[i].desc_begin, items[i].desc_end) == \
            (full[i].lane, full[i].desc_begin, full[i].desc_end)


def test_balanced_plan_does_not_join_non_contiguous_lanes(kk):
    K = kk.kernels()
    descs = (kk.PageDesc * 4)(*[kk.PageDesc(i, 0, 8, 0, 0, 0) for i in range(4)])
    lanes = (kk.AttnLane * 2)()
    lanes[0].desc_offset, lanes[0].desc_count = 2, 2   # lane 0 uses descriptors 2, 3
    lanes[1].desc_offset, lanes[1].desc_count = 0, 2   # lane 1 uses descriptors 0, 1
    items = (kk.AttnItem * 8)()
    n = K["attention_plan_balanced"](descs, lanes, 2, 1, items, 8)
    assert n == 2
    assert (items[0].lane, items[0].desc_begin, items[0].desc_end) == (0, 2, 4)
    assert (items[1].lane, items[1].desc_begin, items[1].desc_end) == (1, 0, 2)


@pytest.mark.parametrize("target", [8, 64, 256, 1000])
def test_per_lane_plan_covers(kk, target):
    K = kk.kernels()
    contexts = [17, 100, 513, 2000, 0, 64, 4096]
    descs, lanes, nd = make_tables(kk, contexts, 7)
    items = (kk.AttnItem * 8192)()
    n = K["attention_plan"](descs, lanes, len(contexts), target, items, 8192)
    check_cover(kk, descs, lanes, items, n, multi_lane=False)
