"""Helpers shared by the GPU tests: torch tensors as kernel arguments, random
paged KV layouts, and plain-PyTorch FP32 references for the numerics tests."""
from __future__ import annotations

import ctypes as C
import math
import random

import numpy as np
import torch


def p(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def make_pools(kk, layers, kv_heads, head_dim, micro_cap, extent_cap, device="cuda", seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    micro = (torch.randn(micro_cap, layers, 2, 8, kv_heads, head_dim, generator=g) / 8).half()
    extent = (torch.randn(max(extent_cap, 1), layers, 2, 64, kv_heads, head_dim, generator=g) / 8).half()
    micro, extent = micro.to(device), extent.to(device)
    pools = kk.KvPools(p(micro), p(extent), micro_cap, extent_cap, layers, kv_heads, head_dim, 0)
    return pools, micro, extent


def build_tables(contexts, micro_cap, extent_cap, rng: random.Random):
    """Per lane: ctx tokens as floor(ctx/64) extent pages then micro pages
    (last one partial), at random distinct slots. Returns list of entry lists
    (slot, begin, valid, kind)."""
    micro_slots = list(range(micro_cap))
    extent_slots = list(range(extent_cap))
    rng.shuffle(micro_slots)
    rng.shuffle(extent_slots)
    tables = []
    for ctx in contexts:
        entries = []
        t = 0
        for _ in range(ctx // 64):
            entries.append((extent_slots.pop(), t, 64, 1))
            t += 64
        while t < ctx:
            n = min(8, ctx - t)
            entries.append((micro_slots.pop(), t, n, 0))
            t += n
        tables.append(entries)
    return tables


def descs_and_lanes(kk, tables):
    flat = [e for tbl in tables for e in tbl]
    descs = (kk.PageDesc * max(len(flat), 1))()
    for i, (slot, begin, valid, kind) in enumerate(flat):
        descs[i] = kk.PageDesc(slot, begin, valid, kind, 0, 0)
    lanes = (kk.AttnLane * len(tables))()
    off = 0
    for b, tbl in enumerate(tables):
        lanes[b].desc_offset = off
        lanes[b].desc_count = len(tbl)
        lanes[b].token_count = sum(e[2] for e in tbl)
        lanes[b].query_row = b
        off += len(tbl)
    return descs, lanes


def to_device_bytes(struct_array) -> torch.Tensor:
    raw = bytes(struct_array)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda()


def gather_kv(micro, extent, table, layer):
    """[T, kv_heads, D] K and V of one lane, FP32."""
    ks, vs = [], []
    for slot, begin, valid, kind in table:
        pool = micro if kind == 0 else extent
        ks.append(pool[slot, layer, 0, :valid].float())
        vs.append(pool[slot, layer, 1, :valid].float())
    return torch.cat(ks), torch.cat(vs)


def attention_ref(q, k, v, scale):
    """q [Hq, D], k/v [T, Hkv, D] -> [Hq, D] (FP32, GQA)."""
    hq, hkv = q.shape[0], k.shape[1]
    g = hq // hkv
    kk_ = k.repeat_interleave(g, dim=1)  # [T, Hq, D]
    vv = v.repeat_interleave(g, dim=1)
    s = torch.einsum("hd,thd->ht", q.float(), kk_) * scale
    w = torch.softmax(s, dim=-1)
    return torch.einsum("ht,thd->hd", w, vv)


def rope_ref(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """x [N, H, D] fp16 -> rotate-half RoPE in fp32 with fp16 inputs, fp16 out."""
    n, h, d = x.shape
    half = d // 2
    dim = torch.arange(half, dtype=torch.float32, device=x.device)
    inv = torch.pow(torch.tensor(theta, device=x.device), -2.0 * dim / d)
    ang = positions.float()[:, None] * inv[None, :]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    a, b = x[..., :half].float(), x[..., half:].float()
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1).half()
