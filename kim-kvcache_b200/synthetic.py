"""Seeded random-init TinyLlama-shaped weight archives in the reference's
manifest format (reference src/model/weight_manifest.cpp:361-600;
converter scripts/convert_tinyllama_weights.py writes the same format).

There is no network and no checkpoint, so benchmarks and tests use
random-init weights of the exact architecture: matrices ~ N(0, std) in FP16
(std 0.02 by default) and RMSNorm weights = 1.0 (a N(0, 0.02) norm scale
would shrink every activation and leave the top-2 logit gap below the FP16
comparison tolerance).
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import numpy as np

TINYLLAMA = dict(hidden=2048, intermediate=5632, layers=22, q_heads=32, kv_heads=4, head_dim=64,
                 vocab=32000, max_positions=2048, eps=1e-5, theta=10000.0, bos=1, eos=2)


def tensor_list(cfg: dict) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) in the oracle's order: embed, lm_head, final norm, then per
    layer input norm, post norm, q, k, v, o, gate, up, down."""
    H, I, V = cfg["hidden"], cfg["intermediate"], cfg["vocab"]
    KV = cfg["kv_heads"] * cfg["head_dim"]
    out = [("model.embed_tokens.weight", (V, H)), ("lm_head.weight", (V, H)),
           ("model.norm.weight", (H,))]
    for l in range(cfg["layers"]):
        p = f"model.layers.{l}."
        out += [(p + "input_layernorm.weight", (H,)), (p + "post_attention_layernorm.weight", (H,)),
                (p + "self_attn.q_proj.weight", (H, H)), (p + "self_attn.k_proj.weight", (KV, H)),
                (p + "self_attn.v_proj.weight", (KV, H)), (p + "self_attn.o_proj.weight", (H, H)),
                (p + "mlp.gate_proj.weight", (cfg["intermediate"], H)),
                (p + "mlp.up_proj.weight", (cfg["intermediate"], H)),
                (p + "mlp.down_proj.weight", (H, I))]
    return out


def make_tensor(name: str, shape, rng: np.random.Generator, std: float) -> np.ndarray:
    if name.endswith("norm.weight"):
        return np.full(shape, 1.0, dtype=np.float16).view(np.uint16)
    vals = rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(std)
    return vals.astype(np.float16).view(np.uint16).reshape(shape)


def write_archive(directory: str | os.PathLike, cfg: dict, seed: int, std: float = 0.02,
                  keep_weights: bool = False):
    """Writes model.manifest + model.weights under `directory` (reused when an
    identical archive is already there). Returns (manifest, data, weights)
    where weights is the oracle-ordered list of uint16 arrays if requested."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    manifest, data = d / "model.manifest", d / "model.weights"
    stamp = d / "stamp.json"
    key = json.dumps({"cfg": cfg, "seed": seed, "std": std}, sort_keys=True)
    tensors = tensor_list(cfg)
    rng = np.random.default_rng(seed)
    if stamp.exists() and stamp.read_text() == key and manifest.exists() and data.exists():
        if not keep_weights:
            return str(manifest), str(data), None
        return str(manifest), str(data), [make_tensor(n, s, rng, std) for n, s in tensors]
    records, kept = [], []
    offset = 0
    with open(data, "wb") as f:
        for name, shape in tensors:
            t = make_tensor(name, shape, rng, std)
            raw = t.tobytes()
            f.write(raw)
            records.append((name, offset, len(raw), shape, hashlib.sha256(raw).hexdigest()))
            offset += len(raw)
            if keep_weights:
                kept.append(t)
    lines = ["version=1", "checkpoint=synthetic/tinyllama-shape",
             f"checkpoint_revision=seed{seed}", f"tokenizer_revision=seed{seed}",
             "config_sha256=" + hashlib.sha256(key.encode()).hexdigest(), "dtype=fp16",
             f"data_file={data.name}", f"data_bytes={offset}",
             f"hidden_size={cfg['hidden']}", f"intermediate_size={cfg['intermediate']}",
             f"layer_count={cfg['layers']}", f"attention_head_count={cfg['q_heads']}",
             f"kv_head_count={cfg['kv_heads']}", f"head_dimension={cfg['head_dim']}",
             f"vocabulary_size={cfg['vocab']}", f"max_position_embeddings={cfg['max_positions']}",
             f"bos_token_id={cfg.get('bos', 1)}", f"eos_token_id={cfg.get('eos', 2)}",
             f"rms_norm_epsilon={cfg['eps']}", f"rope_theta={cfg['theta']}",
             "tied_word_embeddings=0", f"tensor_count={len(records)}"]
    for name, off, size, shape, digest in records:
        lines.append(f"tensor={name}|{off}|{size}|{','.join(map(str, shape))}|{digest}")
    manifest.write_text("\n".join(lines) + "\n")
    stamp.write_text(key)
    return str(manifest), str(data), (kept if keep_weights else None)


# ---- decode workloads of the benchmark configs --------------------------------

# The reference benchmark seed (include/kim-kv/benchmark/benchmark.h:123).
BENCH_SEED = 0x4B564341434845


def decode_workload(config: str) -> dict:
    """Seeded decode workload of a BASELINE config: name, batch and per-lane
    context lengths. Every replica (rank) gets the same contexts, so per-GPU
    work is identical and the max-over-ranks time measures the GPUs, not the
    draw."""
    import random
    rng = random.Random(BENCH_SEED)
    if config == "c2":
        return dict(name="c2: TinyLlama-shape greedy decode, batch 1, prompt 6 (+32 new)",
                    batch=1, contexts=[6])
    if config == "c5":
        return dict(name="c5: TinyLlama-shape decode replicas, 64 requests/GPU, ctx~U[64,1024]",
                    batch=64, contexts=[rng.randint(64, 1024) for _ in range(64)])
    return dict(name="c4: TinyLlama-shape decode, 32 lanes/GPU, ctx~U[1024,4096] extent+micro pages",
                batch=32, contexts=[rng.randint(1024, 4096) for _ in range(32)])


def pool_capacities(contexts: list[int], extra_tokens: int) -> tuple[int, int]:
    """(micro, extent) page capacities for lanes of these contexts that decode
    `extra_tokens` more tokens each with auto-promotion on: room for every
    64-token run that promotion folds, plus micro pages for the tails."""
    B = len(contexts)
    extent = sum((c + extra_tokens) // 64 for c in contexts) + B
    micro = B * 16 + (sum(contexts) + B * extra_tokens) // 8 + 64
    return micro, extent


def build_decode_prefixes(R: dict, K: dict, backend, pools, contexts: list[int], cfg: dict,
                          fill_seed: int, stream) -> None:
    """Lane i (request i + 1) gets contexts[i] tokens of committed KV: the
    runtime's own append -> seal -> promote path lays out the pages (64-token
    extents for the body, 8-token micro pages for the tail), then every page
    of both pools is filled with seeded FP16 values in [-0.35, 0.35) (the
    prefix K/V a prefill would have written)."""
    import ctypes as C
    for i, ctx in enumerate(contexts):
        rid = i + 1
        assert R["backend_create_request"](backend, rid) == 0
        assert R["backend_append"](backend, rid, ctx) == 0
        R["backend_seal"](backend, rid)
        for begin in range(0, (ctx // 64) * 64, 64):
            assert R["backend_promote"](backend, rid, begin, stream) == 0
    row = cfg["kv_heads"] * cfg["head_dim"]
    L = cfg["layers"]
    micro_elems = pools.micro_capacity * L * 2 * 8 * row
    extent_elems = pools.extent_capacity * L * 2 * 64 * row
    assert K["fill_fp16"](C.c_void_p(pools.micro), micro_elems, fill_seed, 0.35, stream) == 0
    assert K["fill_fp16"](C.c_void_p(pools.extent), extent_elems, fill_seed + 1, 0.35, stream) == 0


# ---- single-layer paged attention + one-token append ----

C1_CONTEXTS = [17, 100, 513, 2000]
C1_POOL_PAGES = 4096
C1_SHAPE = dict(layers=1, kv_heads=4, head_dim=64, q_heads=32)


def c1_layout(create, append, seal, promote, release, seed: int, pool_pages: int = C1_POOL_PAGES,
              contexts: list[int] = C1_CONTEXTS) -> None:
    """The config-1 page layout through a page-table API (the product backend
    or a KvCacheManager, same calls; each returns 0 on success): every extent
    slot and then every micro slot is allocated once and released in a seeded
    order, so the pools' LIFO free lists hand out slots in a seeded
    permutation; then lane i (request i + 1) appends its context, seals, and
    promotes every full 64-token run (body = extents, tail = 8-token micro
    pages). Both pools hold pool_pages pages."""
    import random
    rng = random.Random(seed)
    base = 1 << 20
    ids = []
    for i in range(pool_pages):
        rid = base + i
        assert create(rid) == 0 and append(rid, 64) == 0
        seal(rid)
        assert promote(rid, 0) == 0
        ids.append(rid)
    rng.shuffle(ids)
    for rid in ids:
        assert release(rid) == 0
    ids = []
    for i in range(pool_pages):
        rid = 2 * base + i
        assert create(rid) == 0 and append(rid, 8) == 0
        ids.append(rid)
    rng.shuffle(ids)
    for rid in ids:
        assert release(rid) == 0
    for i, ctx in enumerate(contexts):
        rid = i + 1
        assert create(rid) == 0 and append(rid, ctx) == 0
        seal(rid)
        for begin in range(0, (ctx // 64) * 64, 64):
            assert promote(rid, begin) == 0


def c1_data(seed: int, pool_pages: int = C1_POOL_PAGES, lanes: int = len(C1_CONTEXTS)) -> dict:
    """Seeded FP16 contents (uint16 bits), all N(0, 1) / 8: both pools
    ([slot][layer][K|V][tokens][kv_head][dim]), the step's queries
    [lane][q_head * dim] and the appended token's K and V [lane][kv_head * dim]."""
    rng = np.random.default_rng(seed)
    L, H, D, Q = C1_SHAPE["layers"], C1_SHAPE["kv_heads"], C1_SHAPE["head_dim"], C1_SHAPE["q_heads"]

    def normal(shape):
        out = np.empty(shape, np.float16)
        flat = out.reshape(-1)
        for i in range(0, flat.size, 1 << 24):
            n = min(1 << 24, flat.size - i)
            flat[i:i + n] = (rng.standard_normal(n, dtype=np.float32) / 8).astype(np.float16)
        return out.view(np.uint16)

    return {"micro": normal((pool_pages, L, 2, 8, H, D)), "extent": normal((pool_pages, L, 2, 64, H, D)),
            "q": normal((lanes, Q * D)), "k": normal((lanes, H * D)), "v": normal((lanes, H * D))}
