"""Decode-throughput benchmark of the kim-kvcache token loop on B200.

Workload (default, config c4): TinyLlama-1.1B-shaped random-init FP16 decoder,
32 lanes per GPU, per-lane context ~ U[1024, 4096] stored as 64-token extent
pages (built by append + promotion) with 8-token micro-page tails; each step
decodes one token for every lane through the reference-facing runner API
(generationForwardBatch) and the fused sm_100a step. N GPUs = N independent
replicas (one process per GPU, no collective on the data path).

Prints one JSON line (rank 0): value = whole-job decode tok/s from the device
time of the fused steps (CUDA events, max over ranks); e2e = the same through
the host API with the per-step host->device input upload and device->host
token readback inside the CUDA-event-timed region; roofline of the dominant
kernel; the CPU oracle baseline on this box's host cores; SM clocks sampled
during the timed region.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4|c2|c5]
  python bench.py --impl reference ...   # the reference path on the host CPU
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import math
import os
import random
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "decode tok/s/GPU TinyLlama-shape c4/c32; paged-attn HBM GB/s vs 8 TB/s"
SEED = 0x4B564341434845  # the reference benchmark seed (include/kim-kv/benchmark/benchmark.h:123)
# Wall-time bound of the reference arm's timed steps (the whole arm then ends
# within a few minutes on the box's host cores).
REFERENCE_BUDGET_S = 90.0
# Positions per fused prefill call in the prompted decode workload (c5).
PREFILL_CHUNK = 64


def load_pkg(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def gpu_id(torch, dev) -> str:
    """nvidia-smi --id of this process's GPU (UUID: immune to CUDA_VISIBLE_DEVICES)."""
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        return uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
        return str(dev.index)


class ClockSampler:
    """nvidia-smi SM clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        # nvidia-smi takes a moment to start: wait (up to 3 s) for its first
        # sample, so that a short timed region is still sampled.
        deadline = time.time() + 3.0
        while time.time() < deadline and self.proc.poll() is None:
            self.file.flush()
            if os.path.getsize(self.file.name) > 0:
                break
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.flush()
        rows = [r.split(",") for r in open(self.file.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4)
                          if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


# ---------------------------------------------------------------------------
# our arm


def run_ours(args, rank, world, local_rank):
    import torch

    kk = load_pkg("kim_kvcache_b200", ROOT / "kim-kvcache_b200" / "__init__.py")
    synth = load_pkg("kk_synthetic", ROOT / "kim-kvcache_b200" / "synthetic.py")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        dist = dist_mod
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))

    wl = synth.decode_workload(args.config)
    B = wl["batch"]
    contexts = wl["contexts"]
    # c5 as BASELINE states it: the lanes' contexts are their prompts, run
    # through the fused prefill before decoding (c4/c2: synthetic prefixes).
    prompted = args.config == "c5" and args.pages == "hetero"
    cfg = dict(synth.TINYLLAMA)
    cfg["max_positions"] = max(4608, max(contexts) + args.steps + args.warmup + 8)
    archive_dir = Path(tempfile.gettempdir()) / f"kk_bench_archive_{cfg['max_positions']}"
    if rank == 0 or dist is None:
        manifest, data, _ = synth.write_archive(archive_dir, cfg, seed=SEED % (2 ** 31))
    if dist is not None:
        dist.barrier()
        manifest, data = str(archive_dir / "model.manifest"), str(archive_dir / "model.weights")

    K = kk.kernels()
    R = kk.runtime()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    total_tokens = sum(contexts) + B * (args.steps + args.warmup + 2)
    hq, hkv, D, L = cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"], cfg["layers"]
    row = hkv * D
    fixed = 0 if args.pages == "hetero" else int(args.pages[len("fixed"):])
    if fixed:
        # Fixed-page backend: every page holds `fixed` tokens (the reference's
        # strategy baseline); prefixes are appended, nothing is promoted.
        page_cap = sum(-(-(c + args.steps + args.warmup + 2) // fixed) for c in contexts) + B
        backend = R["fixed_backend_create"](L, hkv, D, hq, hq * cfg["max_positions"] * 4, fixed, page_cap)
        assert backend, "backend allocation failed"
        for i, ctx in enumerate(contexts):
            assert R["backend_create_request"](backend, i + 1) == 0
            assert R["backend_append"](backend, i + 1, ctx) == 0
        pools = kk.KvPools()
        assert R["backend_pools"](backend, C.byref(pools))
        assert K["fill_fp16"](C.c_void_p(pools.micro), page_cap * L * 2 * fixed * row, SEED + rank, 0.35,
                              sptr) == 0
    else:
        # Room for every 64-token run that auto-promotion folds during the run:
        # with too few extents, promotion fails and the tails grow as micro pages.
        micro_cap, extent_cap = synth.pool_capacities(contexts, args.steps + args.warmup + 3)
        if prompted:
            micro_cap += PREFILL_CHUNK // 8 + 8  # a chunk's pages before promotion folds them
        backend = R["backend_create"](L, hkv, D, hq, hq * cfg["max_positions"] * 4, micro_cap, extent_cap)
        assert backend, "backend allocation failed"
        pools = kk.KvPools()
        assert R["backend_pools"](backend, C.byref(pools))
        if not prompted:
            # Prefix state: append ctx tokens, seal, promote every full
            # 64-token run, then seeded KV contents in every page.
            synth.build_decode_prefixes(R, K, backend, pools, contexts, cfg, SEED + 2 * rank, sptr)
    torch.cuda.synchronize(dev)

    status = C.c_int(0)
    detail = C.create_string_buffer(512)
    runner = R["runner_create"](manifest.encode(), data.encode(), backend, sptr,
                                max(B, PREFILL_CHUNK if prompted else 1), 1, 1, C.byref(status), detail, 512)
    assert runner, f"runner creation failed: {status.value} {detail.value.decode()}"
    # Fold each lane's 8 sealed micro pages into an extent whenever decode
    # completes a 64-token run, so tails stay short (8 micro -> 1 extent).
    assert R["runner_set_auto_promote"](runner, 0 if fixed else 1) == 1

    ids = (C.c_uint64 * B)(*range(1, B + 1))
    tokens = (C.c_uint32 * B)(*[random.Random(SEED + b).randrange(3, 32000) for b in range(B)])
    positions = (C.c_uint32 * B)(*contexts)
    prefill = None
    if prompted:
        # The prompts go through the fused chunked prefill (the runner's
        # multi-position step, PREFILL_CHUNK positions per call), timed with
        # CUDA events around the API calls (prompt upload included); each
        # call returns the lane's first generated token.
        rng = random.Random(SEED)
        prompts = [(C.c_uint32 * n)(*[rng.randrange(3, 32000) for _ in range(n)]) for n in contexts]
        out1 = C.c_uint32(0)
        pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pe0.record(stream)
        for i, n in enumerate(contexts):
            assert R["backend_create_request"](backend, i + 1) == 0
            if not R["runner_prefill"](runner, i + 1, prompts[i], n, 0, C.byref(out1)):
                buf = C.create_string_buffer(512)
                R["runner_last_error"](runner, buf, 512)
                raise RuntimeError(f"prefill of lane {i} failed: {buf.value.decode()}")
            tokens[i] = out1.value
        pe1.record(stream)
        torch.cuda.synchronize(dev)
        pms = pe0.elapsed_time(pe1)
        prefill = {"prompt_tokens": sum(contexts), "ms": round(pms, 3),
                   "tok_per_s": round(sum(contexts) / (pms / 1e3), 1), "chunk": PREFILL_CHUNK,
                   "calls": len(contexts)}
    out_tok = (C.c_uint32 * B)()
    out_ok = (C.c_uint8 * B)()

    # numpy views of the call's buffers: the caller's per-step bookkeeping
    # (check every lane, feed the tokens back, advance the positions) is three
    # vector operations instead of per-lane Python.
    tokens_v, positions_v = np.ctypeslib.as_array(tokens), np.ctypeslib.as_array(positions)
    out_tok_v, out_ok_v = np.ctypeslib.as_array(out_tok), np.ctypeslib.as_array(out_ok)
    forward = R["runner_forward_batch"]

    def step():
        ok = forward(runner, B, ids, tokens, positions, out_tok, out_ok)
        if not (ok and out_ok_v.all()):
            buf = C.create_string_buffer(512)
            R["runner_last_error"](runner, buf, 512)
            raise RuntimeError(f"decode step failed: {buf.value.decode()}")
        tokens_v[:] = out_tok_v
        positions_v[:] += 1

    warm_ms = 0.0
    for _ in range(args.warmup):
        step()
        warm_ms += R["runner_last_step_ms"](runner)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    sampler = ClockSampler(gpu_id(torch, dev))
    sampler.start()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    device_ms = []
    h2d, d2h = C.c_uint64(0), C.c_uint64(0)
    h2d_total = d2h_total = 0
    host_us = (C.c_float * 5)()
    host_phases = []
    ev0.record(stream)
    for _ in range(args.steps):
        step()
        device_ms.append(R["runner_last_step_ms"](runner))
        R["runner_last_transfer_bytes"](runner, C.byref(h2d), C.byref(d2h))
        h2d_total += h2d.value
        d2h_total += d2h.value
        R["runner_last_host_us"](runner, host_us)
        host_phases.append(list(host_us))
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    launches = R["runner_last_launches"](runner)
    dev_ms = sum(device_ms)

    if args.trace:
        trace_step(kk, step, torch, dev, args.trace)

    # Dominant-kernel roofline: replay the attention of one step (all 22 layers,
    # same work list) and time it with CUDA events on the launching stream.
    roof = attention_roofline(kk, K, R, backend, pools, B, contexts, positions, cfg, stream, sptr)

    t = torch.tensor([dev_ms, e2e_ms], device=dev)
    per_rank_ms = [dev_ms]
    if dist is not None:
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        per_rank_ms = [round(float(g[0]) / args.steps, 4) for g in gathered]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
    dev_ms, e2e_ms = float(t[0]), float(t[1])
    if rank != 0:
        R["runner_destroy"](runner)
        R["backend_destroy"](backend)
        return None
    # After timing (untimed): one more decode step of every lane, checked lane
    # by lane against the CPU oracle fed the GPU's own K/V; the oracle's pass
    # over the same lanes is the CPU baseline at N = 1.
    check = None
    if not args.no_cpu_baseline and not fixed:
        check = oracle_check(kk, R, runner, backend, cfg, B, ids, tokens_v, positions_v, synth,
                             sptr, torch)
    R["runner_destroy"](runner)
    R["backend_destroy"](backend)
    tokens_total = B * args.steps * world
    line = {
        "metric": METRIC,
        "value": round(tokens_total / (dev_ms / 1e3), 1),
        "value_scope": f"whole job: decode tok/s summed over {world} GPU(s)",
        "per_gpu_value": round(B * args.steps / (dev_ms / 1e3), 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (random-init TinyLlama-shape weights, seeded contexts and KV)",
        "config": {
            "workload": wl["name"],
            "model": "TinyLlama-1.1B shape (22 layers, hidden 2048, 32q/4kv heads, vocab 32000)",
            "global_batch": B * world,
            "batch_per_gpu": B,
            "ctx_mean": round(sum(contexts) / len(contexts), 1),
            "parallelism": f"replicas x{world}",
            "pages": "micro 8 + extent 64, auto-promotion" if not fixed else f"fixed {fixed}-token pages",
            "l2": "inputs larger than L2 every step (2.07 GB weights + paged KV)",
            "cuda_graphs": True,
        },
        "e2e": {"value": round(tokens_total / (e2e_ms / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": round(h2d_total / args.steps), "d2h_bytes_per_step": round(d2h_total / args.steps)},
        "gpu_launches": launches * args.steps,
        # Median host wall time per step inside the runner's decode call (µs).
        "host_us_per_step": {name: round(statistics.median(p[i] for p in host_phases), 1)
                             for i, name in enumerate(("reserve", "record", "launch", "wait", "commit"))},
        "roofline": roof,
        "clocks": clocks,
    }
    if world > 1:
        line["per_rank_ms_per_step"] = per_rank_ms
    if prefill is not None:
        # The whole c5 job of this GPU: prompts through prefill, then every
        # decode step (warm-up included), device time; new tokens = the one
        # each prefill returns + one per decode step.
        job_ms = prefill["ms"] + warm_ms + dev_ms
        new_tok = B * (1 + args.warmup + args.steps)
        line["config"]["workload"] = wl["name"].replace("ctx~", "prompts~") + ", fused prefill then decode"
        line["prefill"] = prefill
        line["job"] = {"prompt_tokens": prefill["prompt_tokens"], "new_tokens": new_tok,
                       "device_ms": round(job_ms, 3), "new_tok_per_s": round(new_tok / (job_ms / 1e3), 1),
                       "scope": "one GPU (each replica runs the same job)"}
    if check is not None:
        line["parity"] = check["parity"]
        if world == 1:
            line["cpu_baseline"] = check["cpu_baseline"]
    return line


# DRAM traffic / algorithmic K+V bytes of one K1 launch, from an ncu capture of
# `bench.py --kernel-only attention --variant tma --plan balanced` (the same
# kernel, balanced work list and context distribution as the c4 step).
K1_TRAFFIC_PER_ALGORITHMIC_BYTE = 80.686848 / 78.297088


def attention_roofline(kk, K, R, backend, pools, B, contexts, positions, cfg, stream, sptr):
    import torch
    hq, D, L = cfg["q_heads"], cfg["head_dim"], cfg["layers"]
    # Current block tables of all lanes (committed prefix = what attention reads).
    descs_list, lanes = [], (kk.AttnLane * B)()
    buf = (kk.KkEntry * 8192)()
    for b in range(B):
        t = kk.KkTableOut(C.cast(buf, C.POINTER(kk.KkEntry)), 8192, 0, 0)
        assert R["backend_block_table"](backend, b + 1, C.byref(t))
        lanes[b].desc_offset = len(descs_list)
        lanes[b].desc_count = t.count
        lanes[b].token_count = sum(buf[i].valid_tokens for i in range(t.count))
        lanes[b].query_row = b
        for i in range(t.count):
            e = buf[i]
            descs_list.append(kk.PageDesc(e.slot, e.logical_token_begin, e.valid_tokens, e.kind, 0, 0))
    descs = (kk.PageDesc * len(descs_list))(*descs_list)
    items = (kk.AttnItem * 16384)()
    # the runner's own work list: one token-balanced run per SM
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    n_items = K["attention_plan_balanced"](descs, lanes, B, sms, items, 16384)
    tokens = sum(lanes[b].token_count for b in range(B))
    to_dev = lambda arr: torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).cuda()
    d_descs, d_lanes, d_items = to_dev(descs), to_dev(lanes), to_dev(items)
    q = torch.randn(B, hq * D, device="cuda").half() / 8
    out = torch.empty_like(q)
    ws_b = K["attention_workspace_bytes"](B, n_items, hq, D)
    ws = torch.zeros(ws_b, dtype=torch.uint8, device="cuda")

    def launch_all(sp):
        for layer in range(L):
            rc = K["paged_decode_attention"](C.byref(pools), layer, hq, d_descs.data_ptr(),
                                             d_lanes.data_ptr(), B, d_items.data_ptr(), n_items,
                                             q.data_ptr(), hq * D, out.data_ptr(), hq * D, 0.125,
                                             ws.data_ptr(), ws_b, sp)
            assert rc == 0
    for _ in range(3):
        launch_all(sptr)
    torch.cuda.synchronize()
    # One launch per layer, replayed from a CUDA graph with programmatic
    # dependent launch (as in the decode step), timed with events on the
    # stream the graph runs on.
    graph = torch.cuda.CUDAGraph()
    K["set_pdl"](1)
    with torch.cuda.graph(graph):
        launch_all(C.c_void_p(torch.cuda.current_stream().cuda_stream))
    K["set_pdl"](0)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    assert K["device_status"](sptr) == 0
    avg_ms = e0.elapsed_time(e1) / (reps * L)
    bytes_per_launch = tokens * cfg["kv_heads"] * D * 2 * 2  # K and V of every attended token
    peak, peak_note = measured_peaks()
    achieved = bytes_per_launch / (avg_ms / 1e3) / 1e9
    return {"kernel": "paged_attention_tma_kernel (K1), one layer, all lanes, balanced plan",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_note,
            "algorithmic_bytes_per_launch": bytes_per_launch, "avg_launch_us": round(avg_ms * 1e3, 2),
            "traffic": round(bytes_per_launch * K1_TRAFFIC_PER_ALGORITHMIC_BYTE),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of "
                              "the same kernel and work list on the kernel-only c4 case "
                              "(80.69 MB for 78.30 MB algorithmic), scaled by the bytes processed"}


# ---------------------------------------------------------------------------
# Phase trace (library built with `build.py --trace`)

# Stamps of a projection CTA: entry, dependency wait returned, accumulator
# complete, partial tile in shared memory, cluster wait passed, peers'
# partials received, reduced, epilogue stored, exit. Attention CTA: entry,
# producer's wait returned, producer done, first stage taken, consumers done,
# exit (aux = stages | split-combine flag << 31).
GEMM_PHASES = ["wait", "acc", "part", "cl_wait", "recv", "reduced", "epi", "exit", "xnorm", "rnorm", "x_land",
               "x_done", "mma0", "x_first_done", "x_last_land"]
ATTN_PHASES = ["wait", "prod_done", "first_stage", "cons_done", "exit"]


def trace_step(kk, step, torch, dev, path):
    """One decode step with per-CTA phase stamps: saves the records to `path`
    (.npz) and prints, per kernel, the median time of each phase after the
    launch's first dependency-wait return (medians over CTAs, then over the
    inner layers), the launch's span to its last exit, and the hand-off from
    the previous launch's last exit."""
    lib = kk.load_library()
    if not hasattr(lib, "kk_trace_read_gemm"):
        raise SystemExit("--trace needs the trace build: python kim-kvcache_b200/build.py --trace")
    rec = np.dtype([("tag", "<u4"), ("block", "<u4"), ("smid", "<u4"), ("aux", "<u4"), ("t", "<u8", 16)])
    readers = {"gemm": lib.kk_trace_read_gemm, "attn": lib.kk_trace_read_attn}
    for fn in readers.values():
        fn.restype = C.c_uint32
        fn.argtypes = [C.c_void_p, C.c_uint32, C.c_int]
        fn(None, 0, 1)
    step()
    torch.cuda.synchronize(dev)
    out = {}
    for name, fn in readers.items():
        buf = np.zeros(1 << 16, dtype=rec)
        out[name] = buf[:fn(C.c_void_p(buf.ctypes.data), 1 << 16, 1)]
    np.savez(path, **out)
    g, a = out["gemm"], out["attn"]
    kind, layer = g["tag"] >> 16, g["tag"] & 0xFFFF
    launches = []  # (start, name, layer, records)
    names = {4: "qkv", 3: "gate/up", 5: "lm_head"}
    for key in sorted(set(zip(kind.tolist(), layer.tolist(), g["aux"].tolist()))):
        k, l, kd = key
        nm = names.get(k, "o" if kd == 2048 else "down")
        r = g[(kind == k) & (layer == l) & (g["aux"] == kd)]
        launches.append((int(r["t"][:, 0].min()), nm, l, r, GEMM_PHASES))
    al = a["tag"] & 0xFFFF
    for l in sorted(set(al.tolist())):
        r = a[al == l]
        launches.append((int(r["t"][:, 0].min()), "attention", l, r, ATTN_PHASES))
    launches.sort(key=lambda x: x[0])
    rows, prev_end = {}, None
    for _, nm, l, r, phases in launches:
        t = r["t"].astype(np.int64)
        waits = t[:, 1][t[:, 1] > 0]
        w0 = int(waits.min()) if len(waits) else int(t[:, 0].min())
        # GEMM stamps 9-12: the fused RMSNorm's release, RMS factors, first X
        # tile landed, transforms done; 13: the first MMA issued.
        cols = list(range(1, 16)) if phases is GEMM_PHASES else [1, 2, 3, 4, 5]
        med = [float(np.median(t[:, c][t[:, c] > 0] - w0)) / 1e3 if (t[:, c] > 0).any() else float("nan")
               for c in cols]
        end = int(t[:, 8 if phases is GEMM_PHASES else 5].max())
        handoff = (w0 - prev_end) / 1e3 if prev_end is not None else float("nan")
        prev_end = end
        if 0 < l < max(layer.max(), al.max()):
            rows.setdefault(nm, []).append(med + [(end - w0) / 1e3, handoff, len(r)])
    print(f"phase trace of one step -> {path} (us after the launch's first dependency-wait return; "
          "medians over CTAs and over the inner layers)")
    for nm in ["qkv", "attention", "o", "gate/up", "down"]:
        if nm not in rows:
            continue
        m = np.nanmedian(np.array(rows[nm], dtype=float), axis=0)
        phases = ATTN_PHASES if nm == "attention" else GEMM_PHASES
        cells = "  ".join(f"{p} {v:.2f}" for p, v in zip(phases, m[:len(phases)]))
        print(f"  {nm:9s} CTAs {int(m[-1]):4d} | {cells} | span {m[-3]:.2f} | hand-off {m[-2]:.2f}")


# ---------------------------------------------------------------------------
# CPU oracle baseline / reference arm


def cpu_model(synth, cfg, threads):
    sys.path.insert(0, str(ROOT / "oracle"))
    import kk_oracle_py as ko
    archive_dir = Path(tempfile.gettempdir()) / f"kk_bench_archive_{cfg['max_positions']}"
    _, _, weights = synth.write_archive(archive_dir, cfg, seed=SEED % (2 ** 31), keep_weights=True)
    model = ko.Model(cfg, weights, threads=threads)
    del weights
    return ko, model


def oracle_check(kk, R, runner, backend, cfg, B, ids, tokens_v, positions_v, synth, sptr, torch):
    """One decode step of all B lanes through the batched-logits call,
    compared with the CPU oracle (the restatement of the reference decoder)
    that attends over the K/V the GPU holds for every lane (read back with the
    backend's gather). Returns the parity record (logits within 2e-2 on every
    lane, greedy tokens identical wherever the top-2 gap exceeds 2e-2) and
    the oracle's time for the same B-lane step as the CPU baseline."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import lane_parity as lp
    threads = os.cpu_count() or 1
    _, model = cpu_model(synth, cfg, threads)
    contexts_now = [int(x) for x in positions_v]
    toks_in = [int(x) for x in tokens_v]
    parity = lp.LaneParity(model, R, backend, list(ids), contexts_now, cfg, sptr, torch)
    got, ok, logits = lp.forward_with_logits(R, runner, list(ids), toks_in, contexts_now, cfg["vocab"])
    assert all(ok), "a lane of the checked step failed"
    t0 = time.perf_counter()
    parity.step(toks_in, contexts_now, got, logits)
    dt = time.perf_counter() - t0
    rec = parity.record()
    rec["lanes"] = len(rec["lanes"])
    parity.close()
    model.close()
    return {"parity": rec,
            "cpu_baseline": {"value": round(B / dt, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"one decode step of all {B} lanes (the GPU arm's lanes and "
                                       f"contexts, on the K/V the GPU holds), C restatement of the "
                                       f"reference FP16 decoder, {dt:.1f} s"}}


def run_reference(args, rank, world):
    """The reference arm: the reference's own model arithmetic, ReferenceModel
    of its runner contract test (tests/cuda/cuda_model_runner_test.cpp:
    213-420), compiled from the reference tree into oracle/_ref (kind
    "reference"); where that library is absent, the C restatement of it
    (kind "port"). The same B lanes and contexts as our arm, one
    ReferenceModel per lane holding that lane's K/V (seeded), lanes spread
    over every host core; a step decodes one token of every lane. The timed
    steps stop at --steps or when the next step would pass REFERENCE_BUDGET_S
    (stated in the sample). Rank 0 only."""
    if rank != 0:
        return None
    synth = load_pkg("kk_synthetic", ROOT / "kim-kvcache_b200" / "synthetic.py")
    sys.path.insert(0, str(ROOT / "oracle"))
    import kk_oracle_py as ko
    wl = synth.decode_workload(args.config)
    B, contexts = wl["batch"], wl["contexts"]
    cfg = dict(synth.TINYLLAMA)
    cfg["max_positions"] = max(4608, max(contexts) + args.steps + args.warmup + 8)
    threads = os.cpu_count() or 1
    archive_dir = Path(tempfile.gettempdir()) / f"kk_bench_archive_{cfg['max_positions']}"
    _, _, weights = synth.write_archive(archive_dir, cfg, seed=SEED % (2 ** 31), keep_weights=True)
    kind = "reference" if ko.REF_LIB.exists() else "port"
    model = ko.RefModel(cfg, weights) if kind == "reference" else ko.Model(cfg, weights, threads=threads)
    del weights
    L, row = cfg["layers"], cfg["kv_heads"] * cfg["head_dim"]
    rng = np.random.default_rng(5)
    longest = max(contexts)
    k = rng.uniform(-0.35, 0.35, (longest, L, row)).astype(np.float16).view(np.uint16)
    v = rng.uniform(-0.35, 0.35, (longest, L, row)).astype(np.float16).view(np.uint16)
    lanes = []
    for b, ctx in enumerate(contexts):
        if kind == "reference":
            lane = model.lane_create()
            model.lane_append_kv(lane, k[:ctx], v[:ctx])
        else:
            lane = b + 1
            model.create(lane)
            model.append_kv(lane, k[:ctx], v[:ctx])
        lanes.append(lane)
    del k, v

    def forward(toks, pos):
        if kind == "reference":
            return model.forward_lanes(lanes, toks, pos, threads)
        greedy, _, _ = model.forward(lanes, toks, pos, want_logits=False, want_hidden=False)
        return [int(x) for x in greedy]

    toks = [3 + (7919 * b) % 31997 for b in range(B)]
    pos = list(contexts)
    warm = min(args.warmup, 1)
    for _ in range(warm):
        toks = forward(toks, pos)
        pos = [p + 1 for p in pos]
    times = []
    begin = time.perf_counter()
    while len(times) < args.steps:
        if times and time.perf_counter() - begin + statistics.fmean(times) > REFERENCE_BUDGET_S:
            break
        t0 = time.perf_counter()
        toks = forward(toks, pos)
        times.append(time.perf_counter() - t0)
        pos = [p + 1 for p in pos]
    model.close()
    total_t = sum(times)
    value = B * len(times) / total_t
    what = ("ReferenceModel (the reference's test-local FP16 decoder, compiled from its source), one per lane"
            if kind == "reference" else "C restatement of the reference FP16 decoder")
    sample = (f"{len(times)} timed decode steps of all {B} lanes (after {warm} warm-up; bounded by "
              f"{REFERENCE_BUDGET_S:.0f} s of the requested {args.steps}), {what}, {threads} host threads, "
              "seeded K/V of the workload's contexts")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s",
            "n_gpus": world, "steps": len(times), "steps_requested": args.steps, "warmup": warm,
            "ms_per_step": round(total_t / max(len(times), 1) * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": wl["name"], "batch": B, "ctx_mean": round(sum(contexts) / B, 1),
                       "same_config": True},
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def run_c3(args):
    """TinyLlama shape, 4 concurrent requests through the
    iteration scheduler, prompts seeded uniform in [128, 512], chunked
    prefill in 64-token chunks mixed with decode, 128 new tokens each. Two
    requests share a prompt prefix of 256 + k tokens (k seeded in [1, 7], so
    the shared tail page is partial): it is prefilled once under request 1,
    forked to request 2 in the KV backend, and both are submitted with that
    prefix already in the cache, so each one's first write copies the shared
    partial tail. The scheduler hands every prompt chunk to the runner's
    fused prefill. Timed with CUDA events around the whole workload (prefix
    prefill, fork, submissions, drain), host calls included: value = output
    tokens per second; prompt and total token rates are reported beside it."""
    import torch
    kk = load_pkg("kim_kvcache_b200", ROOT / "kim-kvcache_b200" / "__init__.py")
    synth = load_pkg("kk_synthetic", ROOT / "kim-kvcache_b200" / "synthetic.py")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cfg = dict(synth.TINYLLAMA)
    cfg["max_positions"] = 4608
    archive_dir = Path(tempfile.gettempdir()) / f"kk_bench_archive_{cfg['max_positions']}"
    manifest, data, _ = synth.write_archive(archive_dir, cfg, seed=SEED % (2 ** 31))
    R = kk.runtime()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    hq, hkv, D, L = cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"], cfg["layers"]
    rng = random.Random(SEED)
    k = rng.randint(1, 7)
    P = 256 + k
    lengths = [rng.randint(128, 512) for _ in range(4)]
    lengths[0], lengths[1] = max(lengths[0], P + 1), max(lengths[1], P + 1)
    prefix = [rng.randrange(3, 32000) for _ in range(P)]
    prompts = [prefix + [rng.randrange(3, 32000) for _ in range(n - P)] if i < 2
               else [rng.randrange(3, 32000) for _ in range(n)] for i, n in enumerate(lengths)]
    new_tokens, chunk = 128, 64
    runs = args.steps if args.steps <= 8 else 3
    backend = R["backend_create"](L, hkv, D, hq, hq * cfg["max_positions"] * 4, 4 * (512 + 128) // 8 + 64,
                                  4 * (512 + 128) // 64 + 8)
    status, detail = C.c_int(0), C.create_string_buffer(512)
    runner = R["runner_create"](manifest.encode(), data.encode(), backend, sptr, chunk, 1, 1,
                                C.byref(status), detail, 512)
    assert runner, f"runner creation failed: {status.value} {detail.value.decode()}"
    assert R["runner_set_auto_promote"](runner, 1) == 1
    out = C.c_uint32(0)

    def workload(base):
        ids = [base + i for i in range(4)]
        assert R["backend_create_request"](backend, ids[0]) == 0
        pre = (C.c_uint32 * P)(*prefix)
        if not R["runner_prefill"](runner, ids[0], pre, P, 0, C.byref(out)):
            raise RuntimeError("prefix prefill failed")
        assert R["backend_fork"](backend, ids[0], ids[1]) == 0
        sched = kk.Scheduler(R, backend, runner, 4, 4 * chunk, 10 ** 6, chunk, fused_prefill=True)
        for i, rid in enumerate(ids):
            assert sched.submit(rid, prompts[i], new_tokens, -1, kv_prefix=P if i < 2 else 0) == 0
        terms = sched.drain()
        sched.close()
        return terms

    for w in range(max(1, args.warmup // 3)):
        workload(1000 * (w + 1))
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_id(torch, dev))
    sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    produced = 0
    ev0.record(stream)
    for r in range(runs):
        terms = workload(100000 * (r + 1))
        assert all(t["error"] == 0 for t in terms), terms
        produced += sum(len(t["tokens"]) for t in terms)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    snap = kk.BackendSnapshot()
    R["backend_snapshot"](backend, C.byref(snap))
    assert snap.request_count == 0 and R["backend_check_invariants"](backend) == 1
    R["runner_destroy"](runner)
    R["backend_destroy"](backend)
    prompt_tok = runs * sum(lengths)
    print(json.dumps({
        "metric": "scheduler output tok/s TinyLlama-shape c3 (4 requests, chunked fused prefill + decode)",
        "value": round(produced / (ms / 1e3), 1), "unit": "tok/s", "n_gpus": 1, "steps": runs,
        "warmup": max(1, args.warmup // 3), "ms_per_step": round(ms / runs, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": "c3: 4 requests, prompts ~U[128,512] (two share a forked 256+k prefix), "
                               "chunk 64, 128 new tokens each", "prompt_lengths": lengths, "shared_prefix": P,
                   "k": k, "fused_prefill": True, "auto_promote": True},
        "prompt_tok_per_s": round(prompt_tok / (ms / 1e3), 1),
        "total_tok_per_s": round((prompt_tok + produced) / (ms / 1e3), 1),
        "e2e": {"value": round(produced / (ms / 1e3), 1), "unit": "tok/s",
                "note": "host scheduler calls inside the CUDA-event-timed region"},
        "clocks": clocks}), flush=True)


# ---------------------------------------------------------------------------
# config 1: single-layer GQA paged decode attention + one-token KV append

C1_METRIC = "c1 attention+append step latency (1 layer, 4 lanes, ctx 17/100/513/2000)"


class _DevArray:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<u2", "data": (ptr, False), "version": 3}


def c1_reference(kk, synth, seed: int, data: dict):
    """The reference's config-1 CPU path (oracle/_ref): its KvCacheManager
    laid out like the GPU arm's backend, host pools holding the same seeded
    K/V, and kref_c1_step (reserveToken, K/V store, gather, referenceAttention
    per query head, rollback). Returns (step(threads) -> output, manager)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import kk_oracle_py as ko
    lib = C.CDLL(str(ko.REF_LIB))
    mgr = kk.Manager(lib, "kref_", synth.C1_POOL_PAGES, synth.C1_POOL_PAGES)

    def promote(rid, begin):
        err, pid, _, _ = mgr.prepare_promotion(rid, begin)
        return err if err else mgr.commit_promotion(pid)

    synth.c1_layout(mgr.create, mgr.append, mgr.seal, promote, mgr.release, seed)
    f = lib.kref_c1_step
    u16p = C.POINTER(C.c_uint16)
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(C.c_uint64), C.POINTER(C.c_uint32), u16p, u16p,
                  C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, u16p, u16p, u16p, u16p,
                  C.c_int, C.c_uint32]
    B = len(synth.C1_CONTEXTS)
    micro, extent = data["micro"].copy(), data["extent"].copy()
    out = np.zeros((B, synth.C1_SHAPE["q_heads"] * synth.C1_SHAPE["head_dim"]), np.uint16)
    ids = (C.c_uint64 * B)(*range(1, B + 1))
    expected = (C.c_uint32 * B)(*synth.C1_CONTEXTS)
    p = lambda a: a.ctypes.data_as(u16p)

    def step(threads):
        assert f(mgr.h, B, ids, expected, p(micro), p(extent), synth.C1_SHAPE["layers"], 0, synth.C1_SHAPE["kv_heads"],
                 synth.C1_SHAPE["head_dim"], synth.C1_SHAPE["q_heads"], p(data["k"]), p(data["v"]), p(data["q"]), p(out),
                 0, threads) == 1, "reference config-1 step failed"
        return out

    return step, mgr


def run_c1(args):
    """BASELINE config 1 on one GPU: a 1-layer backend (4 KV heads, head_dim
    64, 32 query heads) over a 4096-page micro and a 4096-page extent pool
    laid out by synthetic.c1_layout, 4 lanes of context 17 / 100 / 513 / 2000, seeded
    N(0,1)/8 contents. A step is the reference-facing per-layer token
    transaction of every lane: reserveToken, writeLayer of the new token's K/V,
    one attendLayerBatch over the 4 lanes (the paged decode-attention
    kernel), then rollback, so every step sees the same tables. value = mean
    device-timed latency of a step with the inputs resident (CUDA events on
    the stream, host calls inside); e2e = the same with the queries and the
    new K/V uploaded from pinned host memory and the outputs read back every
    step. After timing: the page tables equal the reference KvCacheManager's
    entry for entry, and the outputs are within 2e-2 of the reference's own
    CPU path on the same contents (its timing is the CPU baseline)."""
    import torch
    kk = load_pkg("kim_kvcache_b200", ROOT / "kim-kvcache_b200" / "__init__.py")
    synth = load_pkg("kk_synthetic", ROOT / "kim-kvcache_b200" / "synthetic.py")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    R = kk.runtime()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    L, H, D, Q = synth.C1_SHAPE["layers"], synth.C1_SHAPE["kv_heads"], synth.C1_SHAPE["head_dim"], synth.C1_SHAPE["q_heads"]
    B = len(synth.C1_CONTEXTS)
    ws_bytes = Q * 4096 * 4
    backend = R["backend_create"](L, H, D, Q, ws_bytes, synth.C1_POOL_PAGES, synth.C1_POOL_PAGES)
    assert backend, "backend allocation failed"
    synth.c1_layout(lambda r: R["backend_create_request"](backend, r), lambda r, n: R["backend_append"](backend, r, n),
              lambda r: R["backend_seal"](backend, r), lambda r, b: R["backend_promote"](backend, r, b, sptr),
              lambda r: R["backend_release"](backend, r), SEED)
    data = synth.c1_data(SEED)
    pools = kk.KvPools()
    assert R["backend_pools"](backend, C.byref(pools))
    for name, ptr in (("micro", pools.micro), ("extent", pools.extent)):
        host = torch.from_numpy(data[name].reshape(-1).view(np.int16))
        torch.as_tensor(_DevArray(ptr, host.numel()), device=dev).view(torch.int16).copy_(host)
    q_h, k_h, v_h = (torch.from_numpy(data[n].view(np.int16)).pin_memory() for n in ("q", "k", "v"))
    q_d, k_d, v_d = q_h.to(dev), k_h.to(dev), v_h.to(dev)
    out_d = torch.zeros_like(q_d)
    out_h = torch.zeros_like(q_h).pin_memory()
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(dev)
    st = C.c_int(0)
    statuses = (C.c_int * B)()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def step(upload: bool, tables: list | None = None):
        if upload:
            q_d.copy_(q_h, non_blocking=True)
            k_d.copy_(k_h, non_blocking=True)
            v_d.copy_(v_h, non_blocking=True)
        txns = []
        for i in range(B):
            t = R["txn_reserve"](backend, i + 1, synth.C1_CONTEXTS[i], sptr, C.byref(st))
            assert t and st.value == 0, f"reserve failed: {st.value}"
            txns.append(t)
        for i, t in enumerate(txns):
            assert R["txn_write_layer"](t, 0, k_d[i].data_ptr(), v_d[i].data_ptr()) == 0
        ev[2].record(stream)
        R["txn_attend_batch"]((C.c_void_p * B)(*txns), B, 0, q_d.data_ptr(), out_d.data_ptr(), Q * D * 2,
                              ws.data_ptr(), ws_bytes, 1.0 / math.sqrt(D), statuses)
        ev[3].record(stream)
        assert list(statuses) == [0] * B, list(statuses)
        if upload:
            out_h.copy_(out_d, non_blocking=True)
        if tables is not None:
            for t in txns:
                buf = (kk.KkEntry * 64)()
                tt = kk.KkTableOut(C.cast(buf, C.POINTER(kk.KkEntry)), 64, 0, 0)
                assert R["txn_reserved_table"](t, C.byref(tt)) == 1
                tables.append(kk.Manager._entries(tt, buf)[1])
        for t in txns:
            assert R["txn_rollback"](t) == 0
            R["txn_destroy"](t)

    def timed(upload: bool, n: int):
        lat, attend = [], []
        for _ in range(n):
            ev[0].record(stream)
            step(upload)
            ev[1].record(stream)
            ev[1].synchronize()
            lat.append(ev[0].elapsed_time(ev[1]) * 1e3)
            attend.append(ev[2].elapsed_time(ev[3]) * 1e3)
        return lat, attend

    # The first step's reserved tables: compared below with the reference
    # KvCacheManager's after the same layout (generations count allocations,
    # so they are compared before the steps' COW pages cycle).
    tables = []
    step(False, tables)
    timed(False, args.warmup)
    timed(True, args.warmup)
    sampler = ClockSampler(gpu_id(torch, dev))
    sampler.start()
    lat, attend = timed(False, args.steps)
    lat_e2e, _ = timed(True, args.steps)
    clocks = sampler.stop()

    # Checks (untimed): one more step and its outputs.
    step(True)
    torch.cuda.synchronize(dev)
    got = out_h.numpy().view(np.uint16).view(np.float16).astype(np.float32)
    ref_step, mgr = c1_reference(kk, synth, SEED, data)
    # As the GPU step does: every lane reserved, then every lane rolled back.
    ref_tables, ref_ids = [], []
    for i in range(B):
        err, rid, _, reserved = mgr.reserve(i + 1, synth.C1_CONTEXTS[i])
        assert err == 0
        ref_tables.append(reserved[1])
        ref_ids.append(rid)
    for rid in ref_ids:
        assert mgr.rollback(rid) == 0
    threads = os.cpu_count() or 1
    want = ref_step(threads).view(np.float16).astype(np.float32)
    err = float(np.max(np.abs(got - want)))
    t0, n_ref = time.perf_counter(), 0
    while n_ref < 3 or (time.perf_counter() - t0 < 10.0 and n_ref < args.steps):
        ref_step(threads)
        n_ref += 1
    ref_us = (time.perf_counter() - t0) / n_ref * 1e6
    mgr.close()
    R["backend_destroy"](backend)
    parity = {"lanes": B, "max_abs_err": round(err, 6), "tolerance": 2e-2,
              "tables_equal_reference": tables == ref_tables, "ok": err <= 2e-2 and tables == ref_tables}
    kv_bytes = sum((c + 1) * H * D * 2 * 2 for c in synth.C1_CONTEXTS) * L
    mean = statistics.fmean(lat)
    return {
        "metric": C1_METRIC, "value": round(mean, 2), "unit": "us", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(mean / 1e3, 5), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic (seeded N(0,1)/8)",
        "config": {"workload": "c1: 1 layer, 4 KV heads x 64, 32 query heads, 4 lanes ctx "
                               "17/100/513/2000, 4096-page micro + 4096-page extent pools, seeded "
                               "permutation; reserve + writeLayer + attendLayerBatch + rollback per step",
                   "l2": "working set (2.7 MB) stays in L2: a latency figure, not a bandwidth one"},
        "latency_us": {"p50": round(statistics.median(lat), 2), "p90": round(float(np.percentile(lat, 90)), 2),
                       "attend_call_p50": round(statistics.median(attend), 2)},
        "e2e": {"value": round(statistics.fmean(lat_e2e), 2), "unit": "us",
                "p50": round(statistics.median(lat_e2e), 2),
                "h2d_bytes_per_step": int(q_h.numel() * 2 + k_h.numel() * 2 + v_h.numel() * 2),
                "d2h_bytes_per_step": int(out_h.numel() * 2)},
        "algorithmic_kv_bytes_per_step": kv_bytes,
        "gpu_launches": None,
        "parity": parity,
        "cpu_baseline": {"value": round(ref_us, 2), "unit": "us", "cores": threads, "kind": "reference",
                         "sample": f"{n_ref} steps of the reference's CPU path on the same layout and "
                                   "contents (KvCacheManager reserve/rollback + gather + "
                                   "referenceAttention per query head, std::thread over lanes x KV heads)"},
        "clocks": clocks,
    }


def run_reference_c1(args):
    """Reference arm of config 1: the reference's own CPU path (kref_c1_step,
    oracle/_ref) on the same layout and contents as run_c1, all host cores."""
    kk = load_pkg("kim_kvcache_b200", ROOT / "kim-kvcache_b200" / "__init__.py")
    synth = load_pkg("kk_synthetic", ROOT / "kim-kvcache_b200" / "synthetic.py")
    data = synth.c1_data(SEED)
    step, mgr = c1_reference(kk, synth, SEED, data)
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        step(threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step(threads)
    us = (time.perf_counter() - t0) / max(args.steps, 1) * 1e6
    mgr.close()
    return {"impl": "reference", "metric": C1_METRIC, "value": round(us, 2), "unit": "us", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded N(0,1)/8)", "config": {"workload": "c1 (as the GPU arm)"},
            "cpu_baseline": {"value": round(us, 2), "unit": "us", "cores": threads, "kind": "reference",
                             "sample": f"{args.steps} steps after {args.warmup} warm-up: KvCacheManager "
                                       "reserve/rollback + gather + referenceAttention per query head"},
            "e2e": {"value": round(us, 2), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_prefill(args):
    """Prompt throughput of the fused multi-token prefill (kkrt_runner_prefill):
    --prefill-requests prompts of --prompt tokens each, every prompt fed in
    chunks of --prefill-chunk consecutive positions (the runner's batch size),
    causal attention over the request's pages. Timed with CUDA events around
    the API calls, so the prompt upload and the per-chunk token readback are
    inside the timed region (value = e2e)."""
    import torch
    kk = load_pkg("kim_kvcache_b200", ROOT / "kim-kvcache_b200" / "__init__.py")
    synth = load_pkg("kk_synthetic", ROOT / "kim-kvcache_b200" / "synthetic.py")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cfg = dict(synth.TINYLLAMA)
    P, nreq, chunk = args.prompt, args.prefill_requests, args.prefill_chunk
    cfg["max_positions"] = max(4608, P + 8)
    archive_dir = Path(tempfile.gettempdir()) / f"kk_bench_archive_{cfg['max_positions']}"
    manifest, data, _ = synth.write_archive(archive_dir, cfg, seed=SEED % (2 ** 31))
    R = kk.runtime()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    hq, hkv, D, L = cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"], cfg["layers"]
    micro_cap = (nreq + 1) * (P // 8 + 2)
    extent_cap = (nreq + 1) * (P // 64 + 1)
    backend = R["backend_create"](L, hkv, D, hq, hq * cfg["max_positions"] * 4, micro_cap, extent_cap)
    assert backend, "backend allocation failed"
    status, detail = C.c_int(0), C.create_string_buffer(512)
    runner = R["runner_create"](manifest.encode(), data.encode(), backend, sptr, chunk, 1, 1,
                                C.byref(status), detail, 512)
    assert runner, f"runner creation failed: {status.value} {detail.value.decode()}"
    assert R["runner_set_auto_promote"](runner, 1) == 1
    rng = random.Random(SEED)
    prompts = [(C.c_uint32 * P)(*[rng.randrange(3, 32000) for _ in range(P)]) for _ in range(nreq + 1)]
    out = C.c_uint32(0)

    def prefill(rid, prompt):
        assert R["backend_create_request"](backend, rid) == 0
        if not R["runner_prefill"](runner, rid, prompt, P, 0, C.byref(out)):
            buf = C.create_string_buffer(512)
            R["runner_last_error"](runner, buf, 512)
            raise RuntimeError(f"prefill failed: {buf.value.decode()}")

    for w in range(max(1, args.warmup // 3)):
        prefill(1000 + w, prompts[-1])
        assert R["backend_release"](backend, 1000 + w) == 0
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_id(torch, dev))
    sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for r in range(nreq):
        prefill(r + 1, prompts[r])
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    R["runner_destroy"](runner)
    R["backend_destroy"](backend)
    tok = nreq * P
    steps = nreq * -(-P // chunk)
    print(json.dumps({
        "metric": "prefill prompt tok/s/GPU TinyLlama-shape (fused causal chunks)",
        "value": round(tok / (ms / 1e3), 1), "unit": "tok/s", "n_gpus": 1, "steps": steps,
        "warmup": max(1, args.warmup // 3), "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": f"prefill: {nreq} prompts x {P} tokens, chunk {chunk}",
                   "model": "TinyLlama-1.1B shape", "auto_promote": True},
        "e2e": {"value": round(tok / (ms / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": None, "d2h_bytes_per_step": 4 * chunk},
        "clocks": clocks}), flush=True)


GEMM_SHAPES = {  # name: (M, K, epilogue) of the TinyLlama projections at N = 32
    "qkv": (2560, 2048, "f16"), "o": (2048, 2048, "f16"), "gu": (11264, 2048, "silu"),
    "down": (2048, 5632, "f16"), "lm": (32000, 2048, "f32"),
}


def run_kernel_only(args):
    """Small standalone cases of the hot kernels for profiling (no model):
    attention = one layer of K1 over config-4 shaped paged tables (32 lanes,
    ctx ~ U[1024, 4096], 22-layer pages so the pools exceed L2);
    gemm = one projection shape (--shape) at N = 32, cycling through enough
    weight copies that every launch streams its weights from HBM."""
    import torch
    kk = load_pkg("kim_kvcache_b200", ROOT / "kim-kvcache_b200" / "__init__.py")
    K = kk.kernels()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    sptr = C.c_void_p(stream.cuda_stream)
    label = {"kernel": args.kernel_only}
    if args.kernel_only == "gemm":
        M, Kd, epi = GEMM_SHAPES[args.shape]
        N = 32
        packed = args.layout == "packed"
        nbytes = M * Kd * 2
        copies = max(2, -(-256 * 2**20 // nbytes))
        x = torch.randn(64, Kd, device="cuda").half()
        out = torch.empty(64, M, device="cuda", dtype=torch.float32)
        descs = []
        keep = []
        for i in range(copies):
            w = torch.empty(M * Kd, dtype=torch.int16, device="cuda")
            K["fill_fp16"](C.c_void_p(w.data_ptr()), w.numel(), 10 + i, 0.02, sptr)
            d = kk.GemmDesc()
            if packed:
                pk = torch.empty(K["gemm_packed_bytes"](M, Kd) // 2, dtype=torch.int16, device="cuda")
                assert K["gemm_pack_weight"](w.data_ptr(), M, Kd, pk.data_ptr(), sptr) == 0
                d.weight, d.weight_layout = pk.data_ptr(), kk.W_PACKED
                keep.append(pk)
                del w
            else:
                d.weight = w.data_ptr()
                keep.append(w)
            d.M, d.K, d.x, d.N, d.x_stride, d.x_rows = M, Kd, x.data_ptr(), N, Kd, 64
            d.epilogue = {"f16": kk.EPI_STORE_F16, "silu": kk.EPI_SILU_PAIRS,
                          "f32": kk.EPI_STORE_F32}[epi]
            d.out, d.out_stride = out.data_ptr(), M // 2 if epi == "silu" else M
            descs.append(d)
        state = {"i": 0}

        def launch():
            d = descs[state["i"] % copies]
            state["i"] += 1
            return K["gemm"](C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream))
        label.update(shape=args.shape, layout=args.layout, M=M, K=Kd, N=N, weight_copies=copies)
    elif args.kernel_only == "gather":
        # K6: one 4096-token sequence (extent body + micro tail) of the
        # 22-layer TinyLlama KV gathered into a contiguous tensor.
        L, hkv, D, T = 22, 4, 64, 4096 + 40
        n_ext, n_mic = T // 64, (T % 64 + 7) // 8
        row = hkv * D
        micro = torch.empty(n_mic * 2 * L * 2 * 8 * row, dtype=torch.int16, device="cuda")
        extent = torch.empty(n_ext * 2 * L * 2 * 64 * row, dtype=torch.int16, device="cuda")
        K["fill_fp16"](C.c_void_p(micro.data_ptr()), micro.numel(), 1, 0.35, sptr)
        K["fill_fp16"](C.c_void_p(extent.data_ptr()), extent.numel(), 2, 0.35, sptr)
        pools = kk.KvPools(micro.data_ptr(), extent.data_ptr(), n_mic * 2, n_ext * 2, L, hkv, D, 0)
        rng = random.Random(SEED)
        es, ms = rng.sample(range(n_ext * 2), n_ext), rng.sample(range(n_mic * 2), n_mic)
        descs_list, t = [], 0
        for slot in es:
            descs_list.append(kk.PageDesc(slot, t, 64, 1, 0, 0))
            t += 64
        for slot in ms:
            n = min(8, T - t)
            descs_list.append(kk.PageDesc(slot, t, n, 0, 0, 0))
            t += n
        descs = (kk.PageDesc * len(descs_list))(*descs_list)
        dd = torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).cuda()
        out = torch.empty(L * 2 * T * row, dtype=torch.int16, device="cuda")

        def launch():
            return K["kv_gather"](C.byref(pools), dd.data_ptr(), len(descs_list), T, out.data_ptr(),
                                  C.c_void_p(torch.cuda.current_stream().cuda_stream))
        nbytes = 2 * L * 2 * T * row * 2  # read + write
        label.update(tokens=T, descriptors=len(descs_list), note="bytes = read + write")
    else:
        variant = {"auto": kk.ATTN_AUTO, "direct": kk.ATTN_DIRECT, "tma": kk.ATTN_TMA}[args.variant]
        assert K["attention_set_variant"](variant) == 0
        label.update(variant=args.variant)
        rng = random.Random(SEED)
        contexts = [rng.randint(1024, 4096) for _ in range(32)]
        L, hkv, D, hq = 22, 4, 64, 32
        extent_cap = sum(c // 64 for c in contexts)
        micro_cap = 32 * 8 + 8
        row = hkv * D
        micro = torch.empty(micro_cap * L * 2 * 8 * row, dtype=torch.int16, device="cuda")
        extent = torch.empty(extent_cap * L * 2 * 64 * row, dtype=torch.int16, device="cuda")
        K["fill_fp16"](C.c_void_p(micro.data_ptr()), micro.numel(), 1, 0.35, sptr)
        K["fill_fp16"](C.c_void_p(extent.data_ptr()), extent.numel(), 2, 0.35, sptr)
        pools = kk.KvPools(micro.data_ptr(), extent.data_ptr(), micro_cap, extent_cap, L, hkv, D, 0)
        descs_list, lanes = [], (kk.AttnLane * 32)()
        es, ms = list(range(extent_cap)), list(range(micro_cap))
        rng.shuffle(es)
        rng.shuffle(ms)
        for b, ctx in enumerate(contexts):
            lanes[b].desc_offset, lanes[b].query_row, lanes[b].token_count = len(descs_list), b, ctx
            t = 0
            while t + 64 <= ctx:
                descs_list.append(kk.PageDesc(es.pop(), t, 64, 1, 0, 0))
                t += 64
            while t < ctx:
                n = min(8, ctx - t)
                descs_list.append(kk.PageDesc(ms.pop(), t, n, 0, 0, 0))
                t += n
            lanes[b].desc_count = len(descs_list) - lanes[b].desc_offset
        descs = (kk.PageDesc * len(descs_list))(*descs_list)
        items = (kk.AttnItem * 8192)()
        if args.plan == "balanced":
            n_items = K["attention_plan_balanced"](descs, lanes, 32, torch.cuda.get_device_properties(0).multi_processor_count, items, 8192)
        else:
            n_items = K["attention_plan"](descs, lanes, 32, args.target_tokens, items, 8192)
        to_dev = lambda arr: torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).cuda()
        dd, dl, di = to_dev(descs), to_dev(lanes), to_dev(items)
        q = (torch.randn(32, hq * D, device="cuda") / 8).half()
        out = torch.empty_like(q)
        ws_b = K["attention_workspace_bytes"](32, n_items, hq, D)
        ws = torch.zeros(ws_b, dtype=torch.uint8, device="cuda")
        state = {"i": 0}

        def launch():
            layer = state["i"] % L  # a different layer's K/V every launch: HBM, not L2
            state["i"] += 1
            return K["paged_decode_attention"](
                C.byref(pools), layer, hq, dd.data_ptr(), dl.data_ptr(), 32, di.data_ptr(), n_items,
                q.data_ptr(), hq * D, out.data_ptr(), hq * D, 0.125, ws.data_ptr(), ws_b,
                C.c_void_p(torch.cuda.current_stream().cuda_stream))
        nbytes = sum(contexts) * row * 2 * 2
        label.update(items=n_items, plan=args.plan, target_tokens=args.target_tokens)
    for _ in range(args.warmup):
        assert launch() == 0
    torch.cuda.synchronize()
    # The timed launches are replayed from a CUDA graph, so the device time is
    # not inflated by host launch overhead between short kernels.
    graph = torch.cuda.CUDAGraph()
    K["set_pdl"](1 if args.pdl else 0)
    with torch.cuda.graph(graph):
        for _ in range(args.steps):
            assert launch() == 0
    K["set_pdl"](0)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    label.update(pdl=bool(args.pdl))
    us = e0.elapsed_time(e1) / args.steps * 1e3
    peak, _ = measured_peaks()
    assert K["device_status"](sptr) == 0
    label.update(avg_us=round(us, 2), bytes=nbytes, gbs=round(nbytes / us / 1e3, 1),
                 frac=round(nbytes / us / 1e3 / peak, 4))
    print(json.dumps(label))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4", choices=["c4", "c2", "c5", "c3", "c1"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-only", choices=["attention", "gemm", "gather"], default=None,
                    help="time one hot kernel on a standalone case (profiling)")
    ap.add_argument("--shape", default="gu", choices=sorted(GEMM_SHAPES),
                    help="--kernel-only gemm: projection shape")
    ap.add_argument("--layout", default="packed", choices=["packed", "rowmajor"],
                    help="--kernel-only gemm: weight layout")
    ap.add_argument("--variant", default="auto", choices=["auto", "direct", "tma"],
                    help="--kernel-only attention: kernel variant")
    ap.add_argument("--target-tokens", type=int, default=256,
                    help="--kernel-only attention: tokens per work item (--plan lane)")
    ap.add_argument("--pdl", action="store_true",
                    help="--kernel-only: launch with programmatic dependent launch (as the runner does)")
    ap.add_argument("--plan", default="balanced", choices=["balanced", "lane"],
                    help="--kernel-only attention: one token-balanced run per SM, or per-lane items")
    ap.add_argument("--pages", default="hetero", choices=["hetero", "fixed8", "fixed16", "fixed32", "fixed64"],
                    help="KV backend of the decode step: two pools (8-token micro + 64-token extent pages, "
                         "the default) or a fixed-page backend (reference Fixed-8/16/32/64)")
    ap.add_argument("--trace", default=None, metavar="OUT.npz",
                    help="after the timed steps, record per-CTA phase stamps of one more step "
                         "(needs the library built with build.py --trace)")
    ap.add_argument("--prefill", action="store_true",
                    help="time the fused multi-token prefill instead of decode (one GPU)")
    ap.add_argument("--prompt", type=int, default=1024, help="--prefill: tokens per prompt")
    ap.add_argument("--prefill-requests", type=int, default=8, help="--prefill: prompts timed")
    ap.add_argument("--prefill-chunk", type=int, default=64,
                    help="--prefill: positions per fused step (the runner batch size)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.kernel_only:
        run_kernel_only(args)
        return
    if args.prefill:
        run_prefill(args)
        return
    if args.config == "c3" and args.impl == "ours":
        run_c3(args)
        return
    if args.config == "c1":
        line = None
        if rank == 0:
            line = run_reference_c1(args) if args.impl == "reference" else run_c1(args)
    else:
        line = run_reference(args, rank, world) if args.impl == "reference" else run_ours(
            args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)
        if "parity" in line and not line["parity"]["ok"]:
            sys.exit("parity gate failed: the checked step disagrees with the CPU reference")


if __name__ == "__main__":
    main()
