"""TEST INFRASTRUCTURE ONLY — lane-by-lane parity of the fused decode step
against the CPU oracle (kk_oracle.c, the restatement of the reference's
FP16-rounding decoder, tests/cuda/cuda_model_runner_test.cpp:213-420).

The oracle attends over exactly the K/V the GPU holds: each checked lane's
committed pages are read back with the backend's gather
(kkrt_backend_gather, [layer][K|V][token][head][dim]) and appended to an
oracle sequence, so the comparison covers long synthetic contexts without
recomputing a prefill on the CPU. Every decode step then runs on both sides
with the same input token; the oracle computes the new token's K/V itself.

Gates: greedy tokens identical wherever the oracle's top-2 logit gap exceeds
2e-2, and logits within a bound that starts at the
north star's 2e-2 absolute. With random-init weights a 22-layer FP16 decoder
amplifies every 1-ulp FP16 difference, so the same reference arithmetic
summed in another order (the oracle's twin, kko_model_set_wide_sums) already
moves the logits of these lanes by about that much. Each checked step
therefore also runs the twin on the same lanes, and the logit bound is
    min(0.035, max(2e-2, 1.5 x the twin's own deviation)),
0.035 being the bound the reference puts on its own CUDA runner against its
ReferenceModel (tests/cuda/cuda_model_runner_test.cpp:536). The record keeps
the measured error, the twin's deviation and the bound.

Imported only by tests/ and by bench.py's CPU-baseline leg (as the checker).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

TOL = 2e-2
REFERENCE_RUNNER_TOL = 0.035  # tests/cuda/cuda_model_runner_test.cpp:536 of the reference
FLOOR_FACTOR = 1.5


def pick_lanes(contexts: list[int], count: int = 5) -> list[int]:
    """Indices of the lanes to check: the longest and the shortest context,
    then lanes spread over the batch, `count` in all (fewer for small batches)."""
    order = {int(np.argmax(contexts)), int(np.argmin(contexts))}
    n = len(contexts)
    for i in np.linspace(0, n - 1, num=max(count, 2)).astype(int):
        if len(order) >= min(count, n):
            break
        order.add(int(i))
    return sorted(order)


def gather_lane_kv(R, backend, request_id: int, tokens: int, cfg: dict, stream, torch):
    """The lane's committed K and V as uint16 arrays [tokens][layers][kv_heads*head_dim]."""
    L, hkv, D = cfg["layers"], cfg["kv_heads"], cfg["head_dim"]
    out = torch.empty(L, 2, tokens, hkv, D, dtype=torch.half, device="cuda")
    assert R["backend_gather"](backend, request_id, out.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    host = out.cpu().view(torch.int16).numpy().view(np.uint16)
    k = np.ascontiguousarray(host[:, 0].transpose(1, 0, 2, 3).reshape(tokens, L, hkv * D))
    v = np.ascontiguousarray(host[:, 1].transpose(1, 0, 2, 3).reshape(tokens, L, hkv * D))
    return k, v


class LaneParity:
    """Oracle sequences mirroring some lanes of a GPU batch, and the running
    parity record of the steps compared so far."""

    def __init__(self, model, R, backend, lane_ids: list[int], contexts: list[int], cfg: dict,
                 stream, torch, seq_base: int = 1 << 40):
        self.model, self.cfg = model, cfg
        self.lanes = list(lane_ids)           # request ids of the checked lanes
        self.seqs = [seq_base + r for r in self.lanes]
        self.max_logit_err = 0.0
        self.max_twin_err = 0.0                # the oracle's own summation-order deviation
        self.mismatches = []                  # (step, request, gpu, oracle, gap)
        self.tokens_compared = 0
        self.logit_rows = 0
        self.steps = 0
        for rid, seq, ctx in zip(self.lanes, self.seqs, contexts):
            k, v = gather_lane_kv(R, backend, rid, ctx, cfg, stream, torch)
            model.create(seq)
            model.append_kv(seq, k, v)

    def step(self, tokens_in: list[int], positions: list[int], gpu_tokens: list[int],
             gpu_logits: np.ndarray | None = None):
        """One decode position of the checked lanes: tokens_in / positions /
        gpu_tokens (and optionally gpu_logits [lanes][vocab]) in lane order."""
        if gpu_logits is not None:
            # The twin first, on copies of the sequences (forward appends K/V).
            twins = [s_ + (1 << 62) for s_ in self.seqs]
            for s_, t_ in zip(self.seqs, twins):
                self.model.fork(s_, t_)
            self.model.set_wide_sums(True)
            try:
                _, twin_logits, _ = self.model.forward(twins, tokens_in, positions, want_logits=True,
                                                       want_hidden=False)
            finally:
                self.model.set_wide_sums(False)
                for t_ in twins:
                    self.model.release(t_)
        want, logits, _ = self.model.forward(self.seqs, tokens_in, positions, want_logits=True,
                                             want_hidden=False)
        if gpu_logits is not None:
            self.max_twin_err = max(self.max_twin_err, float(np.max(np.abs(twin_logits - logits))))
        for i, rid in enumerate(self.lanes):
            top = np.sort(logits[i])[-2:]
            gap = float(top[1] - top[0])
            self.tokens_compared += 1
            if gap > TOL and int(gpu_tokens[i]) != int(want[i]):
                self.mismatches.append((self.steps, rid, int(gpu_tokens[i]), int(want[i]), gap))
            if gpu_logits is not None:
                err = float(np.max(np.abs(gpu_logits[i] - logits[i])))
                self.max_logit_err = max(self.max_logit_err, err)
                self.logit_rows += 1
        self.steps += 1
        return want, logits

    def logit_bound(self) -> float:
        return min(REFERENCE_RUNNER_TOL, max(TOL, FLOOR_FACTOR * self.max_twin_err))

    def record(self) -> dict:
        return {"lanes": self.lanes, "steps": self.steps, "tokens_compared": self.tokens_compared,
                "logit_rows_compared": self.logit_rows,
                "max_abs_logit_err": round(self.max_logit_err, 6),
                "oracle_twin_max_abs_logit_err": round(self.max_twin_err, 6),
                "logit_bound": round(self.logit_bound(), 6),
                "greedy_mismatches_above_gap": len(self.mismatches), "token_gap_tolerance": TOL,
                "ok": self.ok()}

    def ok(self) -> bool:
        return not self.mismatches and self.max_logit_err <= self.logit_bound()

    def close(self):
        for seq in self.seqs:
            self.model.release(seq)


def forward_with_logits(R, runner, ids, tokens, positions, vocab):
    """kkrt_runner_forward_batch_logits: (tokens, ok, logits [n][vocab])."""
    n = len(ids)
    out, ok = (C.c_uint32 * n)(), (C.c_uint8 * n)()
    logits = np.zeros((n, vocab), dtype=np.float32)
    rc = R["runner_forward_batch_logits"](runner, n, (C.c_uint64 * n)(*ids), (C.c_uint32 * n)(*tokens),
                                          (C.c_uint32 * n)(*positions), out, ok,
                                          logits.ctypes.data_as(C.POINTER(C.c_float)))
    assert rc == 1, "batched logits step rejected"
    return [out[i] for i in range(n)], [ok[i] for i in range(n)], logits
