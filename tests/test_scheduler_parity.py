"""Scheduler and single-request generation parity against the reference's own
IterationSchedulerRuntime / SingleRequestGenerationRuntime (compiled from its
sources into oracle/_ref), both driven by identical SPI test doubles: the
sequence of model batches (every item), the per-iteration counters and the
terminals (reason, error, output tokens, usage) must be identical.
Scenarios follow the reference contract tests (tests/engine/
iteration_scheduler_test.cpp:240-412): FIFO join/exit, chunked-prefill budget,
admission gates, cancel, stop, model failure isolation, EOS, batch splitting."""
import ctypes as C
import random

import pytest


def bind_scheduler(kk, lib, prefix):
    # The reference exposes the common entry points; this library's
    # extensions (fused prefill, KV-prefix requests) are bound where present.
    return kk.bind(lib, prefix, {k: v for k, v in kk.RUNTIME_SIGNATURES.items()
                                 if k.startswith(("sched_", "fake_", "generate"))
                                 and hasattr(lib, prefix + k)})


def both(kk, kk_lib, ref_lib):
    return [bind_scheduler(kk, kk_lib, "kkrt_"), bind_scheduler(kk, ref_lib, "kref_")]


def batch_log(f, runner):
    sizes = (C.c_uint32 * 65536)()
    items = (C.c_uint64 * (3 * 1 << 18))()
    n = f["fake_runner_log"](runner, sizes, 65536, items, 3 << 18)
    total = sum(sizes[i] for i in range(n))
    return [sizes[i] for i in range(n)], [items[i] for i in range(3 * total)]


def comparable(terms):
    return [(t["request_id"], t["reason"], t["error"], tuple(t["tokens"]), t["prompt_tokens"],
             t["completion_tokens"], t["ttft_ns"] > 0 if t["tokens"] else None) for t in terms]


def run_scenario(kk, fns, cfg, requests, actions, vocab=97, max_batch=4, eos=5, fail=0):
    f = fns
    backend = f["fake_backend_create"]()
    runner = f["fake_runner_create"](vocab, max_batch, eos, cfg.get("max_pos", 4096), fail)
    s = kk.Scheduler(f, backend, runner, cfg["max_active"], cfg["max_tokens"], cfg["max_kv"],
                     cfg["chunk"])
    admissions = [s.submit(rid, prompt, max_new, e) for rid, prompt, max_new, e in requests]
    iters = []
    for step in range(cfg.get("iterations", 10 ** 6)):
        if f["sched_idle"](s.h):
            break
        for kind, when, arg in actions:
            if when == step:
                if kind == "cancel":
                    s.cancel(arg)
                elif kind == "stop":
                    s.stop()
                elif kind == "submit":
                    admissions.append(s.submit(*arg))
        iters.append(s.run_iteration())
    terms = s.drain()
    log = batch_log(f, runner)
    s.close()
    f["fake_runner_destroy"](runner)
    f["fake_backend_destroy"](backend)
    return admissions, iters, comparable(terms), log


def check(kk, kk_lib, ref_lib, *args, **kw):
    a, b = both(kk, kk_lib, ref_lib)
    ra = run_scenario(kk, a, *args, **kw)
    rb = run_scenario(kk, b, *args, **kw)
    assert ra[0] == rb[0], "admission results differ"
    assert ra[3] == rb[3], "model batch sequence differs"
    assert ra[1] == rb[1], "iteration counters differ"
    assert ra[2] == rb[2], "terminals differ"
    return ra


def _random_scenario(seed):
    rng = random.Random(seed)
    cfg = dict(max_active=rng.randint(1, 10), max_tokens=rng.randint(1, 40),
               max_kv=rng.randint(50, 2000), chunk=rng.randint(1, 16))
    reqs = []
    for rid in range(1, rng.randint(2, 14)):
        reqs.append((rid, [rng.randrange(0, 97) for _ in range(rng.randint(1, 40))],
                     rng.randint(1, 20), rng.choice([-1, -1, 5, 96, 200])))
    actions = [("cancel", rng.randint(0, 20), rng.randint(1, 14)) for _ in range(rng.randint(0, 3))]
    return (cfg, reqs, actions), dict(vocab=97, max_batch=rng.randint(1, 8), eos=rng.choice([5, 60]),
                                      fail=rng.choice([0, 0, 3]))


_CANCEL_CFG = dict(max_active=8, max_tokens=8, max_kv=10 ** 6, chunk=2)
_CANCEL_REQS = [(i, [i + 3] * (i % 5 + 1), 6, -1) for i in range(1, 9)]

# (name, positional args after `fns`, keyword args) of every scheduler
# scenario; shared with the golden-fixture generator (tests/golden).
SCENARIOS = [
    ("fifo_chunked_prefill", (dict(max_active=4, max_tokens=16, max_kv=100000, chunk=4),
                              [(1, [3, 4, 6, 7, 8, 9, 10], 5, -1), (2, [11] * 12, 3, -1), (3, [12], 8, -1),
                               (4, [13, 14], 1, -1)], []), {}),
    ("admission_gates_late_join", (dict(max_active=2, max_tokens=6, max_kv=40, chunk=3),
                                   [(1, [3] * 10, 10, -1), (2, [4] * 20, 5, -1), (3, [5] * 30, 30, -1),
                                    (0, [1], 1, -1), (1, [3], 1, -1), (7, [], 1, -1), (8, [96, 97], 1, -1)],
                                   [("submit", 3, (9, [6, 7], 4, -1)), ("submit", 6, (10, [8], 3, -1))]), {}),
    ("cancel_and_model_failure", (_CANCEL_CFG, _CANCEL_REQS, [("cancel", 2, 3), ("cancel", 4, 6)]),
     dict(fail=5)),
    ("stop", (_CANCEL_CFG, _CANCEL_REQS, [("stop", 3, None)]), {}),
] + [(f"random_{seed}",) + _random_scenario(seed) for seed in range(8)]


def test_fifo_chunked_prefill_and_decode(kk, kk_lib, ref_lib):
    _, args, kw = SCENARIOS[0]
    admissions, iters, terms, log = check(kk, kk_lib, ref_lib, *args, **kw)
    assert admissions == [0, 0, 0, 0]
    assert {t[0] for t in terms} == {1, 2, 3, 4}


@pytest.mark.parametrize("index", range(1, len(SCENARIOS)), ids=[s[0] for s in SCENARIOS[1:]])
def test_scenarios_match_reference(kk, kk_lib, ref_lib, index):
    _, args, kw = SCENARIOS[index]
    check(kk, kk_lib, ref_lib, *args, **kw)


def test_single_request_generation(kk, kk_lib, ref_lib):
    a, b = both(kk, kk_lib, ref_lib)
    outs = []
    for f in (a, b):
        res = []
        for rid, prompt, max_new, eos, fail in [(1, [3, 4, 5], 6, -1, 0), (2, [9] * 20, 40, 60, 0),
                                                (3, [7], 5, -1, 3), (4, [], 3, -1, 0),
                                                (5, [200], 3, -1, 0), (6, [4, 4], 1, -1, 0)]:
            backend = f["fake_backend_create"]()
            runner = f["fake_runner_create"](97, 4, 5, 64, fail)
            term = kk.Terminal()
            toks = (C.c_uint32 * 256)()
            n = f["generate"](backend, runner, rid, kk._u32(prompt), len(prompt), max_new, eos,
                              C.byref(term), toks, 256)
            res.append((n, term.reason, term.error, list(toks[:term.token_count]),
                        term.prompt_tokens, term.completion_tokens, batch_log(f, runner)))
            f["fake_runner_destroy"](runner)
            f["fake_backend_destroy"](backend)
        outs.append(res)
    assert outs[0] == outs[1]
