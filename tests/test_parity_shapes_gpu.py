"""Parity of the fused sm_100a decode step at the shapes that bench.py
measures (BASELINE configs 4 and 5): TinyLlama-1.1B shape (22 layers, hidden
2048, 32 query / 4 KV heads, vocab 32000), the bench's own seeded contexts,
pools and auto-promotion, batch 32 with ctx ~ U[1024, 4096] and batch 64
with ctx ~ U[64, 1024].

Lanes are checked against the CPU oracle (the restatement of the
reference's FP16-rounding decoder, tests/cuda/cuda_model_runner_test.cpp
:213-420) fed the K/V the GPU holds for them (read back with the backend's
gather). Gates (oracle/lane_parity.py): greedy tokens identical wherever the
oracle's top-2 gap exceeds 2e-2 on every step (the captured-graph steps
included); logits within 2e-2 absolute on the steps that return logits, or
within 1.5 x the deviation of the oracle's own summation-order twin on the
same rows where that floor is higher (never above the 0.035 the reference
allows its own CUDA runner, cuda_model_runner_test.cpp:536); every lane
committed.
"""
import ctypes as C
import importlib.util
import os
import tempfile
from pathlib import Path

import pytest
import torch

import kk_oracle_py as ko
import lane_parity as lp

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

ROOT = Path(__file__).resolve().parent.parent
STEPS = 5           # steps 0 and STEPS-1 return logits; the ones between replay the graph


def _synth():
    spec = importlib.util.spec_from_file_location("kk_synth", ROOT / "kim-kvcache_b200" / "synthetic.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.fixture(scope="module")
def tinyllama():
    """The bench's model: random-init TinyLlama shape, archive + oracle (shared
    by the tests of this module)."""
    synth = _synth()
    cfg = dict(synth.TINYLLAMA)
    cfg["max_positions"] = 4608
    d = Path(tempfile.gettempdir()) / "kk_parity_archive"
    manifest, data, weights = synth.write_archive(d, cfg, seed=synth.BENCH_SEED % (2 ** 31),
                                                  keep_weights=True)
    model = ko.Model(cfg, weights, threads=os.cpu_count() or 8)
    del weights
    yield synth, cfg, manifest, data, model
    model.close()


@pytest.mark.parametrize("config", ["c4", "c5"])
def test_fused_step_matches_oracle_at_bench_shape(kk, tinyllama, config):
    synth, cfg, manifest, data, model = tinyllama
    R, K = kk.runtime(), kk.kernels()
    wl = synth.decode_workload(config)
    B, contexts = wl["batch"], wl["contexts"]
    L, hkv, D, hq = cfg["layers"], cfg["kv_heads"], cfg["head_dim"], cfg["q_heads"]
    micro_cap, extent_cap = synth.pool_capacities(contexts, STEPS + 8)
    backend = R["backend_create"](L, hkv, D, hq, hq * cfg["max_positions"] * 4, micro_cap, extent_cap)
    assert backend
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    pools = kk.KvPools()
    assert R["backend_pools"](backend, C.byref(pools))
    synth.build_decode_prefixes(R, K, backend, pools, contexts, cfg, synth.BENCH_SEED, stream)
    torch.cuda.synchronize()
    st, det = C.c_int(0), C.create_string_buffer(512)
    runner = R["runner_create"](manifest.encode(), data.encode(), backend, stream, B, 1, 0,
                                C.byref(st), det, 512)
    assert runner, det.value.decode()
    assert R["runner_set_auto_promote"](runner, 1) == 1

    sel = lp.pick_lanes(contexts, 5)
    parity = lp.LaneParity(model, R, backend, [i + 1 for i in sel], [contexts[i] for i in sel], cfg,
                           stream, torch)
    ids = list(range(1, B + 1))
    toks = [3 + (7919 * b) % 31997 for b in range(B)]
    pos = list(contexts)
    for step in range(STEPS):
        if step in (0, STEPS - 1):
            got, ok, logits = lp.forward_with_logits(R, runner, ids, toks, pos, cfg["vocab"])
            gpu_logits = logits[sel]
        else:
            out, okc = (C.c_uint32 * B)(), (C.c_uint8 * B)()
            assert R["runner_forward_batch"](runner, B, (C.c_uint64 * B)(*ids), (C.c_uint32 * B)(*toks),
                                             (C.c_uint32 * B)(*pos), out, okc)
            got, ok, gpu_logits = list(out), list(okc), None
        assert all(ok), f"step {step}: a lane failed"
        parity.step([toks[i] for i in sel], [pos[i] for i in sel], [got[i] for i in sel], gpu_logits)
        toks, pos = got, [p_ + 1 for p_ in pos]
    rec = parity.record()
    print(config, rec)
    assert rec["logit_rows_compared"] == 2 * len(sel)
    assert rec["max_abs_logit_err"] <= parity.logit_bound(), rec
    assert not parity.mismatches, parity.mismatches
    snap = kk.BackendSnapshot()
    R["backend_snapshot"](backend, C.byref(snap))
    assert snap.committed_token_count == sum(contexts) + STEPS * B
    assert snap.active_transaction_count == 0
    assert R["backend_check_invariants"](backend) == 1
    parity.close()
    R["runner_destroy"](runner)
    R["backend_destroy"](backend)
