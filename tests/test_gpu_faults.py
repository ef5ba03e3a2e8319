"""Failure detection on the GPU, with no GPU fault: every failure is made on
the host (a fake of the failing call) or is a bounded device-side wait made
to run out by an arrival that never comes.

* A drift check whose grid barriers wait for an injected arrival returns
  within its (short) limit, HC_ERR_TIMEOUT reaches the host through the error
  flag, ``check_errors`` raises and zero-fills the workspace, and the next
  check -- with the default limits -- gives exactly what an untouched twin
  cache gives.
* A failed pinned host allocation for the full KV tier raises a clear
  ``RuntimeError`` naming the layer and the size.
"""
import time

import pytest
import torch

from heterocache_b200 import ops
from heterocache_b200.cache import HeteroCache, HeteroCacheConfig
from heterocache_b200.synthetic import DriftingDecode
from scenarios import SCENARIOS, make_config, scenario_inputs

pytestmark = pytest.mark.gpu


def _prefilled(sc, dev, real_offload=False):
    kw = dict(vars(make_config(sc)))
    kw["real_offload"] = real_offload
    cfg = HeteroCacheConfig(**kw)
    cfg.record_checks = True
    cache = HeteroCache(cfg)
    geo, tdt, inputs = scenario_inputs(sc)
    for layer, (q, k, v) in enumerate(inputs):
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        cache.update(kd, vd, layer)
        cache.init_coefficient(qd, kd, layer)
        cache.prefill_select(qd, kd, vd, layer)
    return cache, geo, tdt, inputs


def test_drift_check_timeout_is_reported_and_the_next_check_recovers(cuda_device):
    sc = SCENARIOS["llama_bf16_avg5"]
    dev = cuda_device
    a, geo, tdt, inputs = _prefilled(sc, dev)
    b, _, _, _ = _prefilled(sc, dev)
    gens = [DriftingDecode(geo, seed=5, q0=inputs[0][0][:, :, -1:, :], dtype=tdt) for _ in range(2)]
    S = sc["steps"]
    for step in range(S - 1):  # up to the step before the first check
        for c, g in zip((a, b), gens):
            q, k, v = (t.to(dev) for t in g.step())
            c.update(k, v, 0)
            c.attention(q, 0)
            c.decode_select(q, 0)
    torch.cuda.synchronize()
    qs = []
    for c, g in zip((a, b), gens):
        q, k, v = (t.to(dev) for t in g.step())
        c.update(k, v, 0)
        c.attention(q, 0)
        qs.append(q)
    b.decode_select(qs[1], 0)  # the twin checks normally
    torch.cuda.synchronize()
    ops.set_wait_limits(5_000_000, inject_stall=True)  # 5 ms, and an arrival that never comes
    try:
        t0 = time.perf_counter()
        a.decode_select(qs[0], 0)  # this step's check on `a` stalls at its first grid barrier
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        ops.set_wait_limits(0, inject_stall=False)
    assert elapsed < 1.0, elapsed  # the limit, not the 2 s default, ended the wait
    with pytest.raises(RuntimeError, match="timed out"):
        a.check_errors()
    a.check_errors()  # flag cleared
    # the check again, with the default limits, on the reset workspace
    jobs = a._jobs[0]
    a._drift_and_retrieve(0, jobs, qs[0])
    torch.cuda.synchronize()
    a.check_errors()
    la, lb = a.check_log[-1], b.check_log[-1]
    assert torch.equal(la["trigger"], lb["trigger"])
    assert torch.equal(la["coeffs"], lb["coeffs"])
    assert torch.equal(la["retrieved"], lb["retrieved"])
    assert torch.equal(a.prefill_topk_set[0], b.prefill_topk_set[0])
    assert torch.equal(a.key_pools[0], b.key_pools[0]) and torch.equal(a.value_pools[0], b.value_pools[0])


def test_failed_pinned_allocation_raises_a_clear_error(cuda_device, monkeypatch):
    sc = SCENARIOS["llama_bf16_avg5"]
    real_empty = torch.empty

    def failing_empty(*args, **kwargs):
        if kwargs.get("pin_memory"):
            raise RuntimeError("CUDA error: out of memory (injected)")
        return real_empty(*args, **kwargs)

    import heterocache_b200.cache as cache_mod
    monkeypatch.setattr(cache_mod.torch, "empty", failing_empty)
    with pytest.raises(RuntimeError, match=r"Layer 0: pinned host allocation of \d+ bytes"):
        _prefilled(sc, cuda_device, real_offload=True)
