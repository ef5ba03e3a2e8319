"""Failure detection on the GPU, with no GPU fault: every failure is made on
the host (a fake of the failing call) or is a bounded device-side wait made
to run out by an arrival that never comes.

* A drift check whose grid barriers wait for an injected arrival returns
  within its (short) limit, HC_ERR_TIMEOUT reaches the host through the error
  flag, ``check_errors`` raises and zero-fills the workspace, and the next
  check -- with the default limits -- gives exactly what an untouched twin
  cache gives.
* The same for a batch of drift checks (``hc_drift_check_batch``) and for
  the prefill attention (whose injected stall loads no key tile, so its
  mbarrier waits run out): the flag reaches the host, and the next launch
  gives the untouched result.
* A failed pinned host allocation for the full KV tier raises a clear
  ``RuntimeError`` naming the layer and the size.
"""
import time

import pytest
import torch

from heterocache_b200 import ops
from heterocache_b200.ops import Workspace
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


TIMEOUT_BIT = 1 << 7  # HC_ERR_TIMEOUT in the error flag


def test_drift_batch_timeout_is_reported_and_the_next_batch_recovers(cuda_device):
    """Two checks in one batch launch stall at their first grid barrier; the
    batch run again with the default limits on a zeroed workspace gives what
    a batch that never stalled gives."""
    from test_gpu_drift_batch import S, _layer
    from heterocache_b200.synthetic import LLAMA_8B
    dev, geo, tdt = cuda_device, LLAMA_8B, torch.bfloat16
    L, K, ml = 2048, 300, 64
    _, _, kp, bt, qb = _layer(geo, L, tdt, 3)
    qb, kp, bt = qb.to(dev), kp.to(dev), bt.to(dev)
    i32 = dict(dtype=torch.int32, device=dev)

    def outputs():
        return [dict(bm=torch.zeros(L // 32, **i32), ref=torch.arange(K, **i32), trig=torch.zeros(1, **i32),
                     rpos=torch.zeros(ml, **i32)) for _ in range(2)]

    def run(outs, ws, err):
        jobs = [ops.drift_job(qb, kp, bt, pivot_head=h, max_len=ml, ref_bitmap=o["bm"], ref_positions=o["ref"],
                              trigger=o["trig"], retrieve_positions=o["rpos"]) for h, o in zip((2, 5), outs)]
        ops.drift_check_batch(ops.drift_jobs_array(jobs), dtype=tdt, device=dev, num_kv_heads=geo.num_kv_heads,
                              groups=geo.groups, steps=S, seq_len=L, pooling="avgpool", kernel_size=5, topk=K,
                              threshold=0.9, workspace=ws, err=err)

    ref_outs, ws0, err0 = outputs(), Workspace(dev), torch.zeros(1, **i32)
    run(ref_outs, ws0, err0)
    outs, ws, err = outputs(), Workspace(dev), torch.zeros(1, **i32)
    ops.set_wait_limits(5_000_000, inject_stall=True)
    try:
        t0 = time.perf_counter()
        run(outs, ws, err)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        ops.set_wait_limits(0, inject_stall=False)
    assert elapsed < 1.0, elapsed
    assert int(err.item()) & TIMEOUT_BIT
    err.zero_()
    ws.reset()
    outs = outputs()
    run(outs, ws, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(err0.item()) == 0
    for o, r in zip(outs, ref_outs):
        for name in o:
            assert torch.equal(o[name], r[name]), name


def test_prefill_attention_timeout_is_reported_and_the_next_launch_recovers(cuda_device):
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(2)
    q = torch.randn(1, 8, 700, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, 2, 700, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, 2, 700, 128, generator=g, device=dev).to(torch.bfloat16)
    good = ops.prefill_attention(q, k, v)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.set_wait_limits(5_000_000, inject_stall=True)
    try:
        t0 = time.perf_counter()
        ops.prefill_attention(q, k, v, err=err)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        ops.set_wait_limits(0, inject_stall=False)
    assert elapsed < 1.0, elapsed
    assert int(err.item()) & TIMEOUT_BIT
    err.zero_()
    again = ops.prefill_attention(q, k, v, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(again, good)


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
