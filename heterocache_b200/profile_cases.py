"""Small, fixed launches of single kernels for profiler captures.

    python -m heterocache_b200.profile_cases <case> [--reps N]

Each case builds seeded synthetic inputs on ``cuda:0`` and issues ``reps``
launches of one entry point (the first ones warm the launch caches), so that
a profiler can capture one launch of a known shape without running the whole
benchmark:

* ``drift_batch``   -- hc_drift_check_batch: 8 drift checks (one layer's 8 KV
  heads as pivots) at 131072 tokens, Llama-3.1-8B geometry, bf16, one launch;
* ``drift_single``  -- hc_drift_check: one pivot at 131072 tokens;
* ``prefill_attention`` -- hc_prefill_attention: causal, 32 query / 8 KV
  heads, 8192 tokens, bf16;
* ``prefill_select_w32`` -- hc_prefill_select with an observation window of
  32 queries (128 query rows per KV head, the tcgen05 path): 5 compressed KV
  heads of a Llama-3.1-8B layer at 131072 tokens, max-pool 7, keep 0.4 L,
  bf16.
"""
from __future__ import annotations

import argparse
import math

import torch

from . import ops
from .ops import Workspace

L_DRIFT, KV, G, D, S = 131072, 8, 4, 128, 5


def _drift_inputs(dev):
    n = L_DRIFT // 256
    gen = torch.Generator(device=dev).manual_seed(0)
    pool = torch.randn(KV * n, 256, 1, D, device=dev, generator=gen).to(torch.bfloat16)
    bt = torch.arange(KV * n, dtype=torch.int32, device=dev).view(KV, n)
    qb = torch.randn(S, KV * G, D, device=dev, generator=gen).to(torch.bfloat16)
    return pool, bt, qb


def drift_batch(dev, reps):
    pool, bt, qb = _drift_inputs(dev)
    i32 = dict(dtype=torch.int32, device=dev)
    K, ml = 1024 * 4, 8192
    keep = []
    jobs = []
    for h in range(KV):
        o = dict(bm=torch.zeros((L_DRIFT + 31) // 32, **i32), ref=torch.zeros(K, **i32),
                 trig=torch.zeros(1, **i32), rpos=torch.zeros(ml, **i32))
        keep.append(o)
        jobs.append(ops.drift_job(qb, pool, bt, pivot_head=h, max_len=ml, ref_bitmap=o["bm"],
                                  ref_positions=o["ref"], trigger=o["trig"], retrieve_positions=o["rpos"]))
    arr = ops.drift_jobs_array(jobs)
    ws, err = Workspace(dev), torch.zeros(1, **i32)
    for _ in range(reps):
        ops.drift_check_batch(arr, dtype=torch.bfloat16, device=dev, num_kv_heads=KV, groups=G, steps=S,
                              seq_len=L_DRIFT, pooling="avgpool", kernel_size=5, topk=K, threshold=0.5,
                              workspace=ws, err=err)
    torch.cuda.synchronize()
    return int(err.item())


def drift_single(dev, reps):
    pool, bt, qb = _drift_inputs(dev)
    i32 = dict(dtype=torch.int32, device=dev)
    K, ml = 1024 * 4, 8192
    bm = torch.zeros(1, (L_DRIFT + 31) // 32, **i32)
    ref = torch.zeros(1, K, **i32)
    trig, rpos = torch.zeros(1, **i32), torch.zeros(1, ml, **i32)
    ws, err = Workspace(dev), torch.zeros(1, **i32)
    for _ in range(reps):
        ops.drift_check(qb, pool, bt, num_kv_heads=KV, groups=G, steps=S, seq_len=L_DRIFT, pooling="avgpool",
                        kernel_size=5, topk=K, threshold=0.5, pivot_heads=torch.tensor([7], **i32),
                        ref_slots=torch.tensor([0], **i32), max_len=torch.tensor([ml], **i32), max_len_cap=ml,
                        ref_bitmap=bm, ref_positions=ref, trigger=trig, retrieve_positions=rpos, workspace=ws,
                        err=err)
    torch.cuda.synchronize()
    return int(err.item())


def prefill_attention(dev, reps):
    L, H = 8192, KV * G
    gen = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(1, L, H, D, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(1, L, KV, D, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
    v = torch.randn(1, L, KV, D, generator=gen, device=dev).to(torch.bfloat16).transpose(1, 2)
    out = torch.empty(1, L, H, D, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(reps):
        ops.prefill_attention(q, k, v, scale=1.0 / math.sqrt(D), out=out, err=err)
    torch.cuda.synchronize()
    return int(err.item())


def prefill_select_w32(dev, reps):
    L, H, nc = L_DRIFT, KV * G, 5
    gen = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(1, H, 64, D, device=dev, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, KV, L, D, device=dev, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, KV, L, D, device=dev, generator=gen).to(torch.bfloat16)
    keep_len = int(0.4 * L)
    keep = torch.full((nc,), keep_len, dtype=torch.int32, device=dev)
    npg = (keep_len + 255) // 256
    bt = torch.full((KV, L // 256 + 2), -1, dtype=torch.int32)
    for h in range(nc):
        bt[h, :npg] = torch.arange(h * npg, (h + 1) * npg, dtype=torch.int32)
    bt = bt.to(dev)
    kp = torch.zeros(nc * npg, 256, 1, D, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    hl = torch.zeros(KV, dtype=torch.int32, device=dev)
    ws, err = Workspace(dev), torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(reps):
        ops.prefill_select(q, k, v, keep, keep_len, n_heads=nc, groups=G, window=32, pooling="maxpool",
                           kernel_size=7, k_pool=kp, v_pool=vp, block_table=bt, heads_len=hl, workspace=ws, err=err)
    torch.cuda.synchronize()
    return int(err.item())


CASES = {"drift_batch": drift_batch, "drift_single": drift_single, "prefill_attention": prefill_attention,
         "prefill_select_w32": prefill_select_w32}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    err = CASES[a.case](dev, a.reps)
    print(f"{a.case}: {a.reps} launches, err flag {err}")
    if err:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
