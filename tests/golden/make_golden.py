"""Generate the golden fixtures by running the reference's own code.

Run in the build container, where the reference checkout is importable:

    python tests/golden/make_golden.py --reference <path to HeteroCache checkout>

For every scenario in ``scenarios.py`` this imports the reference's
``heterocache.cache_utils.HeteroCache`` unchanged, drives it on CPU with the
seeded inputs, and writes ``<scenario>.json`` next to this file.  The one shim:
with ``real_offload=False`` the reference builds index tensors with
``torch.arange(..., device="cuda")`` (heterocache/cache_utils.py:637, :772);
while a scenario runs, that call is redirected to the CPU.  ``real_offload=False`` keeps the full-KV tier in
memory (pinned host buffers need a driver); its arithmetic equals the
pinned-host branch.

It also pins the observation-window math (W > 1) against the reference's
``SnapKVCluster.update_kv`` (heterocache/kv_cluster.py:138-199): the kept key
rows are matched back to positions and stored as ``snapkv_*.json``.

The reference is not available where the GPU tests run; only these JSON
files travel.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from scenarios import SCENARIOS, _recover, _row_index, make_config, run_scenario  # noqa: E402

SNAPKV_CASES = {
    "snapkv_f32_w32_max7": dict(L=1024, dtype="float32", window=32, k=7, pooling="maxpool", seed=21, cap=400),
    "snapkv_bf16_w32_max7": dict(L=1024, dtype="bfloat16", window=32, k=7, pooling="maxpool", seed=22, cap=400),
    "snapkv_f32_w8_avg5": dict(L=600, dtype="float32", window=8, k=5, pooling="avgpool", seed=23, cap=200),
}


def snapkv_inputs(case):
    g = torch.Generator("cpu").manual_seed(case["seed"])
    H, D, L = 4, 128, case["L"]
    q = torch.randn(1, H, L, D, generator=g)
    k = torch.randn(1, H, L, D, generator=g)
    v = torch.randn(1, H, L, D, generator=g)
    dt = getattr(torch, case["dtype"])
    return q.to(dt), k.to(dt), v.to(dt)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    orig_arange = torch.arange

    def cpu_arange(*a, **k):
        if k.get("device") == "cuda":
            k["device"] = "cpu"
        return orig_arange(*a, **k)

    import heterocache.cache_utils as cu
    from heterocache.kv_cluster import SnapKVCluster

    for name, sc in SCENARIOS.items():
        if args.only and name != args.only:
            continue
        cfg = make_config(sc, cu.HeteroCacheConfig)
        torch.arange = cpu_arange
        try:
            cache = cu.HeteroCache(cfg)
            rec = run_scenario(cache, sc, cfg.data)
        finally:
            torch.arange = orig_arange
        rec["scenario"] = sc
        rec["base_compress_len"] = cache.base_compress_len
        with open(os.path.join(HERE, f"{name}.json"), "w") as f:
            json.dump(rec, f, separators=(",", ":"))
        print(name, "decode steps", len(rec["decode"]), "oom_step", rec["oom_step"])

    for name, case in SNAPKV_CASES.items():
        if args.only and name != args.only:
            continue
        q, k, v = snapkv_inputs(case)
        cl = SnapKVCluster(window_size=case["window"], kernel_size=case["k"], pooling=case["pooling"])
        cl.max_capacity_prompt = case["cap"]
        ck, cv = cl.update_kv(k, q, v, None, 1)
        W = case["window"]
        kept = []
        for h in range(k.shape[1]):
            index = _row_index(k[0, h])
            kept.append(_recover(ck[0, h], 0, case["cap"] - W, index))
        with open(os.path.join(HERE, f"{name}.json"), "w") as f:
            json.dump({"case": case, "kept": kept}, f, separators=(",", ":"))
        print(name, "ok")


if __name__ == "__main__":
    main()
