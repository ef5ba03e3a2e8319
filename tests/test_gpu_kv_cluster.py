"""The ``SnapKVCluster`` drop-in (heterocache/kv_cluster.py:138-199) on the GPU.

* Against the committed goldens (``tests/golden/snapkv_*.json``: positions
  kept by the unmodified reference on seeded inputs): the kept set must be
  the reference's, except at ties with the k-th score (the reference's
  ``torch.topk`` order among equal values is unspecified), and the returned
  rows must be the input rows at those positions followed by the window.
* Against the oracle at larger sizes (bf16 and fp32, avg and max pooling).
* The reference's capacity rule and early return.
"""
import json
import os

import numpy as np
import pytest
import torch

from heterocache_b200.kv_cluster import SnapKVCluster
from oracle.hc_oracle import snapkv_scores
from parity import compare_selection, scores_close

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _check(q, k, v, *, window, ks, pooling, cap, dtype, gold_kept=None):
    dev = torch.device("cuda", 0)
    cl = SnapKVCluster(window_size=window, kernel_size=ks, pooling=pooling)
    cl.max_capacity_prompt = cap
    cl.record_scores = True
    ko, vo = cl.update_kv(k.to(dev), q.to(dev), v.to(dev), None, 1)
    torch.cuda.synchronize()
    cl.check_errors()
    bsz, H, L, D = k.shape
    assert tuple(ko.shape) == (bsz, H, cap, D) and tuple(vo.shape) == (bsz, H, cap, D)
    ref = snapkv_scores(q, k, window=window, kernel_size=ks, pooling=pooling)  # [bsz, H, L - W]
    idx = cl.last_indices.cpu()
    dsc = cl.last_scores.float().cpu()[..., :L - window]
    ko, vo = ko.cpu(), vo.cpu()
    keep = cap - window
    for b in range(bsz):
        for h in range(H):
            sel = idx[b, h].tolist()
            assert sel == sorted(sel) and len(set(sel)) == keep
            assert all(0 <= t < L - window for t in sel)
            r = ref[b, h].double().numpy()
            res = compare_selection(r, dsc[b, h].numpy(), sel, keep, dtype)
            assert res["ok"], (b, h, res)
            assert scores_close(res, dtype, terms=window), {k: res[k] for k in ("flips", "L", "max_rel")}
            if gold_kept is not None:
                # the reference's own set, except positions tied with its k-th
                # score or whose device score differs from the oracle's
                assert len(gold_kept[h]) == keep
                t_ref = np.partition(r, r.size - keep)[r.size - keep] if keep else np.inf
                d = dsc[b, h].double().numpy()
                for t in set(sel) ^ set(gold_kept[h]):
                    tied = abs(r[t] - t_ref) <= 1e-6 * abs(t_ref)
                    flipped = d[t] != r[t]
                    assert tied or flipped, (h, t, r[t], t_ref)
            assert torch.equal(ko[b, h, :keep], k[b, h, sel])
            assert torch.equal(vo[b, h, :keep], v[b, h, sel])
            assert torch.equal(ko[b, h, keep:], k[b, h, L - window:])
            assert torch.equal(vo[b, h, keep:], v[b, h, L - window:])


@pytest.mark.parametrize("name", ["snapkv_f32_w32_max7", "snapkv_bf16_w32_max7", "snapkv_f32_w8_avg5"])
def test_snapkv_matches_reference_goldens(cuda_device, name):
    from make_golden import snapkv_inputs
    gold = json.load(open(os.path.join(GOLDEN, f"{name}.json")))
    case = gold["case"]
    q, k, v = snapkv_inputs(case)
    _check(q, k, v, window=case["window"], ks=case["k"], pooling=case["pooling"], cap=case["cap"],
           dtype=case["dtype"], gold_kept=gold["kept"])


@pytest.mark.parametrize("dtype,L,H,window,ks,pooling,cap", [
    ("bfloat16", 8192, 8, 32, 7, "maxpool", 2048),
    ("bfloat16", 6000, 4, 64, 5, "avgpool", 3000),
    ("float32", 4096, 4, 32, 7, "maxpool", 1500),
    ("float16", 3000, 2, 16, 5, "avgpool", 16),  # keeps only the window
])
def test_snapkv_matches_oracle(cuda_device, dtype, L, H, window, ks, pooling, cap):
    tdt = getattr(torch, dtype)
    g = torch.Generator().manual_seed(L + window)
    q = torch.randn(2, H, L, 128, generator=g).to(tdt)
    k = torch.randn(2, H, L, 128, generator=g)
    # planted heavy hitters: 1% of positions aligned with the window queries
    hot = torch.randperm(L - window, generator=g)[: max(1, L // 100)]
    k[:, :, hot] += 4 * torch.nn.functional.normalize(q[:, :, -window:].float().mean(2), dim=-1)[:, :, None]
    k = k.to(tdt)
    v = torch.randn(2, H, L, 128, generator=g).to(tdt)
    _check(q, k, v, window=window, ks=ks, pooling=pooling, cap=cap, dtype=dtype)


def test_snapkv_capacity_rule_and_short_prompts(cuda_device):
    dev = cuda_device
    q = torch.randn(1, 4, 100, 128, device=dev).to(torch.bfloat16)
    k = torch.randn(1, 4, 100, 128, device=dev).to(torch.bfloat16)
    v = torch.randn(1, 4, 100, 128, device=dev).to(torch.bfloat16)
    cl = SnapKVCluster(window_size=8, compression_ratio=0.5)
    ko, vo = cl.update_kv(k, q, v, None, 2)  # capacity int(0.5 * 100 / 2) = 25
    assert cl.max_capacity_prompt == 25 and ko.shape[2] == 25
    cl2 = SnapKVCluster(window_size=8)
    cl2.max_capacity_prompt = 101  # longer than the prompt: returned unchanged
    ko2, vo2 = cl2.update_kv(k, q, v, None, 1)
    assert ko2 is k and vo2 is v
    with pytest.raises(RuntimeError, match="own key head"):
        SnapKVCluster(window_size=8).update_kv(k[:, :2], q, v[:, :2], None, 2)
