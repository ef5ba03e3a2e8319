"""hc_drift_check_batch: several pivots' drift checks -- of different layers,
i.e. different query buffers, pools and page tables -- in few launches.

Every job is checked against the oracle exactly as a single drift check is
(per-step overlap within the tie range, trigger, new reference set and
retrieval list from the last step's scores; ``tests/parity.py`` rules), and
with one job per launch the results equal single hc_drift_check launches bit
for bit (the same split of each check over the SMs).
"""
import math

import numpy as np
import pytest
import torch

from heterocache_b200 import ops
from heterocache_b200.ops import Workspace
from heterocache_b200.synthetic import LLAMA_8B, prefill_inputs
from parity import compare_selection, scores_close

pytestmark = pytest.mark.gpu

DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
S = 5


def _layer(geo, L, tdt, seed):
    """One layer: prefill q/k, the pivots' keys in a paged pool (pages of a
    head contiguous, heads in reverse order so page ids are not the head's
    own), and drifting decode queries [S, H, D]."""
    KV, D, H = geo.num_kv_heads, geo.head_dim, geo.num_heads
    q, k, _ = prefill_inputs(geo, L, seed=seed, dtype=tdt)
    n = (L + 255) // 256
    bt = torch.full((KV, n + 1), -1, dtype=torch.int32)
    kp = torch.zeros(KV * n, 256, 1, D, dtype=tdt)
    for h in range(KV):
        first = (KV - 1 - h) * n
        bt[h, :n] = torch.arange(first, first + n, dtype=torch.int32)
        kp.view(-1, D)[first * 256:first * 256 + L] = k[0, h]
    g = torch.Generator().manual_seed(seed + 1)
    qb = torch.empty(S, H, D)
    cur = q[0, :, -1, :].float()
    for s in range(S):
        cur = 0.6 * cur + 0.4 * torch.randn(H, D, generator=g)
        qb[s] = cur
    return q, k, kp, bt, qb.to(tdt)


def _oracle(geo, q, k, qb, pivot, K):
    """Pooled scores [S, L] of the buffered queries (heterocache/cache_utils.py:
    1033-1061) and a reference set from the prefill's last query."""
    G, D = geo.groups, geo.head_dim
    keys = k[:, pivot:pivot + 1]
    q_sub = qb.transpose(0, 1).unsqueeze(0)[:, pivot * G:(pivot + 1) * G]  # [1, G, S, D]
    logits = torch.matmul(q_sub, keys.transpose(-1, -2)) / math.sqrt(D)
    p = torch.softmax(logits, dim=-1, dtype=torch.float32).to(q.dtype)
    shp = p.shape
    p = torch.nn.functional.avg_pool1d(p.reshape(-1, shp[-1]).unsqueeze(1), 5, 1, 2).squeeze(1).view(shp)
    scores = p.max(dim=1).values[0]
    pre = q[0, pivot * G, -1].float() @ k[0, pivot].float().T
    ref_set = pre.topk(K).indices.sort().values
    return scores, ref_set


def _overlap_range(sc, ref_mask, K):
    x = sc.double()
    t = x.topk(K).values[-1]
    above, tie = x > t, x == t
    need = K - int(above.sum())
    base = int((above & ref_mask).sum())
    tie_in = int((tie & ref_mask).sum())
    tie_out = int(tie.sum()) - tie_in
    return base + max(0, need - tie_out), base + min(need, tie_in)


@pytest.mark.parametrize("dtype,per_launch", [("bfloat16", 0), ("bfloat16", 2), ("bfloat16", 1),
                                              ("float16", 0), ("float32", 3)])
def test_drift_batch_matches_oracle(cuda_device, dtype, per_launch):
    dev, geo, tdt = cuda_device, LLAMA_8B, DT[dtype]
    G, KV, D, H = geo.groups, geo.num_kv_heads, geo.head_dim, geo.num_heads
    L = 4096
    K = int(0.2 * L)
    words = (L + 31) // 32
    layers = [_layer(geo, L, tdt, seed) for seed in (31, 57)]
    # (layer, pivot, retrieval length): five checks over two layers
    spec = [(0, 1, 600), (0, 6, 819), (1, 3, 400), (1, 0, 1024), (0, 2, 1)]
    i32 = dict(dtype=torch.int32, device=dev)
    dev_layers = [(qb.to(dev), kp.to(dev), bt.to(dev)) for (_, _, kp, bt, qb) in layers]
    jobs, outs, exp = [], [], []
    for li, pivot, ml in spec:
        q, k, _, _, qb = layers[li]
        scores, ref_set = _oracle(geo, q, k, qb, pivot, K)
        bm = torch.zeros(words, dtype=torch.int32)
        for t in ref_set.tolist():
            bm[t // 32] |= (1 << (t % 32)) if (t % 32) < 31 else -(1 << 31)
        o = {"bm": bm.to(dev), "ref": ref_set.to(torch.int32).to(dev), "trig": torch.zeros(1, **i32),
             "rpos": torch.full((ml,), -1, **i32), "coeffs": torch.zeros(S, dtype=torch.float32, device=dev),
             "med": torch.zeros(1, dtype=torch.float64, device=dev),
             "sc": torch.zeros(S, L, dtype=tdt, device=dev)}
        init = {n: t.clone() for n, t in o.items()}
        qbd, kpd, btd = dev_layers[li]
        jobs.append(ops.drift_job(qbd, kpd, btd, pivot_head=pivot, max_len=ml, ref_bitmap=o["bm"],
                                  ref_positions=o["ref"], trigger=o["trig"], retrieve_positions=o["rpos"],
                                  coeffs=o["coeffs"], median=o["med"], out_scores=o["sc"]))
        outs.append(o)
        ref_mask = torch.zeros(L, dtype=torch.bool)
        ref_mask[ref_set] = True
        exp.append((scores, [_overlap_range(scores[s], ref_mask, K) for s in range(S)], init))
    err = torch.zeros(1, **i32)
    ops.drift_check_batch(ops.drift_jobs_array(jobs), dtype=tdt, device=dev, num_kv_heads=KV, groups=G, steps=S,
                          seq_len=L, pooling="avgpool", kernel_size=5, topk=K, threshold=0.999,
                          workspace=Workspace(dev), err=err, jobs_per_launch=per_launch)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for (li, pivot, ml), o, (scores, ranges, init) in zip(spec, outs, exp):
        dsc = o["sc"].float().cpu()
        counts = (o["coeffs"].cpu().double() * K).round().long().tolist()
        for s in range(S):
            res = compare_selection(scores[s].float().numpy(), dsc[s].numpy(), [], K, dtype, scores_only=True)
            assert scores_close(res, dtype), (li, pivot, res)
            lo, hi = ranges[s]
            slack = res["flips"] if dtype != "float32" else res["flips"] + res["boundary"]
            assert lo - slack <= counts[s] <= hi + slack, (li, pivot, s, counts[s], ranges[s])
        c = sorted(o["coeffs"].cpu().tolist())
        assert o["med"].item() == pytest.approx(c[S // 2], abs=0.0)
        assert int(o["trig"].item()) == 1
        new_ref = o["ref"].cpu().tolist()
        assert new_ref == sorted(new_ref) and len(set(new_ref)) == K
        res = compare_selection(scores[-1].float().numpy(), dsc[-1].numpy(), new_ref, K, dtype)
        assert res["ok"], res
        bits = o["bm"].cpu().numpy().view(np.uint32)
        assert [w * 32 + b for w in range(words) for b in range(32) if (int(bits[w]) >> b) & 1] == new_ref
        rl = o["rpos"].cpu().tolist()
        assert rl == sorted(rl) and len(set(rl)) == ml
        res = compare_selection(scores[-1].float().numpy(), dsc[-1].numpy(), rl, ml, dtype)
        assert res["ok"], res

    if per_launch != 1:
        return
    # one job per launch: each check split over the SMs as a single launch
    # splits it, so the single entry point gives the same bits
    for (li, pivot, ml), o, (_, _, init) in zip(spec, outs, exp):
        qbd, kpd, btd = dev_layers[li]
        one = {n: t.clone() for n, t in init.items()}
        ops.drift_check(qbd, kpd, btd, num_kv_heads=KV, groups=G, steps=S, seq_len=L, pooling="avgpool",
                        kernel_size=5, topk=K, threshold=0.999, pivot_heads=torch.tensor([pivot], **i32),
                        ref_slots=torch.tensor([0], **i32), max_len=torch.tensor([ml], **i32), max_len_cap=ml,
                        ref_bitmap=one["bm"].view(1, words), ref_positions=one["ref"].view(1, K),
                        trigger=one["trig"], retrieve_positions=one["rpos"].view(1, ml), workspace=Workspace(dev),
                        err=err, coeffs=one["coeffs"].view(1, S), median=one["med"], out_scores=one["sc"].view(1, S, L))
        torch.cuda.synchronize()
        for n in o:
            assert torch.equal(o[n], one[n]), (li, pivot, n)


def test_drift_batch_leaves_other_layers_alone(cuda_device):
    """A batch writes only its jobs' rows: a second reference slot of the same
    bitmap tensor, not named by any job, keeps its bits."""
    dev, geo, tdt = cuda_device, LLAMA_8B, torch.bfloat16
    G, KV = geo.groups, geo.num_kv_heads
    L, K = 2048, 300
    q, k, kp, bt, qb = _layer(geo, L, tdt, 5)
    words = L // 32
    i32 = dict(dtype=torch.int32, device=dev)
    bm = torch.randint(-2**31, 2**31 - 1, (2, words), dtype=torch.int32, device=dev)
    ref = torch.randint(0, L, (2, K), dtype=torch.int32, device=dev)
    keep_bm, keep_ref = bm[1].clone(), ref[1].clone()
    trig = torch.zeros(1, **i32)
    rpos = torch.zeros(16, **i32)
    job = ops.drift_job(qb.to(dev), kp.to(dev), bt.to(dev), pivot_head=4, max_len=16, ref_bitmap=bm[0],
                        ref_positions=ref[0], trigger=trig, retrieve_positions=rpos)
    err = torch.zeros(1, **i32)
    ops.drift_check_batch(ops.drift_jobs_array([job]), dtype=tdt, device=dev, num_kv_heads=KV, groups=G, steps=S,
                          seq_len=L, pooling="maxpool", kernel_size=7, topk=K, threshold=1.5,
                          workspace=Workspace(dev), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(trig.item()) == 1
    assert torch.equal(bm[1], keep_bm) and torch.equal(ref[1], keep_ref)
    assert int(bm[0].cpu().numpy().view(np.uint32).astype(np.uint64).sum()) > 0
