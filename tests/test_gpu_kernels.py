"""Kernel-level parity: each C-ABI entry point against the CPU oracle.

Inputs are the seeded synthetic tensors (generated on the CPU, copied to the
device), so both sides see identical bits.  Tolerances:
  * selections: ``tests/parity.py`` (agreement wherever oracle scores are
    separated by more than 1e-6 relative; device-score flips counted and
    bounded below);
  * attention outputs: 2e-2 max-abs for bf16/fp16, 1e-5 for fp32.
"""
import math

import numpy as np
import pytest
import torch

from heterocache_b200 import ops
from heterocache_b200.ops import Workspace
from heterocache_b200.synthetic import LLAMA_8B, QWEN_7B, LayerGeometry, prefill_inputs
from oracle.hc_oracle import paged_attention, window_scores
from parity import compare_selection, scores_close

pytestmark = pytest.mark.gpu

DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
ATOL = {"float32": 1e-5, "bfloat16": 2e-2, "float16": 2e-2}


def _contiguous_pages(lengths, bsz, KV, max_blocks):
    """Per-row contiguous prefill pages (the reference layout)."""
    bt = torch.full((bsz * KV, max_blocks), -1, dtype=torch.int32)
    ptr = 0
    for r in range(bsz * KV):
        n = (int(lengths[r % KV]) + 255) // 256
        if n:
            bt[r, :n] = torch.arange(ptr, ptr + n, dtype=torch.int32)
            ptr += n
    return bt, ptr


@pytest.mark.parametrize("dtype,L,pooling,ks,window,geo", [
    ("bfloat16", 2048, "avgpool", 5, 1, LLAMA_8B),
    ("float16", 2048, "avgpool", 5, 1, LLAMA_8B),
    ("float32", 2048, "avgpool", 5, 1, LLAMA_8B),
    ("bfloat16", 1000, "maxpool", 7, 1, LLAMA_8B),
    ("float32", 8192, "maxpool", 7, 32, LLAMA_8B),
    ("bfloat16", 4096, "maxpool", 7, 32, LLAMA_8B),
    ("bfloat16", 1536, "avgpool", 5, 1, QWEN_7B),
    ("bfloat16", 32768, "avgpool", 5, 1, LLAMA_8B),
    # GQA group sizes 1, 2 and 8 (the pooling's group max over 1, 2 and 8 lanes)
    ("bfloat16", 2048, "avgpool", 5, 1, LayerGeometry(8, 8, 128)),
    ("float16", 2500, "avgpool", 5, 1, LayerGeometry(16, 8, 128)),
    ("bfloat16", 2048, "maxpool", 7, 1, LayerGeometry(64, 8, 128)),
    # observation window of 32 (128 query rows per KV head) at long context
    ("bfloat16", 131072, "maxpool", 7, 32, LLAMA_8B),
    ("float16", 20000, "avgpool", 5, 32, QWEN_7B),
])
def test_prefill_select_matches_oracle(cuda_device, dtype, L, pooling, ks, window, geo):
    tdt = DT[dtype]
    G, KV, D = geo.groups, geo.num_kv_heads, geo.head_dim
    q, k, v = prefill_inputs(geo, L, seed=L + window, window=window, dtype=tdt)
    nc = max(1, KV - 3)
    keep = [max(1, int(L * f)) for f in np.linspace(0.05, 0.45, nc)]
    keep[0] = min(L, 256)  # exactly one page
    ref = window_scores(q[:, :nc * G, L - window:, :], k[:, :nc], groups=G, pooling=pooling, kernel_size=ks)
    max_blocks = (L + 255) // 256 + 2
    bt, nb = _contiguous_pages(keep + [0] * (KV - nc), 1, KV, max_blocks)
    dev = cuda_device
    kp = torch.zeros(nb, 256, 1, D, dtype=tdt, device=dev)
    vp = torch.zeros_like(kp)
    hl = torch.zeros(KV, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out_idx = torch.full((1, nc, max(keep)), -7, dtype=torch.int32, device=dev)
    out_sc = torch.zeros(1, nc, L, dtype=tdt, device=dev)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    ops.prefill_select(qd, kd, vd, torch.tensor(keep, dtype=torch.int32, device=dev), max(keep), n_heads=nc,
                       groups=G, window=window, pooling=pooling, kernel_size=ks, k_pool=kp, v_pool=vp,
                       block_table=bt.to(dev), heads_len=hl, workspace=Workspace(dev), err=err,
                       out_indices=out_idx, out_scores=out_sc)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert hl[:nc].tolist() == keep
    idx = out_idx.cpu()
    dsc = out_sc.float().cpu()
    kflat, vflat = kp.cpu().view(-1, D), vp.cpu().view(-1, D)
    for h in range(nc):
        sel = idx[0, h, :keep[h]].tolist()
        assert sel == sorted(sel) and len(set(sel)) == keep[h]
        assert idx[0, h, keep[h]:].eq(-1).all()
        res = compare_selection(ref[0, h].float().numpy(), dsc[0, h].numpy(), sel, keep[h], dtype)
        assert res["ok"], res
        assert scores_close(res, dtype, terms=window), {k: res[k] for k in ("flips", "L", "max_rel")}
        start = int(bt[h, 0]) * 256
        assert torch.equal(kflat[start:start + keep[h]], k[0, h, sel]), h
        assert torch.equal(vflat[start:start + keep[h]], v[0, h, sel]), h


@pytest.mark.parametrize("dtype,L,pooling,ks", [("bfloat16", 4096, "avgpool", 5), ("float32", 3000, "maxpool", 7)])
def test_pivot_init_matches_oracle(cuda_device, dtype, L, pooling, ks):
    tdt = DT[dtype]
    geo = LLAMA_8B
    G, KV = geo.groups, geo.num_kv_heads
    q, k, _ = prefill_inputs(geo, L, seed=5, dtype=tdt)
    first, npiv = 6, 2
    K = int(0.2 * L)
    ref = window_scores(q[:, first * G:(first + npiv) * G, -1:, :], k[:, first:first + npiv], groups=G,
                        pooling=pooling, kernel_size=ks)
    dev = cuda_device
    pos = torch.full((1, npiv, K), -1, dtype=torch.int32, device=dev)
    words = (L + 31) // 32
    bm = torch.zeros(1, npiv, words, dtype=torch.int32, device=dev)
    sc = torch.zeros(1, npiv, L, dtype=tdt, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.pivot_init(q.to(dev), k.to(dev), first_pivot=first, n_pivots=npiv, groups=G, pooling=pooling,
                   kernel_size=ks, topk=K, ref_positions=pos, ref_bitmap=bm, workspace=Workspace(dev), err=err,
                   out_scores=sc)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for i in range(npiv):
        sel = pos[0, i].cpu().tolist()
        assert sel == sorted(sel) and len(set(sel)) == K
        bits = bm[0, i].cpu().numpy().view(np.uint32)
        from_bits = [w * 32 + b for w in range(words) for b in range(32) if (int(bits[w]) >> b) & 1]
        assert from_bits == sel
        res = compare_selection(ref[0, i].float().numpy(), sc[0, i].float().cpu().numpy(), sel, K, dtype)
        assert res["ok"], res


def _random_paged(lengths, G_geo: LayerGeometry, tdt, dev, seed):
    KV, D = G_geo.num_kv_heads, G_geo.head_dim
    bsz = len(lengths) // KV
    g = torch.Generator().manual_seed(seed)
    max_blocks = max((l + 255) // 256 for l in lengths) + 1
    nb = sum((l + 255) // 256 for l in lengths) + 3
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    bt = torch.full((len(lengths), max_blocks), -1, dtype=torch.int32)
    ptr = 0
    for r, l in enumerate(lengths):
        n = (l + 255) // 256
        bt[r, :n] = perm[ptr:ptr + n]
        ptr += n
    kp = torch.randn(nb, 256, 1, D, generator=g).to(tdt)
    vp = torch.randn(nb, 256, 1, D, generator=g).to(tdt)
    q = torch.randn(bsz, G_geo.num_heads, 1, D, generator=g).to(tdt)
    return q, kp, vp, bt, torch.tensor(lengths, dtype=torch.int32)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("geo", [LLAMA_8B, QWEN_7B], ids=["llama", "qwen"])
def test_flash_decode_matches_oracle(cuda_device, dtype, geo):
    tdt = DT[dtype]
    KV = geo.num_kv_heads
    lens = [0, 1, 15, 16, 17, 255, 256, 257, 4099, 30000, 777, 12][: 2 * KV]
    lens += [513] * (2 * KV - len(lens))
    q, kp, vp, bt, hl = _random_paged(lens, geo, tdt, cuda_device, seed=3)
    dev = cuda_device
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.flash_decode(q.to(dev), kp.to(dev), vp.to(dev), bt.to(dev), hl.to(dev), num_kv_heads=KV,
                           workspace=Workspace(dev), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = paged_attention(q, kp, vp, bt, hl, KV)
    diff = (out.float().cpu() - ref).abs().max().item()
    assert diff <= ATOL[dtype], diff
    # a row with no tokens gives zeros
    assert out.view(2, KV, -1)[0, 0].float().abs().max().item() == 0.0


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_flash_decode_with_new_token_and_query_stage(cuda_device, dtype):
    """The step's token merged from k_new/v_new (not in the pages) equals the
    oracle over the pages with that token appended; q_stage receives the
    query rows bit for bit."""
    geo = LLAMA_8B
    KV, H, D = geo.num_kv_heads, geo.num_heads, geo.head_dim
    tdt = DT[dtype]
    dev = cuda_device
    lens = [0, 1, 255, 256, 4099, 30000, 777, 12]
    q, kp, vp, bt, hl = _random_paged(lens, geo, tdt, dev, seed=11)
    g = torch.Generator().manual_seed(12)
    kn = torch.randn(1, KV, 1, D, generator=g).to(tdt)
    vn = torch.randn(1, KV, 1, D, generator=g).to(tdt)
    stage = torch.zeros(H, D, dtype=tdt, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.flash_decode(q.to(dev), kp.to(dev), vp.to(dev), bt.to(dev), hl.to(dev), num_kv_heads=KV,
                           workspace=Workspace(dev), err=err, k_new=kn.to(dev), v_new=vn.to(dev), q_stage=stage)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(stage.cpu(), q[0, :, 0, :])
    # oracle: the token written after each row's last page token (a fresh page
    # where the row's pages are full)
    n_extra = sum(1 for l in lens if l % 256 == 0)
    kp2 = torch.cat([kp, torch.zeros(n_extra, *kp.shape[1:], dtype=tdt)])
    vp2 = torch.cat([vp, torch.zeros(n_extra, *vp.shape[1:], dtype=tdt)])
    bt2 = torch.cat([bt, torch.full((bt.shape[0], 1), -1, dtype=torch.int32)], dim=1)
    nxt = kp.shape[0]
    for r, l in enumerate(lens):
        page, off = l // 256, l % 256
        if off == 0:
            bt2[r, page] = nxt
            nxt += 1
        blk = int(bt2[r, page])
        kp2[blk, off, 0] = kn[0, r, 0]
        vp2[blk, off, 0] = vn[0, r, 0]
    ref = paged_attention(q, kp2, vp2, bt2, hl + 1, KV)
    diff = (out.float().cpu() - ref).abs().max().item()
    assert diff <= ATOL[dtype], diff


def test_flash_decode_strided_query(cuda_device):
    """Queries as the attention layer produces them: a transposed projection view."""
    geo = LLAMA_8B
    dev = cuda_device
    lens = [300, 5000, 17, 1024, 2048, 999, 1, 4096]
    q, kp, vp, bt, hl = _random_paged(lens, geo, torch.bfloat16, dev, seed=9)
    qs = q.view(1, 1, geo.num_heads, geo.head_dim).transpose(1, 2).to(dev)  # [1, H, 1, D] non-contiguous
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.flash_decode(qs, kp.to(dev), vp.to(dev), bt.to(dev), hl.to(dev), num_kv_heads=8,
                           workspace=Workspace(dev), err=err)
    ref = paged_attention(q, kp, vp, bt, hl, 8)
    assert (out.float().cpu() - ref).abs().max().item() <= 2e-2


@pytest.mark.parametrize("bsz", [1, 5])
def test_decode_append_allocates_in_row_order(cuda_device, bsz):
    """Up to 32 rows take the one-warp bookkeeping path, more the block-scan path."""
    dev = cuda_device
    KV, D = 8, 128
    # rows 1,3,5 (of each batch entry) sit at a page boundary with the next page unmapped
    lens = [10, 256, 300, 512, 0, 256, 7, 100] * bsz
    R = KV * bsz
    max_blocks = 4
    bt = torch.full((R, max_blocks), -1, dtype=torch.int32)
    ptr = 0
    for r, l in enumerate(lens):
        n = max(1, (l + 255) // 256) if l % 256 else l // 256
        bt[r, :n] = torch.arange(ptr, ptr + n, dtype=torch.int32)
        ptr += n
    n_free = 6 * bsz
    free = torch.arange(ptr, ptr + n_free, dtype=torch.int32)
    nb = ptr + n_free
    kp = torch.zeros(nb, 256, 1, D, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    k = torch.randn(bsz, KV, 1, D).to(torch.bfloat16)
    v = torch.randn(bsz, KV, 1, D).to(torch.bfloat16)
    btd, hld = bt.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev)
    fp = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.decode_append(k.to(dev), v.to(dev), kp, vp, btd, hld, free.to(dev), fp, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    need = [r for r, l in enumerate(lens) if bt[r, l // 256] == -1]
    exp_bt = bt.clone()
    for i, r in enumerate(need):
        exp_bt[r, lens[r] // 256] = int(free[i])
    assert torch.equal(btd.cpu(), exp_bt)
    assert hld.cpu().tolist() == [l + 1 for l in lens]
    assert int(fp.item()) == len(need)
    for r, l in enumerate(lens):
        slot = int(exp_bt[r, l // 256]) * 256 + l % 256
        assert torch.equal(kp.cpu().view(-1, D)[slot], k[r // KV, r % KV, 0])
        assert torch.equal(vp.cpu().view(-1, D)[slot], v[r // KV, r % KV, 0])
    # exhaust the free list: nothing changes, OOM flag set
    fp.fill_(n_free)
    before = (btd.clone(), hld.clone())
    hld.copy_(torch.tensor([256 * 2] * R, dtype=torch.int32))
    ops.decode_append(k.to(dev), v.to(dev), kp, vp, btd, hld, free.to(dev), fp, err)
    torch.cuda.synchronize()
    assert int(err.item()) & (1 << 3)
    assert hld.cpu().tolist() == [512] * R
    assert torch.equal(btd, before[0])


def test_decode_append_stages_the_query(cuda_device):
    """With q / q_stage the append launch also stores the step's query rows."""
    dev = cuda_device
    KV, H, D = 8, 32, 128
    bt = torch.arange(KV, dtype=torch.int32, device=dev).view(KV, 1)
    kp = torch.zeros(KV, 256, 1, D, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    hl = torch.full((KV,), 3, dtype=torch.int32, device=dev)
    fp = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    k = torch.randn(1, KV, 1, D, device=dev).to(torch.bfloat16)
    v = torch.randn(1, KV, 1, D, device=dev).to(torch.bfloat16)
    # a transposed view, as the attention modules hand it over: head stride D
    q = torch.randn(1, 1, H, D, device=dev).to(torch.bfloat16).transpose(1, 2)
    qbuf = torch.zeros(5, H, D, dtype=torch.bfloat16, device=dev)
    ops.decode_append(k, v, kp, vp, bt, hl, torch.zeros(1, dtype=torch.int32, device=dev), fp, err,
                      q=q, q_stage=qbuf[2])
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(qbuf[2], q[0, :, 0, :])
    assert not qbuf[[0, 1, 3, 4]].any()
    assert torch.equal(kp[:, 3, 0], k[0, :, 0]) and hl.tolist() == [4] * KV


@pytest.mark.parametrize("dtype,geo,L", [("bfloat16", LLAMA_8B, 8192), ("bfloat16", QWEN_7B, 3000),
                                         ("float32", LLAMA_8B, 2048),
                                         # 5 and 10 query rows; 40 rows (G = 8, the largest
                                         # tensor-core case, query fragments in shared memory)
                                         ("bfloat16", LayerGeometry(8, 8, 128), 4096),
                                         ("float16", LayerGeometry(16, 8, 128), 3000),
                                         ("bfloat16", LayerGeometry(64, 8, 128), 5000)])
def test_drift_check_matches_oracle(cuda_device, dtype, geo, L):
    """Scoring of S buffered queries over a pivot's pages, overlap, median, trigger."""
    tdt = DT[dtype]
    dev = cuda_device
    G, KV, D, H = geo.groups, geo.num_kv_heads, geo.head_dim, geo.num_heads
    S = 5
    q, k, v = prefill_inputs(geo, L, seed=21, dtype=tdt)
    pivot = KV - 1
    K = int(0.2 * L)
    # pivot pages: contiguous keep-head layout
    n = (L + 255) // 256
    max_blocks = n + 2
    bt = torch.full((KV, max_blocks), -1, dtype=torch.int32)
    bt[pivot, :n] = torch.arange(n, dtype=torch.int32)
    kp = torch.zeros(n, 256, 1, D, dtype=tdt)
    kp.view(-1, D)[:L] = k[0, pivot]
    # reference set from the prefill scores, decode queries drifting away
    pre = window_scores(q[:, pivot * G:(pivot + 1) * G, -1:, :], k[:, pivot:pivot + 1], groups=G,
                        pooling="avgpool", kernel_size=5)[0, 0]
    ref_set = pre.float().topk(K).indices.sort().values
    g = torch.Generator().manual_seed(4)
    qb = torch.empty(S, H, D)
    cur = q[0, :, -1, :].float()
    for s in range(S):
        cur = 0.6 * cur + 0.4 * torch.randn(H, D, generator=g)
        qb[s] = cur
    qb = qb.to(tdt)
    # oracle (heterocache/cache_utils.py:1033-1078)
    keys = k[:, pivot:pivot + 1]
    q_sub = qb.transpose(0, 1).unsqueeze(0)[:, pivot * G:(pivot + 1) * G]  # [1, G, S, D]
    logits = torch.matmul(q_sub, keys.transpose(-1, -2)) / math.sqrt(D)
    p = torch.softmax(logits, dim=-1, dtype=torch.float32).to(tdt)
    shp = p.shape
    p = torch.nn.functional.avg_pool1d(p.reshape(-1, shp[-1]).unsqueeze(1), 5, 1, 2).squeeze(1).view(shp)
    scores = p.max(dim=1).values[0]  # [S, L]
    ref_mask = torch.zeros(L, dtype=torch.bool)
    ref_mask[ref_set] = True

    def overlap_range(sc):
        """Overlap with the reference set over every valid resolution of ties at the k-th score."""
        x = sc.double()
        t = x.topk(K).values[-1]
        above, tie = x > t, x == t
        need = K - int(above.sum())
        base = int((above & ref_mask).sum())
        tie_in = int((tie & ref_mask).sum())
        tie_out = int(tie.sum()) - tie_in
        return base + max(0, need - tie_out), base + min(need, tie_in)

    ranges = [overlap_range(scores[s]) for s in range(S)]
    max_len = int(0.15 * L)
    # device
    words = (L + 31) // 32
    bm = torch.zeros(1, words, dtype=torch.int32)
    for t in ref_set.tolist():
        bm[0, t // 32] |= (1 << (t % 32)) if (t % 32) < 31 else -(1 << 31)
    refpos = ref_set.to(torch.int32).view(1, K).clone()
    i32 = dict(dtype=torch.int32, device=dev)
    trig = torch.zeros(1, **i32)
    rpos = torch.full((1, max_len), -1, **i32)
    coeffs = torch.zeros(1, S, dtype=torch.float32, device=dev)
    med = torch.zeros(1, dtype=torch.float64, device=dev)
    sc = torch.zeros(1, S, L, dtype=tdt, device=dev)
    err = torch.zeros(1, **i32)
    bmd, refd = bm.to(dev), refpos.to(dev)
    thr = 0.999  # forces the trigger path
    ops.drift_check(qb.to(dev), kp.to(dev), bt.to(dev), num_kv_heads=KV, groups=G, steps=S, seq_len=L,
                    pooling="avgpool", kernel_size=5, topk=K, threshold=thr,
                    pivot_heads=torch.tensor([pivot], **i32), ref_slots=torch.tensor([0], **i32),
                    max_len=torch.tensor([max_len], **i32), max_len_cap=max_len, ref_bitmap=bmd,
                    ref_positions=refd, trigger=trig, retrieve_positions=rpos, workspace=Workspace(dev), err=err,
                    coeffs=coeffs, median=med, out_scores=sc)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    dsc = sc[0].float().cpu()
    dev_counts = (coeffs[0].cpu().double() * K).round().long().tolist()
    for s in range(S):
        res = compare_selection(scores[s].float().numpy(), dsc[s].numpy(), [], K, dtype, scores_only=True)
        assert scores_close(res, dtype), res
        lo, hi = ranges[s]
        # each flipped score can move one position across the boundary
        slack = res["flips"] if dtype != "float32" else res["flips"] + res["boundary"]
        assert lo - slack <= dev_counts[s] <= hi + slack, (s, dev_counts[s], ranges[s], res)
    assert int(trig.item()) == 1
    # after a trigger the reference set is the last step's top-K
    new_ref = refd[0].cpu().tolist()
    assert new_ref == sorted(new_ref) and len(set(new_ref)) == K
    res = compare_selection(scores[-1].float().numpy(), dsc[-1].numpy(), new_ref, K, dtype)
    assert res["ok"], res
    bits = bmd[0].cpu().numpy().view(np.uint32)
    assert [w * 32 + b for w in range(words) for b in range(32) if (int(bits[w]) >> b) & 1] == new_ref
    # retrieval list: top-max_len of the last step, ascending
    rl = rpos[0].cpu().tolist()
    assert rl == sorted(rl) and len(set(rl)) == max_len
    res = compare_selection(scores[-1].float().numpy(), dsc[-1].numpy(), rl, max_len, dtype)
    assert res["ok"], res


def test_drift_check_quiet_when_stable(cuda_device):
    """Queries equal to the prefill query: overlap 1.0 per step, no trigger."""
    geo, tdt, dev = LLAMA_8B, torch.bfloat16, cuda_device
    G, KV, D, H, L, S = geo.groups, geo.num_kv_heads, geo.head_dim, geo.num_heads, 4096, 5
    q, k, _ = prefill_inputs(geo, L, seed=8, dtype=tdt)
    pivot, K = 7, int(0.2 * L)
    n = L // 256
    bt = torch.full((KV, n + 1), -1, dtype=torch.int32)
    bt[pivot, :n] = torch.arange(n, dtype=torch.int32)
    kp = k[0, pivot].reshape(n, 256, 1, D).contiguous()
    i32 = dict(dtype=torch.int32, device=dev)
    words = L // 32
    pos = torch.zeros(1, 1, K, **i32)
    bm = torch.zeros(1, 1, words, **i32)
    ws = Workspace(dev)
    err = torch.zeros(1, **i32)
    qd = q.to(dev)
    ops.pivot_init(qd, k.to(dev), first_pivot=pivot, n_pivots=1, groups=G, pooling="avgpool", kernel_size=5,
                   topk=K, ref_positions=pos, ref_bitmap=bm, workspace=ws, err=err)
    qb = qd[0, :, -1, :].unsqueeze(0).expand(S, H, D).contiguous()
    trig = torch.full((1,), 7, **i32)
    coeffs = torch.zeros(1, S, dtype=torch.float32, device=dev)
    rpos = torch.zeros(1, 16, **i32)
    ops.drift_check(qb, kp.to(dev), bt.to(dev), num_kv_heads=KV, groups=G, steps=S, seq_len=L, pooling="avgpool",
                    kernel_size=5, topk=K, threshold=0.5, pivot_heads=torch.tensor([pivot], **i32),
                    ref_slots=torch.tensor([0], **i32), max_len=torch.tensor([16], **i32), max_len_cap=16,
                    ref_bitmap=bm.view(1, words), ref_positions=pos.view(1, K), trigger=trig,
                    retrieve_positions=rpos, workspace=ws, err=err, coeffs=coeffs)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(trig.item()) == 0
    assert coeffs.min().item() == 1.0


@pytest.mark.parametrize("tier", ["device", "host"])
def test_retrieve_gathers_only_on_trigger(cuda_device, tier):
    dev = cuda_device
    KV, D, L = 8, 128, 1000
    full_k = torch.randn(1, KV, L, D).to(torch.bfloat16)
    full_v = torch.randn(1, KV, L, D).to(torch.bfloat16)
    if tier == "device":
        fk, fv = full_k.to(dev), full_v.to(dev)
    else:
        fk, fv = full_k.pin_memory(), full_v.pin_memory()
    bt = torch.full((KV, 4), -1, dtype=torch.int32)
    bt[2, :2] = torch.tensor([0, 1])
    bt[3, :1] = torch.tensor([2])
    kp = torch.zeros(3, 256, 1, D, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    i32 = dict(dtype=torch.int32, device=dev)
    positions = torch.tensor([sorted(torch.randperm(L)[:400].tolist())], **i32)
    args = dict(member_job=torch.tensor([0, 0], **i32), member_head=torch.tensor([2, 3], **i32),
                member_len=torch.tensor([400, 200], **i32), max_member_len=400,
                retrieve_positions=positions, full_k=fk, full_v=fv, k_pool=kp, v_pool=vp,
                block_table=bt.to(dev), num_kv_heads=KV, err=torch.zeros(1, **i32))
    ops.retrieve(trigger=torch.zeros(1, **i32), **args)
    torch.cuda.synchronize()
    assert kp.abs().sum().item() == 0
    ops.retrieve(trigger=torch.ones(1, **i32), **args)
    torch.cuda.synchronize()
    pos = positions[0].cpu()
    kf = kp.cpu().view(-1, D)
    assert torch.equal(kf[0:400], full_k[0, 2, pos])
    assert torch.equal(kf[512:712], full_k[0, 3, pos[:200]])
    assert torch.equal(vp.cpu().view(-1, D)[512:712], full_v[0, 3, pos[:200]])


def test_retrieve_delta_matches_full_retrieval(cuda_device):
    """Delta retrieval from a pinned-host tier: after each of several
    retrievals (overlapping position lists, one with the trigger off) the
    pools are bit-identical to the full retrieval's, and the slot maps hold
    the positions of the retrieved rows."""
    dev = cuda_device
    KV, D, L = 8, 128, 3000
    g = torch.Generator().manual_seed(7)
    full_k = torch.randn(1, KV, L, D, generator=g).to(torch.bfloat16)
    full_v = torch.randn(1, KV, L, D, generator=g).to(torch.bfloat16)
    fk, fv = full_k.pin_memory(), full_v.pin_memory()
    heads, lens, keep = [2, 5, 6], [700, 300, 1], [650, 300, 0]
    bt = torch.full((KV, 6), -1, dtype=torch.int32)
    bt[2, :4] = torch.tensor([0, 1, 2, 3])
    bt[5, :2] = torch.tensor([4, 5])
    bt[6, :1] = torch.tensor([6])
    kp = torch.zeros(7, 256, 1, D, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    # prefill: each satellite holds its kept rows in slots [0, keep)
    kept = [sorted(torch.randperm(L, generator=g)[:n].tolist()) for n in keep]
    for h, kh in zip(heads, kept):
        s = int(bt[h, 0]) * 256
        kp.view(-1, D)[s:s + len(kh)] = full_k[0, h, kh]
        vp.view(-1, D)[s:s + len(kh)] = full_v[0, h, kh]
    i32 = dict(dtype=torch.int32, device=dev)
    reuse = [min(k, n) for k, n in zip(keep, lens)]
    slot = torch.zeros(3, max(reuse), dtype=torch.int32)
    for i, (kh, r) in enumerate(zip(kept, reuse)):
        slot[i, :r] = torch.tensor(kh[:r], dtype=torch.int32)
    slot = slot.to(dev)
    offs = torch.tensor([0, 700, 1000], **i32)
    rows = sum(lens)
    stage = (torch.empty(rows, D, dtype=torch.bfloat16, device=dev),
             torch.empty(rows, D, dtype=torch.bfloat16, device=dev), torch.empty(rows, **i32))
    kp_d, vp_d = kp.to(dev), vp.to(dev)       # delta path
    kp_f, vp_f = kp.to(dev), vp.to(dev)       # full-retrieval path
    common = dict(member_job=torch.zeros(3, **i32), member_head=torch.tensor(heads, **i32),
                  member_len=torch.tensor(lens, **i32), max_member_len=max(lens), full_k=fk, full_v=fv,
                  block_table=bt.to(dev), num_kv_heads=KV)
    err = torch.zeros(1, **i32)
    # first list: many of the first satellite's kept rows plus new ones; then
    # a list overlapping the first; then one with the trigger off
    p1 = sorted(set(kept[0][:500]) | set(torch.randperm(L, generator=g)[:400].tolist()))[:700]
    p2 = sorted(set(p1[::2]) | set(torch.randperm(L, generator=g)[:600].tolist()))[:700]
    p3 = sorted(torch.randperm(L, generator=g)[:700].tolist())
    for pos_list, trig in ((p1, 1), (p2, 1), (p3, 0)):
        positions = torch.tensor([pos_list], **i32)
        trigger = torch.tensor([trig], **i32)
        ops.retrieve_delta(member_stage_offset=offs, reuse_len=torch.tensor(reuse, **i32), trigger=trigger,
                           retrieve_positions=positions, slot_positions=slot, k_pool=kp_d, v_pool=vp_d,
                           stage_k=stage[0], stage_v=stage[1], stage_src=stage[2], err=err, **common)
        ops.retrieve(trigger=trigger, retrieve_positions=positions, k_pool=kp_f, v_pool=vp_f, err=err, **common)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(kp_d.cpu(), kp_f.cpu())
        assert torch.equal(vp_d.cpu(), vp_f.cpu())
        if trig:
            sl = slot.cpu()
            for i, r in enumerate(reuse):
                assert sl[i, :r].tolist() == pos_list[:r]
    # the pools hold the second list's rows
    assert torch.equal(kp_d.cpu().view(-1, D)[0:700], full_k[0, 2, p2])


@pytest.mark.parametrize("window", [1, 8])
def test_scoring_reads_the_last_queries_of_a_short_query(cuda_device, window):
    """A query holding only the last positions (the scoring reads only those)
    gives the same pivot sets and prefill selection as the full-length query,
    reading inside its own buffer."""
    geo = LLAMA_8B
    G, KV, D = geo.groups, geo.num_kv_heads, geo.head_dim
    dev = cuda_device
    L, nc = 3000, 3
    q, k, v = prefill_inputs(geo, L, seed=91, dtype=torch.bfloat16)
    q_short = q[:, :, -32:, :].contiguous()
    kd, vd = k.to(dev), v.to(dev)
    keep = [700, 300, 1500]
    results = []
    for qq in (q.to(dev), q_short.to(dev)):
        n = sum((x + 255) // 256 for x in keep)
        bt = torch.full((KV, (L + 255) // 256 + 1), -1, dtype=torch.int32)
        ptr = 0
        for h, x in enumerate(keep):
            pages = (x + 255) // 256
            bt[h, :pages] = torch.arange(ptr, ptr + pages, dtype=torch.int32)
            ptr += pages
        kp = torch.zeros(n, 256, 1, D, dtype=torch.bfloat16, device=dev)
        vp = torch.zeros_like(kp)
        hl = torch.zeros(KV, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        idx = torch.empty(1, nc, max(keep), dtype=torch.int32, device=dev)
        ops.prefill_select(qq, kd, vd, torch.tensor(keep, dtype=torch.int32, device=dev), max(keep), n_heads=nc,
                           groups=G, window=window, pooling="avgpool", kernel_size=5, k_pool=kp, v_pool=vp,
                           block_table=bt.to(dev), heads_len=hl, workspace=Workspace(dev), err=err,
                           out_indices=idx)
        K = 600
        pos = torch.empty(1, 1, K, dtype=torch.int32, device=dev)
        bm = torch.zeros(1, 1, (L + 31) // 32, dtype=torch.int32, device=dev)
        ops.pivot_init(qq, kd, first_pivot=KV - 1, n_pivots=1, groups=G, pooling="avgpool", kernel_size=5,
                       topk=K, ref_positions=pos, ref_bitmap=bm, workspace=Workspace(dev), err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        results.append((idx.cpu(), kp.cpu(), pos.cpu(), bm.cpu()))
    for a, b in zip(*results):
        assert torch.equal(a, b)
    with pytest.raises(ValueError):
        ops.pivot_init(q_short[:, :, :0].to(dev), kd, first_pivot=KV - 1, n_pivots=1, groups=G, pooling="avgpool",
                       kernel_size=5, topk=600, ref_positions=pos, ref_bitmap=bm, workspace=Workspace(dev),
                       err=err)
