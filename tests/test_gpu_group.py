"""CacheGroup: independent sequences whose pages share one pool per layer,
attended in one decode launch (``attention_together``), against the same
sequences in caches of their own (one launch each).  The split of the tokens
over the launch differs, so outputs agree within the bf16 tolerance; the
drift-check triggers and every page (read through each cache's own page
table) are identical."""
import pytest
import torch

from heterocache_b200.ops import PAGE
from heterocache_b200.cache import (CacheGroup, HeteroCache, HeteroCacheConfig, attention_together,
                                    flush_checks_together)
from heterocache_b200.roles import derive_runtime_data, synthetic_roles
from heterocache_b200.synthetic import LLAMA_8B, DriftingDecode, prefill_inputs

pytestmark = pytest.mark.gpu


def _config(geo):
    KV = geo.num_kv_heads
    data = derive_runtime_data(synthetic_roles(1, KV, seed=13), 1, KV)
    return HeteroCacheConfig(data, compression_ratio=0.5, stable_threshold=0.9, real_offload=False,
                             max_gen_len=32, decode_step=5, pooling="avgpool", kernel_size=5,
                             num_attn_heads=geo.num_heads, num_kv_heads=KV, num_layers=1)


def _prefill(c, geo, L, seed, dev):
    q, k, v = prefill_inputs(geo, L, seed=seed, dtype=torch.bfloat16, q_positions=32)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    c.update(kd, vd, 0)
    c.init_coefficient(qd, kd, 0)
    c.prefill_select(qd, kd, vd, 0)
    return q[:, :, -1:, :]


def _pages(c):
    """Every mapped page of the cache, in page-table order."""
    bt = c.block_tables[0].cpu()
    hl = c.heads_len[0].cpu()
    ks, vs = [], []
    for r in range(bt.shape[0]):
        n = (int(hl[r]) + PAGE - 1) // PAGE
        ids = bt[r, :n].long().to(c.key_pools[0].device)
        ks.append(c.key_pools[0][ids])
        vs.append(c.value_pools[0][ids])
    return ks, vs


@pytest.mark.parametrize("rows", [True, False], ids=["rows-of-one-buffer", "separate-tensors"])
def test_group_matches_independent_caches(cuda_device, rows):
    dev, geo = cuda_device, LLAMA_8B
    H, KV, D, L, n_steps = geo.num_heads, geo.num_kv_heads, geo.head_dim, 3000, 12
    seeds = (301, 302, 303)
    own = [HeteroCache(_config(geo)) for _ in seeds]
    grp_caches = [HeteroCache(_config(geo)) for _ in seeds]
    group = CacheGroup(grp_caches)
    q0 = [_prefill(c, geo, L, s, dev) for c, s in zip(own, seeds)]
    for c, s in zip(grp_caches, seeds):
        _prefill(c, geo, L, s, dev)
    assert grp_caches[1].key_pools[0].data_ptr() == grp_caches[0].key_pools[0].data_ptr()
    gens = [DriftingDecode(geo, seed=s + 7, q0=q, dtype=torch.bfloat16) for s, q in zip(seeds, q0)]
    n_trig = 0
    for step in range(n_steps):
        qkv = [tuple(t.to(dev) for t in g.step()) for g in gens]
        if rows:  # every sequence's q/k/v a row of one batch buffer (as the graphed step feeds them)
            qb = torch.stack([q for q, _, _ in qkv])
            kb = torch.stack([k for _, k, _ in qkv])
            vb = torch.stack([v for _, _, v in qkv])
            qkv = [(qb[i], kb[i], vb[i]) for i in range(len(seeds))]
        defer = step % 3 != 2  # some steps append at update time (nothing pending at attention)
        res = []
        for c, (q, k, v) in zip(own, qkv):
            c.update(k, v, 0, {"query_states": q, "defer_append": defer})
            res.append(c.attention(q, 0))
            c.decode_select(q, 0, defer=True)
        flush_checks_together(own)
        for c, (q, k, v) in zip(grp_caches, qkv):
            c.update(k, v, 0, {"query_states": q, "defer_append": defer})
        q_all = torch.cat([q for q, _, _ in qkv], 0)
        out = attention_together(group, q_all, 0)
        for c, (q, _, _) in zip(grp_caches, qkv):
            c.decode_select(q, 0, defer=True)
        flush_checks_together(grp_caches)
        torch.cuda.synchronize()
        ref = torch.cat(res, 0)
        assert out.shape == (len(seeds), H, D)
        assert (ref.float() - out.float()).abs().max().item() <= 2e-2, step
        for a, b in zip(own, grp_caches):
            ja, jb = a._jobs[0], b._jobs[0]
            assert torch.equal(ja.trigger[:ja.n_jobs], jb.trigger[:jb.n_jobs]), step
            n_trig += int(jb.trigger[:jb.n_jobs].sum())
            assert torch.equal(a.heads_len[0], b.heads_len[0]), step
            ka, va = _pages(a)
            kb_, vb_ = _pages(b)
            for x, y in zip(ka + va, kb_ + vb_):
                assert torch.equal(x, y), step
    for c in own + grp_caches:
        c.join_retrievals()
        c.check_errors()
    assert n_trig > 0


def test_group_needs_adoption_before_prefill(cuda_device):
    c = HeteroCache(_config(LLAMA_8B))
    _prefill(c, LLAMA_8B, 600, 7, cuda_device)
    with pytest.raises(RuntimeError, match="before their prefill"):
        CacheGroup([c])
