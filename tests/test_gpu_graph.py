"""Decode steps replayed from CUDA graphs (``DecodeStepGraph``, the path the
benchmark times) against the same steps run eagerly through the cache:
identical attention outputs and cache state, bit for bit, across two drift
checks, in the Llama (drift check after attention) and Qwen2 (before) order.
"""
import pytest
import torch

from heterocache_b200.cache import HeteroCache, HeteroCacheConfig
from heterocache_b200.graph import DecodeStepGraph
from heterocache_b200.roles import derive_runtime_data, synthetic_roles
from heterocache_b200.synthetic import LLAMA_8B, QWEN_7B, DriftingDecode, prefill_inputs

pytestmark = pytest.mark.gpu


def _cache(geo, layers, L, dev, threshold):
    KV = geo.num_kv_heads
    data = derive_runtime_data(synthetic_roles(layers, KV, seed=13), layers, KV)
    cfg = HeteroCacheConfig(data, compression_ratio=0.5, stable_threshold=threshold, real_offload=False,
                            max_gen_len=32, decode_step=5, pooling="avgpool", kernel_size=5,
                            num_attn_heads=geo.num_heads, num_kv_heads=KV, num_layers=layers)
    cache = HeteroCache(cfg)
    q_last = []
    for layer in range(layers):
        q, k, v = prefill_inputs(geo, L, seed=40 + layer, dtype=torch.bfloat16, q_positions=32)
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        cache.update(kd, vd, layer)
        cache.init_coefficient(qd, kd, layer)
        cache.prefill_select(qd, kd, vd, layer)
        q_last.append(q[:, :, -1:, :])
    return cache, q_last


@pytest.mark.parametrize("order,geo", [("llama", LLAMA_8B), ("qwen", QWEN_7B)])
def test_graph_decode_matches_eager(cuda_device, order, geo):
    dev = cuda_device
    layers, L, n_steps = 2, 3000, 12  # two drift checks (decode_step 5)
    eager, q_last = _cache(geo, layers, L, dev, threshold=0.9)
    graphed, _ = _cache(geo, layers, L, dev, threshold=0.9)
    gens = [DriftingDecode(geo, seed=70 + l, q0=q_last[l], dtype=torch.bfloat16) for l in range(layers)]
    steps = [[tuple(t.to(dev) for t in g.step()) for g in gens] for _ in range(n_steps)]
    torch.cuda.synchronize()

    # eager: the same calls the graph captures
    H, D = geo.num_heads, geo.head_dim
    outs_e = []
    for s in range(n_steps):
        row = []
        for l in range(layers):
            q, k, v = steps[s][l]
            out = torch.empty(1, H, D, dtype=torch.bfloat16, device=dev)
            eager.update(k, v, l, {"query_states": q, "defer_append": True})
            if order == "qwen":
                eager.decode_select(q, l)
            eager.attention(q, l, out=out)
            if order == "llama":
                eager.decode_select(q, l, defer=True)  # as the graph: one batch at the step's end
            row.append(out)
        eager.join_retrievals()
        outs_e.append(torch.stack(row).clone())

    graph = DecodeStepGraph(graphed, list(range(layers)), order=order)
    outs_g = []
    for s in range(n_steps):
        for l in range(layers):
            q, k, v = steps[s][l]
            graph.q[l].copy_(q), graph.k[l].copy_(k), graph.v[l].copy_(v)
        outs_g.append(graph.step().clone())
    torch.cuda.synchronize()
    eager.check_errors()
    graphed.check_errors()

    for s in range(n_steps):
        assert torch.equal(outs_g[s], outs_e[s]), f"step {s}"
    assert graphed.get_seq_length() == eager.get_seq_length() == L + n_steps
    for l in range(layers):
        assert torch.equal(graphed.heads_len[l], eager.heads_len[l])
        assert torch.equal(graphed.block_tables[l], eager.block_tables[l])
        assert torch.equal(graphed.key_pools[l], eager.key_pools[l])
        assert torch.equal(graphed.value_pools[l], eager.value_pools[l])
        if len(eager.prefill_topk_set[l]):
            assert torch.equal(graphed.prefill_topk_set[l], eager.prefill_topk_set[l])


@pytest.mark.parametrize("per_launch", [1, 0])
def test_deferred_checks_match_per_layer_checks(cuda_device, per_launch):
    """Llama order: drift checks put off to one batch (run by the next step's
    first update, and by join_retrievals at the end) against each layer's
    check run where it falls due.  One check per launch splits every check
    over the SMs as a single check does: bit-identical results.  The default
    batching splits each check over fewer CTAs, so its softmax sums are added
    in another order (fp32 rounding): same triggers, attention outputs within
    the bf16 tolerance, reference sets within a few boundary swaps."""
    dev, geo = cuda_device, LLAMA_8B
    layers, L, n_steps = 4, 3000, 11  # two checks per layer (decode_step 5)
    per_layer, q_last = _cache(geo, layers, L, dev, threshold=0.9)
    batched, _ = _cache(geo, layers, L, dev, threshold=0.9)
    batched.drift_batch_per_launch = per_launch
    gens = [DriftingDecode(geo, seed=90 + l, q0=q_last[l], dtype=torch.bfloat16) for l in range(layers)]
    steps = [[tuple(t.to(dev) for t in g.step()) for g in gens] for _ in range(n_steps)]
    H, D = geo.num_heads, geo.head_dim
    outs = {}
    for name, cache, defer in (("per_layer", per_layer, False), ("batched", batched, True)):
        outs[name] = []
        for s in range(n_steps):
            row = []
            for l in range(layers):
                q, k, v = steps[s][l]
                out = torch.empty(1, H, D, dtype=torch.bfloat16, device=dev)
                cache.update(k, v, l, {"query_states": q, "defer_append": True})
                cache.attention(q, l, out=out)
                cache.decode_select(q, l, defer=defer)
                row.append(out)
            outs[name].append(torch.stack(row).clone())
        cache.join_retrievals()
    torch.cuda.synchronize()
    per_layer.check_errors()
    batched.check_errors()
    assert not batched._deferred
    for l in range(layers):
        assert torch.equal(batched.heads_len[l], per_layer.heads_len[l])
        assert torch.equal(batched.block_tables[l], per_layer.block_tables[l])
        jb, jp = batched._jobs[l], per_layer._jobs[l]
        if jp is not None:
            assert torch.equal(jb.trigger, jp.trigger)
    for s in range(n_steps):
        if per_launch == 1:
            assert torch.equal(outs["batched"][s], outs["per_layer"][s]), f"step {s}"
        else:
            err = (outs["batched"][s].float() - outs["per_layer"][s].float()).abs().max().item()
            assert err <= 2e-2, (s, err)
    for l in range(layers):
        if not len(per_layer.prefill_topk_set[l]):
            continue
        a, b = batched.prefill_topk_set[l], per_layer.prefill_topk_set[l]
        if per_launch == 1:
            assert torch.equal(a, b)
            assert torch.equal(batched.key_pools[l], per_layer.key_pools[l])
        else:
            for x, y in zip(a.reshape(-1, a.shape[-1]).tolist(), b.reshape(-1, b.shape[-1]).tolist()):
                assert len(set(x) ^ set(y)) <= max(4, len(x) // 100), l


def test_run_host_matches_step_by_step(cuda_device):
    """DecodeStepGraph.run_host (copies overlapped with the replays on two
    copy streams, the path the benchmark's end-to-end figure times) gives the
    outputs and cache state of copying each step in and out around step()."""
    dev, geo = cuda_device, LLAMA_8B
    layers, L, n_steps = 2, 3000, 13
    a, q_last = _cache(geo, layers, L, dev, threshold=0.9)
    b, _ = _cache(geo, layers, L, dev, threshold=0.9)
    gens = [DriftingDecode(geo, seed=50 + l, q0=q_last[l], dtype=torch.bfloat16) for l in range(layers)]
    steps = [[g.step() for g in gens] for _ in range(n_steps)]
    hq = torch.stack([torch.stack([st[l][0] for l in range(layers)]) for st in steps]).pin_memory()
    hk = torch.stack([torch.stack([st[l][1] for l in range(layers)]) for st in steps]).pin_memory()
    hv = torch.stack([torch.stack([st[l][2] for l in range(layers)]) for st in steps]).pin_memory()
    ga = DecodeStepGraph(a, list(range(layers)))
    gb = DecodeStepGraph(b, list(range(layers)))
    out_a = torch.empty((n_steps,) + tuple(ga.out.shape), dtype=ga.out.dtype).pin_memory()
    ga.run_host(hq, hk, hv, out_a)
    out_b = []
    for s in range(n_steps):
        gb.q.copy_(hq[s]), gb.k.copy_(hk[s]), gb.v.copy_(hv[s])
        out_b.append(gb.step().cpu())
    torch.cuda.synchronize()
    a.check_errors()
    b.check_errors()
    for s in range(n_steps):
        assert torch.equal(out_a[s], out_b[s]), f"step {s}"
    for l in range(layers):
        assert torch.equal(a.key_pools[l], b.key_pools[l])
        assert torch.equal(a.heads_len[l], b.heads_len[l])


@pytest.mark.parametrize("per_launch", [1, 0])
def test_checks_of_several_caches_in_one_batch(cuda_device, per_launch):
    """flush_checks_together: the put-off drift checks of three independent
    caches (three sequences) in one batch, against each cache flushing its
    own.  One check per launch: bit-identical; the default batching adds the
    softmax sums in another order: same triggers, outputs within the bf16
    tolerance."""
    from heterocache_b200.cache import flush_checks_together
    dev, geo = cuda_device, LLAMA_8B
    KV, H, D, L, n_steps = geo.num_kv_heads, geo.num_heads, geo.head_dim, 3000, 11

    def make(seed):
        data = derive_runtime_data(synthetic_roles(1, KV, seed=13), 1, KV)
        cfg = HeteroCacheConfig(data, compression_ratio=0.5, stable_threshold=0.9, real_offload=False,
                                max_gen_len=32, decode_step=5, pooling="avgpool", kernel_size=5,
                                num_attn_heads=H, num_kv_heads=KV, num_layers=1)
        c = HeteroCache(cfg)
        q, k, v = prefill_inputs(geo, L, seed=seed, dtype=torch.bfloat16, q_positions=32)
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        c.update(kd, vd, 0)
        c.init_coefficient(qd, kd, 0)
        c.prefill_select(qd, kd, vd, 0)
        return c, q[:, :, -1:, :]

    seeds = (201, 202, 203)
    own = [make(s)[0] for s in seeds]
    both = [make(s) for s in seeds]
    tog = [c for c, _ in both]
    tog[0].drift_batch_per_launch = per_launch
    for c in own:
        c.drift_batch_per_launch = per_launch
    gens = [DriftingDecode(geo, seed=s + 7, q0=q0, dtype=torch.bfloat16) for s, (_, q0) in zip(seeds, both)]
    n_trig = 0
    for step in range(n_steps):
        qkv = [tuple(t.to(dev) for t in g.step()) for g in gens]
        outs = {}
        for name, caches in (("own", own), ("tog", tog)):
            res = []
            for c, (q, k, v) in zip(caches, qkv):
                c.update(k, v, 0)
                res.append(c.attention(q, 0))
                c.decode_select(q, 0, defer=True)
            if name == "own":
                for c in caches:
                    c.flush_checks()
            else:
                flush_checks_together(caches)
            outs[name] = torch.stack(res)
        torch.cuda.synchronize()
        if per_launch == 1:
            assert torch.equal(outs["own"], outs["tog"]), step
        else:
            assert (outs["own"].float() - outs["tog"].float()).abs().max().item() <= 2e-2, step
        for a, b in zip(own, tog):
            ja, jb = a._jobs[0], b._jobs[0]
            assert torch.equal(ja.trigger[:ja.n_jobs], jb.trigger[:jb.n_jobs]), step
            n_trig += int(jb.trigger[:jb.n_jobs].sum())
            if per_launch == 1:
                assert torch.equal(a.key_pools[0], b.key_pools[0]), step
                assert torch.equal(a.prefill_topk_set[0], b.prefill_topk_set[0]), step
    for c in own + tog:
        c.check_errors()
    assert n_trig > 0
