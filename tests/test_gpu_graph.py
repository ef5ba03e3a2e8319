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
                eager.decode_select(q, l)
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
