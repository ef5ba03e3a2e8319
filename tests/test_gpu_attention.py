"""The drop-in attention classes on the GPU.

Decode outputs of ``LlamaAttention`` / ``Qwen2Attention`` must equal
``o_proj`` of the oracle's paged attention over the cache's own pages
(2e-2 max-abs in bf16 before o_proj, checked after o_proj with the same
bound scaled by the projection), and the cache state built through the
module must match the CPU oracle fed with the module's keys and values.
A tiny random-init transformers model also runs prefill + greedy decode with
the classes patched in.
"""
import pytest
import torch

from heterocache_b200.attention import LlamaAttention, Qwen2Attention, patch_transformers
from heterocache_b200.cache import HeteroCache, HeteroCacheConfig
from heterocache_b200.roles import derive_runtime_data, synthetic_roles
from oracle.hc_oracle import OracleCache, paged_attention

pytestmark = pytest.mark.gpu


def _config(kind):
    if kind == "llama":
        from transformers import LlamaConfig
        return LlamaConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=4, head_dim=128,
                           intermediate_size=2048, num_hidden_layers=2, vocab_size=512, rope_theta=500000.0,
                           max_position_embeddings=4096)
    from transformers import Qwen2Config
    return Qwen2Config(hidden_size=1024, num_attention_heads=8, num_key_value_heads=4, intermediate_size=2048,
                       num_hidden_layers=2, vocab_size=512, rope_theta=1e6, max_position_embeddings=4096)


def _rope(cfg, positions, device):
    if hasattr(cfg, "rope_theta"):
        theta = cfg.rope_theta
    else:
        theta = cfg.rope_parameters["rope_theta"]
    d = 128
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    f = positions.float()[:, None] * inv[None]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos()[None].to(device, torch.bfloat16), emb.sin()[None].to(device, torch.bfloat16)


@pytest.mark.parametrize("kind", ["llama", "qwen"])
def test_attention_module_decode_matches_oracle(cuda_device, kind):
    torch.manual_seed(0)
    cfg = _config(kind)
    cls = LlamaAttention if kind == "llama" else Qwen2Attention
    attn = cls(cfg, layer_idx=0).to(cuda_device, torch.bfloat16).eval()
    data = derive_runtime_data(synthetic_roles(1, 4, seed=3, star_size=3), 1, 4)
    hc = HeteroCacheConfig(data, compression_ratio=0.5, stable_threshold=0.999, real_offload=False, max_gen_len=32,
                           decode_step=5, num_attn_heads=8, num_kv_heads=4, num_layers=1)
    cache = HeteroCache(hc)
    orc = OracleCache(hc)
    L = 700
    h = torch.randn(1, L, 1024, device=cuda_device, dtype=torch.bfloat16)
    pos = torch.arange(L)
    cos, sin = _rope(cfg, pos, cuda_device)
    with torch.no_grad():
        out = attn(h, position_embeddings=(cos, sin), past_key_values=cache)[0]
        q = attn.q_proj(h).view(1, L, -1, 128).transpose(1, 2)
        k = attn.k_proj(h).view(1, L, -1, 128).transpose(1, 2)
        v = attn.v_proj(h).view(1, L, -1, 128).transpose(1, 2)
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
    assert out.shape == (1, L, 1024) and torch.isfinite(out.float()).all()
    orc.update(k.cpu(), v.cpu(), 0)
    orc.init_coefficient(q.cpu(), k.cpu(), 0)
    orc.prefill_select(q.cpu(), k.cpu(), v.cpu(), 0)
    torch.cuda.synchronize()
    assert torch.equal(cache.heads_len[0].cpu(), orc.heads_len[0])
    assert torch.equal(cache.block_tables[0].cpu(), orc.block_tables[0])
    for step in range(9):
        x = torch.randn(1, 1, 1024, device=cuda_device, dtype=torch.bfloat16)
        c1, s1 = _rope(cfg, torch.tensor([L + step]), cuda_device)
        check_step = (step + 1) % 5 == 0
        with torch.no_grad():
            y = attn(x, position_embeddings=(c1, s1), past_key_values=cache)[0]
            qd = attn.q_proj(x).view(1, 1, -1, 128).transpose(1, 2)
            kd = attn.k_proj(x).view(1, 1, -1, 128).transpose(1, 2)
            qd, _ = apply_rotary_pos_emb(qd, kd, c1, s1)
        torch.cuda.synchronize()
        cache.check_errors()
        # Llama attends before decode_select: on check steps the pages changed after the attention
        if kind == "llama" and check_step:
            continue
        ref = paged_attention(qd.cpu(), cache.key_pools[0].cpu(), cache.value_pools[0].cpu(),
                              cache.block_tables[0].cpu(), cache.heads_len[0].cpu(), 4)
        with torch.no_grad():
            ref_out = attn.o_proj(ref.view(1, 1, -1).to(cuda_device, torch.bfloat16))
        diff = (y.float() - ref_out.float()).abs().max().item()
        assert diff <= 5e-2, (kind, step, diff)


@pytest.mark.parametrize("kind", ["llama", "qwen"])
def test_tiny_model_prefill_and_greedy_decode(cuda_device, kind):
    """transformers model with the classes patched in, driven token by token."""
    import transformers
    patch_transformers()
    torch.manual_seed(0)
    cfg = _config(kind)
    cfg._attn_implementation = "sdpa"
    model_cls = transformers.LlamaForCausalLM if kind == "llama" else transformers.Qwen2ForCausalLM
    model = model_cls(cfg).to(cuda_device, torch.bfloat16).eval()
    attn0 = model.model.layers[0].self_attn
    assert isinstance(attn0, LlamaAttention if kind == "llama" else Qwen2Attention)
    data = derive_runtime_data(synthetic_roles(2, 4, seed=5, star_size=3), 2, 4)
    hc = HeteroCacheConfig(data, compression_ratio=0.5, stable_threshold=0.5, real_offload=False, max_gen_len=16,
                           decode_step=5, num_attn_heads=8, num_kv_heads=4, num_layers=2)
    cache = HeteroCache(hc)
    ids = torch.randint(0, 512, (1, 600), device=cuda_device)
    with torch.no_grad():
        out = model(input_ids=ids, past_key_values=cache, use_cache=True)
        tok = out.logits[:, -1:].argmax(-1)
        for t in range(7):
            pos = torch.tensor([[600 + t]], device=cuda_device)
            out = model(input_ids=tok, past_key_values=cache, use_cache=True, position_ids=pos,
                        cache_position=pos[0])
            assert torch.isfinite(out.logits.float()).all()
            tok = out.logits[:, -1:].argmax(-1)
    torch.cuda.synchronize()
    cache.check_errors()
    assert cache.get_seq_length() == 607
    for layer in range(2):
        assert cache.heads_len[layer].cpu().tolist() == [int(x) for x in cache._hlen[layer]]


@pytest.mark.parametrize("kind", ["llama", "qwen"])
def test_model_decode_graph_matches_eager(cuda_device, kind):
    """Whole-model decode replayed from CUDA graphs (ModelDecodeGraph) gives
    the eager token-by-token run's tokens and cache state."""
    import transformers

    from heterocache_b200.graph import ModelDecodeGraph
    patch_transformers()
    torch.manual_seed(0)
    cfg = _config(kind)
    cfg._attn_implementation = "sdpa"
    model_cls = transformers.LlamaForCausalLM if kind == "llama" else transformers.Qwen2ForCausalLM
    model = model_cls(cfg).to(cuda_device, torch.bfloat16).eval()
    data = derive_runtime_data(synthetic_roles(2, 4, seed=5, star_size=3), 2, 4)
    ids = torch.randint(0, 512, (1, 600), device=cuda_device)
    n_tok = 12  # two drift checks (decode_step 5)

    def new_cache():
        hc = HeteroCacheConfig(data, compression_ratio=0.5, stable_threshold=0.9, real_offload=False,
                               max_gen_len=32, decode_step=5, num_attn_heads=8, num_kv_heads=4, num_layers=2)
        c = HeteroCache(hc)
        with torch.no_grad():
            out = model(input_ids=ids, past_key_values=c, use_cache=True, logits_to_keep=1)
        return c, out.logits[:, -1:].argmax(-1)

    eager, tok = new_cache()
    toks_e = []
    with torch.no_grad():
        for t in range(n_tok):
            pos = torch.tensor([[600 + t]], device=cuda_device)
            out = model(input_ids=tok, past_key_values=eager, use_cache=True, position_ids=pos,
                        cache_position=pos[0], logits_to_keep=1)
            tok = out.logits[:, -1:].argmax(-1)
            toks_e.append(int(tok.item()))
    graphed, tok0 = new_cache()
    tok_buf = tok0.clone()
    pos_buf = torch.tensor([[600]], device=cuda_device)
    runner = ModelDecodeGraph(model, graphed, tok_buf, pos_buf)
    toks_g = [int(runner.step().item()) for _ in range(n_tok)]
    torch.cuda.synchronize()
    eager.check_errors()
    graphed.check_errors()
    assert toks_g == toks_e
    assert int(pos_buf.item()) == 600 + n_tok
    assert graphed.get_seq_length() == eager.get_seq_length() == 600 + n_tok
    for layer in range(2):
        assert torch.equal(graphed.heads_len[layer].cpu(), eager.heads_len[layer].cpu())
        assert torch.equal(graphed.block_tables[layer].cpu(), eager.block_tables[layer].cpu())
        assert (graphed.key_pools[layer].float() - eager.key_pools[layer].float()).abs().max().item() <= 2e-2
