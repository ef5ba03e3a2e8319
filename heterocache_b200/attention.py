"""Drop-in patched attention classes for transformers' Llama and Qwen2.

Same projections, RoPE and call order as the reference's patched classes
(heterocache/llama_model.py:279-405, heterocache/qwen_model.py:93-212):

* prefill (q_len > 1): ``cache.update`` -> ``init_coefficient`` ->
  ``prefill_select`` -> causal attention over the uncompressed prompt;
* decode (q_len == 1): ``cache.update`` (page append) -> paged decode
  attention over each (batch, KV head) row's compressed pages; Llama runs
  ``decode_select`` after the attention (llama_model.py:391), Qwen2 before it
  (qwen_model.py:178).

Decode attention is ``HeteroCache.attention`` (the sm_100a split-K kernel) in
place of ``flash_attn_with_kvcache``.  The prefill attention over the full
prompt (the reference's flash-attn forward, llama_model.py:353-361,
qwen_model.py:161-169) is ``ops.prefill_attention``, a causal grouped-query
attention on the tcgen05 tensor cores, for 16-bit models; fp32 models use
PyTorch's ``scaled_dot_product_attention``.

``patch_transformers()`` installs the classes the way the reference's loader
does (heterocache/utils.py:195-197); call it before building the model.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

try:
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
except Exception:  # pragma: no cover
    def apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=1):
        cos, sin = cos.unsqueeze(unsqueeze_dim), sin.unsqueeze(unsqueeze_dim)

        def rot(x):
            x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
            return torch.cat((-x2, x1), dim=-1)

        return q * cos + rot(q) * sin, k * cos + rot(k) * sin


def _causal_attention(q, k, v, groups: int, scale: float) -> torch.Tensor:
    """Causal attention over the uncompressed prompt, [bsz, L, H, D] out.

    16-bit CUDA inputs with head_dim 128 (the models of this path) run the
    sm_100a kernel (``ops.prefill_attention``: tcgen05 tensor cores, TMA,
    grouped-query without expanding K/V).  fp32 models take PyTorch's SDPA,
    with K/V heads expanded to the query heads so every SDPA backend can take
    it."""
    if q.is_cuda and q.dtype in (torch.bfloat16, torch.float16) and q.shape[-1] == ops.HEAD_DIM:
        return ops.prefill_attention(q, k, v, scale=scale)
    if groups > 1 and q.shape[-2] > 1:
        k = k.repeat_interleave(groups, dim=1)
        v = v.repeat_interleave(groups, dim=1)
        out = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale)
    else:
        out = F.scaled_dot_product_attention(q, k, v, is_causal=q.shape[-2] > 1, scale=scale,
                                             enable_gqa=groups > 1)
    return out.transpose(1, 2)


class _HeteroAttention(nn.Module):
    decode_select_before_attention = False
    qkv_bias = False
    o_bias = False

    def __init__(self, config, layer_idx: Optional[int] = None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = getattr(config, "head_dim", None) or self.hidden_size // self.num_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.scaling = self.head_dim ** -0.5
        self.attention_dropout = getattr(config, "attention_dropout", 0.0)
        self.is_causal = True
        qb = self._qkv_bias(config)
        self.q_proj = nn.Linear(self.hidden_size, self.num_heads * self.head_dim, bias=qb)
        self.k_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=qb)
        self.v_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=qb)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, self.hidden_size, bias=self._o_bias(config))

    def _qkv_bias(self, config) -> bool:
        return getattr(config, "attention_bias", False)

    def _o_bias(self, config) -> bool:
        return getattr(config, "attention_bias", False)

    def forward(self, hidden_states: torch.Tensor, position_embeddings: Tuple[torch.Tensor, torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None, past_key_values=None,
                cache_position: Optional[torch.LongTensor] = None, **kwargs):
        bsz, q_len, _ = hidden_states.shape
        hidden_shape = (bsz, q_len, -1, self.head_dim)
        q = self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        k = self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        v = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        cos, sin = position_embeddings
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        cache = past_key_values
        if cache is not None and not hasattr(cache, "prefill_select"):
            # another transformers cache (e.g. the DynamicCache a model builds by
            # default): plain causal attention over what it returns
            k, v = cache.update(k, v, self.layer_idx, {"cache_position": cache_position})
            out = F.scaled_dot_product_attention(q, k, v, is_causal=q_len > 1, scale=self.scaling,
                                                 enable_gqa=self.num_key_value_groups > 1)
            return self.o_proj(out.transpose(1, 2).reshape(bsz, q_len, -1).contiguous()), None
        if cache is None or q_len != 1:
            if cache is not None:
                k, v = cache.update(k, v, self.layer_idx, {"cache_position": cache_position})
                cache.init_coefficient(q, k, self.layer_idx)
                cache.prefill_select(q, k, v, self.layer_idx)
            out = _causal_attention(q, k, v, self.num_key_value_groups, self.scaling)
            return self.o_proj(out.reshape(bsz, q_len, -1).contiguous()), None
        # the query rides along so the page-append launch also stores it for
        # the drift check; the append itself is deferred: attention merges the
        # new token from k/v and appends it on the side stream
        cache.update(k, v, self.layer_idx, {"cache_position": cache_position, "query_states": q,
                                            "defer_append": True})
        if self.decode_select_before_attention:
            cache.decode_select(q, self.layer_idx)
        out = cache.attention(q, self.layer_idx, scale=self.scaling)  # [bsz, H, D]
        if not self.decode_select_before_attention:
            # the layer's attention is done: its drift check may wait for the
            # batch at the end of the step (or the next step's first update)
            if getattr(cache, "defer_checks", False):
                cache.decode_select(q, self.layer_idx, defer=True)
            else:
                cache.decode_select(q, self.layer_idx)
        return self.o_proj(out.reshape(bsz, 1, -1)), None


class LlamaAttention(_HeteroAttention):
    """Patched Llama attention (heterocache/llama_model.py:279-405)."""

    decode_select_before_attention = False


class Qwen2Attention(_HeteroAttention):
    """Patched Qwen2 attention (heterocache/qwen_model.py:93-212): q/k/v with
    bias, o_proj without; decode_select before the decode attention."""

    decode_select_before_attention = True

    def _qkv_bias(self, config) -> bool:
        return True

    def _o_bias(self, config) -> bool:
        return False


def patch_transformers() -> None:
    """Install the classes into transformers (heterocache/utils.py:195-197)."""
    import transformers
    transformers.models.llama.modeling_llama.LlamaAttention = LlamaAttention
    transformers.models.qwen2.modeling_qwen2.Qwen2Attention = Qwen2Attention
