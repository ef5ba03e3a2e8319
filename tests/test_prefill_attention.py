"""The drop-in attention's prompt attention for fp32 models (K/V heads
expanded to the query heads before SDPA; 16-bit CUDA inputs take the sm_100a
kernel, tested in test_gpu_prefill_attention.py) against a plain fp32 causal
grouped-query softmax.  Output layout [bsz, L, H, D]."""
import math

import torch

from heterocache_b200.attention import _causal_attention


def _reference(q, k, v, groups, scale):
    L = q.shape[-2]
    k = k.repeat_interleave(groups, dim=1).float()
    v = v.repeat_interleave(groups, dim=1).float()
    logits = torch.matmul(q.float(), k.transpose(-1, -2)) * scale
    mask = torch.ones(L, L, dtype=torch.bool).triu(1)
    logits = logits.masked_fill(mask, float("-inf"))
    return torch.matmul(torch.softmax(logits, dim=-1), v)


def test_causal_attention_grouped_query_prompt():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 8, 37, 128, generator=g)
    k = torch.randn(1, 2, 37, 128, generator=g)
    v = torch.randn(1, 2, 37, 128, generator=g)
    out = _causal_attention(q, k, v, 4, 1 / math.sqrt(128))
    assert out.shape == (1, 37, 8, 128)
    ref = _reference(q, k, v, 4, 1 / math.sqrt(128)).transpose(1, 2)
    assert torch.allclose(out, ref, atol=1e-5, rtol=1e-5)


def test_causal_attention_single_query_attends_to_all_keys():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 8, 1, 128, generator=g)
    k = torch.randn(1, 2, 9, 128, generator=g)
    v = torch.randn(1, 2, 9, 128, generator=g)
    out = _causal_attention(q, k, v, 4, 0.1)
    kk, vv = k.repeat_interleave(4, dim=1), v.repeat_interleave(4, dim=1)
    ref = torch.matmul(torch.softmax(torch.matmul(q, kk.transpose(-1, -2)) * 0.1, dim=-1), vv)
    assert torch.allclose(out, ref.transpose(1, 2), atol=1e-5, rtol=1e-5)
