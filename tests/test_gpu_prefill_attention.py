"""hc_prefill_attention (tcgen05 causal grouped-query attention) against an
fp32 PyTorch reference of the same op: softmax(q k^T * scale, causal) v with
K/V heads shared by G query heads.  Tolerance: 2e-2 max-abs for bf16/fp16
outputs (the reference's flash-attn forward keeps P in the 16-bit type too)."""
import math

import pytest
import torch

from heterocache_b200 import ops

pytestmark = pytest.mark.gpu


def _reference(q, k, v, scale):
    """fp32 causal attention, [bsz, L, H, D] out."""
    bsz, H, L, D = q.shape
    G = H // k.shape[1]
    out = torch.empty(bsz, L, H, D, dtype=torch.float32, device=q.device)
    mask = torch.ones(L, L, dtype=torch.bool, device=q.device).tril()
    for h in range(H):
        qh = q[:, h].float()
        kh, vh = k[:, h // G].float(), v[:, h // G].float()
        s = torch.matmul(qh, kh.transpose(-1, -2)) * scale
        s = s.masked_fill(~mask, float("-inf"))
        out[:, :, h] = torch.matmul(torch.softmax(s, dim=-1), vh)
    return out


@pytest.mark.parametrize("dtype,H,KV,L,bsz", [
    ("bfloat16", 32, 8, 1, 1),
    ("bfloat16", 32, 8, 127, 1),
    ("bfloat16", 32, 8, 128, 1),
    ("bfloat16", 32, 8, 129, 1),
    ("bfloat16", 32, 8, 1000, 1),
    ("bfloat16", 32, 8, 4096, 1),
    ("float16", 28, 4, 3000, 1),
    ("bfloat16", 8, 8, 700, 2),
    ("float16", 16, 2, 513, 2),
])
def test_prefill_attention_matches_fp32_reference(cuda_device, dtype, H, KV, L, bsz):
    torch.backends.cuda.matmul.allow_tf32 = False
    tdt = getattr(torch, dtype)
    g = torch.Generator(device=cuda_device).manual_seed(L * 7 + H)
    D = 128
    # the projections' layout: [bsz, L, H, D] viewed as [bsz, H, L, D]
    q = torch.randn(bsz, L, H, D, generator=g, device=cuda_device).to(tdt).transpose(1, 2)
    k = torch.randn(bsz, L, KV, D, generator=g, device=cuda_device).to(tdt).transpose(1, 2)
    v = torch.randn(bsz, L, KV, D, generator=g, device=cuda_device).to(tdt).transpose(1, 2)
    # a few large logits, so that the running max grows and O is rescaled
    q[:, :, L // 2:] *= 3
    scale = 1.0 / math.sqrt(D)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = ops.prefill_attention(q, k, v, scale=scale, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = _reference(q, k, v, scale)
    diff = (out.float() - ref).abs().max().item()
    assert diff <= 2e-2, diff


def test_prefill_attention_contiguous_heads_and_default_scale(cuda_device):
    """[bsz, H, L, D]-contiguous inputs, scale 0 (= 1/sqrt(D)), into a given out."""
    tdt, dev = torch.bfloat16, cuda_device
    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(1, 4, 600, 128, generator=g, device=dev).to(tdt)
    k = torch.randn(1, 2, 600, 128, generator=g, device=dev).to(tdt)
    v = torch.randn(1, 2, 600, 128, generator=g, device=dev).to(tdt)
    out = torch.full((1, 600, 4, 128), 7.0, dtype=tdt, device=dev)
    ops.prefill_attention(q, k, v, out=out)
    torch.cuda.synchronize()
    diff = (out.float() - _reference(q, k, v, 1 / math.sqrt(128))).abs().max().item()
    assert diff <= 2e-2, diff
