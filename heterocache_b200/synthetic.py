"""Seeded synthetic inputs with the shapes of the benchmark configurations.

No dataset or checkpoint is used.  Every tensor is generated in fp32 on the
CPU from ``torch.Generator("cpu").manual_seed(seed)`` and only then cast, so a
device run and a CPU check see identical bits.

* ``prefill_inputs``: Q/K/V ~ N(0, 1) in the attention layer's
  ``[bsz, heads, L, head_dim]`` layout.  In each KV head, 1% of the key
  positions are planted heavy hitters: ``K += 4 * normalize(mean of the
  group's query heads over the last ``window`` queries)``.
* ``DriftingDecode``: per step a query that drifts,
  ``q_t = 0.9 * q_{t-1} + 0.1 * N(0, 1)``, plus fresh N(0, 1) keys/values.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch


@dataclass
class LayerGeometry:
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128

    @property
    def groups(self) -> int:
        return self.num_heads // self.num_kv_heads


LLAMA_8B = LayerGeometry(32, 8, 128)
QWEN_7B = LayerGeometry(28, 4, 128)


def prefill_inputs(geo: LayerGeometry, seq_len: int, *, bsz: int = 1, seed: int = 0,
                   window: int = 32, planted_frac: float = 0.01, planted_scale: float = 4.0,
                   dtype: torch.dtype = torch.float32,
                   q_positions: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Seeded q/k/v [bsz, heads, seq_len, D] with planted heavy hitters.  With
    ``q_positions`` only the last that many query positions are generated
    (q is [bsz, H, q_positions, D]): the path reads the window queries only,
    which keeps long-context inputs small."""
    g = torch.Generator("cpu").manual_seed(seed)
    H, KV, D, G = geo.num_heads, geo.num_kv_heads, geo.head_dim, geo.groups
    qn = seq_len if q_positions is None else min(q_positions, seq_len)
    q = torch.randn(bsz, H, qn, D, generator=g)
    k = torch.randn(bsz, KV, seq_len, D, generator=g)
    v = torch.randn(bsz, KV, seq_len, D, generator=g)
    n_plant = max(1, int(round(planted_frac * seq_len)))
    w = min(window, qn)
    for b in range(bsz):
        for h in range(KV):
            mean_q = q[b, h * G:(h + 1) * G, qn - w:, :].mean(dim=(0, 1))
            direction = mean_q / mean_q.norm().clamp_min(1e-12)
            pos = torch.randperm(seq_len, generator=g)[:n_plant]
            k[b, h, pos, :] += planted_scale * direction
    return q.to(dtype), k.to(dtype), v.to(dtype)


def prefill_kv_device(geo: LayerGeometry, seq_len: int, q_last: torch.Tensor, *, seed: int, device,
                      dtype: torch.dtype = torch.bfloat16, planted_frac: float = 0.01,
                      planted_scale: float = 4.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Benchmark-size K/V generated on the device (same recipe as
    ``prefill_inputs``: N(0,1) plus planted heavy hitters along the group's
    mean query direction over the window ``q_last`` [bsz, H, W, D])."""
    g = torch.Generator(device=device).manual_seed(seed)
    bsz = q_last.shape[0]
    KV, D, G = geo.num_kv_heads, geo.head_dim, geo.groups
    k = torch.randn(bsz, KV, seq_len, D, generator=g, device=device, dtype=torch.float32)
    v = torch.randn(bsz, KV, seq_len, D, generator=g, device=device, dtype=torch.float32)
    n_plant = max(1, int(round(planted_frac * seq_len)))
    mean_q = q_last.float().view(bsz, KV, G, -1, D).mean(dim=(2, 3))  # [bsz, KV, D]
    direction = mean_q / mean_q.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    pos = torch.randint(0, seq_len, (bsz, KV, n_plant), generator=g, device=device)
    add = torch.zeros_like(k)
    add.scatter_(2, pos.unsqueeze(-1).expand(-1, -1, -1, D), (planted_scale * direction).unsqueeze(2)
                 .expand(-1, -1, n_plant, -1).contiguous())
    k += add
    return k.to(dtype), v.to(dtype)


class DriftingDecode:
    """Per-step decode inputs: ``q_t = 0.9 q_{t-1} + 0.1 noise``; fresh k, v."""

    def __init__(self, geo: LayerGeometry, *, bsz: int = 1, seed: int = 1,
                 q0: torch.Tensor = None, dtype: torch.dtype = torch.float32):
        self.geo, self.bsz, self.dtype = geo, bsz, dtype
        self.g = torch.Generator("cpu").manual_seed(seed)
        H, D = geo.num_heads, geo.head_dim
        self.q = (q0.float().clone() if q0 is not None
                  else torch.randn(bsz, H, 1, D, generator=self.g))

    def step(self) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        H, KV, D = self.geo.num_heads, self.geo.num_kv_heads, self.geo.head_dim
        noise = torch.randn(self.bsz, H, 1, D, generator=self.g)
        self.q = 0.9 * self.q + 0.1 * noise
        k = torch.randn(self.bsz, KV, 1, D, generator=self.g)
        v = torch.randn(self.bsz, KV, 1, D, generator=self.g)
        return self.q.to(self.dtype), k.to(self.dtype), v.to(self.dtype)
