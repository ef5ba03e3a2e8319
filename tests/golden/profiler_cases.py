"""Seeded synthetic attention dumps for the offline head profiler.

The reference's profiler (tools/get_cluster.py) reads ``attn_weights_{layer}_
{step}.pt`` files that tools/get_weights.py dumps from an eager forward of a
real model: softmax attention [bsz, heads, q_len, keys] in the model dtype,
one file per layer and sequence length (the prefill length, then each decode
length).  No model or dataset is available here, so these cases build dumps
of that shape from a seeded generator with the structure the profiler looks
for: per layer some heads keep their heavy hitters over the decode steps
(stable), some redraw them (volatile), and star groups of heads share a
pivot's profile (similar).  Every (layer, step, batch row, effective head)
row is checked to have no equal pooled values at the top-k boundary, so that
the reference's torch.topk and any tie rule pick the same set.

Used by tests/golden/make_profiler_golden.py (which runs the reference on
them) and by the profiler tests (which rebuild the same dumps).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

CASES = {
    # Llama-like GQA dumps (every query head saved): the mean over 4 heads
    "llama_gqa_f16": dict(layers=3, q_heads=32, kv_heads=8, saved="q", dtype="float16", bsz=1, prefill=512,
                          decode=8, q_rows=3, max_length=512, topk=48, stable=0.5, sim=0.5, decode_step=516,
                          seed=101),
    # Qwen-like groups of 7, two batch rows, bf16, a max_length below the
    # prompt, the spatial step absent (the last step is used)
    "qwen_gqa_bf16_b2": dict(layers=2, q_heads=28, kv_heads=4, saved="q", dtype="bfloat16", bsz=2, prefill=300,
                             decode=6, q_rows=2, max_length=280, topk=32, stable=0.6, sim=0.4, decode_step=999,
                             seed=202),
    # dumps of the KV heads only (no mean), fp16
    "kv_saved_f16": dict(layers=2, q_heads=32, kv_heads=8, saved="kv", dtype="float16", bsz=1, prefill=256,
                         decode=5, q_rows=1, max_length=1000, topk=40, stable=0.5, sim=0.5, decode_step=258,
                         seed=303),
}

_DT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def steps_of(case: dict) -> list[int]:
    p = case["prefill"]
    return [p] + [p + 1 + i for i in range(case["decode"])]


def _head_roles(gen: torch.Generator, n: int) -> list[tuple[str, int]]:
    """(role, leader) per effective head: one or two star groups, the rest
    split between stable and volatile."""
    perm = torch.randperm(n, generator=gen).tolist()
    roles: list[tuple[str, int]] = [("", -1)] * n
    i = 0
    for _ in range(1 + (n >= 8)):
        size = 2 + int(torch.randint(0, 2, (1,), generator=gen))
        lead = perm[i]
        roles[lead] = ("stable", lead)
        for m in perm[i + 1:i + size]:
            roles[m] = ("member", lead)
        i += size
    for j, h in enumerate(perm[i:]):
        roles[h] = ("stable" if j % 2 == 0 else "volatile", h)
    return roles


def make_dumps(case: dict) -> dict[int, dict[int, torch.Tensor]]:
    """{layer: {step: attention [bsz, saved heads, q_rows or 1, step]}} in the case's dtype."""
    gen = torch.Generator().manual_seed(case["seed"])
    dt = _DT[case["dtype"]]
    kv, qh, bsz = case["kv_heads"], case["q_heads"], case["bsz"]
    G = qh // kv
    saved = qh if case["saved"] == "q" else kv
    steps = steps_of(case)
    Lmax = steps[-1]
    out: dict[int, dict[int, torch.Tensor]] = {}
    for layer in range(case["layers"]):
        roles = _head_roles(gen, kv)
        base = torch.randn(bsz, kv, Lmax, generator=gen)
        hot = torch.rand(bsz, kv, Lmax, generator=gen) < 0.08
        base = base + 5.0 * hot
        out[layer] = {}
        for si, step in enumerate(steps):
            prof = base.clone()
            for h, (role, lead) in enumerate(roles):
                if role == "member":
                    prof[:, h] = base[:, lead] + 0.35 * torch.randn(bsz, Lmax, generator=gen)
                elif role == "volatile" and si > 0:
                    redraw = torch.randn(bsz, Lmax, generator=gen)
                    prof[:, h] = redraw + 5.0 * (torch.rand(bsz, Lmax, generator=gen) < 0.08)
                else:
                    prof[:, h] = base[:, h] + 0.3 * torch.randn(bsz, Lmax, generator=gen)
            q_rows = case["q_rows"] if si == 0 else 1
            # query heads: the effective profile plus a little noise each
            logits = prof[:, :, None, None, :step].expand(bsz, kv, G, q_rows, step).clone()
            logits = logits + 0.2 * torch.randn(bsz, kv, G, q_rows, step, generator=gen)
            attn = torch.softmax(logits.reshape(bsz, qh, q_rows, step), dim=-1, dtype=torch.float32).to(dt)
            if saved == kv:
                attn = attn.view(bsz, kv, G, q_rows, step)[:, :, 0].contiguous()
            out[layer][step] = attn
    return out


def boundary_ties(case: dict, dumps: dict) -> int:
    """Rows whose pooled values tie at the top-k boundary (0 for a usable case)."""
    kv, qh = case["kv_heads"], case["q_heads"]
    ties = 0
    for layer in dumps.values():
        for attn in layer.values():
            B, Hs, _, L = attn.shape
            if qh != kv and Hs == qh:
                rows = torch.mean(attn.view(B, kv, qh // kv, -1, L), dim=2)
            else:
                rows = attn
            n = min(case["max_length"], L)
            for h in range(rows.shape[1]):
                vec = rows[:, h, -1:, :n].sum(-2).float()
                ks = min(5, n)
                vec = F.avg_pool1d(vec, kernel_size=ks, padding=ks // 2, stride=1)
                k = min(case["topk"], vec.shape[-1])
                srt = vec.sort(dim=-1, descending=True).values
                if k < vec.shape[-1]:
                    ties += int((srt[:, k - 1] == srt[:, k]).sum())
    return ties
