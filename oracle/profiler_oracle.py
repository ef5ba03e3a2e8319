"""CPU oracle for the offline head profiler (tools/get_cluster.py).

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module: the
profiler tests run it beside heterocache_b200.profiler (CUDA kernels for the
top-k sets and their intersections, host code for the rest).  It restates
the reference's analysis in plain PyTorch/numpy on the CPU:

  per dumped (layer, step): the last query row of each head (the mean over a
  GQA group when every query head was saved), avg_pool1d k = 5, the top-k
  positions as a set                                    -- :13-60
  overlap ratio |a & b| / |a|                           -- :62-69
  per head: the median over decode steps of the overlap with the prefill
  set -> anchor (>= stable threshold) or volatile       -- :200-231
  at one decode step: heads i -> j with overlap >= sim threshold, greedy star
  clusters (highest degree leads; ties to the lowest index) -> pivot and
  satellites                                            -- :71-115, :233-254
  allocation: inverse median over anchors and satellites, normalised to
  their count                                           -- :256-305

Equal pooled values at the top-k boundary go to the lowest positions (the
reference's torch.topk leaves that order unspecified; the fixtures have no
such ties).

Parity pin: tests/golden/make_profiler_golden.py runs the reference's own
analyze_combined_heads on seeded synthetic dumps (tests/golden/
profiler_cases.py) and commits its JSON; tests/test_profiler_oracle.py checks
this module against it exactly.
"""
from __future__ import annotations

from collections import defaultdict
from typing import Dict, List, Optional, Sequence, Set, Tuple

import numpy as np
import torch
import torch.nn.functional as F

TYPE_MAP = {"anchor": 1, "volatile": 2, "pivot": 3, "satellite": 4}  # tools/get_cluster.py:133-138


def head_topk_sets(attn: torch.Tensor, num_q_heads: int, num_kv_heads: int, topk: int,
                   max_length: int) -> Tuple[List[List[Set[int]]], int, int]:
    """get_head_topk_exact (tools/get_cluster.py:13-60) on a loaded dump."""
    if attn.dim() == 3:
        attn = attn.unsqueeze(2)
    B, Hs, _, L = attn.shape
    if num_q_heads != num_kv_heads and Hs == num_q_heads:
        G = num_q_heads // num_kv_heads
        rows = torch.mean(attn.view(B, num_kv_heads, G, -1, L), dim=2)
        He = num_kv_heads
    else:
        rows = attn
        He = Hs
    sets: List[List[Set[int]]] = [[set() for _ in range(B)] for _ in range(He)]
    for h in range(He):
        vec = rows[:, h, -1:, :max_length].sum(-2)
        if vec.shape[-1] == 0:
            continue
        ks = min(5, vec.shape[-1])
        vec = F.avg_pool1d(vec.float(), kernel_size=ks, padding=ks // 2, stride=1)
        k = min(topk, vec.shape[-1])
        if k == 0:
            continue
        for b in range(B):
            v = vec[b]
            # largest first, equal values by position
            order = sorted(range(v.shape[0]), key=lambda t: (-float(v[t]), t))
            sets[h][b] = set(order[:k])
    return sets, B, He


def overlap_ratio(a: Set[int], b: Set[int], topk: int) -> float:
    """calculate_overlap_ratio (tools/get_cluster.py:62-69)."""
    if not a or not b:
        return 0.0
    return len(a & b) / (len(a) if len(a) > 0 else topk)


def star_clusters(adjacency: Dict[int, Set[int]], heads: Sequence[int]) -> Tuple[Dict[int, List[int]], Set[int]]:
    """find_star_clusters_greedy (tools/get_cluster.py:71-115)."""
    unassigned = set(heads)
    clusters: Dict[int, List[int]] = {}
    assigned: Set[int] = set()
    while unassigned:
        cands = []
        for n in unassigned:
            nb = adjacency.get(n, set()) & unassigned
            cands.append((len(nb), n, nb))
        if not cands:
            break
        cands.sort(key=lambda x: (-x[0], x[1]))
        deg, lead, members = cands[0]
        if deg == 0:
            break
        clusters[lead] = sorted(members)
        unassigned.remove(lead)
        assigned.add(lead)
        for m in clusters[lead]:
            unassigned.remove(m)
            assigned.add(m)
    return clusters, assigned


def analyze(dumps: Dict[int, Dict[int, torch.Tensor]], *, num_layers: int, num_q_heads: int, num_kv_heads: int,
            topk: int, max_length: int, stable_threshold: float, sim_threshold: float, decode_step: int) -> dict:
    """analyze_combined_heads (tools/get_cluster.py:117-330) on in-memory dumps
    {layer: {step: attention}}; returns the JSON object it writes."""
    total = num_q_heads
    cls = [[0] * total for _ in range(num_layers)]
    alloc = [[-1.0] * total for _ in range(num_layers)]
    relations: List[dict] = [{} for _ in range(num_layers)]
    counts = {k: 0 for k in TYPE_MAP}
    all_steps = sorted({s for by in dumps.values() for s in by})
    if not all_steps:
        raise ValueError("no dumps")
    prefill, decode_steps = all_steps[0], all_steps[1:]
    spatial = decode_step if decode_step in all_steps else all_steps[-1]

    def sets_of(t):
        return head_topk_sets(t, num_q_heads, num_kv_heads, topk, max_length)

    for layer in range(num_layers):
        if layer not in dumps or prefill not in dumps[layer]:
            continue
        base, B, H = sets_of(dumps[layer][prefill])
        if H != total and layer == 0:
            cls = [[0] * H for _ in range(num_layers)]
            alloc = [[-1.0] * H for _ in range(num_layers)]
        history = defaultdict(list)
        for step in decode_steps:
            if step not in dumps[layer]:
                continue
            cur, _, _ = sets_of(dumps[layer][step])
            for h in range(H):
                ovs = [overlap_ratio(base[h][b], cur[h][b], topk) for b in range(B)]
                history[h].append(sum(ovs) / len(ovs) if ovs else 0)
        dyn, med = {}, {}
        for h in range(H):
            hist = history[h]
            if not hist:
                dyn[h], med[h] = "volatile", 0.0
            else:
                m = np.median(hist)
                dyn[h] = "volatile" if m < stable_threshold else "anchor"
                med[h] = float(m)
        sp, _, _ = sets_of(dumps[layer][spatial])
        adj = defaultdict(set)
        for i in range(H):
            for j in range(H):
                if i == j:
                    continue
                s = sum(overlap_ratio(sp[i][b], sp[j][b], topk) for b in range(B))
                if s / B >= sim_threshold:
                    adj[i].add(j)
        clusters, assigned = star_clusters(adj, list(range(H)))
        relations[layer] = clusters
        for h in range(H):
            alloc[layer][h] = med[h]
            if h in clusters:
                cls[layer][h] = TYPE_MAP["pivot"]
                counts["pivot"] += 1
                alloc[layer][h] = -1.0
            elif h in assigned:
                cls[layer][h] = TYPE_MAP["satellite"]
                counts["satellite"] += 1
            elif dyn[h] == "anchor":
                cls[layer][h] = TYPE_MAP["anchor"]
                counts["anchor"] += 1
            else:
                cls[layer][h] = TYPE_MAP["volatile"]
                counts["volatile"] += 1
                alloc[layer][h] = -1.0
    targets = [v for row in alloc for v in row if v > -0.5]
    n = len(targets)
    eps = 1e-6
    inv_total = 0.0
    for v in targets:
        inv_total += 1.0 / (v + eps)
    if n > 0 and inv_total > 1e-9:
        for r in range(len(alloc)):
            for c in range(len(alloc[r])):
                v = alloc[r][c]
                if v > -0.5:
                    alloc[r][c] = (1.0 / (v + eps)) / inv_total * n
    return {"meta": {"type_map": TYPE_MAP, "counts": counts}, "classification_matrix": cls,
            "allocation_matrix": alloc, "leader_member_relations": relations}


def to_json_obj(result: dict) -> dict:
    """The object as it reads back from the reference's JSON file (dict keys
    become strings)."""
    import json
    return json.loads(json.dumps(result))
