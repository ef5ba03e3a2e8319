"""Head-role files: seeded synthetic generation and the runtime metadata derivation.

A role file is the JSON document HeteroCache's offline profiler writes
(tools/get_cluster.py:306-330): ``meta``, ``classification_matrix``,
``allocation_matrix`` and ``leader_member_relations``.  At load time the
reference permutes each layer's KV heads into the order
anchor -> satellite -> volatile -> pivot and derives four per-layer lists from
the permuted classification (heterocache/utils.py:71-175 and :300-343).  The
cache object only ever sees the derived, permuted document.

``synthetic_roles`` produces a role file without a model: a seeded star group
(one pivot plus satellites) and a seeded split of the remaining heads into
anchors and volatiles, with the profiler's inverse-stability allocation rule
(tools/get_cluster.py:281-305).  ``derive_runtime_data`` then applies the
load-time permutation and derivation exactly as the reference does.
"""
from __future__ import annotations

import copy
import json
from typing import Dict, List, Optional

import numpy as np

TYPE_MAP = {"anchor": 1, "volatile": 2, "pivot": 3, "satellite": 4}
# Sort key of the load-time permutation (heterocache/utils.py:101).
SORT_PRIORITY = {1: 0, 4: 1, 2: 2, 3: 3}


def synthetic_roles(num_layers: int, num_kv_heads: int, seed: int, *,
                    star_size: int = 4, n_anchor: Optional[int] = None,
                    n_stars: int = 1) -> Dict:
    """Seeded role file in the profiler's (un-permuted) layout.

    Per layer: a seeded permutation of the KV heads; the first ``n_stars``
    groups of ``star_size`` heads become stars (head 0 of a group is the
    pivot, the rest satellites); the remaining heads are split into
    ``n_anchor`` anchors (default: half, rounded down) and volatiles.
    Stability medians: anchor ~ U(0.5, 0.9), volatile ~ U(0.1, 0.5),
    satellites drawn 50/50 from the two ranges.  The profiler's precedence is
    pivot > satellite > unique (tools/get_cluster.py:254-274); pivots and
    volatiles get allocation -1 and every other head gets the model-wide
    inverse-stability share (tools/get_cluster.py:281-305).
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    cls: List[List[int]] = []
    med: List[List[float]] = []
    rel: List[Dict[str, List[int]]] = []
    counts = {k: 0 for k in TYPE_MAP}
    for _ in range(num_layers):
        perm = [int(x) for x in rng.permutation(num_kv_heads)]
        row_c = [0] * num_kv_heads
        row_m = [0.0] * num_kv_heads
        layer_rel: Dict[str, List[int]] = {}
        used = 0
        for s in range(n_stars):
            grp = perm[used:used + star_size]
            if len(grp) < 2:
                break
            used += len(grp)
            pivot, members = grp[0], sorted(grp[1:])
            layer_rel[str(pivot)] = members
            row_c[pivot] = TYPE_MAP["pivot"]
            row_m[pivot] = -1.0
            for m in members:
                row_c[m] = TYPE_MAP["satellite"]
                row_m[m] = float(rng.uniform(0.5, 0.9) if rng.random() < 0.5
                                 else rng.uniform(0.1, 0.5))
        rest = perm[used:]
        na = len(rest) // 2 if n_anchor is None else min(n_anchor, len(rest))
        for i, h in enumerate(rest):
            if i < na:
                row_c[h] = TYPE_MAP["anchor"]
                row_m[h] = float(rng.uniform(0.5, 0.9))
            else:
                row_c[h] = TYPE_MAP["volatile"]
                row_m[h] = -1.0
        for c in row_c:
            counts[{v: k for k, v in TYPE_MAP.items()}[c]] += 1
        cls.append(row_c)
        med.append(row_m)
        rel.append(layer_rel)

    # Inverse-stability allocation over every target head of the model.
    eps = 1e-6
    targets = [v for row in med for v in row if v > -0.5]
    total_inv = sum(1.0 / (v + eps) for v in targets)
    alloc = []
    for row in med:
        out = []
        for v in row:
            if v > -0.5 and total_inv > 1e-9:
                out.append((1.0 / (v + eps)) / total_inv * len(targets))
            else:
                out.append(v)
        alloc.append(out)
    return {
        "meta": {"type_map": dict(TYPE_MAP), "counts": counts},
        "classification_matrix": cls,
        "allocation_matrix": alloc,
        "leader_member_relations": rel,
    }


def layer_permutation(classification_row: List[int], num_kv_heads: int) -> List[int]:
    """Stable sort of one layer's KV heads by role priority
    (heterocache/utils.py:103-116): returns old head ids in new order."""
    row = classification_row[:num_kv_heads]
    return [i for i, _ in sorted(enumerate(row), key=lambda x: SORT_PRIORITY.get(x[1], 99))]


def derive_runtime_data(raw: Dict, num_layers: int, num_kv_heads: int) -> Dict:
    """Permute and derive the lists the cache object reads
    (heterocache/utils.py:300-343).

    Returns a deep copy holding the permuted ``allocation_matrix`` and
    ``classification_matrix``, the remapped ``leader_member_relations`` (keys
    keep the role file's insertion order, members are sorted) and, per layer:
    ``need_to_compress_counts`` (number of anchor + satellite heads, which sort
    first), ``need_to_select_counts`` (pivot ids), ``need_to_update_counts``
    (satellite ids) and ``need_to_keep_counts`` (volatile + pivot ids).
    """
    data = copy.deepcopy(raw)
    for key in ("need_to_update_counts", "need_to_select_counts",
                "need_to_compress_counts", "need_to_keep_counts"):
        data.setdefault(key, [])
    for layer in range(num_layers):
        perm = layer_permutation(data["classification_matrix"][layer], num_kv_heads)
        cls = [data["classification_matrix"][layer][i] for i in perm]
        alloc = [data["allocation_matrix"][layer][i] for i in perm]
        data["classification_matrix"][layer] = cls
        data["allocation_matrix"][layer] = alloc
        data["need_to_compress_counts"].append(cls.count(1) + cls.count(4))
        data["need_to_select_counts"].append([i for i, x in enumerate(cls) if x == 3])
        data["need_to_update_counts"].append([i for i, x in enumerate(cls) if x == 4])
        data["need_to_keep_counts"].append([i for i, x in enumerate(cls) if x in (2, 3)])
        old_to_new = {old: new for new, old in enumerate(perm)}
        new_rel = {}
        for old_leader, old_members in data["leader_member_relations"][layer].items():
            ol = int(old_leader)
            if ol in old_to_new:
                members = sorted(old_to_new[m] for m in old_members if m in old_to_new)
                new_rel[str(old_to_new[ol])] = members
        data["leader_member_relations"][layer] = new_rel
    return data


def full_head_count(data: Dict) -> int:
    """Model-wide volatile + pivot count (heterocache/cache_utils.py:640)."""
    c = data["meta"]["counts"]
    return int(c["volatile"]) + int(c["pivot"])


def check_budget(data: Dict, compression_ratio: float, num_layers: int, num_kv_heads: int) -> None:
    """The load-time feasibility assert (heterocache/utils.py:345-353)."""
    total = num_kv_heads * num_layers
    full = full_head_count(data)
    if not int(compression_ratio * total) > full:
        raise ValueError(
            "Too many full KV cache heads retained (volatile+pivot) to satisfy the "
            "compression ratio; lower the ratio or adjust clustering hyperparameters")


def load_role_file(path: str) -> Dict:
    with open(path, "r", encoding="utf-8") as f:
        raw = json.load(f)
    for key in ("meta", "classification_matrix", "allocation_matrix", "leader_member_relations"):
        if key not in raw:
            raise ValueError(f"role file {path!r} lacks {key!r}")
    counts = raw["meta"].get("counts", {})
    for key in ("volatile", "pivot"):
        if key not in counts:
            raise KeyError(f"role file {path!r}: meta.counts has no {key!r} entry")
    return raw
