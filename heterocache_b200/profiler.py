"""Offline head profiler: a HeteroCache role file (head classification,
allocation ratios, star clusters) from dumped attention weights -- the job of
the reference's tools/get_cluster.py -- with the per-dump work on the GPU.

For every dumped (layer, step) the top-k set of each head's last attention
row is computed on the device as a bitmap (``ops.profile_topk``: the mean
over a GQA group, avg-pool 5, top-k; tools/get_cluster.py:13-60), and set
overlaps are popcounts of bitmap intersections (``ops.profile_overlap``;
:62-69).  What follows -- medians of the overlaps with the prefill set,
the similarity graph at one decode step, greedy star clustering, the
inverse-stability allocation -- is a few hundred numbers per model and runs
on the host in the reference's order and arithmetic, so the JSON written is
the reference's (:117-330).  Equal pooled values at the top-k boundary go to
the lowest positions (torch.topk leaves their order unspecified).

    python -m heterocache_b200.profiler --tensor_save_dir ./tensor --model_path <model dir> \\
        --topk 1024 --max_length 5000 --stable_threshold 0.5 --sim_threshold 0.5 --decode_step 5000

Dumps already on the GPU (attention hooked in a live forward) go through
``HeadProfiler.analyze`` without touching the disk.
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import pathlib
from collections import defaultdict
from typing import Callable, Dict, List, Mapping, Optional, Set, Tuple, Union

import numpy as np
import torch

from . import ops
from .ops import Workspace

TYPE_MAP = {"anchor": 1, "volatile": 2, "pivot": 3, "satellite": 4}  # tools/get_cluster.py:133-138

Dump = Union[torch.Tensor, str]


def star_clusters(adjacency: Mapping[int, Set[int]], heads: List[int]) -> Tuple[Dict[int, List[int]], Set[int]]:
    """Greedy star clustering (tools/get_cluster.py:71-115): the unassigned
    head with the most unassigned neighbours (ties: the lowest index) leads,
    its unassigned neighbours become its satellites; until no head has one."""
    unassigned = set(heads)
    clusters: Dict[int, List[int]] = {}
    assigned: Set[int] = set()
    while unassigned:
        best = None
        for n in unassigned:
            nb = set(adjacency.get(n, set())) & unassigned
            key = (-len(nb), n)
            if best is None or key < best[0]:
                best = (key, n, nb)
        (neg_deg, _), lead, members = best
        if neg_deg == 0:
            break
        clusters[lead] = sorted(members)
        unassigned.remove(lead)
        assigned.add(lead)
        for m in clusters[lead]:
            unassigned.remove(m)
            assigned.add(m)
    return clusters, assigned


class HeadProfiler:
    """Head statistics of one model's dumps on one GPU.

    ``num_q_heads`` / ``num_kv_heads`` decide the GQA mean as the reference
    does: dumps that hold every query head of a GQA model are averaged over
    each KV head's group; any other dump is taken head by head.
    """

    def __init__(self, num_layers: int, num_q_heads: int, num_kv_heads: Optional[int] = None, *, topk: int = 1024,
                 max_length: int = 5000, device=None):
        self.num_layers = int(num_layers)
        self.num_q_heads = int(num_q_heads)
        self.num_kv_heads = int(num_kv_heads if num_kv_heads is not None else num_q_heads)
        self.topk = int(topk)
        self.max_length = int(max_length)
        self.device = torch.device(device if device is not None else "cuda")
        if self.device.type != "cuda":
            raise ValueError("heterocache_b200.profiler: the profiler runs on a CUDA device")
        self.ws = Workspace(self.device)

    # ---- per dump, on the device
    def head_bitmaps(self, attn: torch.Tensor) -> Tuple[torch.Tensor, int, int]:
        """Top-k bitmaps [bsz, effective heads, words] of one dump, with bsz
        and the effective head count.  A host tensor sends only its last
        query row, cut to max_length, to the device."""
        if attn.dim() == 3:
            attn = attn.unsqueeze(2)
        B, Hs, _, L = attn.shape
        g = self.num_q_heads // self.num_kv_heads if (
            self.num_q_heads != self.num_kv_heads and Hs == self.num_q_heads) else 1
        if not attn.is_cuda:
            attn = attn[:, :, -1:, :self.max_length].contiguous().to(self.device)
        bits = ops.profile_topk(attn, groups=g, topk=self.topk, max_length=self.max_length, workspace=self.ws)
        return bits, B, Hs // g

    def head_topk_sets(self, attn: torch.Tensor) -> Tuple[List[List[Set[int]]], int, int]:
        """The reference's get_head_topk_exact result (sets[head][batch row])
        from the device bitmaps."""
        bits, B, H = self.head_bitmaps(attn)
        words = bits.cpu().numpy().view(np.uint32)
        sets = [[set() for _ in range(B)] for _ in range(H)]
        for h in range(H):
            for b in range(B):
                pos = np.nonzero(np.unpackbits(words[b, h].view(np.uint8), bitorder="little"))[0]
                sets[h][b] = set(int(t) for t in pos)
        return sets, B, H

    @staticmethod
    def _ratios(inter: torch.Tensor, size_a: torch.Tensor, size_b: torch.Tensor) -> np.ndarray:
        """|a & b| / |a|, 0 where either set is empty (calculate_overlap_ratio)."""
        i, a, b = (x.cpu().numpy().astype(np.int64) for x in (inter, size_a, size_b))
        out = np.zeros(i.shape, dtype=np.float64)
        ok = (a > 0) & (b > 0)
        out[ok] = i[ok] / a[ok]
        return out

    # ---- the analysis
    def analyze(self, dumps: Mapping[int, Mapping[int, Dump]], *, stable_threshold: float = 0.5,
                sim_threshold: float = 0.5, decode_step: int = 5000,
                loader: Optional[Callable[[str], torch.Tensor]] = None) -> dict:
        """analyze_combined_heads (tools/get_cluster.py:117-330) over
        ``dumps[layer][step]`` (tensors, or file paths read by ``loader``);
        returns the JSON object the reference writes."""
        load = loader or (lambda path: torch.load(path, map_location="cpu"))
        total = self.num_q_heads
        cls = [[0] * total for _ in range(self.num_layers)]
        alloc = [[-1.0] * total for _ in range(self.num_layers)]
        relations: List[dict] = [{} for _ in range(self.num_layers)]
        counts = {k: 0 for k in TYPE_MAP}
        all_steps = sorted({s for by in dumps.values() for s in by})
        if not all_steps:
            raise ValueError("heterocache_b200.profiler: no dumps")
        prefill, decode_steps = all_steps[0], all_steps[1:]
        spatial = decode_step if decode_step in all_steps else all_steps[-1]

        def bitmaps_of(d: Dump):
            try:
                t = load(d) if isinstance(d, str) else d
            except Exception:
                return None
            return self.head_bitmaps(t)

        for layer in range(self.num_layers):
            if layer not in dumps or prefill not in dumps[layer]:
                continue
            got = bitmaps_of(dumps[layer][prefill])
            if got is None:
                continue
            base, B, H = got
            if H != total and layer == 0:
                cls = [[0] * H for _ in range(self.num_layers)]
                alloc = [[-1.0] * H for _ in range(self.num_layers)]
            base2 = base.reshape(B * H, -1)
            size_base = ops.profile_overlap(base2, base2, diagonal=True)
            history = defaultdict(list)
            spatial_bits = None
            for step in decode_steps:
                if step not in dumps[layer]:
                    continue
                got = bitmaps_of(dumps[layer][step])
                if got is None:
                    continue
                cur = got[0]
                if step == spatial:
                    spatial_bits = cur
                cur2 = cur.reshape(B * H, -1)
                r = self._ratios(ops.profile_overlap(base2, cur2, diagonal=True), size_base,
                                 ops.profile_overlap(cur2, cur2, diagonal=True)).reshape(B, H)
                for h in range(H):
                    ovs = [float(r[b, h]) for b in range(B)]
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
            # similarity graph at the spatial step (the reference indexes the
            # layer's dumps by that step: a missing one raises KeyError)
            src = dumps[layer][spatial]
            if spatial_bits is None or spatial == prefill:
                got = bitmaps_of(src)
                spatial_bits = got[0] if got is not None else None
            adj = defaultdict(set)
            if spatial_bits is not None:
                sim = np.zeros((H, H), dtype=np.float64)
                for b in range(B):
                    sb = spatial_bits[b]
                    c = ops.profile_overlap(sb, sb, diagonal=False).cpu().numpy().astype(np.int64)
                    size = np.diag(c)
                    for i in range(H):
                        for j in range(H):
                            if i != j:
                                sim[i, j] += (c[i, j] / size[i]) if (size[i] > 0 and size[j] > 0) else 0.0
                for i in range(H):
                    for j in range(H):
                        if i != j and sim[i, j] / B >= sim_threshold:
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
        # inverse-stability allocation over anchors and satellites (:256-305)
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
        return {"meta": {"type_map": dict(TYPE_MAP), "counts": counts}, "classification_matrix": cls,
                "allocation_matrix": alloc, "leader_member_relations": relations}


def scan_dumps(tensor_dir: str) -> Dict[int, Dict[int, str]]:
    """``attn_weights_{layer}_{step}.pt`` files by layer and step, parsed as
    the reference does (names that do not parse are skipped)."""
    files: Dict[int, Dict[int, str]] = defaultdict(dict)
    for f in glob.glob(os.path.join(tensor_dir, "attn_weights_*_*.pt")):
        try:
            parts = pathlib.Path(f).stem.split("_")
            files[int(parts[2])][int(parts[3])] = f
        except Exception:
            continue
    return files


def analyze_combined_heads(args, *, device=None, output: Optional[str] = None) -> dict:
    """The reference's entry point (tools/get_cluster.py:117-330) with the
    same arguments; writes the role JSON where the reference does (or to
    ``output``) and returns it."""
    from transformers import AutoConfig

    config = AutoConfig.from_pretrained(args.model_path, trust_remote_code=True)
    prof = HeadProfiler(config.num_hidden_layers, config.num_attention_heads,
                        getattr(config, "num_key_value_heads", config.num_attention_heads), topk=args.topk,
                        max_length=args.max_length, device=device)
    files = scan_dumps(args.tensor_save_dir)
    if not files:
        print("No tensor files found.")
        return {}
    result = prof.analyze(files, stable_threshold=args.stable_threshold, sim_threshold=args.sim_threshold,
                          decode_step=args.decode_step)
    model_name = os.path.basename(os.path.normpath(args.model_path)).lower()
    path = output or (f"./data/clusters/Head_Analysis_{model_name}_topk{args.topk}_th{args.stable_threshold}"
                      f"_sim{args.sim_threshold}_step{args.decode_step}.json")
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w", encoding="utf-8") as f:
        json.dump(result, f, indent=4)
    print(f"Type Counts: {result['meta']['counts']}")
    print(f"Results saved to: '{path}'")
    return result


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--tensor_save_dir", type=str, default="./tensor")
    p.add_argument("--model_path", type=str, default="../models/Llama-3.1-8B-Instruct")
    p.add_argument("--topk", type=int, default=1024)
    p.add_argument("--max_length", type=int, default=5000)
    p.add_argument("--stable_threshold", type=float, default=0.5)
    p.add_argument("--sim_threshold", type=float, default=0.5)
    p.add_argument("--decode_step", type=int, default=5000)
    p.add_argument("--output", type=str, default=None, help="JSON path (default: the reference's)")
    p.add_argument("--raw_tensor_dir", action="store_true",
                   help="read --tensor_save_dir as given (the reference appends <model>_tensors)")
    args = p.parse_args(argv)
    if not args.raw_tensor_dir:
        args.tensor_save_dir = os.path.join(args.tensor_save_dir,
                                            args.model_path.lower().split("/")[-1] + "_tensors")
    analyze_combined_heads(args, output=args.output)


if __name__ == "__main__":
    main()
