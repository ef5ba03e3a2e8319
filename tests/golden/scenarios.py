"""Golden scenarios shared by the fixture generator and the oracle pin test.

Each scenario is a seeded single- or two-layer run of the cache path:
prefill (``update`` -> ``init_coefficient`` -> ``prefill_select`` per layer)
followed by ``n_decode`` decode steps (``update`` -> ``decode_select``).
``run_scenario`` drives any object with the reference cache's method surface
and returns a compact, comparable record of everything the path produces.
"""
from __future__ import annotations

import hashlib
from types import SimpleNamespace
from typing import Dict, List

import numpy as np
import torch

from heterocache_b200.roles import derive_runtime_data, synthetic_roles
from heterocache_b200.synthetic import DriftingDecode, LayerGeometry, prefill_inputs

PAGE = 256

SCENARIOS: Dict[str, Dict] = {
    # Llama-3.1-8B layer geometry, fp32, HeteroCache defaults (avgpool 5).
    "llama_f32_avg5": dict(geo=(32, 8, 128), L=2048, dtype="float32", pooling="avgpool", k=5,
                           thr=0.5, steps=5, n_decode=15, gen=64, role_seed=3, seed=11, layers=1),
    # Same, threshold high enough that every check triggers a retrieval.
    "llama_f32_trigger": dict(geo=(32, 8, 128), L=2048, dtype="float32", pooling="avgpool", k=5,
                              thr=0.999, steps=5, n_decode=10, gen=64, role_seed=3, seed=12, layers=1),
    "llama_bf16_avg5": dict(geo=(32, 8, 128), L=2048, dtype="bfloat16", pooling="avgpool", k=5,
                            thr=0.999, steps=5, n_decode=10, gen=64, role_seed=4, seed=13, layers=1),
    "llama_f32_max7": dict(geo=(32, 8, 128), L=1000, dtype="float32", pooling="maxpool", k=7,
                           thr=0.999, steps=5, n_decode=10, gen=32, role_seed=5, seed=14, layers=1),
    "qwen_bf16": dict(geo=(28, 4, 128), L=1536, dtype="bfloat16", pooling="avgpool", k=5,
                      thr=0.999, steps=5, n_decode=10, gen=32, role_seed=6, seed=15, layers=1),
    # Two layers; layer roles include a star of 8 (1 pivot + 7 satellites).
    "llama_bf16_2layer_star8": dict(geo=(32, 8, 128), L=1280, dtype="bfloat16", pooling="avgpool", k=5,
                                    thr=0.999, steps=4, n_decode=8, gen=16, role_seed=7, seed=16, layers=2,
                                    star=8),
    # Batch of 2, prefill only (decode_select assumes bsz 1).  The pool is
    # sized per KV head, not per batch row (cache_utils.py:704-723), so a
    # batch of 2 only fits when max_gen_len leaves room for the second row.
    "llama_f32_bsz2_prefill": dict(geo=(32, 8, 128), L=777, dtype="float32", pooling="avgpool", k=5,
                                   thr=0.5, steps=5, n_decode=0, gen=1024, role_seed=8, seed=17, layers=1,
                                   bsz=2),
    # Free list exhaustion: keep heads cross a page at step 1 and run out later.
    "llama_f32_oom": dict(geo=(32, 8, 128), L=512, dtype="float32", pooling="avgpool", k=5,
                          thr=0.5, steps=5, n_decode=300, gen=2, role_seed=9, seed=18, layers=1,
                          record_every=25),
}


def make_config(sc: Dict, cfg_cls=None):
    """Config object with the reference ``HeteroCacheConfig`` fields."""
    H, KV, D = sc["geo"]
    layers = sc.get("layers", 1)
    raw = synthetic_roles(layers, KV, sc["role_seed"], star_size=sc.get("star", 4))
    data = derive_runtime_data(raw, layers, KV)
    kw = dict(data=data, compression_ratio=0.5, stable_threshold=sc["thr"], real_offload=False,
              max_gen_len=sc["gen"], decode_step=sc["steps"], pooling=sc["pooling"],
              kernel_size=sc["k"], num_attn_heads=H, num_kv_heads=KV, num_layers=layers)
    if cfg_cls is None:
        return SimpleNamespace(**kw)
    return cfg_cls(**kw)


def scenario_inputs(sc: Dict):
    H, KV, D = sc["geo"]
    geo = LayerGeometry(H, KV, D)
    dtype = getattr(torch, sc["dtype"])
    bsz = sc.get("bsz", 1)
    layers = []
    for layer in range(sc.get("layers", 1)):
        layers.append(prefill_inputs(geo, sc["L"], bsz=bsz, seed=sc["seed"] * 100 + layer, dtype=dtype))
    return geo, dtype, layers


def _bytes(row: torch.Tensor) -> bytes:
    return row.contiguous().view(torch.uint8).numpy().tobytes()


def _row_index(full: torch.Tensor) -> Dict[bytes, int]:
    return {_bytes(full[t]): t for t in range(full.shape[0])}


def _recover(pool_flat: torch.Tensor, start_row: int, n: int, index: Dict[bytes, int]) -> List[int]:
    return [index.get(_bytes(pool_flat[r]), -1) for r in range(start_row, start_row + n)]


def _f64sum(t: torch.Tensor) -> float:
    return float(t.double().sum())


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()[:32]


def run_scenario(cache, sc: Dict, data: Dict) -> Dict:
    """Drive ``cache`` (reference HeteroCache or the oracle) and record results."""
    geo, dtype, layer_inputs = scenario_inputs(sc)
    KV, G, D = geo.num_kv_heads, geo.groups, geo.head_dim
    rec: Dict = {"prefill": [], "decode": [], "oom_step": -1}
    for layer, (q, k, v) in enumerate(layer_inputs):
        cache.update(k, v, layer, None)
        cache.init_coefficient(q, k, layer)
        cache.prefill_select(q, k, v, layer)
    for layer, (q, k, v) in enumerate(layer_inputs):
        bsz = q.shape[0]
        kp = cache.key_pools[layer].view(-1, D)
        kept = {}
        n_comp = data["need_to_compress_counts"][layer]
        for b in range(bsz):
            for h in range(n_comp):
                row = b * KV + h
                n = int(cache.heads_len[layer][row])
                start = int(cache.block_tables[layer][row, 0])
                index = _row_index(k[b, h])
                kept[f"{b}_{h}"] = _recover(kp, start * PAGE, n, index) if start >= 0 else []
        pts = cache.prefill_topk_set[layer]
        rec["prefill"].append({
            "heads_len": cache.heads_len[layer].tolist(),
            "block_table": cache.block_tables[layer].tolist(),
            "kept": kept,
            "topk_set_sorted": (pts.sort(dim=-1).values.tolist() if isinstance(pts, torch.Tensor) else []),
            "k_pool_sum": _f64sum(cache.key_pools[layer]),
            "v_pool_sum": _f64sum(cache.value_pools[layer]),
            "k_pool_digest": _digest(cache.key_pools[layer]),
            "v_pool_digest": _digest(cache.value_pools[layer]),
        })
    if sc["n_decode"] == 0:
        return rec
    gens = [DriftingDecode(geo, bsz=1, seed=sc["seed"] * 1000 + layer,
                           q0=layer_inputs[layer][0][:, :, -1:, :], dtype=dtype)
            for layer in range(len(layer_inputs))]
    for step in range(sc["n_decode"]):
        step_rec = []
        try:
            for layer in range(len(layer_inputs)):
                q, k, v = gens[layer].step()
                cache.update(k, v, layer, None)
                cache.decode_select(q, layer)
                pts = cache.prefill_topk_set[layer]
                sat = {}
                full_k = layer_inputs[layer][1]
                check_step = (step + 1) % sc["steps"] == 0
                for m in (data["need_to_update_counts"][layer] if check_step else []):
                    start = int(cache.block_tables[layer][m, 0])
                    n = int(cache.heads_len[layer][m])
                    sat[str(m)] = _recover(cache.key_pools[layer].view(-1, D), start * PAGE, n,
                                           _row_index(full_k[0, m])) if start >= 0 else []
                step_rec.append({
                    "heads_len": cache.heads_len[layer].tolist(),
                    "block_table_digest": _digest(cache.block_tables[layer]),
                    "topk_set_sorted": (pts.sort(dim=-1).values.tolist() if isinstance(pts, torch.Tensor) else []),
                    "satellite_rows": sat,
                    "k_pool_digest": _digest(cache.key_pools[layer]),
                    "v_pool_digest": _digest(cache.value_pools[layer]),
                })
        except RuntimeError as e:
            if "OOM" in str(e):
                rec["oom_step"] = step
                rec["oom_msg"] = str(e)
                break
            raise
        if step % sc.get("record_every", 1) == 0:
            rec["decode"].append({"step": step, "layers": step_rec})
    return rec
