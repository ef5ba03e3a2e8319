"""The CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py``, which runs the
reference's ``HeteroCache`` and ``SnapKVCluster`` unchanged on the same seeded
inputs.  Every recorded quantity must match bit for bit: kept positions per
compressed head, page tables, lengths, pivot reference sets, retrieved
satellite rows, and SHA-256 digests of the whole key/value pools.
"""
import json
import os

import pytest
import torch

from oracle.hc_oracle import OracleCache, snapkv_indices
from scenarios import SCENARIOS, make_config, run_scenario

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    with open(os.path.join(GOLDEN, f"{name}.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("name", sorted(SCENARIOS))
def test_oracle_matches_reference(name):
    sc = SCENARIOS[name]
    gold = _load(name)
    cfg = make_config(sc)
    cache = OracleCache(cfg)
    rec = run_scenario(cache, sc, cfg.data)
    assert cache.base_compress_len == gold["base_compress_len"]
    assert rec["oom_step"] == gold["oom_step"]
    if "oom_msg" in gold:
        assert rec["oom_msg"] == gold["oom_msg"]
    assert len(rec["prefill"]) == len(gold["prefill"])
    for mine, ref in zip(rec["prefill"], gold["prefill"]):
        for key in ("heads_len", "block_table", "kept", "topk_set_sorted",
                    "k_pool_digest", "v_pool_digest"):
            assert mine[key] == ref[key], (name, key)
    assert len(rec["decode"]) == len(gold["decode"])
    for mine, ref in zip(rec["decode"], gold["decode"]):
        assert mine["step"] == ref["step"]
        for ml, rl in zip(mine["layers"], ref["layers"]):
            for key in ("heads_len", "block_table_digest", "topk_set_sorted",
                        "satellite_rows", "k_pool_digest", "v_pool_digest"):
                assert ml[key] == rl[key], (name, mine["step"], key)


def test_golden_scenarios_exercise_triggers():
    """The fixtures must cover both a fired and a quiet drift check."""
    fired, quiet = 0, 0
    for name, sc in SCENARIOS.items():
        if sc["n_decode"] == 0:
            continue
        cfg = make_config(sc)
        cache = OracleCache(cfg)
        run_scenario(cache, sc, cfg.data)
        for c in cache.checks:
            fired += int(c["trigger"])
            quiet += int(not c["trigger"])
    assert fired > 0 and quiet > 0, (fired, quiet)


@pytest.mark.parametrize("name", ["snapkv_f32_w32_max7", "snapkv_bf16_w32_max7", "snapkv_f32_w8_avg5"])
def test_window_math_matches_reference_snapkv(name):
    gold = _load(name)
    case = gold["case"]
    from make_golden import snapkv_inputs
    q, k, v = snapkv_inputs(case)
    idx = snapkv_indices(q, k, window=case["window"], kernel_size=case["k"], pooling=case["pooling"],
                         capacity=case["cap"])
    assert idx[0].tolist() == gold["kept"]
