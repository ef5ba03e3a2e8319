"""The profiler oracle (oracle/profiler_oracle.py) against the reference's own
output: tests/golden/profiler_*.json were written by running the reference's
tools/get_cluster.py (analyze_combined_heads, get_head_topk_exact) on the
seeded dumps of tests/golden/profiler_cases.py.  Exact equality of the whole
JSON object: classification, allocation ratios (floats), star clusters."""
import json
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from oracle import profiler_oracle as po  # noqa: E402
from profiler_cases import CASES, make_dumps, steps_of  # noqa: E402


def _golden(name):
    with open(os.path.join(HERE, "golden", f"profiler_{name}.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_profiler(name):
    g = _golden(name)
    case = g["case"]
    assert case == CASES[name]
    dumps = make_dumps(case)
    res = po.analyze(dumps, num_layers=case["layers"], num_q_heads=case["q_heads"], num_kv_heads=case["kv_heads"],
                     topk=case["topk"], max_length=case["max_length"], stable_threshold=case["stable"],
                     sim_threshold=case["sim"], decode_step=case["decode_step"])
    assert po.to_json_obj(res) == g["expected"]
    for step, exp in g["layer0_sets"].items():
        sets, B, H = po.head_topk_sets(dumps[0][int(step)], case["q_heads"], case["kv_heads"], case["topk"],
                                       case["max_length"])
        assert [[sorted(sets[h][b]) for b in range(B)] for h in range(H)] == exp


def test_star_clusters_take_the_highest_degree_lowest_index_first():
    adj = {0: {1}, 1: {0, 2, 3}, 2: {1, 3}, 3: {2, 1}, 4: {5}, 5: {4}}
    clusters, assigned = po.star_clusters(adj, list(range(7)))
    # head 1 has degree 3; then 4 and 5 tie at degree 1 and 4 leads
    assert clusters == {1: [0, 2, 3], 4: [5]}
    assert assigned == {0, 1, 2, 3, 4, 5}


def test_overlap_ratio_of_empty_sets_is_zero():
    assert po.overlap_ratio(set(), {1}, 8) == 0.0
    assert po.overlap_ratio({1, 2}, {2, 3}, 8) == 0.5


def test_cases_have_steps_in_order():
    for c in CASES.values():
        s = steps_of(c)
        assert s == sorted(s) and len(s) == c["decode"] + 1
