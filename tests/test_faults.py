"""Failure paths that need no GPU: malformed role files and what the cache
does with them (the reference's ``KeyError`` at heterocache/cache_utils.py:641
and heterocache/utils.py:349 for a file whose ``meta.counts`` uses other role
names, as the shipped Qwen2.5-14B file does), and the library's handling of
a bounded-wait limit set from the host."""
import json

import pytest

from heterocache_b200.cache import HeteroCache, HeteroCacheConfig
from heterocache_b200.roles import check_budget, derive_runtime_data, load_role_file, synthetic_roles


def _write(tmp_path, doc):
    path = tmp_path / "roles.json"
    path.write_text(json.dumps(doc))
    return str(path)


def test_role_file_with_other_role_names_raises_key_error(tmp_path):
    """A file whose meta.counts names the roles differently (e.g.
    Stable_Unique / Unstable_Unique / Leader / Member) lacks the 'volatile'
    and 'pivot' counts the cache reads: KeyError, as in the reference."""
    doc = synthetic_roles(2, 8, seed=1)
    counts = doc["meta"]["counts"]
    doc["meta"]["counts"] = {"Stable_Unique": counts["anchor"], "Unstable_Unique": counts["volatile"],
                             "Leader": counts["pivot"], "Member": counts["satellite"]}
    with pytest.raises(KeyError, match="volatile"):
        load_role_file(_write(tmp_path, doc))
    data = derive_runtime_data(doc, 2, 8)
    with pytest.raises(KeyError):
        HeteroCache(HeteroCacheConfig(data, num_layers=2))


def test_role_file_missing_a_section_is_rejected(tmp_path):
    doc = synthetic_roles(1, 8, seed=2)
    del doc["allocation_matrix"]
    with pytest.raises(ValueError, match="allocation_matrix"):
        load_role_file(_write(tmp_path, doc))


def test_role_file_that_cannot_meet_the_budget_is_rejected():
    """utils.py:345-353: more full (volatile + pivot) heads than the ratio allows."""
    doc = synthetic_roles(1, 8, seed=3, n_anchor=0)  # star of 4 + 4 volatile heads
    data = derive_runtime_data(doc, 1, 8)
    with pytest.raises(ValueError, match="Too many full KV cache heads"):
        check_budget(data, 0.5, 1, 8)


def test_wait_limits_are_set_and_restored_without_a_gpu():
    from heterocache_b200 import ops
    ops.set_wait_limits(1_000_000, inject_stall=True)
    ops.set_wait_limits(0, inject_stall=False)  # the defaults again
