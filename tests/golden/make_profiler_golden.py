"""Generate the offline profiler's golden fixtures by running the reference.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_profiler_golden.py --reference <path to HeteroCache checkout>

For every case in ``profiler_cases.py`` this writes the seeded dumps as
``attn_weights_{layer}_{step}.pt`` into a temporary directory, writes a
model config (``config.json`` with the case's layer and head counts) beside
them, imports the reference's ``tools/get_cluster.py`` unchanged and runs its
``analyze_combined_heads`` on them, then stores the JSON it wrote (and the
per-head top-k sets of get_head_topk_exact for the first layer) as
``profiler_<case>.json`` next to this file.  Only those JSON files travel.
"""
from __future__ import annotations

import argparse
import contextlib
import glob
import importlib.util
import json
import os
import sys
import tempfile
from types import SimpleNamespace

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from profiler_cases import CASES, boundary_ties, make_dumps, steps_of  # noqa: E402


@contextlib.contextmanager
def _cwd(path):
    old = os.getcwd()
    os.chdir(path)
    try:
        yield
    finally:
        os.chdir(old)


def _load_reference(ref_root: str):
    spec = importlib.util.spec_from_file_location("get_cluster", os.path.join(ref_root, "tools", "get_cluster.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_case(ref, name: str, case: dict) -> dict:
    dumps = make_dumps(case)
    assert boundary_ties(case, dumps) == 0, name
    with tempfile.TemporaryDirectory() as tmp:
        model = os.path.join(tmp, "model")
        os.makedirs(model)
        cfg = {"model_type": "llama", "num_hidden_layers": case["layers"], "num_attention_heads": case["q_heads"],
               "num_key_value_heads": case["kv_heads"], "hidden_size": case["q_heads"] * 128,
               "intermediate_size": 256, "vocab_size": 32}
        with open(os.path.join(model, "config.json"), "w") as f:
            json.dump(cfg, f)
        tdir = os.path.join(tmp, "tensors")
        os.makedirs(tdir)
        for layer, by_step in dumps.items():
            for step, t in by_step.items():
                torch.save(t, os.path.join(tdir, f"attn_weights_{layer}_{step}.pt"))
        args = SimpleNamespace(tensor_save_dir=tdir, model_path=model, topk=case["topk"],
                               max_length=case["max_length"], stable_threshold=case["stable"],
                               sim_threshold=case["sim"], decode_step=case["decode_step"])
        with _cwd(tmp):
            os.makedirs(os.path.join("data", "clusters"))
            ref.analyze_combined_heads(args)
            out = glob.glob(os.path.join("data", "clusters", "*.json"))
            assert len(out) == 1, out
            with open(out[0]) as f:
                result = json.load(f)
        # the per-head sets of the first layer's prefill and last step
        from transformers import AutoConfig
        config = AutoConfig.from_pretrained(model)
        sets = {}
        for step in (steps_of(case)[0], steps_of(case)[-1]):
            s, B, H = ref.get_head_topk_exact(os.path.join(tdir, f"attn_weights_0_{step}.pt"), args, config)
            sets[str(step)] = [[sorted(s[h][b]) for b in range(B)] for h in range(H)]
    return {"case": case, "expected": result, "layer0_sets": sets}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    ref = _load_reference(a.reference)
    for name, case in CASES.items():
        res = run_case(ref, name, case)
        with open(os.path.join(HERE, f"profiler_{name}.json"), "w") as f:
            json.dump(res, f, indent=1)
        print(name, res["expected"]["meta"]["counts"])


if __name__ == "__main__":
    main()
