"""Offline head profiler on the GPU (heterocache_b200.profiler, kernels
hc_profile_topk / hc_profile_overlap) against the oracle and the reference's
own output (tests/golden/profiler_*.json, written by the reference's
tools/get_cluster.py on the seeded dumps of tests/golden/profiler_cases.py):
top-k sets bit for bit, and the whole role JSON exactly."""
import json
import os
import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from heterocache_b200 import ops, profiler
from heterocache_b200.ops import Workspace

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from oracle import profiler_oracle as po  # noqa: E402
from profiler_cases import CASES, make_dumps  # noqa: E402

pytestmark = pytest.mark.gpu


def _golden(name):
    with open(os.path.join(HERE, "golden", f"profiler_{name}.json")) as f:
        return json.load(f)


def _sets_from_bits(bits: torch.Tensor):
    w = bits.cpu().numpy().view(np.uint32)
    B, H, _ = w.shape
    return [[set(np.nonzero(np.unpackbits(w[b, h].view(np.uint8), bitorder="little"))[0].tolist())
             for b in range(B)] for h in range(H)]


@pytest.mark.parametrize("name", sorted(CASES))
def test_profiler_matches_reference_json(cuda_device, name):
    g = _golden(name)
    case = g["case"]
    dumps = make_dumps(case)
    prof = profiler.HeadProfiler(case["layers"], case["q_heads"], case["kv_heads"], topk=case["topk"],
                                 max_length=case["max_length"], device=cuda_device)
    res = prof.analyze(dumps, stable_threshold=case["stable"], sim_threshold=case["sim"],
                       decode_step=case["decode_step"])
    assert json.loads(json.dumps(res)) == g["expected"]
    for step, exp in g["layer0_sets"].items():
        sets, B, H = prof.head_topk_sets(dumps[0][int(step)])
        assert [[sorted(sets[h][b]) for b in range(B)] for h in range(H)] == exp


def test_profiler_reads_dump_files_like_the_reference(cuda_device, tmp_path):
    """analyze_combined_heads on files: the reference's file names, config and
    output JSON (indent 4, string keys) from a model directory."""
    name = "llama_gqa_f16"
    g = _golden(name)
    case = g["case"]
    model = tmp_path / "model"
    model.mkdir()
    (model / "config.json").write_text(json.dumps(
        {"model_type": "llama", "num_hidden_layers": case["layers"], "num_attention_heads": case["q_heads"],
         "num_key_value_heads": case["kv_heads"], "hidden_size": case["q_heads"] * 128, "intermediate_size": 256,
         "vocab_size": 32}))
    tdir = tmp_path / "tensors"
    tdir.mkdir()
    for layer, by in make_dumps(case).items():
        for step, t in by.items():
            torch.save(t, tdir / f"attn_weights_{layer}_{step}.pt")
    (tdir / "attn_weights_0_prefill.pt").write_bytes(b"not parsed")  # skipped by name, as the reference does
    out = tmp_path / "roles.json"
    args = SimpleNamespace(tensor_save_dir=str(tdir), model_path=str(model), topk=case["topk"],
                           max_length=case["max_length"], stable_threshold=case["stable"], sim_threshold=case["sim"],
                           decode_step=case["decode_step"])
    profiler.analyze_combined_heads(args, device=cuda_device, output=str(out))
    assert json.loads(out.read_text()) == g["expected"]


@pytest.mark.parametrize("dtype,B,Hs,q,kv,L,max_len,topk,Q", [
    (torch.float16, 1, 32, 32, 8, 5001, 5000, 1024, 1),   # the reference's defaults, GQA mean of 4
    (torch.bfloat16, 2, 28, 28, 4, 3000, 4096, 700, 2),    # groups of 7, all positions used
    (torch.float32, 1, 32, 32, 8, 2048, 2048, 100, 1),     # fp32 dump, groups of 4
    (torch.float16, 3, 8, 32, 8, 777, 500, 600, 1),        # KV heads saved; topk above the row
    (torch.bfloat16, 1, 8, 8, 8, 4, 4, 3, 1),              # 4 positions: pooling kernel 4, 5 pooled values
    (torch.float16, 1, 8, 8, 8, 2, 10, 10, 1),             # 2 positions: kernel 2, 3 pooled values
    (torch.float16, 1, 8, 8, 8, 1, 10, 10, 1),             # 1 position
    (torch.float16, 1, 8, 8, 8, 300, 0, 10, 1),            # max_length 0: empty sets
    (torch.bfloat16, 1, 4, 4, 4, 40000, 131072, 8000, 1),  # long row
])
def test_topk_sets_match_the_oracle(cuda_device, dtype, B, Hs, q, kv, L, max_len, topk, Q):
    gen = torch.Generator().manual_seed(L + topk)
    logits = torch.randn(B, Hs, Q, L, generator=gen) * 3
    attn = torch.softmax(logits, dim=-1).to(dtype)
    exp, eB, eH = po.head_topk_sets(attn, q, kv, topk, max_len)
    g = q // kv if (q != kv and Hs == q) else 1
    bits = ops.profile_topk(attn.to(cuda_device), groups=g, topk=topk, max_length=max_len,
                            workspace=Workspace(cuda_device))
    torch.cuda.synchronize()
    got = _sets_from_bits(bits)
    assert (len(got), len(got[0])) == (eH, eB)
    assert got == exp


def test_topk_ties_take_the_lowest_positions(cuda_device):
    """A row of equal values: the first k positions (the oracle's rule)."""
    attn = torch.full((1, 2, 1, 500), 1 / 500, dtype=torch.float16)
    attn[0, 1, 0, 100:110] = 0.5  # ten larger values, then ties
    bits = ops.profile_topk(attn.to(cuda_device), groups=1, topk=20, max_length=500,
                            workspace=Workspace(cuda_device))
    got = _sets_from_bits(bits)
    exp, _, _ = po.head_topk_sets(attn, 2, 2, 20, 500)
    assert got == exp
    # interior positions pool to equal values (the two at each edge see padding)
    assert got[0][0] == set(range(2, 22))


def test_topk_reads_strided_device_views(cuda_device):
    gen = torch.Generator().manual_seed(9)
    big = torch.softmax(torch.randn(2, 16, 5, 1200, generator=gen), dim=-1).to(torch.bfloat16)
    view = big.to(cuda_device)[:, ::2]  # every other head: a strided view
    bits = ops.profile_topk(view, groups=1, topk=64, max_length=1000, workspace=Workspace(cuda_device))
    exp, _, _ = po.head_topk_sets(big[:, ::2].contiguous(), 8, 8, 64, 1000)
    assert _sets_from_bits(bits) == exp


def test_overlap_counts(cuda_device):
    gen = torch.Generator().manual_seed(3)
    a = torch.randint(-2**31, 2**31 - 1, (5, 37), generator=gen, dtype=torch.int64).to(torch.int32)
    b = torch.randint(-2**31, 2**31 - 1, (7, 37), generator=gen, dtype=torch.int64).to(torch.int32)
    au, bu = a.numpy().view(np.uint32), b.numpy().view(np.uint32)
    pop = np.vectorize(lambda x: bin(int(x)).count("1"))
    full = ops.profile_overlap(a.to(cuda_device), b.to(cuda_device), diagonal=False).cpu().numpy()
    exp = np.array([[pop(au[i] & bu[j]).sum() for j in range(7)] for i in range(5)])
    assert (full == exp).all()
    diag = ops.profile_overlap(a.to(cuda_device), b[:5].to(cuda_device), diagonal=True).cpu().numpy()
    assert (diag == np.array([pop(au[i] & bu[i]).sum() for i in range(5)])).all()
