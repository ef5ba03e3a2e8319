"""End-to-end parity of the drop-in cache: GPU ``HeteroCache`` in lockstep with
the CPU oracle on the golden scenarios.

Per step: lengths and page tables bit-exact; prefill selections, pivot sets
and retrieval lists under the selection rule of ``tests/parity.py``; decode
attention within 2e-2 (bf16) / 1e-5 (fp32) of the oracle's attention over the
same pages.  Drift coefficients (overlap / K) may differ from the oracle's
only by the positions the parity rule leaves open: the exempt positions of
the step's top-K plus the positions where the two reference sets already
differ, divided by K; the triggers must agree unless the oracle's median lies
within that bound of the threshold.
"""
import pytest
import torch

from heterocache_b200.cache import HeteroCache, HeteroCacheConfig
from heterocache_b200.synthetic import DriftingDecode
from oracle.hc_oracle import OracleCache, paged_attention
from parity import compare_exact, compare_selection, exempt_count, near_flip_count, scores_close
from scenarios import SCENARIOS, make_config, scenario_inputs

pytestmark = pytest.mark.gpu

ATOL = {"float32": 1e-5, "bfloat16": 2e-2, "float16": 2e-2}


def _gpu_cache(sc, real_offload=False, ties="topk"):
    ns = make_config(sc)
    kw = dict(vars(ns))
    kw["real_offload"] = real_offload
    cfg = HeteroCacheConfig(**kw)
    cfg.record_checks = True
    return HeteroCache(cfg), OracleCache(ns, ties=ties)


def _compare(ref, dev, sel, k, dtype, exact):
    """The selection rule: tie-aware against the reference's own topk order,
    or, with the oracle breaking ties like the device (exact), identical sets
    up to flips within one rounding step of the k-th score."""
    if exact:
        return compare_exact(ref, dev, sel, k, dtype)
    return compare_selection(ref, dev, sel, k, dtype)


def _check_prefill(gpu, orc, sc, layer_inputs, dtype, exact=False):
    D = 128
    for layer, (q, k, v) in enumerate(layer_inputs):
        assert torch.equal(gpu.heads_len[layer].cpu(), orc.heads_len[layer]), layer
        assert torch.equal(gpu.block_tables[layer].cpu(), orc.block_tables[layer]), layer
        nc = gpu.data["need_to_compress_counts"][layer]
        bsz, KV = q.shape[0], gpu.num_kv_heads
        kp = gpu.key_pools[layer].cpu().view(-1, D)
        vp = gpu.value_pools[layer].cpu().view(-1, D)
        if nc and ("prefill_scores", layer) in gpu.recorded:
            dsc = gpu.recorded[("prefill_scores", layer)].float().cpu()
            idx = gpu.recorded[("prefill_indices", layer)].cpu()
            keep = gpu.recorded[("keep_lens", layer)].tolist()
            for b in range(bsz):
                for h in range(nc):
                    sel = idx[b, h, :keep[h]].tolist()
                    res = _compare(orc.prefill_scores[layer][b, h].float().numpy(), dsc[b, h].numpy(),
                                   sel, keep[h], dtype, exact)
                    assert res["ok"] and scores_close(res, dtype), (layer, b, h, res)
                    start = int(gpu.block_tables[layer][b * KV + h, 0]) * 256
                    assert torch.equal(kp[start:start + keep[h]], k[b, h, sel])
                    assert torch.equal(vp[start:start + keep[h]], v[b, h, sel])
        for h in gpu.data["need_to_keep_counts"][layer]:
            for b in range(bsz):
                start = int(gpu.block_tables[layer][b * KV + h, 0]) * 256
                L = k.shape[2]
                assert torch.equal(kp[start:start + L], k[b, h])
                assert torch.equal(vp[start:start + L], v[b, h])
        pivots = gpu.data["need_to_select_counts"][layer]
        if pivots:
            dsc = gpu.recorded[("pivot_scores", layer)].float().cpu()
            ref = gpu.prefill_topk_set[layer].cpu()
            for b in range(bsz):
                for i in range(len(pivots)):
                    res = _compare(orc.pivot_scores[layer][b, i].float().numpy(), dsc[b, i].numpy(),
                                   ref[b, i].tolist(), gpu.base_compress_len, dtype, exact)
                    assert res["ok"], (layer, b, i, res)


def _run(name, real_offload=False, ties="topk"):
    sc = SCENARIOS[name]
    geo, tdt, layer_inputs = scenario_inputs(sc)
    run_lockstep(sc, geo, tdt, layer_inputs, real_offload, ties)


def _device_query(q, L, dev):
    """The device query tensor [bsz, H, L, D]: zeros except the generated last
    positions (the path reads only the window queries at the end)."""
    if q.shape[2] == L:
        return q.to(dev)
    qd = torch.zeros(q.shape[0], q.shape[1], L, q.shape[3], dtype=q.dtype, device=dev)
    qd[:, :, L - q.shape[2]:] = q.to(dev)
    return qd


CHECKS = []  # drift decisions of the last lockstep run (device vs oracle)


def run_lockstep(sc, geo, tdt, layer_inputs, real_offload=False, ties="topk"):
    exact = ties == "lowest"
    gpu, orc = _gpu_cache(sc, real_offload, ties)
    CHECKS.clear()
    dtype = sc["dtype"]
    dev = torch.device("cuda", 0)
    for layer, (q, k, v) in enumerate(layer_inputs):
        qd, kd, vd = _device_query(q, k.shape[2], dev), k.to(dev), v.to(dev)
        gpu.update(kd, vd, layer)
        gpu.init_coefficient(qd, kd, layer)
        gpu.prefill_select(qd, kd, vd, layer)
        orc.update(k, v, layer)
        orc.init_coefficient(q, k, layer)
        orc.prefill_select(q, k, v, layer)
    torch.cuda.synchronize()
    gpu.check_errors()
    assert gpu.base_compress_len == orc.base_compress_len
    _check_prefill(gpu, orc, sc, layer_inputs, dtype, exact)
    if sc["n_decode"] == 0:
        return
    gens = [DriftingDecode(geo, bsz=1, seed=sc["seed"] * 1000 + l, q0=layer_inputs[l][0][:, :, -1:, :], dtype=tdt)
            for l in range(len(layer_inputs))]
    n_checks = 0
    for step in range(sc["n_decode"]):
        for layer in range(len(layer_inputs)):
            q, k, v = gens[layer].step()
            err_g = err_o = None
            try:
                orc.update(k, v, layer)
            except RuntimeError as e:
                err_o = str(e)
            try:
                gpu.update(k.to(dev), v.to(dev), layer)
            except RuntimeError as e:
                err_g = str(e)
            assert err_g == err_o, (step, err_g, err_o)
            if err_o is not None:
                assert sc.get("record_every") and "OOM" in err_o
                return
            out = gpu.attention(q.to(dev), layer)
            torch.cuda.synchronize()
            ref = paged_attention(q, gpu.key_pools[layer].cpu(), gpu.value_pools[layer].cpu(),
                                  gpu.block_tables[layer].cpu(), gpu.heads_len[layer].cpu(), gpu.num_kv_heads)
            diff = (out.float().cpu() - ref).abs().max().item()
            assert diff <= ATOL[dtype], (step, layer, diff)
            before = len(gpu.check_log)
            dev_sets = gpu.prefill_topk_set[layer]
            dev_sets = dev_sets.cpu() if isinstance(dev_sets, torch.Tensor) else None
            orc_sets = orc.prefill_topk_set[layer]
            orc_sets = orc_sets.clone() if isinstance(orc_sets, torch.Tensor) else None
            gpu.decode_select(q.to(dev), layer)
            n_before = len(orc.checks)
            orc.decode_select(q, layer)
            torch.cuda.synchronize()
            gpu.check_errors()
            assert torch.equal(gpu.heads_len[layer].cpu(), orc.heads_len[layer])
            assert torch.equal(gpu.block_tables[layer].cpu(), orc.block_tables[layer])
            new = orc.checks[n_before:]
            if len(gpu.check_log) > before:
                log = gpu.check_log[-1]
                assert len(new) == len(log["pivots"])
                K = gpu.base_compress_len
                for j, rec in enumerate(new):
                    n_checks += 1
                    trig = bool(log["trigger"][j].item())
                    slot = log["slots"][j]
                    # positions where the two reference sets already differ
                    set_diff = len(set(dev_sets[0, slot].tolist()) ^ set(orc_sets[0, slot].tolist()))
                    dsc = log["scores"][j].float().cpu()
                    S = dsc.shape[0]
                    coeff = log["coeffs"][j].cpu().tolist()
                    bound = []
                    for s_ in range(S):
                        if exact:  # each near-boundary flip moves at most two memberships
                            ex = 2 * near_flip_count(rec["scores"][0, s_].float().numpy(), dsc[s_].numpy(), K,
                                                     dtype)
                        else:
                            ex = exempt_count(rec["scores"][0, s_].float().numpy(), dsc[s_].numpy(), K, dtype)
                        bound.append((ex + set_diff) / K + 1e-7)
                        assert abs(coeff[s_] - rec["coeffs"][s_]) <= bound[-1], (step, s_, coeff, rec["coeffs"])
                    CHECKS.append({"trigger_dev": trig, "trigger_ref": bool(rec["trigger"]),
                                   "median_ref": float(rec["median"]), "bound": max(bound), "set_diff": set_diff})
                    if trig != rec["trigger"]:
                        assert abs(rec["median"] - sc["thr"]) <= max(bound), (step, rec["median"], max(bound))
                        continue
                    if trig:
                        ml = log["max_len"][j]
                        sel = log["retrieved"][j, :ml].cpu().tolist()
                        res = _compare(rec["scores"][0, -1].float().numpy(), dsc[S - 1].numpy(), sel, ml,
                                       dtype, exact)
                        assert res["ok"], (step, res)
                        res = _compare(rec["scores"][0, -1].float().numpy(), dsc[S - 1].numpy(),
                                       log["ref_after"][0, slot].cpu().tolist(), gpu.base_compress_len,
                                       dtype, exact)
                        assert res["ok"], (step, res)
            else:
                assert not new
    if any(gpu.data["leader_member_relations"][l] for l in range(len(layer_inputs))):
        assert n_checks > 0


@pytest.mark.parametrize("ties", ["topk", "lowest"])
@pytest.mark.parametrize("name", [n for n in SCENARIOS])
def test_cache_lockstep_with_oracle(cuda_device, name, ties):
    """ties="topk": the oracle as pinned to the reference (torch.topk's own
    order among equal scores; ties are exempt).  ties="lowest": the oracle
    breaks ties like the device, and the selections must be identical up to
    near-boundary flips."""
    _run(name, ties=ties)


def test_cache_host_tier(cuda_device):
    """Full tier in pinned host memory, retrieval on a side stream."""
    _run("llama_bf16_avg5", real_offload=True)


def test_config3_qwen_224k_host_tier(cuda_device):
    """Config 3 at its full context: Qwen2.5-7B layer geometry (28 query / 4 KV
    heads, G = 7), 229376 tokens, bf16, full tier in pinned host memory, in
    lockstep with the oracle through prefill and 10 decode steps (two drift
    checks; the threshold makes every check retrieve satellites from the host
    tier)."""
    from heterocache_b200.synthetic import QWEN_7B, prefill_inputs
    sc = dict(geo=(28, 4, 128), L=229376, dtype="bfloat16", pooling="avgpool", k=5, thr=0.999, steps=5,
              n_decode=10, gen=16, role_seed=21, seed=31, layers=1)
    inputs = [prefill_inputs(QWEN_7B, sc["L"], seed=sc["seed"] * 100, dtype=torch.bfloat16, q_positions=32)]
    run_lockstep(sc, QWEN_7B, torch.bfloat16, inputs, real_offload=True)


def test_config1_llama_32k_256_drifting_steps(cuda_device):
    """Config 1 exactly: one Llama-3.1-8B attention layer (32 query / 8 KV
    heads), 32768 tokens, bf16, compression ratio 0.5, the full KV in HBM,
    then 256 decode steps with drifting queries (q_t = 0.9 q_{t-1} + 0.1
    noise), a drift check every 5 steps (threshold 0.5, overlap K =
    base_compress_len), in lockstep with the oracle at every step."""
    from heterocache_b200.synthetic import LLAMA_8B, prefill_inputs
    sc = dict(geo=(32, 8, 128), L=32768, dtype="bfloat16", pooling="avgpool", k=5, thr=0.5, steps=5,
              n_decode=256, gen=264, role_seed=41, seed=43, layers=1)
    inputs = [prefill_inputs(LLAMA_8B, sc["L"], seed=sc["seed"] * 100, dtype=torch.bfloat16, q_positions=32)]
    # the oracle breaks score ties toward the lowest positions, as the device
    # does: selections must then be identical up to near-boundary flips
    run_lockstep(sc, LLAMA_8B, torch.bfloat16, inputs, ties="lowest")
    assert len(CHECKS) >= 256 // 5
    agree = sum(c["trigger_dev"] == c["trigger_ref"] for c in CHECKS)
    print(f"config 1: {len(CHECKS)} drift checks, {sum(c['trigger_ref'] for c in CHECKS)} oracle triggers, "
          f"{agree} decisions agree, largest reference-set difference {max(c['set_diff'] for c in CHECKS)}, "
          f"largest coefficient bound {max(c['bound'] for c in CHECKS):.2e}")


@pytest.mark.parametrize("order", ["llama", "qwen"])
def test_deferred_append_matches_immediate(cuda_device, order):
    """update(..., {"defer_append": True}): attention merges the step's token
    from its k/v and the page append runs afterwards on the side stream.
    Against the immediate append on the same inputs: attention outputs within
    the bf16 tolerance, and lengths, page tables, every page row and the drift
    triggers identical, in both call orders (Llama: decode_select after
    attention; Qwen: before)."""
    sc = SCENARIOS["llama_bf16_avg5"]
    geo, tdt, layer_inputs = scenario_inputs(sc)
    dev = torch.device("cuda", 0)
    caches = [_gpu_cache(sc)[0] for _ in range(2)]
    for c in caches:
        for layer, (q, k, v) in enumerate(layer_inputs):
            qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
            c.update(kd, vd, layer)
            c.init_coefficient(qd, kd, layer)
            c.prefill_select(qd, kd, vd, layer)
    gens = DriftingDecode(geo, bsz=1, seed=sc["seed"] * 1000, q0=layer_inputs[0][0][:, :, -1:, :], dtype=tdt)
    n_checks = 0
    for step in range(12):
        q, k, v = (t.to(dev) for t in gens.step())
        outs = []
        for c, defer in zip(caches, (False, True)):
            kw = {"query_states": q, "defer_append": defer}
            c.update(k, v, 0, kw)
            if order == "qwen":
                c.decode_select(q, 0)
            outs.append(c.attention(q, 0).float())
            if order == "llama":
                c.decode_select(q, 0)
            c.join_retrievals()
        torch.cuda.synchronize()
        assert (outs[0] - outs[1]).abs().max().item() <= 2e-2, step
        a, b = caches
        assert torch.equal(a.heads_len[0], b.heads_len[0]) and torch.equal(a.block_tables[0], b.block_tables[0])
        assert torch.equal(a.key_pools[0], b.key_pools[0]) and torch.equal(a.value_pools[0], b.value_pools[0])
        ja, jb = a._jobs[0], b._jobs[0]
        if ja is not None:
            assert torch.equal(ja.trigger, jb.trigger)
            n_checks += int(step % sc["steps"] == sc["steps"] - 1)
    for c in caches:
        c.check_errors()
    assert n_checks > 0


def test_host_tier_holds_only_the_satellites(cuda_device):
    """The pinned-host full tier keeps the satellites' rows only (the reference
    backs up every KV head, cache_utils.py:953-960; only satellites are read
    back): [bsz, n_sat, L, D] from the first satellite head on, bit-equal to
    the prefill K/V of those heads."""
    sc = SCENARIOS["llama_bf16_2layer_star8"]
    geo, tdt, layer_inputs = scenario_inputs(sc)
    gpu, _ = _gpu_cache(sc, real_offload=True)
    dev = cuda_device
    for layer, (q, k, v) in enumerate(layer_inputs):
        gpu.update(k.to(dev), v.to(dev), layer)
    torch.cuda.synchronize()
    for layer, (q, k, v) in enumerate(layer_inputs):
        sats = gpu.data["need_to_update_counts"][layer]
        tier = gpu.full_tier(layer)
        if not sats:
            assert tier is None
            continue
        fk, fv, first = tier
        assert fk.is_pinned() and fv.is_pinned()
        assert first == sats[0] and fk.shape[1] == len(sats) == sats[-1] - sats[0] + 1
        assert torch.equal(fk, k[:, sats[0]:sats[-1] + 1]) and torch.equal(fv, v[:, sats[0]:sats[-1] + 1])
