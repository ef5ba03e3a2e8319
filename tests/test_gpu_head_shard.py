"""Head-sharded mode on 2 GPUs (NCCL) against the single-GPU cache.

Each rank holds 4 of the 8 KV heads (and their 16 query heads); the seeded
roles put a pivot and some of its satellites on different ranks, so the
drift check's position list crosses ranks by broadcast.  Per decode step:
the all-gathered attention output matches the single-GPU cache's (same
kernels; only the split-K partition differs), the drift triggers match, and
every head's page contents (prefill selection, retrieved satellite rows,
appended tokens) are bit-identical.  Skipped with fewer than 2 GPUs.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rows(cache, layer, head):
    D = cache.head_dim
    kp = cache.key_pools[layer].view(-1, D)
    vp = cache.value_pools[layer].view(-1, D)
    n = int(cache.heads_len[layer][head])
    bt = cache.block_tables[layer][head]
    idx = torch.arange(n, device=kp.device)
    slots = bt[(idx // 256)].long() * 256 + idx % 256
    return kp[slots], vp[slots]


def _setup(dev, data, layers, KV, H, L, caches):
    """Prefill the single-GPU cache and the shards on the same inputs."""
    from heterocache_b200.synthetic import LLAMA_8B, DriftingDecode, prefill_inputs
    full, shards = caches
    gens = []
    for layer in range(layers):
        q, k, v = prefill_inputs(LLAMA_8B, L, seed=40 + layer, dtype=torch.bfloat16)
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        full.update(kd, vd, layer)
        full.init_coefficient(qd, kd, layer)
        full.prefill_select(qd, kd, vd, layer)
        for sh in shards:
            ki, qi = sh.head_index(layer, dev), sh.head_index(layer, dev, query=True)
            qs, ksl, vsl = qd.index_select(1, qi), kd.index_select(1, ki), vd.index_select(1, ki)
            sh.update(ksl, vsl, layer)
            sh.init_coefficient(qs, ksl, layer)
            sh.prefill_select(qs, ksl, vsl, layer)
        gens.append(DriftingDecode(LLAMA_8B, seed=70 + layer, q0=q[:, :, -1:, :], dtype=torch.bfloat16))
    return gens


def _config(layers=2, KV=8, H=32):
    from heterocache_b200.cache import HeteroCacheConfig
    from heterocache_b200.roles import derive_runtime_data, synthetic_roles
    # 8 KV heads, one star of 4: the role order puts satellites on both head
    # blocks of 2 ranks and the pivot on the second, so the star crosses ranks
    data = derive_runtime_data(synthetic_roles(layers, KV, 3), layers, KV)
    return HeteroCacheConfig(data, compression_ratio=0.5, stable_threshold=0.999, real_offload=False,
                             max_gen_len=32, decode_step=5, pooling="avgpool", kernel_size=5, num_attn_heads=H,
                             num_kv_heads=KV, num_layers=layers)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("balance", [False, True], ids=["contiguous", "balanced"])
def test_head_sharded_emulated_on_one_gpu(cuda_device, balance, world):
    """Every rank of a 2-, 4- or 8-way head split in one process on one GPU:
    the sharding logic (budgets, local roles, cross-rank position lists,
    remote retrievals; at 8 ranks a cache of one KV head, a pivot whose
    satellites all sit elsewhere) against the single cache.  Contiguous head
    blocks exchange the position lists as copies of the broadcast buffers;
    capacity-balanced head sets through mailboxes (``publish_remote`` into
    every other rank's buffer, ``retrieve_remote_mail``), as the kernel-side
    gather does across GPUs."""
    from heterocache_b200.cache import HeteroCache
    from heterocache_b200.head_shard import HeadShardedCache
    dev = cuda_device
    layers, KV, H, L = 2, 8, 32, 4096
    full = HeteroCache(_config(layers, KV, H))
    shards = [HeadShardedCache(_config(layers, KV, H), r, world, balance=balance) for r in range(world)]
    if balance:
        assert any(sh.kv_heads(0) != list(range(sh.rank * KV // world, (sh.rank + 1) * KV // world))
                   for sh in shards)
    assert sum(len(s) for s in shards[0].remote) > 0
    gens = _setup(dev, full.data, layers, KV, H, L, (full, shards))
    # stand-ins for the ranks' PeerGather mailboxes, all on this GPU
    import types
    base = [sum(shards[0].remote_words(x) for x in range(l)) for l in range(layers)]
    words = sum(shards[0].remote_words(x) for x in range(layers))
    assert all(sum(sh.remote_words(x) for x in range(layers)) == words for sh in shards)
    mails = [torch.full((max(words, 1),), -1, dtype=torch.int32, device=dev) for _ in shards]
    boxes = [types.SimpleNamespace(mail=mails[r], mail_ptrs=[m.data_ptr() for m in mails]) for r in range(world)]
    n_trig = 0
    for step in range(12):
        for layer in range(layers):
            q, k, v = (t.to(dev) for t in gens[layer].step())
            full.update(k, v, layer)
            qi = [sh.head_index(layer, dev, query=True) for sh in shards]
            for sh in shards:
                ki = sh.head_index(layer, dev)
                sh.update(k.index_select(1, ki), v.index_select(1, ki), layer)
            o_full = full.attention(q, layer)
            o = torch.cat([sh.cache.attention(q.index_select(1, qi[sh.rank]), layer) for sh in shards], dim=1)
            order = torch.tensor(shards[0].gathered_heads(layer), device=dev)
            assert (o_full.index_select(1, order).float() - o.float()).abs().max().item() <= 2e-2, (step, layer)
            full.decode_select(q, layer)
            checks = [sh.select_local(q.index_select(1, qi[sh.rank]), layer) for sh in shards]
            assert len(set(checks)) == 1
            if checks[0] and balance:
                # the mailbox path: each pivot rank stores its lists into the
                # other ranks' mailboxes (one GPU, one stream: in order)
                for sh in shards:
                    sh.publish_remote(layer, boxes[sh.rank], base[layer])
                for sh in shards:
                    sh.retrieve_remote_mail(layer, boxes[sh.rank], base[layer])
            elif checks[0]:
                for si, spec in enumerate(shards[0].remote[layer]):
                    bufs = [sh.stage_positions(layer, si) for sh in shards]
                    for r in range(world):
                        if r != spec["src"]:
                            bufs[r].copy_(bufs[spec["src"]])
                    for sh in shards:
                        sh.retrieve_remote(layer, si)
            torch.cuda.synchronize()
            jf = full._jobs[layer]
            for sh in shards:
                js = sh.cache._jobs[layer]
                if jf is not None and js is not None and js.n_jobs:
                    assert torch.equal(jf.trigger[:jf.n_jobs].cpu(), js.trigger[:js.n_jobs].cpu()), (step, layer)
                    n_trig += int(js.trigger[:js.n_jobs].sum())
                for h, g in enumerate(sh.kv_heads(layer)):
                    a, b = _rows(full, layer, g), _rows(sh.cache, layer, h)
                    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]), (step, layer, sh.rank, h)
    full.check_errors()
    for sh in shards:
        sh.check_errors()
    assert n_trig > 0


@pytest.mark.parametrize("balance", [False, True], ids=["contiguous", "balanced"])
def test_head_sharded_two_gpus_match_single_gpu(tmp_path, balance):
    """The real thing: 2 processes, one GPU each, NCCL all-gather and
    broadcast (launched with torch.distributed.run; each rank writes its
    comparison result to a file)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import json
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", HC_SHARD_OUT=str(tmp_path), HC_SHARD_BALANCE=str(int(balance)))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(here, "head_shard_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    (tmp_path / "workers.log").write_text(proc.stdout + proc.stderr)
    errs = [ln for ln in (proc.stdout + proc.stderr).splitlines() if "rror" in ln or "what()" in ln]
    assert proc.returncode == 0, "\n".join(errs[:40]) + proc.stderr[-2000:]
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    for r in res:
        assert "error" not in r, r
        assert r["same_rows"] and r["same_trig"], r
        assert r["max_diff"] <= 2e-2, r
        assert r["crossing"] > 0, r
        # the gather by the decode kernels over NVLink: the NCCL result bit for bit
        assert r["peer_exact"] and r["peer_diff"] <= 2e-2, r
        # position lists through the mailboxes: the same pages and triggers as
        # through NCCL broadcasts
        assert r["mail_rows"] and r["mail_trig"] and r["n_mail"] > 0, r
    assert sum(r["n_trig"] for r in res) > 0


def test_peer_gather_one_rank_writes_the_gathered_output(cuda_device):
    """PeerGather on one rank: the decode combine's mirror stores land in the
    gathered buffer, equal to the returned output (the 2-GPU test covers
    stores into another GPU's memory)."""
    from heterocache_b200.cache import HeteroCache
    from heterocache_b200.head_shard import HeadShardedCache, PeerGather
    dev = cuda_device
    layers, KV, H, L = 1, 8, 32, 2048
    shard = HeadShardedCache(_config(layers, KV, H), 0, 1)
    ref = HeteroCache(_config(layers, KV, H))
    gens = _setup(dev, ref.data, layers, KV, H, L, (ref, [shard]))
    peer = PeerGather(1, H, 128, torch.bfloat16, 0, 1, device=dev)
    for step in range(7):
        q, k, v = (t.to(dev) for t in gens[0].step())
        ref.update(k, v, 0)
        shard.update(k, v, 0)
        o = ref.attention(q, 0)
        peer.barrier()
        shard.attention(q, 0, peer=peer, row0=0)
        peer.barrier()
        torch.cuda.synchronize()
        assert torch.equal(peer.out, o), step
        ref.decode_select(q, 0)
        shard.decode_select(q, 0)
    peer.check_errors()
    assert int(peer.counter.item()) == 14


def test_peer_barrier_times_out_when_a_rank_never_arrives(cuda_device):
    """A 2-rank barrier whose other rank never signals (its flag slot is a
    buffer nothing writes): the bounded wait gives up and reports
    HC_ERR_TIMEOUT; the context stays usable."""
    from heterocache_b200 import ops
    dev = cuda_device
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    other = torch.zeros(2, dtype=torch.int32, device=dev)  # stands for rank 1's flags
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.set_wait_limits(50_000_000)  # 50 ms
    try:
        ops.peer_barrier(0, 2, [flags.data_ptr(), other.data_ptr()], counter, err)
        torch.cuda.synchronize()
    finally:
        ops.set_wait_limits(0)
    assert int(err.item()) & (1 << 7)  # HC_ERR_TIMEOUT in the error flag
    assert int(other[0].item()) == 1 and int(flags[0].item()) == 1  # this rank signalled both
    assert int(counter.item()) == 1
    x = torch.ones(4, device=dev)
    assert float((x * 2).sum().item()) == 8.0


def test_peer_put_stores_the_segments_into_every_destination(cuda_device):
    """hc_peer_put on one GPU (the 2-GPU test covers another GPU's memory):
    the concatenated segments land in every destination, words past them
    are left alone, and nothing is launched without a destination."""
    from heterocache_b200 import ops
    dev = cuda_device
    a = torch.tensor([7], dtype=torch.int32, device=dev)
    b = torch.arange(3000, dtype=torch.int32, device=dev) * 3 - 1000
    c = torch.arange(5, dtype=torch.int32, device=dev) + 40
    d1 = torch.full((3010,), -9, dtype=torch.int32, device=dev)
    d2 = torch.full((3020,), -9, dtype=torch.int32, device=dev)
    ops.peer_put([a, b, c], [d1.data_ptr(), d2[4:].data_ptr()])
    torch.cuda.synchronize()
    want = torch.cat([a, b, c])
    assert torch.equal(d1[:3006], want) and bool((d1[3006:] == -9).all())
    assert torch.equal(d2[4:3010], want) and bool((d2[:4] == -9).all()) and bool((d2[3010:] == -9).all())
    n0 = ops.LAUNCHES[0]
    ops.peer_put([a], [])
    assert ops.LAUNCHES[0] == n0
