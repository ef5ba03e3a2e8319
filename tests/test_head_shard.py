"""Head-sharded mode, host side: role partitioning and the two collectives
(all-gather of head outputs, broadcast of a pivot's position list), the
latter as world-size-2 gloo process groups on the CPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from heterocache_b200.cache import get_compress_len
from heterocache_b200.head_shard import (broadcast_retrieval, gather_heads, head_assignment, head_weights,
                                         local_runtime_data)
from heterocache_b200.roles import derive_runtime_data, full_head_count, synthetic_roles


def _data(layers=3, kv=8, seed=5, star=4):
    return derive_runtime_data(synthetic_roles(layers, kv, seed, star_size=star), layers, kv)


@pytest.mark.parametrize("balance", [False, True], ids=["contiguous", "balanced"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_local_runtime_data_partitions_roles(world, balance):
    layers, KV = 3, 8
    data = _data(layers, KV)
    assign = head_assignment(data, layers, KV, world, balance)
    locs = [local_runtime_data(data, layers, KV, world, r, assignment=assign) for r in range(world)]
    for layer in range(layers):
        heads = assign[layer]
        owner = {h: r for r, hs in enumerate(heads) for h in hs}
        lid = {h: i for hs in heads for i, h in enumerate(hs)}
        # classification / allocation rows reassemble the layer's rows
        order = [h for hs in heads for h in hs]
        cls = sum((locs[r][0]["classification_matrix"][layer] for r in range(world)), [])
        alloc = sum((locs[r][0]["allocation_matrix"][layer] for r in range(world)), [])
        assert cls == [data["classification_matrix"][layer][h] for h in order]
        assert alloc == [data["allocation_matrix"][layer][h] for h in order]
        for r, (loc, remote) in enumerate(locs):
            c = loc["classification_matrix"][layer]
            assert loc["need_to_compress_counts"][layer] == c.count(1) + c.count(4)
            assert loc["need_to_select_counts"][layer] == [i for i, x in enumerate(c) if x == 3]
            assert loc["need_to_update_counts"][layer] == [i for i, x in enumerate(c) if x == 4]
            assert loc["need_to_keep_counts"][layer] == [i for i, x in enumerate(c) if x in (2, 3)]
            # the role order (anchor, satellite, volatile, pivot) holds on every rank
            pri = {1: 0, 4: 1, 2: 2, 3: 3}
            assert [pri[x] for x in c] == sorted(pri[x] for x in c)
        # every satellite is retrieved exactly once: by its pivot's rank (local
        # relation) or, off that rank, through a broadcast spec on its own rank
        for leader, members in data["leader_member_relations"][layer].items():
            lg = int(leader)
            src = owner[lg]
            for m in members:
                loc, remote = locs[owner[m]]
                if owner[m] == src:
                    assert lid[m] in loc["leader_member_relations"][layer][str(lid[lg])]
                else:
                    hits = [s for s in remote[layer] if s["src"] == src and s["leader"] == lid[lg]
                            and (lid[m], data["allocation_matrix"][layer][m]) in s["members"]]
                    assert len(hits) == 1
            off = [data["allocation_matrix"][layer][m] for m in members if owner[m] != src]
            got = locs[src][0]["remote_member_alloc"][layer].get(str(lid[lg]), [])
            assert got == off
            # all ranks hold the same broadcast sequence for the layer
            seqs = [[(s["src"], s["leader"]) for s in locs[r][1][layer]] for r in range(world)]
            assert all(sq == seqs[0] for sq in seqs)
    # the budget uses model-wide counts on every rank
    L = 8192
    kb = get_compress_len(0.5, full_head_count(data), L, KV * layers)
    for loc, _ in locs:
        assert get_compress_len(0.5, full_head_count(loc), L, KV * layers) == kb


@pytest.mark.parametrize("world", [2, 4, 8])
def test_balanced_assignment_partitions_and_evens_the_load(world):
    """Every head on exactly one rank, KV/world per rank, ascending; the
    heaviest rank's cached tokens never above the contiguous blocks' and,
    on these roles (heads kept whole at the end of the role order), lower
    wherever a rank holds more than one head."""
    layers, KV = 3, 8
    data = _data(layers, KV)
    bal = head_assignment(data, layers, KV, world, True)
    con = head_assignment(data, layers, KV, world, False)
    for layer in range(layers):
        w = head_weights(data, layer, 0.5, KV * layers)
        assert sorted(h for hs in bal[layer] for h in hs) == list(range(KV))
        assert all(len(hs) == KV // world and hs == sorted(hs) for hs in bal[layer])
        peak = lambda a: max(sum(w[h] for h in hs) for hs in a[layer])  # noqa: E731
        assert peak(bal) <= peak(con) + 1e-12
        if KV // world > 1 and any(x in (2, 3) for x in data["classification_matrix"][layer]):
            assert peak(bal) < peak(con)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bsz, h, D = 2, 3, 8
        local = torch.full((bsz, h, D), float(rank)) + torch.arange(h).view(1, h, 1) * 0.1
        full = gather_heads(local, world)
        want = torch.cat([torch.full((bsz, h, D), float(r)) + torch.arange(h).view(1, h, 1) * 0.1
                          for r in range(world)], dim=1)
        ok_gather = torch.equal(full, want)
        buf = torch.arange(7, dtype=torch.int32) * (10 if rank == 1 else 0)
        broadcast_retrieval(buf, src=1)
        ok_bcast = buf.tolist() == [10 * i for i in range(7)]
        q.put((rank, ok_gather, ok_bcast))
    finally:
        dist.destroy_process_group()


def test_collectives_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert [r[0] for r in res] == [0, 1]
    assert all(r[1] and r[2] for r in res), res
