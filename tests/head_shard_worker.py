"""Worker of tests/test_gpu_head_shard.py (launched by torch.distributed.run,
one process per GPU): a 2-way head-sharded cache against the single-GPU cache
on the same inputs; writes this rank's comparison to $HC_SHARD_OUT/rank<r>.json."""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

from test_gpu_head_shard import _config, _rows, _setup  # noqa: E402
from heterocache_b200.cache import HeteroCache  # noqa: E402
from heterocache_b200.head_shard import HeadShardedCache, PeerGather  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    res = {"rank": rank}
    try:
        layers, KV, H, L = 2, 8, 32, 4096
        balance = os.environ.get("HC_SHARD_BALANCE", "0") == "1"
        full = HeteroCache(_config(layers, KV, H))
        shard = HeadShardedCache(_config(layers, KV, H), rank, world, balance=balance)
        # a second shard whose head outputs are gathered by the decode kernels
        # over NVLink (PeerGather) instead of the NCCL all-gather, and whose
        # pivots' position lists reach the other rank through its mailbox
        # (publish_remote / retrieve_remote_mail) instead of NCCL broadcasts
        shard_p = HeadShardedCache(_config(layers, KV, H), rank, world, balance=balance)
        # both ranks prefill the full cache and only their own shards
        gens = _setup(dev, full.data, layers, KV, H, L, (full, [shard, shard_p]))
        # mailbox words per layer are known once the budget is (after prefill)
        base = [sum(shard_p.remote_words(x) for x in range(l)) for l in range(layers)]
        mail = sum(shard_p.remote_words(x) for x in range(layers))
        peer = PeerGather(1, H // world, 128, torch.bfloat16, rank, world, device=dev, mail_words=mail)
        print(f"rank {rank}: prefill done", flush=True)
        max_diff, same_rows, same_trig, n_trig = 0.0, True, True, 0
        peer_exact, peer_diff, mail_rows, mail_trig, n_mail = True, 0.0, True, True, 0
        for step in range(12):
            for layer in range(layers):
                q, k, v = (t.to(dev) for t in gens[layer].step())
                # this rank's heads of the layer; the gathered output lists them rank by rank
                ks, hs = shard.head_index(layer, dev), shard.head_index(layer, dev, query=True)
                order = torch.tensor(shard.gathered_heads(layer), device=dev)
                full.update(k, v, layer)
                shard.update(k.index_select(1, ks), v.index_select(1, ks), layer)
                shard_p.update(k.index_select(1, ks), v.index_select(1, ks), layer)
                o_full = full.attention(q, layer).index_select(1, order)
                o_shard = shard.attention(q.index_select(1, hs), layer)
                max_diff = max(max_diff, (o_full.float() - o_shard.float()).abs().max().item())
                peer.barrier()
                shard_p.attention(q.index_select(1, hs), layer, peer=peer, row0=0)
                peer.barrier()
                peer_exact &= bool(torch.equal(peer.out, o_shard))
                peer_diff = max(peer_diff, (o_full.float() - peer.out.float()).abs().max().item())
                full.decode_select(q, layer)
                shard.decode_select(q.index_select(1, hs), layer)
                if shard_p.select_local(q.index_select(1, hs), layer):  # the same on every rank
                    shard_p.publish_remote(layer, peer, base[layer])
                    peer.barrier()
                    shard_p.retrieve_remote_mail(layer, peer, base[layer])
                    n_mail += 1
                torch.cuda.synchronize()
                jp = shard_p.cache._jobs[layer]
                jf, js = full._jobs[layer], shard.cache._jobs[layer]
                if jf is not None and js is not None and js.n_jobs:
                    same_trig &= torch.equal(jf.trigger[:jf.n_jobs].cpu(), js.trigger[:js.n_jobs].cpu())
                    n_trig += int(js.trigger[:js.n_jobs].sum())
                    mail_trig &= torch.equal(jp.trigger[:jp.n_jobs].cpu(), js.trigger[:js.n_jobs].cpu())
                for h, g in enumerate(shard.kv_heads(layer)):
                    a, b = _rows(full, layer, g), _rows(shard.cache, layer, h)
                    same_rows &= bool(torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]))
                    c = _rows(shard_p.cache, layer, h)
                    mail_rows &= bool(torch.equal(c[0], b[0]) and torch.equal(c[1], b[1]))
            print(f"rank {rank}: step {step} done", flush=True)
        full.check_errors()
        shard.check_errors()
        shard_p.check_errors()
        peer.check_errors()
        peer.close()
        res.update(mail_rows=bool(mail_rows), mail_trig=bool(mail_trig), n_mail=n_mail,
                   peer_exact=bool(peer_exact), peer_diff=peer_diff, max_diff=max_diff, same_rows=bool(same_rows), same_trig=bool(same_trig), n_trig=n_trig,
                   crossing=sum(len(s) for s in shard.remote))
    except Exception as e:  # reported through the result file
        res["error"] = repr(e)
    with open(os.path.join(os.environ["HC_SHARD_OUT"], f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()  # every rank has unmapped the others' buffers before any frees its own
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
