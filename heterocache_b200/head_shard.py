"""KV-head-sharded decode over several GPUs (the head-sharded variant of the
multi-GPU configuration).

A layer's KV heads, in the runtime order the role file's derivation produces
(anchor -> satellite -> volatile -> pivot), are split into equal sets, one
per rank: contiguous blocks, or sets balanced by cached tokens
(``head_assignment``); a rank also holds the query heads of its KV heads
(GQA groups stay whole).  Each rank runs the compressed-KV path for its heads
with its own ``HeteroCache``; the budget formula still uses the model-wide
head counts, so every head gets the capacity it would get on one GPU.

Two steps cross ranks:

* attention: each rank's output rows [bsz, H/world, D] are all-gathered
  into [bsz, H, D] for o_proj: by one NCCL all-gather per layer and step, or
  (``PeerGather``) by the decode combine kernel itself, which stores its rows
  into every rank's gathered buffer over NVLink, two device-side barriers a
  step ordering the stores (no collective call on the host, so a whole step
  replays from one CUDA graph);
* retrieval: a pivot and its satellites may sit on different ranks.  The
  pivot's rank runs the drift check; at each check step it broadcasts the
  pivot's trigger and position list (the list heterocache/cache_utils.py:
  1084-1101 builds from the pivot's last buffered step), and every rank
  holding one of its satellites retrieves that satellite's first
  ``lengths[m]`` positions from its own full tier.  The list crosses by an
  NCCL broadcast (``remote_checks``) or, with ``PeerGather``'s mailboxes,
  by the pivot rank's stores into the other ranks' memory
  (``publish_remote``, published by the step barrier, then
  ``retrieve_remote_mail``), which keeps a check step inside the step's
  graph too.

Every rank issues the same collectives in the same order: one all-gather per
``attention`` call and, at check steps, one broadcast per star group of the
layer (in relation order); with ``PeerGather`` the same holds for its
barriers.
"""
from __future__ import annotations

import copy
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from . import ops
from .cache import HeteroCache, HeteroCacheConfig


def head_blocks(num_kv_heads: int, world: int) -> List[range]:
    """Contiguous, equal blocks of KV heads per rank."""
    if world < 1 or num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world} ranks")
    n = num_kv_heads // world
    return [range(r * n, (r + 1) * n) for r in range(world)]


def head_weights(data: Dict, layer: int, compression_ratio: float, total_kv_heads: int) -> List[float]:
    """Cached tokens of each KV head of the layer per prompt token: 1 for a
    head kept whole (volatile, pivot), else its budget share
    ``min(alloc * base / L, 1)`` with base the budget formula of
    heterocache/cache_utils.py:15-16 (linear in L)."""
    from .roles import full_head_count
    F = full_head_count(data)
    c = (compression_ratio * total_kv_heads - F) / (total_kv_heads - F)
    cls = data["classification_matrix"][layer]
    alloc = data["allocation_matrix"][layer]
    return [1.0 if x in (2, 3) else max(min(a * c, 1.0), 0.0) for x, a in zip(cls, alloc)]


def head_assignment(data: Dict, num_layers: int, num_kv_heads: int, world: int, balance: bool = False,
                    compression_ratio: float = 0.5, total_kv_heads: Optional[int] = None) -> List[List[List[int]]]:
    """Per layer, per rank: the rank's KV heads (ascending ids, KV/world each).

    ``balance=False``: contiguous blocks (``head_blocks``).  ``balance=True``:
    the heads spread so that the ranks hold about the same number of cached
    tokens (largest head first onto the least-loaded rank with room; ties to
    the lower rank): in the role order the heads kept whole (volatile, pivot)
    sit together at the end, so contiguous blocks put most of a layer's
    bytes, and the decode time, on the last ranks.  A rank's heads keep
    their relative order, so the role order holds on every rank; the
    gathered output lists the ranks' query heads rank by rank
    (``HeadShardedCache.gathered_heads``)."""
    if world < 1 or num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world} ranks")
    n = num_kv_heads // world
    if not balance:
        return [[list(b) for b in head_blocks(num_kv_heads, world)] for _ in range(num_layers)]
    T = total_kv_heads or num_kv_heads * num_layers
    out = []
    for layer in range(num_layers):
        w = head_weights(data, layer, compression_ratio, T)
        load, ranks = [0.0] * world, [[] for _ in range(world)]
        for h in sorted(range(num_kv_heads), key=lambda i: (-w[i], i)):
            r = min((r for r in range(world) if len(ranks[r]) < n), key=lambda r: (load[r], r))
            ranks[r].append(h)
            load[r] += w[h]
        out.append([sorted(x) for x in ranks])
    return out


def local_runtime_data(data: Dict, num_layers: int, num_kv_heads: int, world: int, rank: int,
                       assignment: Optional[List[List[List[int]]]] = None):
    """Runtime role data of one rank's heads, plus its cross-rank retrieval specs.

    ``assignment`` (``head_assignment``; default contiguous blocks) gives
    each layer's heads per rank.  Returns ``(local, remote)``.  ``local`` is
    a derived role document for the rank's heads (local ids 0..n-1 in the
    same order): classification and
    allocation rows sliced, relations kept for local pivots with their local
    satellites, ``remote_member_alloc[layer][local pivot]`` = allocations of
    that pivot's satellites held by other ranks (its position list must cover
    them), and the four ``need_to_*`` lists derived from the sliced rows.
    ``remote[layer]`` lists, in the layer's relation order, every star group
    with satellites off its pivot's rank: ``{"src": pivot rank, "leader":
    pivot's local id there, "alloc": allocations of all its satellites,
    "members": [(local head id, allocation)] of this rank's satellites}``.
    """
    if assignment is None:
        assignment = head_assignment(data, num_layers, num_kv_heads, world)
    local = {"meta": copy.deepcopy(data["meta"]), "classification_matrix": [], "allocation_matrix": [],
             "leader_member_relations": [], "remote_member_alloc": [], "need_to_update_counts": [],
             "need_to_select_counts": [], "need_to_compress_counts": [], "need_to_keep_counts": []}
    remote: List[List[Dict]] = []
    for layer in range(num_layers):
        heads = assignment[layer]
        owner = {h: r for r, hs in enumerate(heads) for h in hs}
        lid = {h: i for hs in heads for i, h in enumerate(hs)}  # local id on the owner's rank
        mine = heads[rank]
        cls = [data["classification_matrix"][layer][h] for h in mine]
        alloc = [data["allocation_matrix"][layer][h] for h in mine]
        local["classification_matrix"].append(cls)
        local["allocation_matrix"].append(alloc)
        local["need_to_compress_counts"].append(cls.count(1) + cls.count(4))
        local["need_to_select_counts"].append([i for i, x in enumerate(cls) if x == 3])
        local["need_to_update_counts"].append([i for i, x in enumerate(cls) if x == 4])
        local["need_to_keep_counts"].append([i for i, x in enumerate(cls) if x in (2, 3)])
        rel: Dict[str, List[int]] = {}
        rem_alloc: Dict[str, List[float]] = {}
        specs: List[Dict] = []
        full_alloc = data["allocation_matrix"][layer]
        for leader, members in data["leader_member_relations"][layer].items():
            lg = int(leader)
            src = owner[lg]
            if src == rank:
                rel[str(lid[lg])] = [lid[m] for m in members if owner[m] == rank]
                off = [full_alloc[m] for m in members if owner[m] != rank]
                if off:
                    rem_alloc[str(lid[lg])] = off
            # a star group crossing ranks: every rank takes part in its broadcast
            if any(owner[m] != src for m in members):
                specs.append({"src": src, "leader": lid[lg],
                              "alloc": [full_alloc[m] for m in members],
                              "members": [(lid[m], full_alloc[m]) for m in members
                                          if owner[m] == rank and src != rank]})
        pivots = [int(x) for x in data["leader_member_relations"][layer]]
        owners = {owner[p] for p in pivots}
        if len(owners) > 1 and pivots != sorted(pivots):
            # the reference pairs relation entry i with the i-th pivot in sorted
            # order (cache_utils.py:1027 with utils.py:326); split over ranks that
            # pairing cannot be kept when the two orders differ
            raise NotImplementedError(f"layer {layer}: pivots in non-sorted relation order span ranks")
        local["leader_member_relations"].append(rel)
        local["remote_member_alloc"].append(rem_alloc)
        remote.append(specs)
    return local, remote


class HeadShardedCache:
    """One rank's share of a head-sharded ``HeteroCache``.

    Inputs are the rank's slices: q [bsz, H/world, L, D], k/v
    [bsz, KV/world, L, D] -- the heads ``q_heads(layer)`` / ``kv_heads(layer)``
    (a contiguous block, or with ``balance=True`` the capacity-balanced
    heads of ``head_assignment``).  ``attention`` returns every head's output
    [bsz, H, D], rank by rank: row j is query head ``gathered_heads(layer)[j]``
    (the identity for contiguous blocks; with ``balance`` the model's o_proj
    input columns are permuted once to that order, as the load-time role
    permutation permutes them).  Method names and call order follow the
    cache object.
    """

    def __init__(self, config: HeteroCacheConfig, rank: int, world: int, group=None, balance: bool = False):
        self.rank, self.world, self.group = rank, world, group
        KV, H = config.num_kv_heads, config.num_attn_heads
        if H % KV:
            raise ValueError("query heads must be a multiple of KV heads")
        T = getattr(config, "total_kv_heads", None) or KV * config.num_layers
        self.assignment = head_assignment(config.data, config.num_layers, KV, world, balance,
                                          config.compression_ratio, T)
        self.groups = H // KV
        local, self.remote = local_runtime_data(config.data, config.num_layers, KV, world, rank,
                                                assignment=self.assignment)
        self.kv_local = KV // world
        self.h_local = H // world
        cfg = HeteroCacheConfig(local, compression_ratio=config.compression_ratio,
                                stable_threshold=config.stable_threshold, real_offload=config.real_offload,
                                max_gen_len=config.max_gen_len, decode_step=config.decode_step,
                                pooling=config.pooling, kernel_size=config.kernel_size,
                                num_attn_heads=self.h_local, num_kv_heads=self.kv_local,
                                num_layers=config.num_layers, window_size=getattr(config, "window_size", 1),
                                total_kv_heads=KV * config.num_layers)
        self.cache = HeteroCache(cfg)
        self.num_layers = config.num_layers
        self.num_attn_heads = H
        self._gather: Dict = {}
        self._bufs: Dict = {}
        self._index: Dict = {}

    # -- which heads -----------------------------------------------------
    def kv_heads(self, layer_idx) -> List[int]:
        """This rank's KV heads of the layer (model ids, ascending)."""
        return self.assignment[layer_idx][self.rank]

    def q_heads(self, layer_idx) -> List[int]:
        """This rank's query heads of the layer (each KV head's GQA group)."""
        G = self.groups
        return [h * G + g for h in self.kv_heads(layer_idx) for g in range(G)]

    def gathered_heads(self, layer_idx) -> List[int]:
        """Model query head of each row of the gathered output (rank by rank)."""
        G = self.groups
        return [h * G + g for hs in self.assignment[layer_idx] for h in hs for g in range(G)]

    def head_index(self, layer_idx, device, query: bool = False) -> torch.Tensor:
        """``kv_heads`` (or ``q_heads``) as an int64 index tensor on ``device``
        (e.g. ``k.index_select(1, ...)`` to slice a layer's inputs)."""
        key = (layer_idx, str(device), query)
        t = self._index.get(key)
        if t is None:
            ids = self.q_heads(layer_idx) if query else self.kv_heads(layer_idx)
            t = torch.tensor(ids, dtype=torch.int64, device=device)
            self._index[key] = t
        return t

    # -- prefill -------------------------------------------------------
    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        return self.cache.update(key_states, value_states, layer_idx, cache_kwargs)

    def init_coefficient(self, query_states, key_states, layer_idx):
        self.cache.init_coefficient(query_states, key_states, layer_idx)

    def prefill_select(self, query_states, key_states, value_states, layer_idx):
        self.cache.prefill_select(query_states, key_states, value_states, layer_idx)

    # -- decode --------------------------------------------------------
    def attention(self, query_states, layer_idx, scale: float = 0.0, out=None, peer: "PeerGather" = None,
                  row0: int = 0):
        """Local flash-decode, then one all-gather: returns [bsz, H, D].

        With ``peer`` the decode kernels store this rank's head rows straight
        into every rank's ``peer.out`` (rows ``row0`` ..) instead, and nothing
        is returned before ``peer.barrier()``: the caller issues one barrier
        before a step's attention calls and one after them, then reads
        ``peer.out``."""
        if peer is not None:
            return self.cache.attention(query_states, layer_idx, scale=scale, mirrors=peer.mirrors(row0),
                                        mirror_batch_stride=peer.mirror_batch_stride)
        local = self.cache.attention(query_states, layer_idx, scale=scale)
        return gather_heads(local, self.world, self.group, out=out, cache=self._gather)

    def decode_select(self, query_states, layer_idx):
        """Local drift checks and retrievals; at a check step, one broadcast per
        star group crossing ranks, then the retrievals of this rank's
        satellites of remote pivots."""
        if self.select_local(query_states, layer_idx):
            self.remote_checks(layer_idx)

    def remote_checks(self, layer_idx) -> None:
        """The cross-rank part of a check step: per star group crossing ranks,
        stage, broadcast and retrieve (every rank, same order)."""
        for si, spec in enumerate(self.remote[layer_idx]):
            buf = self.stage_positions(layer_idx, si)
            broadcast_retrieval(buf, spec["src"], self.group)
            self.retrieve_remote(layer_idx, si)

    # The three phases of decode_select, callable one by one (the broadcast
    # between them is the only cross-rank step).
    def select_local(self, query_states, layer_idx, defer: bool = False) -> bool:
        """The local cache's decode_select; True at a check step with star
        groups that cross ranks.  With ``defer`` a due check is put off (see
        ``HeteroCache.decode_select``); it must be flushed before
        ``remote_checks``."""
        # the local cache counts the buffered queries (its host state, which a
        # captured decode step saves and restores)
        check = self.cache._qcount[layer_idx] + 1 >= self.cache.decode_step
        self.cache.decode_select(query_states, layer_idx, defer=defer)
        return check and bool(self.remote[layer_idx])

    def _max_len(self, spec) -> int:
        c = self.cache
        return max(min(int(c.base_compress_len * a), c.prefill_len) for a in spec["alloc"])

    def stage_positions(self, layer_idx, si) -> torch.Tensor:
        """Buffer [1 + max_len] int32 of star group ``si``: trigger and position
        list, filled on the pivot's rank (the broadcast source)."""
        spec = self.remote[layer_idx][si]
        max_len = self._max_len(spec)
        c = self.cache
        buf = self._bufs.get((layer_idx, si))
        if buf is None:
            buf = torch.zeros(1 + max(max_len, 1), dtype=torch.int32, device=c._dev)
            self._bufs[(layer_idx, si)] = buf
        if spec["src"] == self.rank:
            jobs = c._jobs[layer_idx]
            if jobs is None or spec["leader"] not in jobs.pivot_list:
                raise RuntimeError("pivot job missing on its rank")
            j = jobs.pivot_list.index(spec["leader"])
            buf[0:1].copy_(jobs.trigger[j:j + 1])
            buf[1:1 + max_len].copy_(jobs.retrieve_positions[j, :max_len])
        return buf

    def remote_words(self, layer_idx) -> int:
        """int32 words of the layer's mailbox block (``publish_remote``): per
        star group crossing ranks, its trigger and position list."""
        return sum(1 + max(self._max_len(spec), 1) for spec in self.remote[layer_idx])

    def publish_remote(self, layer_idx, peer: "PeerGather", base: int = 0) -> None:
        """``remote_checks`` over peer memory, pivot side: for each star group
        whose pivot this rank holds, its trigger and position list stored
        straight into words ``base`` .. of every other rank's mailbox
        (hc_peer_put, one launch per group; no collective call, so a check
        step is captured in the step's graph).  Issue after the layer's drift
        check and before the step's closing ``peer.barrier()``, which
        publishes the words; the other ranks then run
        ``retrieve_remote_mail`` with the same ``base``."""
        off = base
        c = self.cache
        for spec in self.remote[layer_idx]:
            max_len = self._max_len(spec)
            if spec["src"] == self.rank:
                jobs = c._jobs[layer_idx]
                if jobs is None or spec["leader"] not in jobs.pivot_list:
                    raise RuntimeError("pivot job missing on its rank")
                j = jobs.pivot_list.index(spec["leader"])
                dsts = [p + off * 4 for r, p in enumerate(peer.mail_ptrs) if r != self.rank]
                segs = [jobs.trigger[j:j + 1]]
                if max_len:
                    segs.append(jobs.retrieve_positions[j, :max_len])
                ops.peer_put(segs, dsts)
            off += 1 + max(max_len, 1)

    def retrieve_remote_mail(self, layer_idx, peer: "PeerGather", base: int = 0) -> None:
        """``remote_checks`` over peer memory, satellite side: this rank's
        satellites of remote pivots retrieved from the trigger and positions
        ``publish_remote`` stored into this rank's mailbox (after the step's
        closing ``peer.barrier()``)."""
        off = base
        for si, spec in enumerate(self.remote[layer_idx]):
            n = 1 + max(self._max_len(spec), 1)
            if spec["members"]:
                self.retrieve_remote(layer_idx, si, buf=peer.mail[off:off + n])
            off += n

    def retrieve_remote(self, layer_idx, si, buf=None) -> None:
        """Retrieve this rank's satellites of star group ``si`` from the staged
        trigger and positions (``buf``: [1 + max_len] int32, by default the
        broadcast buffer of ``stage_positions``)."""
        spec = self.remote[layer_idx][si]
        if not spec["members"]:
            return
        c = self.cache
        if buf is None:
            buf = self._bufs[(layer_idx, si)]
        key = ("members", layer_idx, si)
        if key not in self._bufs:  # device index arrays, made once
            base, L = c.base_compress_len, c.prefill_len
            heads = [h for h, _ in spec["members"]]
            lens = [min(int(base * a), L) for _, a in spec["members"]]
            i32 = dict(dtype=torch.int32, device=c._dev)
            self._bufs[key] = (torch.zeros(len(heads), **i32), torch.tensor(heads, **i32),
                               torch.tensor(lens, **i32), max(lens))
        mj, mh, ml, max_len = self._bufs[key]
        c._wait_retrieval(layer_idx)
        full_k, full_v, first = c.full_tier(layer_idx)
        ops.retrieve(member_job=mj, member_head=mh, member_len=ml, max_member_len=max_len, trigger=buf[0:1],
                     retrieve_positions=buf[1:].view(1, -1), full_k=full_k, full_v=full_v,
                     k_pool=c.key_pools[layer_idx], v_pool=c.value_pools[layer_idx],
                     block_table=c.block_tables[layer_idx], num_kv_heads=c.num_kv_heads, err=c._err,
                     tier_first_head=first)

    def check_errors(self):
        self.cache.check_errors()


def gather_heads(local: torch.Tensor, world: int, group=None, out: Optional[torch.Tensor] = None,
                 cache: Optional[Dict] = None) -> torch.Tensor:
    """All-gather of per-rank head outputs [bsz, h, D] -> [bsz, world*h, D]
    (rank r's heads at rows r*h .. r*h+h-1)."""
    bsz, h, D = local.shape
    if world == 1:
        if out is not None:
            out.copy_(local)
            return out
        return local
    key = (bsz, h, D, local.dtype, local.device)
    stage = cache.get(key) if cache is not None else None
    if stage is None:
        stage = torch.empty(world, bsz, h, D, dtype=local.dtype, device=local.device)
        if cache is not None:
            cache[key] = stage
    if dist.get_backend(group) == "gloo":
        dist.all_gather(list(stage.unbind(0)), local.contiguous(), group=group)
    else:
        dist.all_gather_into_tensor(stage, local.contiguous(), group=group)
    full = stage.permute(1, 0, 2, 3).reshape(bsz, world * h, D)
    if out is not None:
        out.copy_(full)
        return out
    return full


def broadcast_retrieval(buf: torch.Tensor, src: int, group=None) -> None:
    """Trigger and position list of one pivot, from the pivot's rank to all."""
    dist.broadcast(buf, src=src, group=group)


class PeerGather:
    """The all-gather of head outputs done by the attention kernels: every
    rank's gathered output, written by every rank over NVLink.

    Each rank allocates ``out`` [rows, world * h, D] (rows: the batch rows of
    the caches that share it, e.g. one per sequence) and an int32 flag array,
    maps the other ranks' two buffers into its address space through CUDA
    IPC (hc_ipc_export / hc_ipc_open: plain peer mappings for this rank's
    device, no multicast object), and gives each attention call the address of its own
    head block in every rank's ``out`` (``mirrors(row0)``): the decode
    combine kernel stores each output row there as it finishes it.
    ``barrier()`` (hc_peer_barrier) before a step's attention calls and after
    them orders the stores: after the second, ``out`` holds every rank's
    heads on every rank.  All ranks construct it together (one object
    exchange over the process group) and call ``barrier`` equally often.

    ``mail_words`` > 0 adds an int32 mailbox of that size per rank, mapped the
    same way (``mail_ptrs``): the pivots' trigger and position lists reach
    the ranks of their satellites there (``HeadShardedCache.publish_remote``,
    hc_peer_put), published by the same step barrier, so that a check step
    needs no collective call either.
    """

    def __init__(self, rows: int, h: int, D: int, dtype: torch.dtype, rank: int, world: int, group=None,
                 device=None, mail_words: int = 0):
        if not 1 <= world <= 8:
            raise ValueError("PeerGather: 1 to 8 ranks")
        self.rank, self.world, self.h, self.D, self.rows = rank, world, h, D, rows
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.out = torch.zeros(rows, world * h, D, dtype=dtype, device=dev)
        self.flags = torch.zeros(world, dtype=torch.int32, device=dev)
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.mail = torch.zeros(max(int(mail_words), 1), dtype=torch.int32, device=dev)
        self._opened: List[int] = []  # this process's mappings of the other ranks' allocations
        if world == 1:
            self.out_ptrs, self.flag_ptrs = [self.out.data_ptr()], [self.flags.data_ptr()]
            self.mail_ptrs = [self.mail.data_ptr()]
        else:
            import ctypes
            from ._lib import check, lib
            torch.cuda.synchronize(dev)  # the buffers are zero before a peer maps them

            def export(t):
                h, off = ctypes.create_string_buffer(64), ctypes.c_int64(0)
                check("hc_ipc_export", lib().hc_ipc_export(t.data_ptr(), h, ctypes.byref(off)))
                return h.raw, off.value

            mine = (export(self.out), export(self.flags), export(self.mail))
            allh: List = [None] * world
            dist.all_gather_object(allh, mine, group=group)
            opened: Dict[bytes, int] = {}  # one mapping per allocation (out and flags may share one)

            def mapped(handle: bytes, off: int) -> int:
                if handle not in opened:
                    base = ctypes.c_void_p()
                    with torch.cuda.device(dev):  # mapped for this device, peer access enabled as needed
                        check("hc_ipc_open", lib().hc_ipc_open(ctypes.create_string_buffer(handle, 64),
                                                               ctypes.byref(base)))
                    opened[handle] = base.value
                return opened[handle] + off

            self.out_ptrs, self.flag_ptrs, self.mail_ptrs = [], [], []
            for r, ((ho, oo), (hf, of), (hm, om)) in enumerate(allh):
                if r == rank:
                    self.out_ptrs.append(self.out.data_ptr())
                    self.flag_ptrs.append(self.flags.data_ptr())
                    self.mail_ptrs.append(self.mail.data_ptr())
                else:
                    self.out_ptrs.append(mapped(ho, oo))
                    self.flag_ptrs.append(mapped(hf, of))
                    self.mail_ptrs.append(mapped(hm, om))
            self._opened = list(opened.values())
        self.mirror_batch_stride = world * h * D
        self._esz = self.out.element_size()

    def mirrors(self, row0: int = 0) -> List[int]:
        """Where this rank's heads of batch row ``row0`` go in every rank's ``out``."""
        off = (row0 * self.world * self.h + self.rank * self.h) * self.D * self._esz
        return [p + off for p in self.out_ptrs]

    def barrier(self) -> None:
        ops.peer_barrier(self.rank, self.world, self.flag_ptrs, self.counter, self.err)

    def close(self) -> None:
        """Unmap the other ranks' buffers (after this rank's last barrier; every
        rank's own buffers stay until every rank has closed)."""
        if self._opened:
            from ._lib import check, lib
            torch.cuda.synchronize(self.out.device)
            for base in self._opened:
                check("hc_ipc_close", lib().hc_ipc_close(base))
            self._opened = []

    def check_errors(self) -> None:
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"heterocache_b200: peer barrier error flag {e} (a rank did not arrive in time)")
