"""Drop-in ``HeteroCache`` for the B200 path.

Same constructor input, method names and public tensors as the reference
cache (heterocache/cache_utils.py:610-1196): ``update``, ``init_coefficient``,
``prefill_select``, ``decode_select``, ``get_seq_length``; ``key_pools``,
``value_pools``, ``block_tables``, ``heads_len``, ``prefill_topk_set``.
Every data-path step runs in the sm_100a library through the C ABI; Python
keeps only bookkeeping.

Differences in mechanism (not in results):

* The reference reads the device every layer and step (``.item()`` at
  cache_utils.py:801, :985, :1114 and ``.tolist()`` at :1077).  Here the
  per-row lengths and mapped-page counts are mirrored on the host (they evolve
  deterministically), so the free-list check and its ``RuntimeError("Layer N
  OOM.")`` happen before the launch with no device read, and the drift
  decision stays on the device (the retrieval kernel reads the trigger).
* ``prefill_topk_set[layer]`` holds the reference set of each pivot as
  int32 positions in ascending order (the reference keeps the top-k indices
  in score order; only the set is ever used, cache_utils.py:1063-1075).
* With ``real_offload=True`` the full tier lives in pinned host memory and the
  retrieval kernel reads it directly over the host link on a side stream,
  ordered before the next attention of that layer by an event.  The
  reference stages through one shared pinned buffer and copies per satellite
  (cache_utils.py:941-948, :1095-1123), which lets the next satellite's
  host-side gather overwrite a buffer an earlier copy may still be reading;
  here there is no staging buffer.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np
import torch

try:  # the reference subclasses transformers' DynamicCache
    from transformers.cache_utils import DynamicCache as _CacheBase
except Exception:  # pragma: no cover - transformers is optional for the kernels
    _CacheBase = object

from . import ops
from .ops import PAGE, Workspace


def get_compress_len(compression_ratio, full_heads, ori_len, num_kv_heads):
    """Base per-head budget (heterocache/cache_utils.py:15-16)."""
    return int((compression_ratio * num_kv_heads - full_heads) * ori_len / (num_kv_heads - full_heads))


class HeteroCacheConfig:
    """Same fields and defaults as heterocache/cache_utils.py:41-68.

    ``window_size`` (default 1, the HeteroCache behaviour) extends the prefill
    scoring to an observation window of the last W queries with SnapKV's
    in-window causal mask and window sum (heterocache/kv_cluster.py:168-178).

    ``total_kv_heads`` (default: layers x KV heads) is the model-wide KV head
    count of the budget formula; a cache that holds only some of a layer's
    heads (the head-sharded mode) sets it to the whole model's count.
    """

    def __init__(self, data: Optional[Dict], compression_ratio: Optional[float] = 0.5,
                 stable_threshold: Optional[float] = 0.5, real_offload: Optional[bool] = True,
                 max_gen_len: Optional[int] = 128, decode_step: Optional[int] = 4,
                 pooling: Optional[str] = "avgpool", kernel_size: Optional[int] = 5,
                 num_attn_heads: Optional[int] = 32, num_kv_heads: Optional[int] = 8,
                 num_layers: Optional[int] = 32, window_size: int = 1,
                 total_kv_heads: Optional[int] = None):
        self.data = data
        self.stable_threshold = stable_threshold
        self.compression_ratio = compression_ratio
        self.real_offload = real_offload
        self.max_gen_len = max_gen_len
        self.decode_step = decode_step
        self.pooling = pooling
        self.kernel_size = kernel_size
        self.quant_method = None
        self.num_attn_heads = num_attn_heads
        self.num_kv_heads = num_kv_heads
        self.num_layers = num_layers
        self.window_size = window_size
        self.total_kv_heads = total_kv_heads


class _LayerJobs:
    """Device descriptors of one layer's drift-check jobs and satellites."""

    def __init__(self, relations: Dict[str, List[int]], alloc: List[float], base: int, L: int, device,
                 remote_alloc: Optional[Dict[str, List[float]]] = None):
        """``remote_alloc[leader]``: allocations of that pivot's satellites held
        by other caches (head-sharded mode); the pivot's position list is made
        long enough for them too."""
        jobs, slots, max_len = [], [], []
        m_job, m_head, m_len = [], [], []
        remote_alloc = remote_alloc or {}
        for idx, (leader, members) in enumerate(relations.items()):
            far = [min(int(base * a), L) for a in remote_alloc.get(leader, [])]
            if not members and not far:
                continue
            lengths = [min(int(base * alloc[m]), L) for m in members]
            j = len(jobs)
            jobs.append(int(leader))
            slots.append(idx)
            max_len.append(max(lengths + far))
            for m, n in zip(members, lengths):
                if n == 0:
                    continue
                m_job.append(j)
                m_head.append(int(m))
                m_len.append(n)
        self.n_jobs = len(jobs)
        self.pivot_list = list(jobs)
        self.max_len_cap = max(max_len) if max_len else 0
        self.max_member_len = max(m_len) if m_len else 0
        i32 = dict(dtype=torch.int32, device=device)
        self.pivot_heads = torch.tensor(jobs, **i32)
        self.ref_slots = torch.tensor(slots, **i32)
        self.max_len = torch.tensor(max_len, **i32)
        self.member_job = torch.tensor(m_job, **i32)
        self.member_head = torch.tensor(m_head, **i32)
        self.member_len = torch.tensor(m_len, **i32)
        self.m_head_list, self.m_len_list = list(m_head), list(m_len)
        self.delta = None  # slot maps of the delta retrieval (pinned-host tier)
        self.slot_list, self.max_len_list = list(slots), list(max_len)
        self.batch_descs = None  # drift-check batch descriptors (HeteroCache._drift_descs)
        self.trigger = torch.zeros(max(self.n_jobs, 1), **i32)
        self.retrieve_positions = torch.zeros(max(self.n_jobs, 1), max(self.max_len_cap, 1), **i32)
        self.coeffs = None
        self.median = None


class HeteroCache(_CacheBase):
    def __init__(self, cache_config):
        if _CacheBase is not object:
            super().__init__()
        self.config = cache_config
        self.num_attn_heads = cache_config.num_attn_heads
        self.num_kv_heads = cache_config.num_kv_heads
        self.num_layers = cache_config.num_layers
        self.gqa = self.num_kv_heads != self.num_attn_heads
        self.num_key_value_groups = self.num_attn_heads // self.num_kv_heads
        self.total_kv_heads = (getattr(cache_config, "total_kv_heads", None)
                               or self.num_kv_heads * self.num_layers)
        self.page_size = PAGE
        self.compression_ratio = cache_config.compression_ratio
        self.window_size = getattr(cache_config, "window_size", 1)
        n = self.num_layers
        self.key_pools: List[Optional[torch.Tensor]] = [None] * n
        self.value_pools: List[Optional[torch.Tensor]] = [None] * n
        self.block_tables: List[Optional[torch.Tensor]] = [None] * n
        self.free_blocks: List[Optional[torch.Tensor]] = [None] * n
        self.free_block_pointers: List[int] = [0] * n
        self.prefill_boundary_blocks: List[int] = [0] * n
        self.layer_head_capacities: List = [0] * n
        self.heads_len: List[Optional[torch.Tensor]] = [None] * n
        self.head_indices = None
        self.data = cache_config.data
        counts = self.data["meta"]["counts"]
        self.full_heads = counts["volatile"] + counts["pivot"]
        self.key_cache_cpu: List = []
        self.value_cache_cpu: List = []
        self.prefill_topk_set: List = []
        self.query_states_buffer = [[] for _ in range(n)]
        self.bsz = None
        self.head_dim = None
        self.prefill_len = None
        self._seen_tokens = 0
        self.decode_step = cache_config.decode_step
        self.stable_threshold = cache_config.stable_threshold
        self.real_offload = bool(cache_config.real_offload)
        self.device = "cpu" if cache_config.real_offload else "cuda"
        self.pooling = cache_config.pooling
        self.kernel_size = cache_config.kernel_size
        # device-side state
        self._dev = None
        self._err = None
        self._ws_score: Optional[Workspace] = None
        self._ws_fd: Optional[Workspace] = None
        self._free_ptr: List[Optional[torch.Tensor]] = [None] * n
        self._ref_bitmap: List[Optional[torch.Tensor]] = [None] * n
        self._qbuf: List[Optional[torch.Tensor]] = [None] * n
        self._qcount = [0] * n
        # the decode append of this step already stored the query (see update)
        self._q_staged = [False] * n
        # deferred decode appends (update(..., {"defer_append": True})): the
        # step's (k, v, q, query slot) until attention launches it, then the
        # side-stream event of the launched append
        self._pending: List = [None] * n
        self._append_done: List[Optional[torch.cuda.Event]] = [None] * n
        self._jobs: List[Optional[_LayerJobs]] = [None] * n
        # pinned-host tier: prefill kept indices (until the layer's slot maps
        # are built) and the retrieval staging area shared by all layers
        self._kept: List[Optional[tuple]] = [None] * n
        self._stage: Optional[tuple] = None
        # head id held in row 0 of each layer's full tier (pinned-host tier:
        # the first satellite; a device tier keeps every head)
        self._tier_first: List[int] = [0] * n
        self._retrieve_done: List[Optional[torch.cuda.Event]] = [None] * n
        self._side_stream: Optional[torch.cuda.Stream] = None
        # host mirrors of deterministic bookkeeping
        self._hlen: List[Optional[np.ndarray]] = [None] * n
        self._mapped: List[Optional[np.ndarray]] = [None] * n
        # per layer: decode appends that map no new page and stay inside the
        # page table (0: unknown; _append_bookkeeping then checks in full)
        self._slack: List[int] = [0] * n
        # opt-in diagnostics for parity tests: pooled scores and selections
        self.record_checks = bool(getattr(cache_config, "record_checks", False))
        # a CacheGroup this cache's pages live in (shared pool per layer)
        self._group: Optional["CacheGroup"] = None
        self._gidx = 0
        # drift checks put off by decode_select(..., defer=True) until
        # flush_checks(), which runs them as one batch.  Off by default with
        # the pinned-host tier: there a layer's retrieval should start right
        # after its check, to overlap the following layers
        self.defer_checks = bool(getattr(cache_config, "defer_checks",
                                         not getattr(cache_config, "real_offload", False)))
        self._deferred: List[int] = []
        self._batch_arrays: Dict = {}
        # checks per batch launch (0: the library's choice)
        self.drift_batch_per_launch = int(getattr(cache_config, "drift_batch_per_launch", 0))
        self.check_log: List[Dict] = []
        self.recorded: Dict = {}

    def __bool__(self):
        return True

    def __len__(self):
        return self.num_layers

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        if self._seen_tokens is None:
            return 0
        return self._seen_tokens

    # ------------------------------------------------------------------
    def _ensure_device(self, device: torch.device) -> None:
        if self._dev is None:
            self._dev = device
            self._err = torch.zeros(1, dtype=torch.int32, device=device)
            self._ws_score = Workspace(device)
            self._ws_fd = Workspace(device)
            self.head_indices = torch.arange(self.num_kv_heads, device=device)

    def check_errors(self) -> None:
        """Raise if a device-side check fired since the last call (syncs)."""
        if self._err is None:
            return
        code = int(self._err.item())
        if code:
            self._err.zero_()
            if self._ws_score is not None:
                self._ws_score.reset()
            names = {3: "free list exhausted (OOM)", 4: "page-table entry or index out of range",
                     7: "device-side wait timed out"}
            msgs = [v for b, v in names.items() if code & (1 << b)]
            raise RuntimeError("HeteroCache device error: " + ", ".join(msgs or [f"flags {code:#x}"]))

    def _init_layer_storage(self, layer_idx, device, dtype):
        """heterocache/cache_utils.py:693-766 (same sizes, ids and order)."""
        L = self.prefill_len
        gen = self.config.max_gen_len
        alloc = self.data["allocation_matrix"][layer_idx]
        keep = self.data["need_to_keep_counts"][layer_idx]
        caps, total, pre_total = [], 0, 0
        for h in range(self.num_kv_heads):
            if h in keep:
                cap = L
            else:
                cap = max(min(int(self.base_compress_len * alloc[h]), L), 0)
            nblk = (cap + PAGE - 1) // PAGE
            caps.append(nblk * PAGE)
            pre_total += nblk
            total += (cap + gen + PAGE - 1) // PAGE
        max_blocks = (L + gen + PAGE - 1) // PAGE + 1
        rows = self.bsz * self.num_kv_heads
        bt = np.full((rows, max_blocks), -1, dtype=np.int32)
        mapped = np.zeros(rows, dtype=np.int64)
        ptr = 0
        for r in range(rows):
            nb = caps[r % self.num_kv_heads] // PAGE
            if nb > 0:
                bt[r, :nb] = np.arange(ptr, ptr + nb, dtype=np.int32)
                ptr += nb
            mapped[r] = nb
        if ptr > total:
            raise RuntimeError(f"Layer {layer_idx}: Allocation logic error! Used more than allocated.")
        if self._group is not None:
            # pages in the group's shared pool: this cache's ids start at its
            # range's offset; page table and lengths are rows of shared tensors
            kp, vp, off, bt_t, hl_t = self._group._layer_storage(self, layer_idx, total, rows, max_blocks,
                                                                 device, dtype)
            bt_t.copy_(torch.from_numpy(np.where(bt >= 0, bt + off, bt).astype(np.int32)))
            hl_t.zero_()
            self.key_pools[layer_idx], self.value_pools[layer_idx] = kp, vp
            self.block_tables[layer_idx] = bt_t
            self.free_blocks[layer_idx] = torch.arange(off + ptr, off + total, dtype=torch.int32, device=device)
            self.heads_len[layer_idx] = hl_t
        else:
            self.key_pools[layer_idx] = torch.zeros(total, PAGE, 1, self.head_dim, device=device, dtype=dtype)
            self.value_pools[layer_idx] = torch.zeros(total, PAGE, 1, self.head_dim, device=device, dtype=dtype)
            self.block_tables[layer_idx] = torch.from_numpy(bt).to(device)
            self.free_blocks[layer_idx] = torch.arange(ptr, total, dtype=torch.int32, device=device)
            self.heads_len[layer_idx] = torch.zeros(rows, dtype=torch.int32, device=device)
        self.free_block_pointers[layer_idx] = 0
        self._free_ptr[layer_idx] = torch.zeros(1, dtype=torch.int32, device=device)
        self.prefill_boundary_blocks[layer_idx] = pre_total
        self.layer_head_capacities[layer_idx] = caps
        self._hlen[layer_idx] = np.zeros(rows, dtype=np.int64)
        self._mapped[layer_idx] = mapped
        self._slack[layer_idx] = 0

    def _side(self) -> torch.cuda.Stream:
        if self._side_stream is None:
            self._side_stream = torch.cuda.Stream(device=self._dev)
        return self._side_stream

    def _wait_retrieval(self, layer_idx: int) -> None:
        ev = self._retrieve_done[layer_idx]
        if ev is not None:
            torch.cuda.current_stream(self._dev).wait_event(ev)
            self._retrieve_done[layer_idx] = None

    def _wait_append(self, layer_idx: int) -> None:
        ev = self._append_done[layer_idx]
        if ev is not None:
            torch.cuda.current_stream(self._dev).wait_event(ev)
            self._append_done[layer_idx] = None

    def join_retrievals(self) -> None:
        """Make the current stream wait for every side-stream job still running:
        retrievals (host-tier mode) and deferred page appends.  A captured
        decode step ends with this, so each CUDA graph joins the side-stream
        work it forked."""
        self.flush_checks()
        for layer_idx in range(len(self._retrieve_done)):
            self._wait_retrieval(layer_idx)
            self._wait_append(layer_idx)

    # ------------------------------------------------------------------
    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """heterocache/cache_utils.py:884-1005."""
        if self._deferred and layer_idx in self._deferred:
            self.flush_checks()  # the put-off check reads this layer's query buffer
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[-2]
        self._ensure_device(key_states.device)
        if self.bsz is None:
            self.bsz = key_states.shape[0]
            self.head_dim = key_states.shape[-1]
        if not hasattr(self, "base_compress_len"):
            self.prefill_len = key_states.shape[-2]
            self.base_compress_len = get_compress_len(self.compression_ratio, self.full_heads, self.prefill_len,
                                                      self.total_kv_heads)
        if self.key_pools[layer_idx] is None:
            self._init_layer_storage(layer_idx, key_states.device, key_states.dtype)
        seq_len = key_states.shape[-2]
        if seq_len > 1:
            self._slack[layer_idx] = 0  # the prefill sets the lengths anew
            self.prefill_len = seq_len
            keep = self.data["need_to_keep_counts"][layer_idx]
            upd = self.data["need_to_update_counts"][layer_idx]
            if keep:
                keep_t = torch.tensor(keep, dtype=torch.int32, device=key_states.device)
                ops.prefill_keep(key_states, value_states, keep_t, self.key_pools[layer_idx],
                                 self.value_pools[layer_idx], self.block_tables[layer_idx],
                                 self.heads_len[layer_idx], self._err)
                for b in range(self.bsz):
                    for h in keep:
                        self._hlen[layer_idx][b * self.num_kv_heads + h] = seq_len
            if not upd:
                self.key_cache_cpu.append(None)
                self.value_cache_cpu.append(None)
            elif self.real_offload:
                # only the satellites' rows are ever read back (retrieval):
                # after the load-time role permutation they are contiguous
                # heads, so the pinned tier holds [bsz, n_sat, L, D] from
                # head `first` on (the reference backs up every head,
                # cache_utils.py:953-960)
                first, n_tier = 0, self.num_kv_heads
                if list(upd) == list(range(upd[0], upd[0] + len(upd))):
                    first, n_tier = upd[0], len(upd)
                ks = key_states.detach()[:, first:first + n_tier]
                vs = value_states.detach()[:, first:first + n_tier]
                try:
                    kc = torch.empty(ks.shape, dtype=key_states.dtype, pin_memory=True)
                    vc = torch.empty(vs.shape, dtype=value_states.dtype, pin_memory=True)
                except RuntimeError as e:
                    nbytes = 2 * ks.numel() * key_states.element_size()
                    raise RuntimeError(f"Layer {layer_idx}: pinned host allocation of {nbytes} bytes for the "
                                       f"full KV tier failed ({e})") from e
                side = self._side()
                side.wait_stream(torch.cuda.current_stream(key_states.device))
                with torch.cuda.stream(side):
                    kc.copy_(ks, non_blocking=True)
                    vc.copy_(vs, non_blocking=True)
                key_states.record_stream(side)
                value_states.record_stream(side)
                self.key_cache_cpu.append(kc)
                self.value_cache_cpu.append(vc)
                self._tier_first[layer_idx] = first
            else:
                self.key_cache_cpu.append(key_states.detach())
                self.value_cache_cpu.append(value_states.detach())
            return key_states, value_states

        self._append_bookkeeping(layer_idx)
        self._wait_retrieval(layer_idx)
        self._wait_append(layer_idx)
        kw = cache_kwargs or {}
        # A caller that passes the step's query (cache_kwargs["query_states"],
        # as the attention modules of this package do) has a launch it makes
        # anyway store it into the drift-check buffer (the page append, or with
        # a deferred append the attention's combine kernel); decode_select
        # then skips its own copy.
        q = kw.get("query_states") if self.bsz == 1 else None
        if q is not None:
            self._ensure_decode_state(layer_idx, q)
        if kw.get("defer_append"):
            # attention() attends over the pages plus this token, then appends
            # it on the side stream, off the attention's critical path
            # [k, v, q (None once stored), query slot, decode_select of this step already ran]
            self._pending[layer_idx] = [key_states, value_states, q, self._qcount[layer_idx], False]
            return key_states, value_states
        q_stage = None
        if q is not None:
            q_stage = self._qbuf[layer_idx][self._qcount[layer_idx]]
        ops.decode_append(key_states, value_states, self.key_pools[layer_idx], self.value_pools[layer_idx],
                          self.block_tables[layer_idx], self.heads_len[layer_idx], self.free_blocks[layer_idx],
                          self._free_ptr[layer_idx], self._err, q=q, q_stage=q_stage)
        self._q_staged[layer_idx] = q_stage is not None
        return key_states, value_states

    def _append_bookkeeping(self, layer_idx: int) -> None:
        """Host side of a decode append: the free-list check of
        cache_utils.py:981-990 on the mirrored lengths (raises before any
        launch), then the mirrors advance as the device state will.

        After a full check the layer's slack is the number of further appends
        that can map no new page and hit no page-table end (every row grows by
        one token per append): min over rows of min(mapped, table width) x
        256 - length.  Those appends only advance the lengths, so they skip
        the checks, which would find nothing (a few numpy calls per layer and
        step on the host, which sets the pace of a captured decode step over
        many small caches)."""
        hl = self._hlen[layer_idx]
        s = self._slack[layer_idx]
        if s > 0:
            self._slack[layer_idx] = s - 1
            hl += 1
            return
        width = self.block_tables[layer_idx].shape[1]
        logical = hl // PAGE
        if np.any(logical >= width):
            raise IndexError(f"Layer {layer_idx}: block table has no column for the next decode token")
        grow = logical >= self._mapped[layer_idx]
        need = int(np.count_nonzero(grow))
        if need > 0:
            ptr = self.free_block_pointers[layer_idx]
            if ptr + need > self.free_blocks[layer_idx].size(0):
                raise RuntimeError(f"Layer {layer_idx} OOM.")
            self.free_block_pointers[layer_idx] += need
            self._mapped[layer_idx] += grow
        hl += 1
        room = np.minimum(self._mapped[layer_idx], width) * PAGE - hl
        self._slack[layer_idx] = max(int(room.min()), 0) if room.size else 0

    def init_coefficient(self, query_states, key_states, layer_idx):
        """Pivot reference sets (heterocache/cache_utils.py:1149-1190)."""
        pivots = self.data["need_to_select_counts"][layer_idx]
        if len(pivots) == 0:
            self.prefill_topk_set.append([])
            return
        if list(pivots) != list(range(pivots[0], pivots[0] + len(pivots))):
            raise ValueError("pivot heads must be contiguous after the role permutation")
        bsz = key_states.shape[0]
        L = key_states.shape[-2]
        K = self.base_compress_len
        dev = key_states.device
        ref = torch.empty(bsz, len(pivots), K, dtype=torch.int32, device=dev)
        words = (L + 31) // 32
        bitmap = torch.zeros(bsz, len(pivots), words, dtype=torch.int32, device=dev)
        scores = (torch.empty(bsz, len(pivots), L, dtype=key_states.dtype, device=dev)
                  if self.record_checks else None)
        ops.pivot_init(query_states, key_states, first_pivot=pivots[0], n_pivots=len(pivots),
                       groups=self.num_key_value_groups, pooling=self.pooling, kernel_size=self.kernel_size,
                       topk=K, ref_positions=ref, ref_bitmap=bitmap, workspace=self._ws_score, err=self._err,
                       out_scores=scores)
        if scores is not None:
            self.recorded[("pivot_scores", layer_idx)] = scores
        self._ref_bitmap[layer_idx] = bitmap
        self.prefill_topk_set.append(ref)

    def prefill_select(self, query_states, key_states, value_states, layer_idx):
        """Compressed heads (heterocache/cache_utils.py:782-882)."""
        self._slack[layer_idx] = 0  # sets the compressed heads' lengths
        bsz = query_states.shape[0]
        nc = self.data["need_to_compress_counts"][layer_idx]
        if nc == 0:
            return
        ratios = torch.tensor(self.data["allocation_matrix"][layer_idx][:nc], dtype=torch.float32)
        caps = (self.base_compress_len * ratios).int()
        L = key_states.shape[-2]
        keep_lens = torch.clamp(caps, max=L)
        max_k = int(keep_lens.max())
        if max_k == 0:
            self.heads_len[layer_idx][:nc] = 0
            self._hlen[layer_idx][:nc] = 0
            return
        dev = key_states.device
        keep_dev = keep_lens.to(device=dev, dtype=torch.int32)
        scores = idx = None
        # a pinned-host tier keeps the satellites' kept indices: they seed the
        # slot maps of the delta retrieval
        keep_idx = self.real_offload and any(self.data["leader_member_relations"][layer_idx].values())
        if self.record_checks or keep_idx:
            idx = torch.empty(bsz, nc, max_k, dtype=torch.int32, device=dev)
        if self.record_checks:
            scores = torch.empty(bsz, nc, L, dtype=key_states.dtype, device=dev)
            self.recorded[("prefill_scores", layer_idx)] = scores
            self.recorded[("prefill_indices", layer_idx)] = idx
            self.recorded[("keep_lens", layer_idx)] = keep_lens.clone()
        ops.prefill_select(query_states, key_states, value_states, keep_dev, max_k, n_heads=nc,
                           groups=self.num_key_value_groups, window=self.window_size, pooling=self.pooling,
                           kernel_size=self.kernel_size, k_pool=self.key_pools[layer_idx],
                           v_pool=self.value_pools[layer_idx], block_table=self.block_tables[layer_idx],
                           heads_len=self.heads_len[layer_idx], workspace=self._ws_score, err=self._err,
                           out_indices=idx, out_scores=scores)
        kl = keep_lens.numpy().astype(np.int64)
        for b in range(bsz):
            self._hlen[layer_idx][b * self.num_kv_heads:b * self.num_kv_heads + nc] = kl
        if keep_idx:
            self._kept[layer_idx] = (idx, kl.copy())

    # ------------------------------------------------------------------
    def _ensure_decode_state(self, layer_idx, query_states) -> None:
        S = self.decode_step
        if self._qbuf[layer_idx] is None:
            bsz, H, _, D = query_states.shape
            if bsz != 1 and self.data["leader_member_relations"][layer_idx]:
                raise NotImplementedError("decode_select supports batch size 1 (as the reference, "
                                          "cache_utils.py:1093)")
            if self._group is not None:
                self._qbuf[layer_idx] = self._group._query_buffer(self, layer_idx, S, H, D, query_states.dtype,
                                                                  query_states.device)
            else:
                self._qbuf[layer_idx] = torch.empty(S, H, D, dtype=query_states.dtype, device=query_states.device)
        relations = self.data["leader_member_relations"][layer_idx]
        if self._jobs[layer_idx] is None and relations:
            remote = self.data.get("remote_member_alloc")
            jobs = _LayerJobs(relations, self.data["allocation_matrix"][layer_idx], self.base_compress_len,
                              self.prefill_len, query_states.device,
                              remote_alloc=remote[layer_idx] if remote else None)
            if self.record_checks:
                jobs.coeffs = torch.zeros(max(jobs.n_jobs, 1), S, dtype=torch.float32, device=query_states.device)
                jobs.median = torch.zeros(max(jobs.n_jobs, 1), dtype=torch.float64, device=query_states.device)
            self._jobs[layer_idx] = jobs
            if self.real_offload and jobs.member_job.numel() and self._kept[layer_idx] is not None:
                self._init_delta(layer_idx, jobs)

    def _init_delta(self, layer_idx, jobs) -> None:
        """Slot maps of the delta retrieval (pinned-host tier).  Member i holds
        its prefill kept indices in slots [0, R_i), R_i = min(its prefill keep
        length, its retrieval length): decode appends start at the keep length,
        so only prefill selection and retrieval write those slots, and each
        writes them in ascending position order."""
        idx, kl = self._kept[layer_idx]
        self._kept[layer_idx] = None
        dev = idx.device
        nc = idx.shape[1]
        reuse = [min(int(kl[h]), n) if h < nc else 0 for h, n in zip(jobs.m_head_list, jobs.m_len_list)]
        slot = torch.zeros(len(reuse), max(max(reuse), 1), dtype=torch.int32, device=dev)
        for i, (h, r) in enumerate(zip(jobs.m_head_list, reuse)):
            if r:
                slot[i, :r].copy_(idx[0, h, :r])
        offs = np.concatenate([[0], np.cumsum(jobs.m_len_list)[:-1]]).astype(np.int64)
        i32 = dict(dtype=torch.int32, device=dev)
        jobs.delta = {"slot": slot, "reuse": torch.tensor(reuse, **i32), "off": torch.tensor(offs, **i32)}
        if self._stage is None:
            # one staging area for every layer (their retrievals run in order
            # on the side stream), sized for the largest layer
            rows = 0
            for l in range(self.num_layers):
                alloc = self.data["allocation_matrix"][l]
                rows = max(rows, sum(min(int(self.base_compress_len * alloc[m]), self.prefill_len)
                                     for members in self.data["leader_member_relations"][l].values()
                                     for m in members))
            dt = self.key_pools[layer_idx].dtype
            D = self.key_pools[layer_idx].shape[-1]
            self._stage = (torch.empty(rows, D, dtype=dt, device=dev), torch.empty(rows, D, dtype=dt, device=dev),
                           torch.empty(rows, **i32))

    def prepare_decode(self, layers, query_example) -> None:
        """Allocate every layer's decode-time buffers now (before graph capture),
        the scoring workspace included: large enough for a drift-check batch
        of all these layers and for each layer's own check."""
        for l in layers:
            self._ensure_decode_state(l, query_example)
        n = sum(self._jobs[l].n_jobs for l in layers if self._jobs[l] is not None)
        if n and self._ws_score is not None:
            dt = ops.DTYPES[query_example.dtype]
            S, G = self.decode_step, self.num_key_value_groups
            need = max(ops.lib().hc_drift_check_batch_workspace_size(dt, n, S, self.prefill_len, G,
                                                                     self.drift_batch_per_launch),
                       max(ops.lib().hc_drift_check_workspace_size(dt, self._jobs[l].n_jobs, S, self.prefill_len, G)
                           for l in layers if self._jobs[l] is not None))
            self._ws_score.get(need)

    def _host_state(self):
        return {"hlen": [None if h is None else h.copy() for h in self._hlen],
                "mapped": [None if m is None else m.copy() for m in self._mapped], "slack": list(self._slack),
                "free_ptr": list(self.free_block_pointers), "qcount": list(self._qcount),
                "retrieve_done": list(self._retrieve_done), "seen": self._seen_tokens,
                "pending": [None if x is None else list(x) for x in self._pending],
                "append_done": list(self._append_done),
                "q_staged": list(self._q_staged), "deferred": list(self._deferred)}

    def _restore_host_state(self, s) -> None:
        self._hlen, self._mapped, self._slack = s["hlen"], s["mapped"], s["slack"]
        self.free_block_pointers, self._qcount = s["free_ptr"], s["qcount"]
        self._retrieve_done, self._seen_tokens = s["retrieve_done"], s["seen"]
        self._pending, self._append_done, self._q_staged = s["pending"], s["append_done"], s["q_staged"]
        self._deferred = s["deferred"]

    def decode_select(self, query_states, layer_idx, defer: bool = False):
        """Pivot drift check and satellite retrieval (heterocache/cache_utils.py:1007-1147).

        ``defer=True`` (with ``defer_checks`` on) puts a due check off until
        ``flush_checks()``, which runs every put-off layer's check in one
        batch.  The caller guarantees that the layer's attention does not run
        before that (the Llama order, where decode_select follows attention);
        the layer's next update, attention or decode_select flushes first."""
        if self._deferred and layer_idx in self._deferred:
            self.flush_checks()
        S = self.decode_step
        self._ensure_decode_state(layer_idx, query_states)
        pend = self._pending[layer_idx]
        check = self._qcount[layer_idx] + 1 >= S
        if pend is not None:
            # decode_select before attention (Qwen order): this step's
            # attention is still to come; it stores the query, except that a
            # drift check now needs it at once
            pend[4] = True
            if check or pend[2] is None:
                self._qbuf[layer_idx][self._qcount[layer_idx]].copy_(query_states[0, :, 0, :])
                pend[2] = None  # stored
        elif self._q_staged[layer_idx]:
            self._q_staged[layer_idx] = False  # this step's append stored it
        else:
            self._qbuf[layer_idx][self._qcount[layer_idx]].copy_(query_states[0, :, 0, :])
        self._qcount[layer_idx] += 1
        if self._qcount[layer_idx] < S:
            return
        self._qcount[layer_idx] = 0
        jobs = self._jobs[layer_idx]
        if jobs is None or jobs.n_jobs == 0:
            return
        if defer and self.defer_checks:
            self._deferred.append(layer_idx)
            return
        self._drift_and_retrieve(layer_idx, jobs, query_states)

    def flush_checks(self) -> None:
        """Run the drift checks put off by decode_select(..., defer=True): all
        put-off layers' pivots in one hc_drift_check_batch call (a few
        launches instead of one per layer), then each layer's retrieval.
        Every result is the one the check gives where it was put off: no
        update, attention or decode_select of such a layer runs before this."""
        layers, self._deferred = self._deferred, []
        if not layers:
            return
        for l in layers:
            self._wait_retrieval(l)
        key = tuple(layers)
        arr = self._batch_arrays.get(key)
        if arr is None:
            descs = []
            for l in layers:
                descs.extend(self._drift_descs(l))
            arr = ops.drift_jobs_array(descs)
            self._batch_arrays[key] = arr
        dt = self.key_pools[layers[0]].dtype
        ops.drift_check_batch(arr, dtype=dt, device=self._dev, num_kv_heads=self.num_kv_heads,
                              groups=self.num_key_value_groups, steps=self.decode_step, seq_len=self.prefill_len,
                              pooling=self.pooling, kernel_size=self.kernel_size, topk=self.base_compress_len,
                              threshold=self.stable_threshold, workspace=self._ws_score, err=self._err,
                              jobs_per_launch=self.drift_batch_per_launch)
        for l in layers:
            jobs = self._jobs[l]
            if self.record_checks:
                self._log_check(l, jobs, None)
            self._retrieve_layer(l, jobs)

    def _drift_descs(self, layer_idx):
        """The layer's drift-check descriptors (built once: every tensor they
        point into lives as long as the cache)."""
        jobs = self._jobs[layer_idx]
        if jobs.batch_descs is None:
            bm, ref = self._ref_bitmap[layer_idx], self.prefill_topk_set[layer_idx]
            jobs.batch_descs = [
                ops.drift_job(self._qbuf[layer_idx], self.key_pools[layer_idx], self.block_tables[layer_idx],
                              pivot_head=jobs.pivot_list[j], max_len=jobs.max_len_list[j],
                              ref_bitmap=bm[0, jobs.slot_list[j]], ref_positions=ref[0, jobs.slot_list[j]],
                              trigger=jobs.trigger[j:j + 1], retrieve_positions=jobs.retrieve_positions[j],
                              coeffs=None if jobs.coeffs is None else jobs.coeffs[j],
                              median=None if jobs.median is None else jobs.median[j:j + 1])
                for j in range(jobs.n_jobs)]
        return jobs.batch_descs

    def _log_check(self, layer_idx, jobs, scores) -> None:
        self.check_log.append({"layer": layer_idx, "trigger": jobs.trigger.clone(),
                               "coeffs": jobs.coeffs.clone(), "median": jobs.median.clone(),
                               "retrieved": jobs.retrieve_positions.clone(),
                               "pivots": jobs.pivot_heads.tolist(), "slots": jobs.ref_slots.tolist(),
                               "max_len": jobs.max_len.tolist(), "scores": scores,
                               "ref_after": self.prefill_topk_set[layer_idx].clone()})

    def _drift_and_retrieve(self, layer_idx, jobs, query_states):
        S = self.decode_step
        # the step's query is in the buffer: stored on this stream by the
        # attention (deferred append), by the append itself, or just above
        self._wait_retrieval(layer_idx)
        scores = (torch.empty(jobs.n_jobs, S, self.prefill_len, dtype=query_states.dtype,
                              device=query_states.device) if self.record_checks else None)
        ops.drift_check(self._qbuf[layer_idx], self.key_pools[layer_idx], self.block_tables[layer_idx],
                        num_kv_heads=self.num_kv_heads, groups=self.num_key_value_groups, steps=S,
                        seq_len=self.prefill_len, pooling=self.pooling, kernel_size=self.kernel_size,
                        topk=self.base_compress_len, threshold=self.stable_threshold,
                        pivot_heads=jobs.pivot_heads, ref_slots=jobs.ref_slots, max_len=jobs.max_len,
                        max_len_cap=max(jobs.max_len_cap, 1), ref_bitmap=self._ref_bitmap[layer_idx],
                        ref_positions=self.prefill_topk_set[layer_idx], trigger=jobs.trigger,
                        retrieve_positions=jobs.retrieve_positions, workspace=self._ws_score, err=self._err,
                        coeffs=jobs.coeffs, median=jobs.median, out_scores=scores)
        if self.record_checks:
            self._log_check(layer_idx, jobs, scores)
        self._retrieve_layer(layer_idx, jobs)

    def _retrieve_layer(self, layer_idx, jobs) -> None:
        """The satellites' retrieval after the layer's drift check."""
        if jobs.member_job.numel() == 0:
            return
        full_k = self.key_cache_cpu[layer_idx]
        full_v = self.value_cache_cpu[layer_idx]
        first = self._tier_first[layer_idx]
        if jobs.m_head_list and not (first <= min(jobs.m_head_list) and
                                     max(jobs.m_head_list) < first + full_k.shape[1]):
            raise RuntimeError(f"Layer {layer_idx}: a satellite lies outside the full tier's heads")
        if self.real_offload:
            main = torch.cuda.current_stream(self._dev)
            side = self._side()
            side.wait_stream(main)
            if jobs.delta is not None:
                # only rows the satellites do not hold cross the host link
                sk, sv, ss = self._stage
                ops.retrieve_delta(member_job=jobs.member_job, member_head=jobs.member_head,
                                   member_len=jobs.member_len, member_stage_offset=jobs.delta["off"],
                                   reuse_len=jobs.delta["reuse"], max_member_len=jobs.max_member_len,
                                   trigger=jobs.trigger, retrieve_positions=jobs.retrieve_positions,
                                   slot_positions=jobs.delta["slot"], full_k=full_k, full_v=full_v,
                                   tier_first_head=first,
                                   k_pool=self.key_pools[layer_idx], v_pool=self.value_pools[layer_idx],
                                   block_table=self.block_tables[layer_idx], num_kv_heads=self.num_kv_heads,
                                   stage_k=sk, stage_v=sv, stage_src=ss, err=self._err, stream=side)
            else:
                ops.retrieve(member_job=jobs.member_job, member_head=jobs.member_head, member_len=jobs.member_len,
                             max_member_len=jobs.max_member_len, trigger=jobs.trigger,
                             retrieve_positions=jobs.retrieve_positions, full_k=full_k, full_v=full_v,
                             k_pool=self.key_pools[layer_idx], v_pool=self.value_pools[layer_idx],
                             block_table=self.block_tables[layer_idx], num_kv_heads=self.num_kv_heads,
                             err=self._err, stream=side, tier_first_head=first)
            ev = torch.cuda.Event()
            ev.record(side)
            self._retrieve_done[layer_idx] = ev
        else:
            ops.retrieve(member_job=jobs.member_job, member_head=jobs.member_head, member_len=jobs.member_len,
                         max_member_len=jobs.max_member_len, trigger=jobs.trigger,
                         retrieve_positions=jobs.retrieve_positions, full_k=full_k, full_v=full_v,
                         k_pool=self.key_pools[layer_idx], v_pool=self.value_pools[layer_idx],
                         block_table=self.block_tables[layer_idx], num_kv_heads=self.num_kv_heads,
                         err=self._err, tier_first_head=first)

    def full_tier(self, layer_idx):
        """(k, v, first_head): the layer's full KV tier and the head id of its
        row 0 ([bsz, heads, L, D] on the device, or the satellites' rows in
        pinned host memory), or None for a layer without satellites."""
        if self.key_cache_cpu[layer_idx] is None:
            return None
        return self.key_cache_cpu[layer_idx], self.value_cache_cpu[layer_idx], self._tier_first[layer_idx]

    # ------------------------------------------------------------------
    def attention(self, query_states, layer_idx, scale: float = 0.0, out=None, mirrors=None,
                  mirror_batch_stride: int = 0):
        """Decode attention over this layer's pages: q [bsz, H, 1, D] -> [bsz, H, D].

        With a deferred append pending (update(..., {"defer_append": True})),
        the step's token is merged from its k/v and then appended to the pages
        on the side stream; the layer's next use waits for that append.
        ``mirrors`` (device addresses) each receive a copy of the output (see
        ``ops.flash_decode``): the head-sharded mode's gathered outputs on
        every GPU."""
        if self._deferred and layer_idx in self._deferred:
            self.flush_checks()
        self._wait_retrieval(layer_idx)
        self._wait_append(layer_idx)
        total = int(self._hlen[layer_idx].sum())
        pend = self._pending[layer_idx]
        if pend is None:
            return ops.flash_decode(query_states, self.key_pools[layer_idx], self.value_pools[layer_idx],
                                    self.block_tables[layer_idx], self.heads_len[layer_idx],
                                    num_kv_heads=self.num_kv_heads, scale=scale, out=out, workspace=self._ws_fd,
                                    err=self._err, total_tokens_hint=total, mirrors=mirrors,
                                    mirror_batch_stride=mirror_batch_stride)
        self._pending[layer_idx] = None
        k, v, q, slot, selected = pend
        # the step's query goes to the drift-check buffer on this stream (the
        # combine kernel stores it when it is the query attended with), so a
        # drift check right after need not wait for the side-stream append
        same_q = (q is not None and q.data_ptr() == query_states.data_ptr() and q.shape == query_states.shape
                  and q.stride() == query_states.stride())
        if q is not None and not same_q:
            self._qbuf[layer_idx][slot].copy_(q[0, :, 0, :])
        out = ops.flash_decode(query_states, self.key_pools[layer_idx], self.value_pools[layer_idx],
                               self.block_tables[layer_idx], self.heads_len[layer_idx],
                               num_kv_heads=self.num_kv_heads, scale=scale, out=out, workspace=self._ws_fd,
                               err=self._err, k_new=k, v_new=v,
                               q_stage=self._qbuf[layer_idx][slot] if same_q else None, mirrors=mirrors,
                               mirror_batch_stride=mirror_batch_stride)
        main = torch.cuda.current_stream(self._dev)
        side = self._side()
        side.wait_stream(main)
        with torch.cuda.stream(side):
            ops.decode_append(k, v, self.key_pools[layer_idx], self.value_pools[layer_idx],
                              self.block_tables[layer_idx], self.heads_len[layer_idx], self.free_blocks[layer_idx],
                              self._free_ptr[layer_idx], self._err)
        if not torch.cuda.is_current_stream_capturing():  # a graph's buffers are static
            for t in (k, v):
                t.record_stream(side)
        ev = torch.cuda.Event()
        ev.record(side)
        self._append_done[layer_idx] = ev
        if q is not None and not selected:
            self._q_staged[layer_idx] = True  # decode_select of this step comes next
        return out


def flush_checks_together(caches) -> None:
    """``flush_checks`` over several caches at once: every drift check the
    caches put off (``decode_select(..., defer=True)``) in one
    hc_drift_check_batch call, then each cache's retrievals -- e.g. the
    independent sequences of one batch, each with its own cache, whose
    checks would otherwise take a launch each.  The caches must share the
    check's shape: dtype, KV heads, GQA groups, ``decode_step``, prefill
    length, budget, pooling and stable threshold (the same model and prompt
    length).  Results equal per-cache flushes; a device-side error of the
    batch is reported in the first cache's error flag."""
    pend = [(c, c._deferred) for c in caches if c._deferred]
    if not pend:
        return
    first = pend[0][0]
    shape = lambda c: (c.key_pools[c._deferred[0]].dtype, c.num_kv_heads, c.num_key_value_groups,  # noqa: E731
                       c.decode_step, c.prefill_len, c.base_compress_len, c.pooling, c.kernel_size,
                       c.stable_threshold, c._dev)
    want = shape(first)
    for c, _ in pend:
        if shape(c) != want:
            raise ValueError("flush_checks_together: the caches' drift checks differ in shape")
    for c, layers in pend:
        c._deferred = []
        for l in layers:
            c._wait_retrieval(l)
    key = tuple((id(c), tuple(layers)) for c, layers in pend)
    arr = first._batch_arrays.get(key)
    if arr is None:
        descs = []
        for c, layers in pend:
            for l in layers:
                descs.extend(c._drift_descs(l))
        arr = ops.drift_jobs_array(descs)
        first._batch_arrays[key] = arr
    ops.drift_check_batch(arr, dtype=want[0], device=first._dev, num_kv_heads=first.num_kv_heads,
                          groups=first.num_key_value_groups, steps=first.decode_step, seq_len=first.prefill_len,
                          pooling=first.pooling, kernel_size=first.kernel_size, topk=first.base_compress_len,
                          threshold=first.stable_threshold, workspace=first._ws_score, err=first._err,
                          jobs_per_launch=first.drift_batch_per_launch)
    for c, layers in pend:
        for l in layers:
            jobs = c._jobs[l]
            if c.record_checks:
                c._log_check(l, jobs, None)
            c._retrieve_layer(l, jobs)


class CacheGroup:
    """Independent sequences -- one ``HeteroCache`` each, batch 1, as the
    reference's drift check requires (heterocache/cache_utils.py:1093) --
    whose pages share one pool per layer, so that one decode launch
    (``attention_together``) attends over all of them instead of one launch
    per sequence.  Each member's page ids are a range of its own in the
    shared pool, and its page table and lengths are rows of shared tensors;
    everything else (page appends, drift checks, retrievals, free lists) stays
    per member and unchanged.  Adopt the caches before their prefill; they
    must need the same pages per layer (the same model, roles and prompt
    length)."""

    def __init__(self, caches):
        self.members = list(caches)
        for i, c in enumerate(self.members):
            if any(p is not None for p in c.key_pools):
                raise RuntimeError("CacheGroup: adopt caches before their prefill")
            c._group, c._gidx = self, i
        self._layers: Dict[int, dict] = {}
        self._qbufs: Dict[int, torch.Tensor] = {}
        self._ws: Optional[Workspace] = None

    def _query_buffer(self, cache, layer, S, H, D, dtype, device):
        """Member's drift-check query buffer [S, H, D]: row ``cache._gidx`` of
        the layer's [members, S, H, D] buffer, so that a step stages every
        member's query in one copy."""
        qb = self._qbufs.get(layer)
        if qb is None:
            qb = torch.empty(len(self.members), S, H, D, dtype=dtype, device=device)
            self._qbufs[layer] = qb
        if tuple(qb.shape[1:]) != (S, H, D) or qb.dtype != dtype:
            raise ValueError("CacheGroup: the members' query buffers differ in shape")
        return qb[cache._gidx]

    def _workspace(self, device) -> Workspace:
        if self._ws is None:
            self._ws = Workspace(device)
        return self._ws

    def _layer_storage(self, cache, layer, total, rows, max_blocks, device, dtype):
        st = self._layers.get(layer)
        n = len(self.members)
        if st is None:
            D = cache.head_dim
            st = dict(slot=total, rows=rows, mb=max_blocks, dtype=dtype, device=torch.device(device),
                      kp=torch.zeros(n * total, PAGE, 1, D, device=device, dtype=dtype),
                      vp=torch.zeros(n * total, PAGE, 1, D, device=device, dtype=dtype),
                      bt=torch.full((n * rows, max_blocks), -1, dtype=torch.int32, device=device),
                      hl=torch.zeros(n * rows, dtype=torch.int32, device=device))
            self._layers[layer] = st
        if (total > st["slot"] or rows != st["rows"] or max_blocks != st["mb"] or dtype != st["dtype"]):
            raise ValueError("CacheGroup: the members need different pages for this layer")
        i = cache._gidx
        return st["kp"], st["vp"], i * st["slot"], st["bt"][i * rows:(i + 1) * rows], st["hl"][i * rows:(i + 1) * rows]


def _batch_view(ts):
    """[n, ...] view over n batch-1 tensors of one shape and strides that sit
    at a constant distance in one storage (rows of one buffer), else None."""
    t0 = ts[0]
    if len(ts) == 1:
        return t0
    es = t0.element_size()
    d = ts[1].data_ptr() - t0.data_ptr()
    if d <= 0 or d % es:
        return None
    for i, t in enumerate(ts):
        if (t.shape != t0.shape or t.stride() != t0.stride() or t.dtype != t0.dtype
                or t.untyped_storage().data_ptr() != t0.untyped_storage().data_ptr()
                or t.data_ptr() - t0.data_ptr() != i * d):
            return None
    return t0.as_strided((len(ts),) + tuple(t0.shape[1:]), (d // es,) + tuple(t0.stride()[1:]))


def attention_together(group: CacheGroup, query_states, layer_idx, scale: float = 0.0, out=None, mirrors=None,
                       mirror_batch_stride: int = 0):
    """Every member's decode attention for one layer in one launch:
    ``query_states`` [members, H, 1, D] (row i: member i's query) ->
    [members, H, D], as each member's ``attention`` would give (the split of
    the tokens over the launch differs, so the fp32 merge order does too).
    Members with a deferred append (``update(..., {"defer_append": True})``)
    all must have one: the step's tokens are merged from their k/v, then each
    member appends on its own side stream.  ``mirrors`` as for
    ``HeteroCache.attention``, row b of the batch being member b.  A
    device-side error of the launch is reported in the first member's flag."""
    members = group.members
    for c in members:
        if c._deferred and layer_idx in c._deferred:
            c.flush_checks()
        c._wait_retrieval(layer_idx)
        c._wait_append(layer_idx)
    st = group._layers[layer_idx]
    c0 = members[0]
    if query_states.shape[0] != len(members):
        raise ValueError("attention_together: one query row per member")
    ws = group._workspace(c0._dev)
    total = sum(int(c._hlen[layer_idx].sum()) for c in members)
    pends = [c._pending[layer_idx] for c in members]
    if all(p is None for p in pends):
        return ops.flash_decode(query_states, st["kp"], st["vp"], st["bt"], st["hl"], num_kv_heads=c0.num_kv_heads,
                                scale=scale, out=out, workspace=ws, err=c0._err, total_tokens_hint=total,
                                mirrors=mirrors, mirror_batch_stride=mirror_batch_stride)
    if any(p is None for p in pends):
        raise RuntimeError("attention_together: some members have the step's token pending and some not")
    for c in members:
        c._pending[layer_idx] = None
    # the step's queries for the drift checks (this stream): one copy when
    # they all go to the same slot of the group's buffer
    stage = [(c, p[2], p[3]) for c, p in zip(members, pends) if p[2] is not None]
    qg = group._qbufs.get(layer_idx)
    if (qg is not None and len(stage) == len(members) and len({sl for _, _, sl in stage}) == 1
            and all(c._qbuf[layer_idx].data_ptr() == qg[c._gidx].data_ptr() for c in members)):
        qs = _batch_view([q for _, q, _ in stage])
        if qs is None:
            qs = torch.cat([q for _, q, _ in stage], 0)
        qg[:, stage[0][2]].copy_(qs[:, :, 0, :])
    else:
        for c, q, slot in stage:
            c._qbuf[layer_idx][slot].copy_(q[0, :, 0, :])
    k_new = _batch_view([p[0] for p in pends])
    v_new = _batch_view([p[1] for p in pends])
    k_new = torch.cat([p[0] for p in pends], 0) if k_new is None else k_new
    v_new = torch.cat([p[1] for p in pends], 0) if v_new is None else v_new
    out = ops.flash_decode(query_states, st["kp"], st["vp"], st["bt"], st["hl"], num_kv_heads=c0.num_kv_heads,
                           scale=scale, out=out, workspace=ws, err=c0._err, total_tokens_hint=total, k_new=k_new,
                           v_new=v_new, mirrors=mirrors, mirror_batch_stride=mirror_batch_stride)
    main = torch.cuda.current_stream(c0._dev)
    for c, (k, v, q, slot, selected) in zip(members, pends):
        side = c._side()
        side.wait_stream(main)
        with torch.cuda.stream(side):
            ops.decode_append(k, v, c.key_pools[layer_idx], c.value_pools[layer_idx], c.block_tables[layer_idx],
                              c.heads_len[layer_idx], c.free_blocks[layer_idx], c._free_ptr[layer_idx], c._err)
        if not torch.cuda.is_current_stream_capturing():
            for t in (k, v):
                t.record_stream(side)
        ev = torch.cuda.Event()
        ev.record(side)
        c._append_done[layer_idx] = ev
        if q is not None and not selected:
            c._q_staged[layer_idx] = True  # decode_select of this step comes next
    return out
