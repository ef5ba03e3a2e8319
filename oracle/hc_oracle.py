"""CPU oracle for HeteroCache's compressed-KV attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module: it is
the checker that ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` run beside the CUDA path.  It is a restatement in plain
PyTorch-on-CPU of the reference's algorithm (heterocache/cache_utils.py in
ponytaill/HeteroCache), written to keep every rounding point of the reference:

  q.K^T in the model dtype -> / sqrt(d) in the model dtype -> softmax in fp32
  -> cast back to the model dtype -> avg/max pool -> max over the GQA group.

PyTorch on the CPU is used (not numpy) because the reference rounds to bf16 at
each of those points and numpy has no bf16.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
``HeteroCache`` methods (importable in the build container) on seeded inputs
and commits their outputs; ``tests/test_oracle_golden.py`` checks this module
against those fixtures bit for bit.  Decode attention is the one stage whose
reference implementation is a third-party compiled library
(``flash_attn_with_kvcache``, flash-attn 2.7.4.post1); its restatement here
(``paged_attention``) is unpinned by any reference test.
"""
from __future__ import annotations

import math
import statistics
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

PAGE = 256  # heterocache/cache_utils.py:626


def get_compress_len(compression_ratio: float, full_heads: int, ori_len: int, num_kv_heads: int) -> int:
    """Base per-head budget (heterocache/cache_utils.py:15-16)."""
    return int((compression_ratio * num_kv_heads - full_heads) * ori_len / (num_kv_heads - full_heads))


def _pool(x: torch.Tensor, pooling: str, kernel_size: int) -> torch.Tensor:
    """1-D pooling over the last dim of a [N, C, L] tensor, stride 1, padding k//2
    (heterocache/cache_utils.py:821-825)."""
    if pooling == "avgpool":
        return F.avg_pool1d(x, kernel_size=kernel_size, padding=kernel_size // 2, stride=1)
    if pooling == "maxpool":
        return F.max_pool1d(x, kernel_size=kernel_size, padding=kernel_size // 2, stride=1)
    raise ValueError("Pooling method not supported")


def window_scores(q_win: torch.Tensor, k: torch.Tensor, *, groups: int, pooling: str,
                  kernel_size: int) -> torch.Tensor:
    """Pooled, GQA-reduced token scores of one or more KV heads.

    q_win: [bsz, nh*groups, W, D] (the last W queries of the prompt),
    k:     [bsz, nh, L, D]  ->  [bsz, nh, L] in the input dtype.

    W == 1 is HeteroCache's prefill scoring (heterocache/cache_utils.py:808-829,
    :1162-1187).  W > 1 composes the observation-window math of SnapKV
    (heterocache/kv_cluster.py:168-178: causal mask inside the window, fp32
    softmax cast back to the dtype, sum over the W rows) with HeteroCache's
    pooling and GQA max, and scores all L positions.
    """
    bsz, nq, W, D = q_win.shape
    nh, L = k.shape[1], k.shape[2]
    qv = q_win.reshape(bsz, nh, groups, W, D)
    kv = k.reshape(bsz, nh, 1, L, D)
    logits = torch.matmul(qv, kv.transpose(-1, -2)) / math.sqrt(D)  # [bsz, nh, G, W, L]
    if W > 1:
        mask = torch.full((W, W), torch.finfo(logits.dtype).min, dtype=logits.dtype)
        cond = torch.arange(W)
        mask.masked_fill_(cond < (cond + 1).view(W, 1), 0)
        logits[..., L - W:] += mask
    p = F.softmax(logits, dim=-1, dtype=torch.float32).to(q_win.dtype)
    s = p.sum(dim=-2) if W > 1 else p.squeeze(-2)  # [bsz, nh, G, L]
    pooled = _pool(s.reshape(bsz, nh * groups, L), pooling, kernel_size)
    return pooled.view(bsz, nh, groups, L).max(dim=-2).values


def snapkv_scores(q: torch.Tensor, k: torch.Tensor, *, window: int, kernel_size: int,
                  pooling: str) -> torch.Tensor:
    """SnapKV's pooled window sums (heterocache/kv_cluster.py:168-184) for
    per-query-head keys [bsz, H, L, D]: the scores its top-k ranks, over the
    first L - window positions, in the model dtype."""
    W = window
    D = q.shape[-1]
    logits = torch.matmul(q[..., -W:, :], k.transpose(2, 3)) / math.sqrt(D)
    mask = torch.full((W, W), torch.finfo(logits.dtype).min)
    cond = torch.arange(W)
    mask.masked_fill_(cond < (cond + 1).view(W, 1), 0)
    logits[:, :, -W:, -W:] += mask[None, None].to(logits.dtype)
    p = F.softmax(logits, dim=-1, dtype=torch.float32).to(q.dtype)
    s = p[:, :, -W:, :-W].sum(dim=-2)
    return _pool(s, pooling, kernel_size)


def snapkv_indices(q: torch.Tensor, k: torch.Tensor, *, window: int, kernel_size: int,
                   pooling: str, capacity: int) -> torch.Tensor:
    """SnapKV's selection (heterocache/kv_cluster.py:160-186): top-(capacity -
    window) of the pooled window sums, in the reference's (score) order."""
    pooled = snapkv_scores(q, k, window=window, kernel_size=kernel_size, pooling=pooling)
    return pooled.topk(capacity - window, dim=-1).indices


def paged_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_table: torch.Tensor,
                    heads_len: torch.Tensor, num_kv_heads: int, scale: Optional[float] = None) -> torch.Tensor:
    """Restatement of flash_attn_with_kvcache(q[bsz*KV,1,G,D], k_pool, v_pool,
    cache_seqlens=heads_len, block_table, causal=False) as the patched attention
    calls it (heterocache/llama_model.py:370-397): per (batch row, KV head) row,
    fp32 softmax(q K^T * scale) V over the row's first heads_len tokens.
    q [bsz, H, 1, D] -> fp32 [bsz, H, D]."""
    bsz, H, _, D = q.shape
    KV = num_kv_heads
    G = H // KV
    scale = D ** -0.5 if scale is None else scale
    out = torch.zeros(bsz, KV, G, D, dtype=torch.float32)
    kp = k_pool.float().reshape(-1, D)
    vp = v_pool.float().reshape(-1, D)
    for b in range(bsz):
        for h in range(KV):
            row = b * KV + h
            n = int(heads_len[row])
            if n == 0:
                continue
            t = torch.arange(n)
            phys = block_table[row, (t // PAGE)].long() * PAGE + t % PAGE
            qq = q[b, h * G:(h + 1) * G, 0, :].float()
            p = torch.softmax((qq @ kp[phys].T) * scale, dim=-1)
            out[b, h] = p @ vp[phys]
    return out.view(bsz, H, D)


class OracleCache:
    """Restatement of ``HeteroCache`` (heterocache/cache_utils.py:610-1190) on CPU.

    Same constructor input (a ``HeteroCacheConfig``-like object carrying the
    derived role document), same methods and the same public tensors
    (``key_pools``, ``value_pools``, ``block_tables``, ``heads_len``,
    ``prefill_topk_set``).  The full-KV tier is always the in-memory reference
    (the reference's ``real_offload=False`` branch); its arithmetic is the same
    as the pinned-host branch.  For the checks it also records what the
    reference computes but does not keep: pooled scores, per-check overlap
    coefficients, medians, triggers and retrieval index lists.
    """

    def __init__(self, cfg, ties: str = "topk"):
        """``ties``: how a top-k orders positions whose scores are equal, which
        the reference leaves to ``torch.topk`` (unspecified order).  "topk"
        calls it exactly as the reference does (the mode the golden fixtures
        pin); "lowest" breaks such ties toward the lowest positions, one of
        the reference's valid outcomes and the rule the device kernels
        document, so that a lockstep run can require identical selections."""
        if ties not in ("topk", "lowest"):
            raise ValueError("ties must be 'topk' or 'lowest'")
        self.ties = ties
        self.cfg = cfg
        self.data = cfg.data
        self.num_attn_heads = cfg.num_attn_heads
        self.num_kv_heads = cfg.num_kv_heads
        self.num_layers = cfg.num_layers
        self.G = self.num_attn_heads // self.num_kv_heads
        self.gqa = self.G != 1
        self.total_kv_heads = self.num_kv_heads * self.num_layers
        self.ratio = cfg.compression_ratio
        self.pooling = cfg.pooling
        self.kernel_size = cfg.kernel_size
        self.decode_step = cfg.decode_step
        self.stable_threshold = cfg.stable_threshold
        self.max_gen_len = cfg.max_gen_len
        c = self.data["meta"]["counts"]
        self.full_heads = c["volatile"] + c["pivot"]
        n = self.num_layers
        self.key_pools: List[Optional[torch.Tensor]] = [None] * n
        self.value_pools: List[Optional[torch.Tensor]] = [None] * n
        self.block_tables: List[Optional[torch.Tensor]] = [None] * n
        self.heads_len: List[Optional[torch.Tensor]] = [None] * n
        self.free_blocks: List[Optional[torch.Tensor]] = [None] * n
        self.free_ptr = [0] * n
        self.full_k: List[Optional[torch.Tensor]] = [None] * n
        self.full_v: List[Optional[torch.Tensor]] = [None] * n
        self.prefill_topk_set: List = []
        self.qbuf: List[List[torch.Tensor]] = [[] for _ in range(n)]
        self.bsz = None
        self.head_dim = None
        self.prefill_len = None
        self.base_compress_len = None
        self.seen_tokens = 0
        # diagnostics
        self.prefill_scores: Dict[int, torch.Tensor] = {}
        self.prefill_keep_lens: Dict[int, torch.Tensor] = {}
        self.pivot_scores: Dict[int, torch.Tensor] = {}
        self.checks: List[Dict] = []

    def _topk(self, scores: torch.Tensor, k: int) -> torch.Tensor:
        """Indices of the k largest scores along the last dim, by descending
        score (``torch.topk(k, sorted=True)``; with ties="lowest", equal
        scores in ascending position order)."""
        if self.ties == "topk":
            return scores.topk(k, dim=-1, sorted=True).indices
        return torch.sort(scores, dim=-1, descending=True, stable=True).indices[..., :k]

    # -- storage ---------------------------------------------------------
    def _init_layer_storage(self, layer: int, dtype: torch.dtype) -> None:
        """heterocache/cache_utils.py:693-766."""
        L, gen = self.prefill_len, self.max_gen_len
        alloc = self.data["allocation_matrix"][layer]
        keep = self.data["need_to_keep_counts"][layer]
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
        self.key_pools[layer] = torch.zeros(total, PAGE, 1, self.head_dim, dtype=dtype)
        self.value_pools[layer] = torch.zeros(total, PAGE, 1, self.head_dim, dtype=dtype)
        max_blocks = (L + gen + PAGE - 1) // PAGE + 1
        bt = torch.full((self.bsz * self.num_kv_heads, max_blocks), -1, dtype=torch.int32)
        ptr = 0
        for row in range(self.bsz * self.num_kv_heads):
            n = caps[row % self.num_kv_heads] // PAGE
            if n > 0:
                bt[row, :n] = torch.arange(ptr, ptr + n, dtype=torch.int32)
                ptr += n
        if ptr > total:
            raise RuntimeError(f"Layer {layer}: Allocation logic error! Used more than allocated.")
        self.free_blocks[layer] = torch.arange(total, dtype=torch.int32)[ptr:].clone()
        self.free_ptr[layer] = 0
        self.block_tables[layer] = bt
        self.heads_len[layer] = torch.zeros(self.bsz * self.num_kv_heads, dtype=torch.int32)

    def _gather_head(self, layer: int, head: int, length: int, pool=None) -> torch.Tensor:
        """Logical rows [0, length) of one KV head, per batch row
        (heterocache/cache_utils.py:768-780) -> [bsz, 1, length, D]."""
        pool = self.key_pools[layer] if pool is None else pool
        rows = torch.arange(self.bsz) * self.num_kv_heads + head
        nblk = (length + PAGE - 1) // PAGE
        ids = self.block_tables[layer][rows, :nblk].long()
        flat = pool.view(-1, PAGE, self.head_dim)[ids.flatten()]
        return flat.view(self.bsz, nblk * PAGE, self.head_dim)[:, :length, :].unsqueeze(1)

    # -- prefill ---------------------------------------------------------
    def update(self, key_states, value_states, layer, cache_kwargs=None):
        """heterocache/cache_utils.py:884-1005."""
        if layer == 0:
            self.seen_tokens += key_states.shape[-2]
        if self.bsz is None:
            self.bsz = key_states.shape[0]
            self.head_dim = key_states.shape[-1]
        if self.base_compress_len is None:
            self.prefill_len = key_states.shape[-2]
            self.base_compress_len = get_compress_len(self.ratio, self.full_heads, self.prefill_len,
                                                      self.total_kv_heads)
        if self.key_pools[layer] is None:
            self._init_layer_storage(layer, key_states.dtype)
        S = key_states.shape[-2]
        D = self.head_dim
        if S > 1:
            self.prefill_len = S
            keep = self.data["need_to_keep_counts"][layer]
            upd = self.data["need_to_update_counts"][layer]
            fk = self.key_pools[layer].view(-1, D)
            fv = self.value_pools[layer].view(-1, D)
            if keep:
                heads = torch.tensor(keep, dtype=torch.long)
                rows = (torch.arange(self.bsz).unsqueeze(1) * self.num_kv_heads + heads.unsqueeze(0)).view(-1)
                start = self.block_tables[layer][rows, 0].long() * PAGE
                dest = (start.unsqueeze(1) + torch.arange(S).unsqueeze(0)).view(-1)
                fk.index_copy_(0, dest, key_states.index_select(1, heads).reshape(-1, D))
                fv.index_copy_(0, dest, value_states.index_select(1, heads).reshape(-1, D))
                self.heads_len[layer].index_fill_(0, rows, S)
            if upd:
                self.full_k[layer] = key_states.detach()
                self.full_v[layer] = value_states.detach()
            return key_states, value_states
        # decode append (heterocache/cache_utils.py:970-1005)
        flat_k = key_states.reshape(-1, D)
        flat_v = value_states.reshape(-1, D)
        lens = self.heads_len[layer]
        blk = lens // PAGE
        off = lens % PAGE
        seq = torch.arange(flat_k.shape[0])
        phys = self.block_tables[layer][seq, blk.long()]
        need = phys == -1
        n_new = int(need.sum().item())
        if n_new > 0:
            ptr = self.free_ptr[layer]
            if ptr + n_new > self.free_blocks[layer].size(0):
                raise RuntimeError(f"Layer {layer} OOM.")
            new_ids = self.free_blocks[layer][ptr:ptr + n_new]
            self.free_ptr[layer] += n_new
            self.block_tables[layer][seq[need], blk[need].long()] = new_ids
            phys[need] = new_ids
        self.key_pools[layer][phys.long(), off.long(), 0, :] = flat_k
        self.value_pools[layer][phys.long(), off.long(), 0, :] = flat_v
        self.heads_len[layer] += 1
        return key_states, value_states

    def init_coefficient(self, query_states, key_states, layer):
        """Pivot reference sets (heterocache/cache_utils.py:1149-1190)."""
        pivots = self.data["need_to_select_counts"][layer]
        if len(pivots) == 0:
            self.prefill_topk_set.append([])
            return
        G = self.G
        q = query_states[:, pivots[0] * G:(pivots[-1] + 1) * G, -1:, :]
        k = key_states[:, pivots, :, :]
        scores = window_scores(q, k, groups=G, pooling=self.pooling, kernel_size=self.kernel_size)
        self.pivot_scores[layer] = scores
        self.prefill_topk_set.append(self._topk(scores, self.base_compress_len))

    def prefill_select(self, query_states, key_states, value_states, layer):
        """Compressed heads' selection and page write (heterocache/cache_utils.py:782-882)."""
        bsz = query_states.shape[0]
        nc = self.data["need_to_compress_counts"][layer]
        if nc == 0:
            return
        ratios = torch.tensor(self.data["allocation_matrix"][layer][:nc], dtype=torch.float32)
        caps = (self.base_compress_len * ratios).int()
        L = key_states.shape[-2]
        keep_lens = torch.clamp(caps, max=L)
        self.prefill_keep_lens[layer] = keep_lens.clone()
        max_k = int(keep_lens.max().item())
        if max_k == 0:
            self.heads_len[layer][:nc] = 0
            return
        G = self.G
        q = query_states[:, :nc * G, -1:, :]
        k = key_states[:, :nc]
        scores = window_scores(q, k, groups=G, pooling=self.pooling, kernel_size=self.kernel_size)
        self.prefill_scores[layer] = scores
        safe_k = min(max_k, scores.shape[-1])
        idx = self._topk(scores, safe_k)
        grid = torch.arange(safe_k).view(1, 1, -1)
        excess = (grid >= keep_lens.view(1, -1, 1)).expand(bsz, -1, -1)
        idx = idx.masked_fill(excess, L + 1000).sort(dim=-1).values.clamp(max=L - 1)
        gi = idx.unsqueeze(-1).expand(-1, -1, -1, self.head_dim)
        sel_k = torch.gather(k, 2, gi)
        sel_v = torch.gather(value_states[:, :nc], 2, gi)
        rows = torch.arange(bsz).unsqueeze(1) * self.num_kv_heads + torch.arange(nc).unsqueeze(0)
        start = self.block_tables[layer][rows, 0].long() * PAGE
        dest = (start.unsqueeze(-1) + grid).view(-1)
        valid = (~excess).reshape(-1)
        D = self.head_dim
        self.key_pools[layer].view(-1, D).index_copy_(0, dest[valid], sel_k.reshape(-1, D)[valid])
        self.value_pools[layer].view(-1, D).index_copy_(0, dest[valid], sel_v.reshape(-1, D)[valid])
        self.heads_len[layer].index_put_((rows.view(-1),), keep_lens.unsqueeze(0).expand(bsz, -1).reshape(-1).int())

    # -- decode ----------------------------------------------------------
    def decode_select(self, query_states, layer):
        """Pivot drift check and satellite retrieval (heterocache/cache_utils.py:1007-1147)."""
        self.qbuf[layer].append(query_states)
        if len(self.qbuf[layer]) < self.decode_step:
            return
        qb = torch.cat(self.qbuf[layer], dim=2)
        self.qbuf[layer] = []
        relations = self.data["leader_member_relations"][layer]
        if len(relations) == 0:
            return
        bsz, H, S, D = qb.shape
        G = self.G
        fk = self.key_pools[layer].view(-1, D)
        fv = self.value_pools[layer].view(-1, D)
        K = self.base_compress_len
        for idx, (leader, members) in enumerate(relations.items()):
            if not members:
                continue
            head = int(leader)
            keys = self._gather_head(layer, head, self.prefill_len)  # [bsz,1,L,D]
            q = qb[:, head * G:(head + 1) * G]  # [bsz,G,S,D]
            logits = torch.matmul(q, keys.view(bsz, 1, -1, D).transpose(-1, -2)) / math.sqrt(D)
            p = F.softmax(logits, dim=-1, dtype=torch.float32).to(query_states.dtype)
            shp = p.shape
            p = _pool(p.reshape(-1, shp[-1]).unsqueeze(1), self.pooling, self.kernel_size).squeeze(1).view(shp)
            scores = p.max(dim=1).values  # [bsz,S,L]
            cur = self._topk(scores, K)
            ref = self.prefill_topk_set[layer][:, idx, :].unsqueeze(1).sort(dim=-1).values
            ref = ref.expand(-1, S, -1).contiguous()
            pos = torch.searchsorted(ref, cur).clamp(max=K - 1)
            matches = torch.gather(ref, -1, pos) == cur
            coeffs = (matches.sum(dim=-1).float() / K).mean(dim=0)
            coeff_list = coeffs.tolist()
            median = statistics.median(coeff_list)
            rec = {"layer": layer, "pivot": head, "idx": idx, "coeffs": coeff_list,
                   "median": median, "trigger": median < self.stable_threshold,
                   "scores": scores.clone(), "cur_sets": cur.clone()}
            if median < self.stable_threshold:
                self.prefill_topk_set[layer][:, idx, :] = cur[:, -1, :]
                lengths = [min(int(K * self.data["allocation_matrix"][layer][m]), self.prefill_len)
                           for m in members]
                max_len = max(lengths)
                sel = self._topk(scores[:, -1, :], max_len).sort(dim=-1).values.squeeze()
                rec["retrieved"] = sel.clone()
                rec["lengths"] = list(lengths)
                for m, n_tok in zip(members, lengths):
                    if n_tok == 0:
                        continue
                    ii = sel[:n_tok]
                    ks = torch.index_select(self.full_k[layer].select(1, m), 1, ii)
                    vs = torch.index_select(self.full_v[layer].select(1, m), 1, ii)
                    for b in range(bsz):
                        start = int(self.block_tables[layer][b * self.num_kv_heads + m, 0].item())
                        if start == -1:
                            continue
                        fk[start * PAGE:start * PAGE + n_tok].copy_(ks[b])
                        fv[start * PAGE:start * PAGE + n_tok].copy_(vs[b])
            self.checks.append(rec)

    def paged_attention(self, query_states: torch.Tensor, layer: int, scale: Optional[float] = None) -> torch.Tensor:
        """Restatement of the decode attention call (heterocache/llama_model.py:370-397,
        heterocache/qwen_model.py:181-206; library: flash_attn_with_kvcache, causal=False):
        per (batch row, KV head) the first ``heads_len`` rows of its page-table row.
        query_states [bsz, H, 1, D] -> fp32 [bsz, 1, H*D]."""
        bsz, H, _, D = query_states.shape
        G, KV = self.G, self.num_kv_heads
        scale = D ** -0.5 if scale is None else scale
        out = torch.zeros(bsz, KV, G, D, dtype=torch.float32)
        kp = self.key_pools[layer].float().view(-1, D)
        vp = self.value_pools[layer].float().view(-1, D)
        for b in range(bsz):
            for h in range(KV):
                row = b * KV + h
                n = int(self.heads_len[layer][row])
                if n == 0:
                    continue
                t = torch.arange(n)
                phys = self.block_tables[layer][row, (t // PAGE)].long() * PAGE + t % PAGE
                k, v = kp[phys], vp[phys]
                q = query_states[b, h * G:(h + 1) * G, 0, :].float()
                p = torch.softmax((q @ k.T) * scale, dim=-1)
                out[b, h] = p @ v
        return out.view(bsz, 1, H * D)
