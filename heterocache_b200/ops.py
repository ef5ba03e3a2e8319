"""Tensor-level wrappers over the C ABI (one per entry point).

Each wrapper validates devices, dtypes and layouts, then passes raw pointers,
element strides and the current CUDA stream to the library.  Shapes follow
the reference's tensors: q ``[bsz, H, L, D]``, k/v ``[bsz, KV, L, D]``, pools
``[n_blocks, 256, 1, D]``, block tables ``[bsz*KV, max_blocks]`` int32.
"""
from __future__ import annotations

from typing import Optional

import torch

from ._lib import DriftJob, check, lib

DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
POOLING = {"avgpool": 0, "maxpool": 1}
HEAD_DIM = 128
PAGE = 256

# Kernel launches issued through this module (flash-decode is two kernels).
LAUNCHES = [0]


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"heterocache_b200: unsupported dtype {t.dtype}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("heterocache_b200: tensors must live on a CUDA device")


def _rows(t: torch.Tensor, name: str) -> None:
    if t.shape[-1] != HEAD_DIM or t.stride(-1) != 1:
        raise ValueError(f"heterocache_b200: {name} must have a contiguous last dim of {HEAD_DIM}")


def _same_shape(k: torch.Tensor, v: torch.Tensor) -> None:
    if k.shape != v.shape or k.dtype != v.dtype:
        raise ValueError("heterocache_b200: k and v must have the same shape and dtype")


def _i32(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.int32 or not t.is_contiguous():
        raise ValueError(f"heterocache_b200: {name} must be a contiguous int32 tensor")


class Workspace:
    """Grow-only, zero-initialised scratch buffer owned by the caller."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf = torch.zeros(0, dtype=torch.uint8, device=self.device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.zeros(int(nbytes) + (1 << 20), dtype=torch.uint8, device=self.device)
        return self.buf

    def reset(self) -> None:
        self.buf.zero_()


def set_wait_limits(limit_ns: int = 0, inject_stall: bool = False) -> None:
    """Limit of every device-side wait of the library's kernels (0: the
    defaults, 2 s per grid barrier and 1 s per mbarrier wait); with
    ``inject_stall`` the scoring kernels' grid barriers wait for an arrival
    that never comes and the prefill attention loads no key tile, so the
    limit runs out (tests of the timeout path)."""
    check("hc_set_wait_limits", lib().hc_set_wait_limits(int(limit_ns), 1 if inject_stall else 0))


def prefill_keep(k, v, keep_heads, k_pool, v_pool, block_table, heads_len, err):
    _cuda(k, v, keep_heads, k_pool, v_pool, block_table, heads_len, err)
    _rows(k, "k"), _rows(v, "v")
    _i32(keep_heads, "keep_heads"), _i32(block_table, "block_table"), _i32(heads_len, "heads_len")
    _same_shape(k, v)
    bsz, KV, L, D = k.shape
    rc = lib().hc_prefill_keep(dtype_code(k), bsz, KV, L, D, _ptr(keep_heads), keep_heads.numel(),
                               _ptr(k), _ptr(v), k.stride(0), k.stride(1), k.stride(2),
                               v.stride(0), v.stride(1), v.stride(2),
                               _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_table), block_table.shape[1],
                               _ptr(heads_len), _ptr(err), _stream(k))
    check("hc_prefill_keep", rc)
    LAUNCHES[0] += 1


def _need(ok: bool, what: str) -> None:
    """Host-side size check of an argument the kernels index by another
    argument's size (a short buffer would be read or written out of bounds)."""
    if not ok:
        raise ValueError(f"heterocache_b200: {what}")


def _query_rows(q, L: int, rows: int) -> int:
    """Device address of ``q`` for the scoring launches.  They read query
    token positions L - rows .. L - 1, the token axis aligned with the keys'
    (in the reference q and k come from the same prompt).  A query with Lq
    positions is rebased by Lq - L rows, so that those reads are q's own last
    ``rows`` positions, inside the tensor, whatever its length."""
    Lq = q.shape[2]
    if Lq < rows:
        raise ValueError(f"heterocache_b200: the query has {Lq} positions, the scoring reads the last {rows}")
    return q.data_ptr() + (Lq - L) * q.stride(2) * q.element_size()


def prefill_select(q, k, v, keep_lens, max_keep, *, n_heads, groups, window, pooling, kernel_size,
                   k_pool, v_pool, block_table, heads_len, workspace: Workspace, err,
                   out_indices=None, out_scores=None):
    bsz, KV, L = k.shape[0], k.shape[1], k.shape[-2]
    _need(keep_lens.numel() >= n_heads, "keep_lens needs one entry per scored head")
    _need(block_table.shape[0] >= bsz * KV and heads_len.numel() >= bsz * KV,
          "block_table and heads_len need a row per (batch row, KV head)")
    _need(out_indices is None or out_indices.numel() >= bsz * n_heads * max_keep,
          "out_indices needs [bsz, n_heads, max_keep] entries")
    _need(out_scores is None or out_scores.numel() >= bsz * n_heads * L, "out_scores needs [bsz, n_heads, L]")
    _cuda(q, k, v, keep_lens, k_pool, v_pool, block_table, heads_len, err)
    _rows(q, "q"), _rows(k, "k"), _rows(v, "v")
    _i32(keep_lens, "keep_lens"), _i32(block_table, "block_table"), _i32(heads_len, "heads_len")
    _same_shape(k, v)
    bsz, KV, L, D = k.shape
    dt = dtype_code(k)
    nbytes = lib().hc_prefill_select_workspace_size(dt, bsz, n_heads, L, groups, window)
    ws = workspace.get(nbytes)
    rc = lib().hc_prefill_select(dt, bsz, KV, groups, L, D, n_heads, window, POOLING[pooling], kernel_size,
                                 _query_rows(q, L, window), q.stride(0), q.stride(1), q.stride(2),
                                 _ptr(k), _ptr(v), k.stride(0), k.stride(1), k.stride(2),
                                 v.stride(0), v.stride(1), v.stride(2),
                                 _ptr(keep_lens), int(max_keep), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0],
                                 _ptr(block_table), block_table.shape[1], _ptr(heads_len),
                                 _ptr(out_indices), _ptr(out_scores), _ptr(ws), ws.numel(), _ptr(err), _stream(k))
    check("hc_prefill_select", rc)
    LAUNCHES[0] += 1


def snapkv_update_kv(q, k, v, *, window, pooling, kernel_size, capacity, workspace: Workspace, err,
                     out_indices=None, out_scores=None):
    """SnapKV compression (heterocache/kv_cluster.py:155-199) of one layer:
    q, k, v [bsz, H, L, D] -> (k_out, v_out) [bsz, H, capacity, D], the kept
    rows of each head in ascending position order followed by its last
    ``window`` rows."""
    if pooling not in POOLING:
        raise ValueError("Pooling method not supported")
    _same_shape(k, v)
    bsz, H, L, D = k.shape
    if q.shape[1] != H:
        raise RuntimeError(f"heterocache_b200: SnapKV scores every query head against its own key head "
                           f"({q.shape[1]} query heads, {H} key heads)")
    _need(1 <= window < L, f"window {window} must lie in [1, {L})")
    _need(window <= capacity <= L, f"capacity {capacity} must lie in [window, {L}]")
    _need(out_indices is None or (out_indices.dtype == torch.int32 and out_indices.is_contiguous()
                                  and out_indices.numel() >= bsz * H * (capacity - window)),
          "out_indices needs a contiguous int32 [bsz, H, capacity - window]")
    _need(out_scores is None or (out_scores.dtype == k.dtype and out_scores.is_contiguous()
                                 and out_scores.numel() >= bsz * H * L),
          "out_scores needs a contiguous [bsz, H, L] in the key dtype")
    _cuda(q, k, v, err, out_indices, out_scores)
    _rows(q, "q"), _rows(k, "k"), _rows(v, "v")
    if q.dtype != k.dtype:
        raise ValueError("heterocache_b200: q and k must share a dtype")
    k_out = torch.empty(bsz, H, capacity, D, dtype=k.dtype, device=k.device)
    v_out = torch.empty_like(k_out)
    dt = dtype_code(k)
    nbytes = lib().hc_snapkv_update_kv_workspace_size(dt, bsz, H, L, window)
    ws = workspace.get(nbytes)
    rc = lib().hc_snapkv_update_kv(dt, bsz, H, L, D, int(window), POOLING[pooling], int(kernel_size), int(capacity),
                                   _query_rows(q, L, window), q.stride(0), q.stride(1), q.stride(2),
                                   _ptr(k), _ptr(v), k.stride(0), k.stride(1), k.stride(2),
                                   v.stride(0), v.stride(1), v.stride(2), _ptr(k_out), _ptr(v_out),
                                   _ptr(out_indices), _ptr(out_scores), _ptr(ws), ws.numel(), _ptr(err), _stream(k))
    check("hc_snapkv_update_kv", rc)
    LAUNCHES[0] += 1
    return k_out, v_out


def pivot_init(q, k, *, first_pivot, n_pivots, groups, pooling, kernel_size, topk, ref_positions, ref_bitmap,
               workspace: Workspace, err, out_scores=None):
    bsz, L = k.shape[0], k.shape[-2]
    _need(ref_positions.numel() >= bsz * n_pivots * topk, "ref_positions needs [bsz, n_pivots, topk] entries")
    _need(ref_bitmap.numel() >= bsz * n_pivots * ((L + 31) // 32), "ref_bitmap needs [bsz, n_pivots, ceil(L/32)] words")
    _need(out_scores is None or out_scores.numel() >= bsz * n_pivots * L, "out_scores needs [bsz, n_pivots, L]")
    _cuda(q, k, ref_positions, ref_bitmap, err)
    _rows(q, "q"), _rows(k, "k")
    bsz, KV, L, D = k.shape
    dt = dtype_code(k)
    nbytes = lib().hc_pivot_init_workspace_size(dt, bsz, n_pivots, L, groups)
    ws = workspace.get(nbytes)
    rc = lib().hc_pivot_init(dt, bsz, KV, groups, L, D, first_pivot, n_pivots, POOLING[pooling], kernel_size,
                             int(topk), _query_rows(q, L, 1), q.stride(0), q.stride(1), q.stride(2),
                             _ptr(k), k.stride(0), k.stride(1), k.stride(2),
                             _ptr(ref_positions), _ptr(ref_bitmap), _ptr(out_scores), _ptr(ws), ws.numel(),
                             _ptr(err), _stream(k))
    check("hc_pivot_init", rc)
    LAUNCHES[0] += 1


def prefill_attention(q, k, v, *, scale: float = 0.0, out=None, err=None):
    """hc_prefill_attention: causal grouped-query attention of q [bsz, H, L, D]
    over k, v [bsz, KV, L, D] (16-bit, strided, contiguous last dim) on the
    tcgen05 tensor cores.  Returns out [bsz, L, H, D] (the layout the output
    projection reads), or writes the given ``out`` of that shape."""
    _cuda(q, k, v, out, err)
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        _rows(t, name)
    _same_shape(k, v)
    _need(q.dtype in (torch.bfloat16, torch.float16) and k.dtype == q.dtype,
          "prefill_attention takes bf16 or fp16 q, k, v of one dtype")
    bsz, H, L, D = q.shape
    _need(k.shape[0] == bsz and k.shape[2] == L and H % k.shape[1] == 0, "k/v need [bsz, KV, L, D], KV dividing H")
    if out is None:
        out = torch.empty(bsz, L, H, D, dtype=q.dtype, device=q.device)
    _need(out.shape == (bsz, L, H, D) and out.dtype == q.dtype and out.stride(-1) == 1, "out needs [bsz, L, H, D]")
    if err is None:
        err = torch.zeros(1, dtype=torch.int32, device=q.device)
    rc = lib().hc_prefill_attention(dtype_code(q), bsz, H, k.shape[1], L, D, _ptr(q), q.stride(0), q.stride(1),
                                    q.stride(2), _ptr(k), k.stride(0), k.stride(1), k.stride(2), _ptr(v),
                                    v.stride(0), v.stride(1), v.stride(2), float(scale), _ptr(out), out.stride(0),
                                    out.stride(2), out.stride(1), _ptr(err), _stream(q))
    check("hc_prefill_attention", rc)
    LAUNCHES[0] += 1
    return out


def decode_append(k, v, k_pool, v_pool, block_table, heads_len, free_blocks, free_ptr, err, q=None, q_stage=None):
    """Append one token per row; with ``q`` [1, H, 1, D] and ``q_stage`` [H, D]
    the same launch stores the step's query for the drift check."""
    _cuda(k, v, k_pool, v_pool, block_table, heads_len, free_blocks, free_ptr, err, q, q_stage)
    _rows(k, "k"), _rows(v, "v")
    _same_shape(k, v)
    bsz, KV, one, D = k.shape
    if one != 1:
        raise ValueError("heterocache_b200: decode append takes one token per row")
    nq, qsh = 0, 0
    if q_stage is not None:
        _rows(q, "q")
        if q.shape[0] != 1 or q.shape[2] != 1 or q.dtype != k.dtype:
            raise ValueError("heterocache_b200: the staged query must be [1, H, 1, D] in the cache dtype")
        if not q_stage.is_contiguous() or tuple(q_stage.shape) != (q.shape[1], D):
            raise ValueError("heterocache_b200: q_stage must be a contiguous [H, D] tensor")
        nq, qsh = q.shape[1], q.stride(1)
    rc = lib().hc_decode_append(dtype_code(k), bsz, KV, D, _ptr(k), _ptr(v), k.stride(0), k.stride(1),
                                v.stride(0), v.stride(1), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_table),
                                block_table.shape[1], _ptr(heads_len), _ptr(free_blocks), free_blocks.numel(),
                                _ptr(free_ptr), _ptr(q if q_stage is not None else None), qsh, nq, _ptr(q_stage),
                                _ptr(err), _stream(k))
    check("hc_decode_append", rc)
    LAUNCHES[0] += 1


def flash_decode(q, k_pool, v_pool, block_table, heads_len, *, num_kv_heads, out=None, scale: float = 0.0,
                 workspace: Workspace, err, total_tokens_hint: int = 0, k_new=None, v_new=None, q_stage=None,
                 mirrors=None, mirror_batch_stride: int = 0):
    """q: [bsz, H, 1, D] -> out [bsz, H, D] (same dtype).  With k_new/v_new
    [bsz, KV, 1, D] each row also attends to that token (not in the pages);
    then q_stage (bsz 1: a contiguous [H, D] buffer) also receives the query
    rows, and ``mirrors`` (device addresses, e.g. other GPUs' gathered
    outputs) each receive a copy of the output: element (b, head j, d) at
    mirror + (b * mirror_batch_stride + j * D + d) elements."""
    H = q.shape[1]
    _need(num_kv_heads > 0 and H % num_kv_heads == 0,
          f"the {H} query heads do not split evenly over {num_kv_heads} KV heads")
    _cuda(q, k_pool, v_pool, block_table, heads_len, err, k_new, v_new, q_stage)
    _rows(q, "q")
    bsz, H, one, D = q.shape
    if one != 1:
        raise ValueError("heterocache_b200: decode attention takes one query position")
    groups = H // num_kv_heads
    if out is None:
        out = torch.empty(bsz, H, D, dtype=q.dtype, device=q.device)
    _need(out.is_contiguous() and out.numel() == bsz * H * D and out.dtype == q.dtype,
          "out must be a contiguous [bsz, H, D] buffer in the query dtype")
    _need(block_table.shape[0] >= bsz * num_kv_heads and heads_len.numel() >= bsz * num_kv_heads,
          "block_table and heads_len need a row per (batch row, KV head)")
    nbytes = lib().hc_flash_decode_workspace_size(bsz, num_kv_heads, groups, D)
    ws = workspace.get(nbytes)
    if k_new is not None:
        _rows(k_new, "k_new"), _rows(v_new, "v_new")
        _same_shape(k_new, v_new)
        if tuple(k_new.shape) != (bsz, num_kv_heads, 1, D) or k_new.dtype != q.dtype:
            raise ValueError("heterocache_b200: k_new/v_new must be [bsz, KV, 1, D] in the query dtype")
        if q_stage is not None and (bsz != 1 or tuple(q_stage.shape) != (H, D) or q_stage.dtype != q.dtype
                                    or not q_stage.is_contiguous()):
            raise ValueError("heterocache_b200: q_stage must be a contiguous [H, D] buffer in the query dtype (bsz 1)")
        if mirrors:
            import ctypes
            _need(len(mirrors) <= 8, "at most 8 output mirrors")
            arr = (ctypes.c_void_p * len(mirrors))(*[int(m) for m in mirrors])
            rc = lib().hc_flash_decode_peer(dtype_code(q), bsz, num_kv_heads, groups, D, _ptr(q), q.stride(0),
                                            q.stride(1), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0],
                                            _ptr(block_table), block_table.shape[1], _ptr(heads_len), _ptr(k_new),
                                            _ptr(v_new), k_new.stride(0), k_new.stride(1), v_new.stride(0),
                                            v_new.stride(1), float(scale), _ptr(out), _ptr(q_stage), len(mirrors),
                                            arr, int(mirror_batch_stride), _ptr(ws), ws.numel(), _ptr(err),
                                            _stream(q))
            check("hc_flash_decode_peer", rc)
            LAUNCHES[0] += 2
            return out
        rc = lib().hc_flash_decode_with_new(dtype_code(q), bsz, num_kv_heads, groups, D, _ptr(q), q.stride(0),
                                            q.stride(1), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0],
                                            _ptr(block_table), block_table.shape[1], _ptr(heads_len), _ptr(k_new),
                                            _ptr(v_new), k_new.stride(0), k_new.stride(1), v_new.stride(0),
                                            v_new.stride(1), float(scale), _ptr(out), _ptr(q_stage), _ptr(ws),
                                            ws.numel(), _ptr(err), _stream(q))
        check("hc_flash_decode_with_new", rc)
        LAUNCHES[0] += 2
        return out
    if mirrors:
        import ctypes
        _need(len(mirrors) <= 8, "at most 8 output mirrors")
        arr = (ctypes.c_void_p * len(mirrors))(*[int(m) for m in mirrors])
        rc = lib().hc_flash_decode_peer(dtype_code(q), bsz, num_kv_heads, groups, D, _ptr(q), q.stride(0),
                                        q.stride(1), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_table),
                                        block_table.shape[1], _ptr(heads_len), None, None, 0, 0, 0, 0, float(scale),
                                        _ptr(out), None, len(mirrors), arr, int(mirror_batch_stride), _ptr(ws),
                                        ws.numel(), _ptr(err), _stream(q))
        check("hc_flash_decode_peer", rc)
        LAUNCHES[0] += 2
        return out
    rc = lib().hc_flash_decode(dtype_code(q), bsz, num_kv_heads, groups, D, _ptr(q), q.stride(0), q.stride(1),
                               _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_table),
                               block_table.shape[1], _ptr(heads_len), float(scale), _ptr(out),
                               int(total_tokens_hint),
                               _ptr(ws), ws.numel(), _ptr(err), _stream(q))
    check("hc_flash_decode", rc)
    LAUNCHES[0] += 2
    return out


def drift_check(qbuf, k_pool, block_table, *, num_kv_heads, groups, steps, seq_len, pooling, kernel_size, topk,
                threshold, pivot_heads, ref_slots, max_len, max_len_cap, ref_bitmap, ref_positions, trigger,
                retrieve_positions, workspace: Workspace, err, coeffs=None, median=None, out_scores=None):
    """qbuf: [S, H, D] (strided)."""
    n = pivot_heads.numel()
    _need(qbuf.dim() == 3 and qbuf.shape[0] >= steps and qbuf.shape[1] == num_kv_heads * groups,
          "qbuf needs [steps, num_kv_heads * groups, D]")
    _need(block_table.shape[1] * 256 >= seq_len, "block_table rows must cover seq_len tokens")
    _need(ref_slots.numel() >= n and max_len.numel() >= n and trigger.numel() >= n,
          "ref_slots, max_len and trigger need an entry per pivot job")
    _need(ref_positions.shape[-1] >= topk, "ref_positions rows need topk entries")
    _need(ref_bitmap.shape[-1] >= (seq_len + 31) // 32, "ref_bitmap rows need ceil(seq_len/32) words")
    _need(retrieve_positions.numel() >= n * max_len_cap and retrieve_positions.shape[-1] >= max_len_cap,
          "retrieve_positions needs [jobs, max_len_cap]")
    _need(coeffs is None or coeffs.numel() >= n * steps, "coeffs needs [jobs, steps]")
    _need(median is None or median.numel() >= n, "median needs an entry per job")
    _need(out_scores is None or out_scores.numel() >= n * steps * seq_len, "out_scores needs [jobs, steps, seq_len]")
    _cuda(qbuf, k_pool, block_table, pivot_heads, ref_slots, max_len, ref_bitmap, ref_positions, trigger,
          retrieve_positions, err)
    _rows(qbuf, "qbuf")
    dt = dtype_code(qbuf)
    n_jobs = pivot_heads.numel()
    nbytes = lib().hc_drift_check_workspace_size(dt, n_jobs, steps, seq_len, groups)
    ws = workspace.get(nbytes)
    rc = lib().hc_drift_check(dt, num_kv_heads, groups, qbuf.shape[-1], steps, seq_len, POOLING[pooling],
                              kernel_size, int(topk), float(threshold), _ptr(qbuf), qbuf.stride(0),
                              qbuf.stride(1), _ptr(k_pool), k_pool.shape[0], _ptr(block_table),
                              block_table.shape[1], n_jobs,
                              _ptr(pivot_heads), _ptr(ref_slots), _ptr(max_len), int(max_len_cap),
                              _ptr(ref_bitmap), _ptr(ref_positions), _ptr(trigger), _ptr(coeffs), _ptr(median),
                              _ptr(retrieve_positions), _ptr(out_scores), _ptr(ws), ws.numel(), _ptr(err),
                              _stream(qbuf))
    check("hc_drift_check", rc)
    LAUNCHES[0] += 1


def _tier_base(full: torch.Tensor, first_head: int) -> int:
    """Address the kernels index as head 0 of a full tier whose row 0 holds
    head `first_head` (a tier of the satellites only): they read head h at
    base + h * head_stride, so only heads >= first_head are ever addressed."""
    return full.data_ptr() - first_head * full.stride(1) * full.element_size()


def drift_job(qbuf, k_pool, block_table, *, pivot_head, max_len, ref_bitmap, ref_positions, trigger,
              retrieve_positions, coeffs=None, median=None, out_scores=None) -> DriftJob:
    """One check of a drift-check batch: a pivot's query buffer qbuf [S, H, D],
    its layer's key pool and page table, its reference bitmap row and
    reference position row, and its output slots (trigger: one int32,
    retrieve_positions: max_len int32, coeffs: S floats, median: one double,
    out_scores: [S, seq_len] pooled scores in qbuf's dtype).  The tensors must
    stay alive, unmoved, while the batch is in use."""
    _cuda(qbuf, k_pool, block_table, ref_bitmap, ref_positions, trigger, retrieve_positions, coeffs, median,
          out_scores)
    _need(out_scores is None or (out_scores.dtype == qbuf.dtype and out_scores.is_contiguous()),
          "out_scores must be contiguous, in qbuf's dtype")
    _rows(qbuf, "qbuf")
    _need(qbuf.dim() == 3, "qbuf needs [steps, num_kv_heads * groups, D]")
    _i32(block_table, "block_table")
    _need(ref_bitmap.dtype == torch.int32 and ref_bitmap.is_contiguous(), "ref_bitmap must be contiguous 32-bit words")
    for t, name in ((ref_positions, "ref_positions"), (trigger, "trigger"), (retrieve_positions, "retrieve_positions")):
        _i32(t, name)
    _need(trigger.numel() >= 1 and retrieve_positions.numel() >= max_len, "retrieve_positions needs max_len entries")
    _need(coeffs is None or (coeffs.dtype == torch.float32 and coeffs.is_contiguous()), "coeffs must be float32")
    _need(median is None or (median.dtype == torch.float64 and median.numel() >= 1), "median must be float64")
    return DriftJob(_ptr(qbuf), qbuf.stride(0), qbuf.stride(1), _ptr(k_pool), _ptr(block_table), k_pool.shape[0],
                    block_table.shape[1], int(pivot_head), int(max_len), _ptr(ref_bitmap), _ptr(ref_positions),
                    _ptr(trigger), _ptr(retrieve_positions), _ptr(coeffs), _ptr(median), _ptr(out_scores))


def drift_jobs_array(jobs) -> "ctypes.Array":
    """A ctypes array of drift_job descriptors, for drift_check_batch."""
    import ctypes
    return (DriftJob * len(jobs))(*jobs)


def drift_check_batch(jobs, *, dtype, device, num_kv_heads, groups, steps, seq_len, pooling, kernel_size, topk,
                      threshold, workspace: Workspace, err, jobs_per_launch: int = 0, stream=None):
    """hc_drift_check_batch: every job's drift check (the computation of
    drift_check, per job) in ceil(n / per-launch) launches.  ``jobs``: a
    drift_jobs_array; the check lengths and outputs are the jobs' own."""
    n = len(jobs)
    if n == 0:
        return
    _cuda(err)
    dt = DTYPES[dtype]
    nbytes = lib().hc_drift_check_batch_workspace_size(dt, n, steps, seq_len, groups, int(jobs_per_launch))
    _need(nbytes > 0, "drift_check_batch: invalid sizes")
    per = lib().hc_drift_check_batch_per_launch(dt, n, steps, seq_len, groups, int(jobs_per_launch))
    ws = workspace.get(nbytes)
    st = (stream if stream is not None else torch.cuda.current_stream(device)).cuda_stream
    rc = lib().hc_drift_check_batch(dt, num_kv_heads, groups, HEAD_DIM, steps, seq_len, POOLING[pooling],
                                    kernel_size, int(topk), float(threshold), jobs, n, int(jobs_per_launch),
                                    _ptr(ws), ws.numel(), _ptr(err), st)
    check("hc_drift_check_batch", rc)
    LAUNCHES[0] += (n + per - 1) // per


def retrieve(*, member_job, member_head, member_len, max_member_len, trigger, retrieve_positions, full_k, full_v,
             k_pool, v_pool, block_table, num_kv_heads, err, stream: Optional[torch.cuda.Stream] = None,
             tier_first_head: int = 0):
    """full_k/full_v: [1, heads, L, D] on the device or in pinned host memory,
    row 0 holding head `tier_first_head` (every member's head lies in the
    tier)."""
    _need(retrieve_positions.shape[-1] >= max_member_len, "retrieve_positions rows need max_member_len entries")
    _need(member_head.numel() >= member_job.numel() and member_len.numel() >= member_job.numel(),
          "member_head and member_len need an entry per member")
    _cuda(member_job, member_head, member_len, trigger, retrieve_positions, k_pool, v_pool, block_table, err)
    _rows(full_k, "full_k"), _rows(full_v, "full_v")
    if not full_k.is_cuda and not full_k.is_pinned():
        raise ValueError("heterocache_b200: a host-memory full tier must be pinned")
    if full_k.stride() != full_v.stride():
        raise ValueError("heterocache_b200: full_k and full_v must share strides")
    st = (stream or torch.cuda.current_stream(k_pool.device)).cuda_stream
    rc = lib().hc_retrieve(dtype_code(k_pool), num_kv_heads, k_pool.shape[-1], member_job.numel(),
                           _ptr(member_job), _ptr(member_head), _ptr(member_len), int(max_member_len),
                           _ptr(trigger), _ptr(retrieve_positions), retrieve_positions.shape[-1],
                           _tier_base(full_k, tier_first_head), _tier_base(full_v, tier_first_head),
                           full_k.stride(1), full_k.stride(2),
                           _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_table), block_table.shape[1],
                           _ptr(err), st)
    check("hc_retrieve", rc)
    LAUNCHES[0] += 1


def retrieve_delta(*, member_job, member_head, member_len, member_stage_offset, reuse_len, max_member_len, trigger,
                   retrieve_positions, slot_positions, full_k, full_v, k_pool, v_pool, block_table, num_kv_heads,
                   stage_k, stage_v, stage_src, err, stream: Optional[torch.cuda.Stream] = None,
                   tier_first_head: int = 0):
    """Satellite retrieval from a pinned-host tier that moves only rows the
    satellite does not hold yet (same pool contents as ``retrieve``).

    slot_positions [n_members, R] int32: positions held in the first R slots
    of each member (ascending; seeded with the prefill kept indices, kept up
    to date here).  stage_k/stage_v [rows, D] and stage_src [rows] int32:
    device scratch, member m at rows member_stage_offset[m] + [0, len)."""
    m = member_job.numel()
    _need(retrieve_positions.shape[-1] >= max_member_len, "retrieve_positions rows need max_member_len entries")
    _need(member_head.numel() >= m and member_len.numel() >= m and member_stage_offset.numel() >= m
          and reuse_len.numel() >= m and slot_positions.shape[0] >= m,
          "member arrays and slot_positions need an entry per member")
    _cuda(member_job, member_head, member_len, member_stage_offset, reuse_len, trigger, retrieve_positions,
          slot_positions, k_pool, v_pool, block_table, stage_k, stage_v, stage_src, err)
    _rows(full_k, "full_k"), _rows(full_v, "full_v")
    _i32(slot_positions, "slot_positions"), _i32(stage_src, "stage_src")
    if not full_k.is_pinned() or not full_v.is_pinned():
        raise ValueError("heterocache_b200: retrieve_delta reads a pinned host-memory full tier")
    if full_k.stride() != full_v.stride():
        raise ValueError("heterocache_b200: full_k and full_v must share strides")
    if (stage_k.dtype != k_pool.dtype or stage_v.dtype != k_pool.dtype or not stage_k.is_contiguous()
            or not stage_v.is_contiguous() or stage_k.shape != stage_v.shape or stage_k.shape[-1] != k_pool.shape[-1]
            or stage_src.numel() < stage_k.shape[0]):
        raise ValueError("heterocache_b200: staging area must be contiguous [rows, D] in the pool dtype, "
                         "with a stage_src entry per row")
    st = (stream or torch.cuda.current_stream(k_pool.device)).cuda_stream
    rc = lib().hc_retrieve_delta(dtype_code(k_pool), num_kv_heads, k_pool.shape[-1], member_job.numel(),
                                 _ptr(member_job), _ptr(member_head), _ptr(member_len), _ptr(member_stage_offset),
                                 _ptr(reuse_len), int(max_member_len), _ptr(trigger), _ptr(retrieve_positions),
                                 retrieve_positions.shape[-1], _ptr(slot_positions), slot_positions.shape[-1],
                                 _tier_base(full_k, tier_first_head), _tier_base(full_v, tier_first_head),
                                 full_k.stride(1), full_k.stride(2),
                                 _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_table),
                                 block_table.shape[1], _ptr(stage_k), _ptr(stage_v), _ptr(stage_src),
                                 stage_k.shape[0], _ptr(err), st)
    check("hc_retrieve_delta", rc)
    LAUNCHES[0] += 2


def profile_topk(attn: torch.Tensor, *, groups: int, topk: int, max_length: int,
                 workspace: Workspace) -> torch.Tensor:
    """Top-k sets of the heads' last-query attention rows as bitmaps (the
    per-dump step of tools/get_cluster.py:13-60).

    ``attn`` [bsz, saved heads, q_len, keys] (or [bsz, heads, keys]) on the
    GPU, any strides; ``groups`` > 1 averages that many consecutive saved
    heads per effective head (GQA dumps of every query head).  Returns int32
    bitmaps [bsz, heads // groups, words] (bit t of word t // 32); the set of
    a row is empty when ``min(max_length, keys)`` is 0.
    """
    _cuda(attn)
    if attn.dim() == 3:
        attn = attn.unsqueeze(2)
    if attn.dim() != 4:
        raise ValueError("heterocache_b200: attn must be [bsz, heads, q_len, keys]")
    B, Hs, Q, L = attn.shape
    if groups < 1 or Hs % groups:
        raise ValueError("heterocache_b200: saved heads must be a multiple of groups")
    use_len = max(0, min(int(max_length), L))
    He = Hs // groups
    words = (use_len + 1 + 31) // 32 if use_len else 1
    bits = torch.empty(B, He, words, dtype=torch.int32, device=attn.device)
    if B == 0:
        return bits
    nbytes = lib().hc_profile_topk_workspace_size(B, He, use_len)
    ws = workspace.get(nbytes) if nbytes else workspace.get(16)
    sb, sh, sq, st = attn.stride()
    check("hc_profile_topk",
          lib().hc_profile_topk(dtype_code(attn), B, Hs, groups, Q, L, attn.data_ptr(), sb, sh, sq, st, use_len,
                                int(topk), bits.data_ptr(), words, ws.data_ptr(), ws.numel(), _stream(attn)))
    LAUNCHES[0] += 1
    return bits


def profile_overlap(a: torch.Tensor, b: torch.Tensor, *, diagonal: bool) -> torch.Tensor:
    """Intersection sizes of bitmap rows (numerators of the reference's
    calculate_overlap_ratio, tools/get_cluster.py:62-69): ``a`` [na, words],
    ``b`` [nb, words] int32 on the GPU; returns int32 [na, nb], or [na] with
    ``diagonal`` (row i with row i)."""
    _cuda(a, b)
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("heterocache_b200: bitmaps must be [rows, words] with equal words")
    if a.dtype != torch.int32 or b.dtype != torch.int32 or a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("heterocache_b200: bitmaps must be int32 with contiguous words")
    na, nb, words = a.shape[0], b.shape[0], a.shape[1]
    if diagonal and na != nb:
        raise ValueError("heterocache_b200: diagonal overlaps need equal row counts")
    out = torch.empty((na,) if diagonal else (na, nb), dtype=torch.int32, device=a.device)
    if na == 0 or nb == 0:
        return out
    check("hc_profile_overlap",
          lib().hc_profile_overlap(a.data_ptr(), a.stride(0), na, b.data_ptr(), b.stride(0), nb, words,
                                   1 if diagonal else 0, out.data_ptr(), _stream(a)))
    LAUNCHES[0] += 1
    return out


def peer_barrier(rank: int, world: int, flag_ptrs, counter: torch.Tensor, err: torch.Tensor) -> None:
    """One step barrier of a head-sharded cache's ranks (hc_peer_barrier):
    ``flag_ptrs`` the device addresses of every rank's int32 flag array,
    ``counter`` this rank's int32 counter."""
    import ctypes
    _cuda(counter, err)
    _need(1 <= world <= 8 and 0 <= rank < world and len(flag_ptrs) == world, "bad rank or world")
    arr = (ctypes.c_void_p * world)(*[int(p) for p in flag_ptrs])
    check("hc_peer_barrier", lib().hc_peer_barrier(rank, world, arr, _ptr(counter), _ptr(err), _stream(counter)))
    LAUNCHES[0] += 1


def peer_put(segments, dst_ptrs) -> None:
    """hc_peer_put: the concatenation of ``segments`` (up to 4 int32 CUDA
    tensors, each contiguous) stored into every address of ``dst_ptrs`` (up
    to 8 device addresses, e.g. other ranks' buffers mapped through CUDA IPC;
    each must have room for the concatenation), fenced at system scope so
    that a ``peer_barrier`` after it publishes the words.  Runs on the first
    segment's current stream."""
    import ctypes
    _need(1 <= len(segments) <= 4, "peer_put takes 1 to 4 segments")
    _need(len(dst_ptrs) <= 8, "peer_put takes at most 8 destinations")
    _cuda(*segments)
    for t in segments:
        _i32(t, "peer_put segment")
        _need(t.is_contiguous(), "peer_put segments must be contiguous")
    n = len(segments)
    srcs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in segments])
    words = (ctypes.c_int64 * n)(*[t.numel() for t in segments])
    dsts = (ctypes.c_void_p * max(len(dst_ptrs), 1))(*[int(p) for p in dst_ptrs])
    check("hc_peer_put", lib().hc_peer_put(n, srcs, words, len(dst_ptrs), dsts, _stream(segments[0])))
    if dst_ptrs and sum(t.numel() for t in segments):
        LAUNCHES[0] += 1
