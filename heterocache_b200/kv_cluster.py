"""Drop-in ``SnapKVCluster`` (heterocache/kv_cluster.py:138-199).

Same constructor, ``reset`` and ``update_kv(key_states, query_states,
value_states, attention_mask, num_key_value_groups)`` as the reference's
compressor; the scoring, pooling, top-k and the gather of the kept rows run in
one sm_100a launch (``hc_snapkv_update_kv``).

* The capacity rule is the reference's: ``max_capacity_prompt`` defaults to
  ``max(int(compression_ratio * q_len / num_key_value_groups), 2)`` on the
  first call, and a prompt shorter than it is returned unchanged.
* The kept rows of each head come in ascending position order, followed by
  the last ``window_size`` rows.  The reference orders the kept rows by
  descending score (``topk`` sorted); attention over the rows does not depend
  on their order, and the kept set is the same.  Ties at the k-th score go to
  the lowest positions (``torch.topk`` leaves them unspecified).
* As in the reference, every query head is scored against its own key head
  (``key_states`` has as many heads as ``query_states``; the reference's
  ``matmul`` raises otherwise, and so does this).
* ``attention_mask`` is unused, as in the reference (the in-window causal mask
  is built from the window size).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .ops import Workspace


class SnapKVCluster:
    def __init__(self, window_size=64, compression_ratio=0.5, kernel_size=5, pooling="avgpool"):
        self.window_size = window_size
        self.compression_ratio = compression_ratio
        self.kernel_size = kernel_size
        self.pooling = pooling
        self._ws: Optional[Workspace] = None
        self._err: Optional[torch.Tensor] = None
        # kept positions of the last compression, [bsz, H, capacity - window]
        # ascending (diagnostics; None until a call compresses); with
        # record_scores set, also the pooled scores the selection ranked
        # [bsz, H, q_len] (positions q_len - window .. q_len - 1 unset)
        self.last_indices: Optional[torch.Tensor] = None
        self.record_scores = False
        self.last_scores: Optional[torch.Tensor] = None

    def reset(self, window_size=64, max_capacity_prompt=256 + 64, kernel_size=5, pooling="avgpool"):
        self.window_size = window_size
        self.max_capacity_prompt = max_capacity_prompt
        assert self.max_capacity_prompt - self.window_size > 0
        self.kernel_size = kernel_size
        self.pooling = pooling

    def update_kv(self, key_states, query_states, value_states, attention_mask, num_key_value_groups):
        assert key_states.shape[-2] == query_states.shape[-2]
        bsz, num_heads, q_len, head_dim = query_states.shape
        if not hasattr(self, "max_capacity_prompt"):
            self.max_capacity_prompt = int(self.compression_ratio * q_len / num_key_value_groups)
            self.max_capacity_prompt = max(self.max_capacity_prompt, 2)
        if self.max_capacity_prompt > q_len:
            return key_states, value_states
        if self.pooling not in ops.POOLING:
            raise ValueError("Pooling method not supported")
        dev = key_states.device
        if self._ws is None or self._ws.device != dev:
            self._ws = Workspace(dev)
            self._err = torch.zeros(1, dtype=torch.int32, device=dev)
        W, cap = self.window_size, self.max_capacity_prompt
        idx = torch.empty(bsz, num_heads, max(cap - W, 0), dtype=torch.int32, device=dev)
        sc = (torch.zeros(bsz, num_heads, q_len, dtype=key_states.dtype, device=dev) if self.record_scores
              else None)
        k_out, v_out = ops.snapkv_update_kv(query_states, key_states, value_states, window=W, pooling=self.pooling,
                                            kernel_size=self.kernel_size, capacity=cap, workspace=self._ws,
                                            err=self._err, out_indices=idx, out_scores=sc)
        self.last_indices, self.last_scores = idx, sc
        return k_out, v_out

    def check_errors(self) -> None:
        """Raise if a device-side check of the last calls fired (syncs)."""
        if self._err is not None:
            code = int(self._err.item())
            if code:
                self._err.zero_()
                self._ws.reset()
                raise RuntimeError(f"SnapKVCluster device error flags {code:#x}")
