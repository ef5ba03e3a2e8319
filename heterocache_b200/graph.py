"""CUDA-graph decode step over every layer of a ``HeteroCache``.

The eager cache issues a handful of small launches per layer and step from
Python; at batch 1 the host, not the GPU, then sets the pace.  This module
captures one decode step through all layers -- page append, paged
flash-decode, ``decode_select`` -- as CUDA graphs and replays them.  The drift
check runs on every ``decode_step``-th call, so there is one graph per phase
of that cycle; a step replays the graph of the current phase.

Each layer's page append is deferred: attention merges the step's token from
its k/v, and the append runs on the side stream off the critical path (the
graph joins it at the end of the step).

Order per layer follows the patched attention: Llama runs ``decode_select``
after attention (heterocache/llama_model.py:382-391), Qwen2 before it
(heterocache/qwen_model.py:178-201).

Inputs and outputs are static device buffers owned by the graph object:
``q`` [layers, bsz, H, 1, D], ``k``/``v`` [layers, bsz, KV, 1, D] and ``out``
[layers, bsz, H, D].  Host bookkeeping (free-list check, mirrored lengths,
cycle position) still runs per step, so the reference's ``Layer N OOM.`` is
raised before a replay that would need more pages than the free list holds.
"""
from __future__ import annotations

import copy
from typing import List

import torch

from .cache import HeteroCache


class DecodeStepGraph:
    def __init__(self, cache: HeteroCache, layers: List[int], order: str = "llama"):
        if order not in ("llama", "qwen"):
            raise ValueError("order must be 'llama' or 'qwen'")
        if cache.key_pools[layers[0]] is None:
            raise RuntimeError("capture after prefill")
        phases = {cache._qcount[l] for l in layers}
        if len(phases) != 1:
            raise RuntimeError("all layers must be at the same position of the decode_step cycle")
        self.cache, self.layers, self.order = cache, list(layers), order
        dev = cache._dev
        bsz, H, KV, D = cache.bsz, cache.num_attn_heads, cache.num_kv_heads, cache.head_dim
        dt = cache.key_pools[layers[0]].dtype
        n = len(self.layers)
        self.q = torch.zeros(n, bsz, H, 1, D, dtype=dt, device=dev)
        self.k = torch.zeros(n, bsz, KV, 1, D, dtype=dt, device=dev)
        self.v = torch.zeros(n, bsz, KV, 1, D, dtype=dt, device=dev)
        self.out = torch.zeros(n, bsz, H, D, dtype=dt, device=dev)
        cache.prepare_decode(self.layers, self.q[0])
        cache.join_retrievals()  # no capture may wait on work recorded outside it
        S = cache.decode_step
        self.graphs: List[torch.cuda.CUDAGraph] = []
        start = cache._qcount[self.layers[0]]
        torch.cuda.synchronize(dev)
        for phase in range(S):
            saved = cache._host_state()
            for l in self.layers:
                cache._qcount[l] = phase
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._eager_step()
            cache._restore_host_state(saved)
            self.graphs.append(g)
        for l in self.layers:
            cache._qcount[l] = start

    def _eager_step(self) -> None:
        c = self.cache
        for i, l in enumerate(self.layers):
            c.update(self.k[i], self.v[i], l, {"query_states": self.q[i], "defer_append": True})
            if self.order == "qwen":
                c.decode_select(self.q[i], l)
            c.attention(self.q[i], l, out=self.out[i])
            if self.order == "llama":
                c.decode_select(self.q[i], l)
        c.join_retrievals()

    def step(self) -> torch.Tensor:
        """Replay one decode step (inputs already in ``self.q/k/v``)."""
        c = self.cache
        phase = c._qcount[self.layers[0]]
        for l in self.layers:
            c._append_bookkeeping(l)
        self.graphs[phase].replay()
        nxt = (phase + 1) % c.decode_step
        for l in self.layers:
            c._qcount[l] = nxt
        return self.out
