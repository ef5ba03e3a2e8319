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
(heterocache/qwen_model.py:178-201).  In the Llama order a due drift check
is put off to the end of the step, where every layer's check runs in one
batch (``HeteroCache.flush_checks``) before the retrievals.

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

from . import ops
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
        # this library's kernel launches held by each phase's graph
        self.launches_per_phase: List[int] = []
        self.graphs = self._capture((self.q, self.k, self.v, self.out), self.launches_per_phase)
        self._alt = None  # a second buffer set and its graphs (run_host)

    def _capture(self, bufs, launches=None) -> List[torch.cuda.CUDAGraph]:
        """One graph per phase of the drift-check cycle, reading q/k/v from and
        writing out to ``bufs``."""
        cache = self.cache
        start = cache._qcount[self.layers[0]]
        torch.cuda.synchronize(cache._dev)
        graphs = []
        for phase in range(cache.decode_step):
            saved = cache._host_state()
            for l in self.layers:
                cache._qcount[l] = phase
            g = torch.cuda.CUDAGraph()
            n0 = ops.LAUNCHES[0]
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._eager_step(*bufs)
            if launches is not None:
                launches.append(ops.LAUNCHES[0] - n0)
            cache._restore_host_state(saved)
            graphs.append(g)
        for l in self.layers:
            cache._qcount[l] = start
        return graphs

    def _eager_step(self, q=None, k=None, v=None, out=None) -> None:
        c = self.cache
        q = self.q if q is None else q
        k = self.k if k is None else k
        v = self.v if v is None else v
        out = self.out if out is None else out
        for i, l in enumerate(self.layers):
            c.update(k[i], v[i], l, {"query_states": q[i], "defer_append": True})
            if self.order == "qwen":
                c.decode_select(q[i], l)
            c.attention(q[i], l, out=out[i])
            if self.order == "llama":
                c.decode_select(q[i], l, defer=True)
        c.join_retrievals()  # runs the put-off drift checks as one batch first

    def step(self) -> torch.Tensor:
        """Replay one decode step (inputs already in ``self.q/k/v``)."""
        return self._step(self.graphs, self.out)

    def _step(self, graphs, out) -> torch.Tensor:
        c = self.cache
        phase = c._qcount[self.layers[0]]
        for l in self.layers:
            c._append_bookkeeping(l)
        graphs[phase].replay()
        nxt = (phase + 1) % c.decode_step
        for l in self.layers:
            c._qcount[l] = nxt
        if 0 in self.layers:  # as update() of layer 0 counts the token
            c._seen_tokens += 1
        return out

    def prepare_host(self) -> None:
        """Capture the second buffer set's graphs that ``run_host`` alternates
        with (once; ``run_host`` does it on its first call otherwise)."""
        if self._alt is not None:
            return
        dev = self.q.device
        bufs = (torch.zeros_like(self.q), torch.zeros_like(self.k), torch.zeros_like(self.v),
                torch.zeros_like(self.out))
        self.cache.join_retrievals()  # no capture may wait on work recorded outside it
        self._alt = (bufs, self._capture(bufs))
        self._h2d, self._d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def run_host(self, host_q: torch.Tensor, host_k: torch.Tensor, host_v: torch.Tensor,
                 host_out: torch.Tensor) -> None:
        """Decode ``len(host_q)`` steps from host inputs into host outputs
        (pinned memory: ``host_q[s]`` shaped as ``self.q``, ``host_out[s]`` as
        ``self.out``), the host-link copies overlapped with the replays.  Steps
        alternate between two buffer sets, each with its own graphs (the
        second set is captured by ``prepare_host`` or on the first call): step s + 1's inputs cross
        into its set on a copy stream while step s runs, and step s's outputs
        leave from its set on another copy stream while step s + 1 runs; no
        device-side copy is added to the step.  Work already queued on the
        current stream comes first; the current stream waits for the last
        copy back."""
        n = host_q.shape[0]
        if n == 0:
            return
        dev = self.q.device
        cur = torch.cuda.current_stream(dev)
        self.prepare_host()
        sets = [((self.q, self.k, self.v, self.out), self.graphs), self._alt]
        h2d, d2h = self._h2d, self._d2h
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]

        def load(s: int) -> None:
            j = s % 2
            (q, k, v, _), _ = sets[j]
            with torch.cuda.stream(h2d):
                if s >= 2:
                    h2d.wait_event(in_free[j])  # step s - 2 has run on this set
                for dst, src in zip((q, k, v), (host_q[s], host_k[s], host_v[s])):
                    dst.copy_(src, non_blocking=True)
                in_ready[j].record(h2d)

        load(0)
        for s in range(n):
            i = s % 2
            (_, _, _, out), graphs = sets[i]
            if s + 1 < n:
                load(s + 1)
            cur.wait_event(in_ready[i])
            if s >= 2:
                cur.wait_event(out_done[i])  # step s - 2's outputs have left this set
            self._step(graphs, out)
            in_free[i].record(cur)
            out_ready[i].record(cur)
            with torch.cuda.stream(d2h):
                d2h.wait_event(out_ready[i])
                host_out[s].copy_(out, non_blocking=True)
                out_done[i].record(d2h)
        cur.wait_stream(d2h)
        cur.wait_stream(h2d)


class ModelDecodeGraph:
    """CUDA graphs of one greedy decode token through a whole transformers
    causal LM whose attention layers are the patched classes of
    ``heterocache_b200.attention`` over a ``HeteroCache``: embedding, every
    layer (projections, RoPE, the cache's append / attention / drift check /
    retrieval launches, MLP), final norm, LM head and argmax, one graph per
    phase of the drift-check cycle (as ``DecodeStepGraph``).

    The graph reads the current token and position from the static buffers
    ``tok`` [bsz, 1] and ``pos`` [bsz, 1] (int64) and writes the greedy next
    token into ``tok`` and ``pos + 1`` into ``pos``, so consecutive ``step()``
    calls decode token after token with no host work but the cache's
    mirrored bookkeeping.  Capture after prefill, with ``tok``/``pos`` set to
    the first decode token and its position.  The model's own code must not
    synchronise with the host in a decode forward (transformers' Llama and
    Qwen2 do not when no attention mask is passed).
    """

    def __init__(self, model, cache: HeteroCache, tok: torch.Tensor, pos: torch.Tensor):
        layers = [l for l in range(cache.num_layers) if cache.key_pools[l] is not None]
        if len(layers) != cache.num_layers:
            raise RuntimeError("capture after prefill")
        phases = {cache._qcount[l] for l in layers}
        if len(phases) != 1:
            raise RuntimeError("all layers must be at the same position of the decode_step cycle")
        self.model, self.cache = model, cache
        self.tok, self.pos = tok, pos
        dev = cache._dev
        q_example = torch.zeros(cache.bsz, cache.num_attn_heads, 1, cache.head_dim,
                                dtype=cache.key_pools[0].dtype, device=dev)
        cache.prepare_decode(layers, q_example)
        cache.join_retrievals()
        self.layers = layers
        S = cache.decode_step
        start = cache._qcount[layers[0]]
        self.graphs: List[torch.cuda.CUDAGraph] = []
        # this library's kernel launches held by each phase's graph
        self.launches_per_phase: List[int] = []
        torch.cuda.synchronize(dev)
        pool = None
        for phase in range(S):
            saved = cache._host_state()
            for l in layers:
                cache._qcount[l] = phase
            g = torch.cuda.CUDAGraph()
            n0 = ops.LAUNCHES[0]
            with torch.no_grad(), torch.cuda.graph(g, pool=pool, capture_error_mode="thread_local"):
                self._forward()
            self.launches_per_phase.append(ops.LAUNCHES[0] - n0)
            pool = g.pool()
            cache._restore_host_state(saved)
            self.graphs.append(g)
        for l in layers:
            cache._qcount[l] = start

    def _forward(self) -> None:
        out = self.model(input_ids=self.tok, position_ids=self.pos, cache_position=self.pos[0],
                         past_key_values=self.cache, use_cache=True, logits_to_keep=1)
        self.tok.copy_(out.logits[:, -1:].argmax(-1))
        self.pos.add_(1)
        self.cache.join_retrievals()

    def step(self) -> torch.Tensor:
        """Decode one token: returns ``tok`` (now the next token)."""
        c = self.cache
        phase = c._qcount[self.layers[0]]
        for l in self.layers:
            c._append_bookkeeping(l)
        self.graphs[phase].replay()
        nxt = (phase + 1) % c.decode_step
        for l in self.layers:
            c._qcount[l] = nxt
        c._seen_tokens += 1
        return self.tok
