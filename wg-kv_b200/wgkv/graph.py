"""Whole decode steps replayed as CUDA graphs.

The reference runs every decode step eagerly from Python (scripts/profiling.py:392-396):
one step is, per layer, the gate, the ring append, the paged attention and, at layer 0,
the lazy promotion (src/modeling_layers.py:1452-1509), and at batch 1 the host issue
time of those launches is longer than the kernels themselves.  Every launch of this
library is capturable (no host sync, no allocation inside the C calls), and the only
host state a step reads is the ring position (local_length, local_ptr).  With
``cache.wgkv_device_ring`` set, the kernels take that position from ``cache.ring_state``
on the device (``WGKV_RING_ON_DEVICE``) and the last layer advances it there
(``wgkv_ring_advance``), so one captured graph is valid for every later step.

Deferred gating (``g_defer``) rescoring the whole ring happens on the step whose insert
position is window - 1 (:1404-1405); that step replays a second graph captured with the
rescoring launches.  The host copy of the ring position is still advanced on each
replay (plain arithmetic, no sync), so eager calls can follow graph replays.
"""
from __future__ import annotations

import torch

from .pool import advance_host_ring, ring_to_device


def graph_variant(local_length: int, local_ptr: int, window: int, defer: bool) -> str:
    """Which captured step replays next: "refresh" when deferred gating rescores the whole ring on
    this step (its insert position is window - 1, modeling_layers.py:1404-1405), else "plain"."""
    ins = local_length if local_length < window else local_ptr
    return "refresh" if defer and ins == window - 1 else "plain"


class DecodeGraph:
    """Capture ``step_fn`` (one decode step of all layers over static input tensors) and replay it.

    ``step_fn()`` must read its inputs from tensors the caller refills in place before each
    :meth:`replay` and write its outputs to tensors it returns (or that the caller owns).
    :meth:`capture` first runs ``step_fn`` once eagerly as a real decode step (warming the
    workspaces, cuBLAS handles and allocator on the capture stream), then records the graph(s)
    without executing them.  Each :meth:`replay` is one more decode step."""

    def __init__(self, cache, window: int, defer: bool = False, device=None):
        self.cache = cache
        self.W = int(window)
        self.defer = bool(defer)
        self.device = torch.device(device) if device is not None else torch.device("cuda",
                                                                                      torch.cuda.current_device())
        self.stream = torch.cuda.Stream(self.device)
        self.graphs = {}
        self.out = {}
        self.pool = None

    def capture(self, step_fn):
        c = self.cache
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            first = step_fn()  # a real, eager decode step
        self.first = first
        cur.wait_stream(self.stream)
        torch.cuda.synchronize(self.device)
        ring_to_device(c)
        saved = (c.local_length, c.local_ptr)
        # host positions that select the graph's structure only; the kernels read ring_state
        variants = {"plain": (self.W, 0)}
        if self.defer:
            variants["refresh"] = (self.W, self.W - 1)
        c.wgkv_device_ring = True
        try:
            for name, (ln, ptr) in variants.items():
                c.local_length, c.local_ptr = ln, ptr
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=self.pool, stream=self.stream):
                    self.out[name] = step_fn()
                self.pool = g.pool()
                self.graphs[name] = g
        finally:
            c.wgkv_device_ring = False
            c.local_length, c.local_ptr = saved
        return first

    def replay(self):
        """One decode step; returns what ``step_fn`` returned at capture (the graph's outputs)."""
        name = graph_variant(self.cache.local_length, self.cache.local_ptr, self.W, self.defer)
        self.graphs[name].replay()
        advance_host_ring(self.cache, self.W)
        return self.out[name]
