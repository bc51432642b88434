"""Host-buffer decode steps: the layer-step (derive + quad score + select +
split-K decode + merge) replayed as CUDA graphs, with the inputs' host-to-
device copies and the output's device-to-host copy on their own streams so
that they overlap the neighbouring steps' compute.

This is how a serving engine drives the path (the reference runs inside
vLLM's full CUDA graph, backend/builder.py:81-88): fixed device buffers,
graphs captured once per layer, per step only the new query and sequence
lengths move in and the attention output moves out.  q, seq_lens and out
are double-buffered, so step i+1's upload and step i-1's download run while
step i computes; the selection state and split-K partials are shared, which
is safe because the graphs run in order on one compute stream.
"""
from __future__ import annotations

import torch

from . import attention as A
from . import selection as S


class StepPipeline:
    """``submit(layer, q_host, seq_lens_host, out_host)`` queues one
    layer-step; ``synchronize()`` waits for every queued output to reach
    host memory.  Host tensors should be pinned (the copies are
    asynchronous); ``out_host`` must not be read before ``synchronize()``.

    st: a QuadState with its Stage-B buffers (``scorer="clse"``: one built
    with coordinates, ``coords="lse"``); kv_caches: per layer the
    (NB, 2, page, n_kv, d) bf16 cache; block_table (R, MP) int32 on the
    device (fixed for the pipeline's life -- replace its contents between
    steps only after ``synchronize()``)."""

    def __init__(self, st, kv_caches, block_table, *, n_req: int,
                 scale: float, q_shape, device=None, scorer: str = "quad"):
        if scorer not in ("quad", "clse"):
            raise ValueError(f"scorer must be 'quad' or 'clse', got {scorer!r}")
        self.select = S.select_pages_quad if scorer == "quad" else \
            S.select_pages_clse
        dev = torch.device(device) if device is not None else \
            block_table.device
        self.dev, self.st, self.kv = dev, st, list(kv_caches)
        self.bt, self.n_req, self.scale = block_table, int(n_req), float(scale)
        self.q = [torch.zeros(q_shape, dtype=torch.bfloat16, device=dev)
                  for _ in range(2)]
        self.sl = [torch.zeros((n_req,), dtype=torch.int32, device=dev)
                   for _ in range(2)]
        self.out = [torch.zeros(q_shape, dtype=torch.bfloat16, device=dev)
                    for _ in range(2)]
        self.compute = torch.cuda.current_stream(dev)
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.up = [torch.cuda.Event() for _ in range(2)]      # inputs landed
        self.done = [torch.cuda.Event() for _ in range(2)]    # step computed
        self.down = [torch.cuda.Event() for _ in range(2)]    # output copied
        self.i = 0
        # warm-up launch of every layer on a side stream (kernel attributes
        # are set on first use, outside capture), then capture
        side = torch.cuda.Stream(dev)
        side.wait_stream(self.compute)
        with torch.cuda.stream(side):
            for l in range(len(self.kv)):
                self._step(l, 0)
        self.compute.wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graphs = []
        for l in range(len(self.kv)):
            gl = []
            for b in range(2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._step(l, b)
                gl.append(g)
            self.graphs.append(gl)
        torch.cuda.synchronize(dev)
        for e in self.done + self.down:
            e.record(self.compute)

    def _step(self, layer: int, b: int) -> None:
        st, n = self.st, self.n_req
        self.select(st, layer, self.q[b], self.bt, self.sl[b], n, self.scale,
                    derive=True)
        A.sparse_paged_decode_batched_cuda(self.q[b], self.kv[layer], self.bt,
                                           self.sl[b], st, self.out[b],
                                           scale=self.scale)

    def submit(self, layer: int, q_host, seq_lens_host, out_host) -> None:
        b = self.i & 1
        self.i += 1
        # inputs of buffer b: after the step that last read them finished
        self.h2d.wait_event(self.done[b])
        with torch.cuda.stream(self.h2d):
            self.q[b].copy_(q_host, non_blocking=True)
            self.sl[b].copy_(seq_lens_host, non_blocking=True)
        self.up[b].record(self.h2d)
        # compute: inputs landed and the previous output of b copied out
        self.compute.wait_event(self.up[b])
        self.compute.wait_event(self.down[b])
        with torch.cuda.stream(self.compute):     # whatever the caller's stream
            self.graphs[layer][b].replay()
        self.done[b].record(self.compute)
        self.d2h.wait_event(self.done[b])
        with torch.cuda.stream(self.d2h):
            out_host.copy_(self.out[b], non_blocking=True)
        self.down[b].record(self.d2h)

    def synchronize(self) -> None:
        self.compute.wait_stream(self.d2h)
        self.compute.wait_stream(self.h2d)
        torch.cuda.synchronize(self.dev)


__all__ = ["StepPipeline"]
