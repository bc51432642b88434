"""Multi-GPU layouts of the decode hot path (one process per GPU).

Sequence sharding.  Requests share nothing on this path (per-request block
table, summaries, selection and decode; reference attention/decode.py:145-241
works per (request, kv-head)), so a ragged batch is split across ranks by LPT
on each request's algorithmic bytes and every rank runs the unchanged
single-GPU path on its share: no collective on the data path.

KV-head sharding.  Rank g owns kv heads [g*n_kv/N, (g+1)*n_kv/N) of every
request (scores, the GQA combine, selection and decode are per kv-head).
The one exchange is the output: each rank's merge kernel stores its heads'
rows into every rank's output buffer over NVLink (peer-mapped symmetric
memory) and a peer barrier kernel orders those stores before any reader
(``mode="p2p"``); ``mode="nccl"`` decodes into a local slice and calls NCCL
all-gather plus a head permute instead.
"""
from __future__ import annotations

import ctypes
import heapq
from typing import List, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import ptr
from .attention import pps_min_for, split_kv


# --------------------------------------------------------------------------- #
# sequence sharding                                                           #
# --------------------------------------------------------------------------- #
def request_bytes(seq_lens: Sequence[int], *, n_kv: int, page: int,
                  budget: float, b_sum: int, d: int, G: int, sink: int = 1,
                  window: int = 1) -> np.ndarray:
    """Algorithmic bytes of one layer-step per request: summaries of the
    scored pages, their block-table entries, the selected K and V tiles
    (budget pages plus sink and window) and q/out."""
    sl = np.asarray(seq_lens, dtype=np.int64)
    npg = -(-sl // page)
    nsh = np.maximum(npg - window, 0)
    nsel = np.maximum(nsh - sink, 0)
    b = np.where(nsel > 0, np.minimum(np.maximum(np.ceil(nsel * budget), 1),
                                      nsel), 0)
    kept = np.minimum(b + sink + window, npg)
    return (n_kv * nsh * b_sum + 4 * nsh + n_kv * kept * 2 * page * d * 2
            + n_kv * G * d * 2 * 2).astype(np.int64)


def lpt_partition(costs: Sequence[float], world: int) -> List[List[int]]:
    """Longest-processing-time assignment: requests in decreasing cost go to
    the least-loaded rank (lowest rank on ties).  Returns each rank's request
    indices in increasing order."""
    if world < 1:
        raise ValueError("world >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    heap = [(0.0, r) for r in range(world)]
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(p) for p in parts]


# --------------------------------------------------------------------------- #
# kv-head sharding                                                            #
# --------------------------------------------------------------------------- #
def kv_head_range(n_kv: int, world: int, rank: int):
    """[lo, hi) kv heads owned by `rank`; n_kv must divide evenly."""
    if n_kv % world:
        raise ValueError(f"n_kv={n_kv} is not divisible by world={world}")
    per = n_kv // world
    return rank * per, (rank + 1) * per


class HeadGather:
    """The (T, H, d) bf16 output of a kv-head-sharded decode on every rank.

    mode "p2p": two symmetric output buffers (alternating per call, so a
    peer's stores for call k+1 never land in the buffer this rank may still
    be reading from call k) plus peer flag arrays for the barrier; the
    merge kernel writes every rank's buffer directly.
    mode "nccl": a local (T, H/N, d) slice, a (N, T, H/N, d) receive buffer
    and NCCL (or, on CPU process groups, gloo) all-gather + permute."""

    def __init__(self, T: int, H: int, d: int, *, group=None, device=None,
                 mode: str = "p2p"):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if H % self.world:
            raise ValueError(f"H={H} is not divisible by world={self.world}")
        self.T, self.H, self.d, self.Hl = T, H, d, H // self.world
        self.mode = mode
        dev = torch.device(device) if device is not None else None
        if mode == "p2p":
            # plain peer mappings only: no NVLink multicast objects
            import os
            os.environ["TORCH_SYMM_MEM_DISABLE_MULTICAST"] = "1"
            import torch.distributed._symmetric_memory as symm
            if self.world > 8:
                raise ValueError("p2p gather supports up to 8 ranks")
            grp = group if group is not None else dist.group.WORLD
            self.bufs, self._hdl = [], []
            for _ in range(2):
                b = symm.empty((T, H, d), dtype=torch.bfloat16, device=dev)
                b.zero_()
                self.bufs.append(b)
                self._hdl.append(symm.rendezvous(b, grp))
            self.flags = symm.empty((self.world,), dtype=torch.int32,
                                    device=dev)
            self.flags.zero_()
            fh = symm.rendezvous(self.flags, grp)
            torch.cuda.synchronize(dev)
            dist.barrier(group)
            self._peer_out = [(ctypes.c_void_p * self.world)(*h.buffer_ptrs)
                              for h in self._hdl]
            self._peer_flags = (ctypes.c_void_p * self.world)(*fh.buffer_ptrs)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
            self.err = torch.zeros(1, dtype=torch.int32, device=dev)
            self.calls = 0
        elif mode == "nccl":
            self.local = torch.zeros((T, self.Hl, d), dtype=torch.bfloat16,
                                     device=dev)
            self.recv = torch.zeros((self.world, T, self.Hl, d),
                                    dtype=torch.bfloat16, device=dev)
            self.out = torch.zeros((T, H, d), dtype=torch.bfloat16,
                                   device=dev)
        else:
            raise ValueError(f"mode must be 'p2p' or 'nccl', got {mode!r}")

    # -- p2p ------------------------------------------------------------------
    def next_buffer(self):
        """(output tensor, peer pointer array) of the next call.  Under CUDA
        graph capture the buffer is fixed per captured graph: capture an
        even number of alternating graphs (e.g. one per layer)."""
        i = self.calls & 1
        self.calls += 1
        return self.bufs[i], self._peer_out[i]

    def barrier(self, stream=None) -> None:
        st = stream if stream is not None else \
            torch.cuda.current_stream(self.epoch.device).cuda_stream
        _lib.call("amass_peer_barrier",
                  ctypes.cast(self._peer_flags, ctypes.c_void_p), self.world,
                  self.rank, ptr(self.epoch), ptr(self.err), st)

    def check(self) -> None:
        """Raise if a barrier wait timed out (host sync)."""
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"peer barrier timed out waiting for rank "
                               f"{e - 1}")

    # -- nccl -----------------------------------------------------------------
    def all_gather(self) -> torch.Tensor:
        """Gather every rank's local slice into ``out`` (T, H, d)."""
        dist = self.dist
        if dist.get_backend(self.group) == "gloo":
            parts = list(self.recv.unbind(0))
            dist.all_gather(parts, self.local, group=self.group)
            for r, p in enumerate(parts):
                self.recv[r].copy_(p)
        else:
            dist.all_gather_into_tensor(self.recv, self.local,
                                        group=self.group)
        self.out.view(self.T, self.world, self.Hl, self.d).copy_(
            self.recv.permute(1, 0, 2, 3))
        return self.out


def sparse_paged_decode_kvsharded(q_local, kv_local, block_table, seq_lens,
                                  st_local, gather: HeadGather, *, scale,
                                  pps_min=None) -> torch.Tensor:
    """Decode of this rank's kv heads (``st_local`` holds its selection,
    ``q_local`` (T, H/N, d) its query heads, ``kv_local`` its cache slice)
    and the exchange of the outputs; returns this call's (T, H, d) output
    (valid rows [0, n_req))."""
    n_req = seq_lens.shape[0]
    k, v = split_kv(kv_local)
    _, page, n_kv_l, d = k.shape
    if pps_min is None:
        pps_min = pps_min_for(n_req)
    common = (ptr(q_local), q_local.stride(0), q_local.stride(1), ptr(k),
              k.stride(0), k.stride(1), k.stride(2), ptr(v), v.stride(0),
              v.stride(1), v.stride(2), ptr(block_table),
              block_table.stride(0), ptr(st_local.page_table),
              ptr(st_local.page_cnt), ptr(seq_lens), ptr(st_local.m_part),
              ptr(st_local.l_part), ptr(st_local.acc_part),
              int(st_local.split), int(pps_min))
    stream = _lib.stream_of(q_local.device)
    if gather.mode == "p2p":
        out, peers = gather.next_buffer()
        _lib.call("amass_sparse_decode_gather", *common,
                  ctypes.cast(peers, ctypes.c_void_p), gather.world,
                  gather.rank * gather.Hl, out.stride(0), out.stride(1),
                  float(scale), int(n_req), int(n_kv_l), int(st_local.G),
                  int(d), int(page), int(st_local.max_pages), stream)
        gather.barrier(stream)
        return out
    loc = gather.local
    _lib.call("amass_sparse_decode", *common, ptr(loc), loc.stride(0),
              loc.stride(1), float(scale), int(n_req), int(n_kv_l),
              int(st_local.G), int(d), int(page), int(st_local.max_pages),
              stream)
    return gather.all_gather()


__all__ = ["HeadGather", "kv_head_range", "lpt_partition", "request_bytes",
           "sparse_paged_decode_kvsharded"]
