"""Stage B (sparse paged decode) -- host side of the sm_100a kernels.

Mirrors the reference's ``amass.attention`` surface for the hot path:

  ResidentVSource                   attention/decode.py:71-100
  ensure_stage_b_buffers(st, ...)   attention/decode.py:98-114
  sparse_paged_decode_batched_cuda  attention/decode_cuda.py:1376-1465

The split-K partials keep the reference layout (R, n_kv, split, G[, d]).
How a unit's pages are cut into partials is the kernel's own choice (equal
runs of the flat page list, one per warp of the grid, so ragged batches
balance); the reference's chunk rule pps = max(ceil(cnt/split), PPS_MIN)
(decode.py:154-160) is another cut of the same exact softmax re-association.
``pps_min`` here is the floor on pages per run.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr

DEFAULT_SPLIT = 128


def split_kv(kv_cache: torch.Tensor):
    """(K, V) views (num_blocks, page, n_kv, d) for the vLLM cache layouts
    (nb, 2, page, n_kv, d) and (2, nb, page, n_kv, d); V is None for a K-only
    (nb, 1, ...) cache (reference attention/decode.py:59-68)."""
    if kv_cache.shape[0] == 2:
        return kv_cache[0], kv_cache[1]
    if kv_cache.shape[1] == 1:
        return kv_cache.select(1, 0), None
    return kv_cache.select(1, 0), kv_cache.select(1, 1)


class ResidentVSource:
    """AMASS-fast V source: the resident V half of the paged cache."""

    SRC_ID = 0

    def __init__(self, kv_cache: torch.Tensor):
        _, v = split_kv(kv_cache)
        if v is None:
            raise ValueError("ResidentVSource needs a resident V half; this "
                             "cache is K-only -- use a tier V source")
        self._v = v

    def args(self):
        v = self._v
        return v, v.stride(0), v.stride(1), v.stride(2)


def ensure_stage_b_buffers(st, device, split: int = DEFAULT_SPLIT) -> None:
    """Allocate the split-K partials once (outside any graph)."""
    if getattr(st, "m_part", None) is not None:
        st.split = getattr(st, "split", split)
        return
    R, n_kv, G = st.max_reqs, st.n_kv, st.G
    D = getattr(st, "D", None) or st.d
    f32 = torch.float32
    st.split = split
    st.m_part = torch.empty(R, n_kv, split, G, device=device, dtype=f32)
    st.l_part = torch.empty(R, n_kv, split, G, device=device, dtype=f32)
    st.acc_part = torch.empty(R, n_kv, split, G, D, device=device, dtype=f32)


def pps_min_for(n_req: int) -> int:
    """Floor on the pages of one warp run (the run length is otherwise the
    balanced share of the batch's selected pages).  4 for 2..16 requests
    (B200, 8 requests per GPU: 35.1 -> 34.1 us per layer-step), else 8
    (batch 1 and the 64-request batch are unchanged by it)."""
    return 4 if 2 <= n_req <= 16 else 8


def sparse_paged_decode_batched_cuda(q, kv_cache, block_table, seq_lens, st,
                                     out, vsource=None, *, scale=None,
                                     pps_min=None) -> None:
    """Stage B: split-K decode over ``st.page_table``/``st.page_cnt`` and the
    LSE merge into ``out[:n_req]`` (bf16, in place).  Same contract as the
    reference function; ``n_req = seq_lens.shape[0]``."""
    if scale is None:
        # the state's softmax scale, else 1/sqrt(head_dim)
        scale = getattr(st, "scale", None) or q.shape[-1] ** -0.5
    n_req = seq_lens.shape[0]
    k, v = split_kv(kv_cache)
    if vsource is not None:
        v = vsource.args()[0]
    if v is None:
        raise ValueError("no V source")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or \
            out.dtype != torch.bfloat16:
        raise ValueError("q, kv_cache and out must be bf16")
    if getattr(st, "m_part", None) is None:
        raise RuntimeError("ensure_stage_b_buffers(st, ...) was not called")
    _, page, n_kv, d = k.shape
    if pps_min is None:
        pps_min = pps_min_for(n_req)
    _lib.call("amass_sparse_decode", ptr(q), q.stride(0), q.stride(1),
              ptr(k), k.stride(0), k.stride(1), k.stride(2),
              ptr(v), v.stride(0), v.stride(1), v.stride(2),
              ptr(block_table), block_table.stride(0), ptr(st.page_table),
              ptr(st.page_cnt), ptr(seq_lens), ptr(st.m_part),
              ptr(st.l_part), ptr(st.acc_part), int(st.split), int(pps_min),
              ptr(out), out.stride(0), out.stride(1), float(scale),
              int(n_req), int(n_kv), int(st.G), int(d), int(page),
              int(st.max_pages), _lib.stream_of(q.device))


sparse_paged_decode_batched = sparse_paged_decode_batched_cuda
