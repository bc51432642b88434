"""Page summary build / refresh -- host side of the sm_100a summary kernel.

Mirrors the reference's page-finalize builders (``amass.selection``):

  quad_build_tail / quad_build_bulk   selection/quad_build.py:87-121
  r8_build_tail / r8_build_bulk       selection/build.py:435-530
  summarize_pages (the _quad_write / _r8_write core)
                                      selection/quad_build.py:56-84,
                                      selection/build.py:415-432

Every call is one kernel launch over (layer, block, kv-head) pages, with no
host synchronisation (the block lists are built with device ops), so the
builders can run beside the decode on their own stream.  Summaries are a pure
function of the page's keys: rebuilding a page is idempotent.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import ptr


def _layers_arg(K_layers):
    ks = list(K_layers)
    k0 = ks[0]
    if k0.dtype != torch.bfloat16:
        raise ValueError("key caches must be bf16")
    for k in ks:
        if k.stride() != k0.stride() or k.shape != k0.shape:
            raise ValueError("all layers' key caches must share shape/strides")
    arr = (ctypes.c_void_p * len(ks))(*[k.data_ptr() for k in ks])
    return arr, k0


def summarize_pages(st, K_layers, blocks, layer0: int = 0) -> None:
    """Summarise + quantise + scatter the pages ``blocks`` (int32 device
    tensor of physical block ids) of every key cache in ``K_layers`` (each
    (NB, page, n_kv, d) bf16, e.g. ``kv_cache[:, 0]``) into the state's slabs
    at layers layer0, layer0 + 1, ...  Works for a QuadState (quad or CLSE)
    and for an R8State."""
    arr, k0 = _layers_arg(K_layers)
    _, page, n_kv, d = k0.shape
    blocks = blocks.to(torch.int32).contiguous()
    if hasattr(st, "r8_mu"):                       # R8State
        mu, mus, V, Vs = st.r8_mu, st.mu_scale, st.r8_Vk, st.Vk_scale
        v_bits = int(getattr(st, "vk_bits", 8))
        v_tensor = getattr(st, "vk_grain", "col") != "col"
        sig2 = None
        tag = getattr(st, "r8_tag", None)
        c, cs = st.r8_c, st.c_scale
        c_bits = int(st.c_bits)
        c_mode = 0 if getattr(st, "c_grain", "page") == "page" else 1
        resid = None
    else:                                          # QuadState
        mu, mus, V, Vs = st.quad_mu, st.mu_scale, st.quad_V, st.V_scale
        v_bits = int(getattr(st, "v_bits", 8))
        v_tensor = getattr(st, "v_grain", "col") != "col"
        sig2 = st.quad_sig2
        tag = getattr(st, "quad_tag", None)
        c = getattr(st, "quad_c", None)
        cs = getattr(st, "c_scale", None) if c is not None else None
        c_bits = int(getattr(st, "c_bits", 8))
        c_mode = 0 if getattr(st, "c_grain", "token") == "token" else 2
        resid = getattr(st, "quad_resid", None) if c is not None else None
    tagw = int(tag.shape[-1]) if tag is not None else 0
    _lib.call("amass_summarize_pages", ctypes.cast(arr, ctypes.c_void_p),
              len(arr), k0.stride(0), k0.stride(1), k0.stride(2), ptr(blocks),
              int(blocks.numel()), int(layer0), int(mu.shape[1]), int(n_kv),
              int(d), int(page), int(st.r), ptr(mu), ptr(mus), ptr(V),
              ptr(Vs), v_bits, 1 if v_tensor else 0, ptr(sig2), ptr(tag),
              tagw, ptr(c), ptr(cs), c_bits, c_mode, ptr(resid),
              _lib.stream_of(k0.device))


def tail_blocks(block_table, seq_lens, n_req: int, page: int, rows=None):
    """Physical block of each request's last finalized page (index
    seq_len // page - 1, clamped to 0); ``rows`` selects requests
    (reference build.py:371-383).  Device ops only."""
    if rows is None:
        sl = seq_lens[:n_req].to(torch.int64)
        bt = block_table[:n_req]
    else:
        sl = seq_lens[rows].to(torch.int64)
        bt = block_table[rows]
    fin1 = (sl // page - 1).clamp_(min=0)
    return bt.to(torch.int64).gather(1, fin1[:, None]).squeeze(1).to(torch.int32)


def bulk_blocks(block_table, seq_lens, n_req: int, page: int, max_fin: int):
    """Blocks of every finalized page p < min(seq_len // page, max_fin) of
    the first n_req requests (reference build.py:454-464).  Device ops; the
    result is padded with the rows' page-0 blocks (idempotent rebuilds)."""
    sl = seq_lens[:n_req].to(torch.int64)
    fin = (sl // page).clamp_(max=max_fin)
    bt = block_table[:n_req, :max_fin].to(torch.int64)
    p = torch.arange(max_fin, device=bt.device)[None, :]
    sel = torch.where(p < fin[:, None], bt, bt[:, :1])
    return sel.reshape(-1).to(torch.int32)


def quad_build_tail(st, K_layers, block_table, seq_lens, n_req: int,
                    rows=None) -> int:
    """Rebuild the last finalized page of every (selected) request for every
    layer of ``K_layers`` (reference quad_build.py:87-105)."""
    if n_req == 0:
        return 0
    blocks = tail_blocks(block_table, seq_lens, n_req, st.page, rows)
    if blocks.numel() == 0:
        return 0
    summarize_pages(st, K_layers, blocks)
    return len(K_layers) * int(blocks.numel())


def quad_build_bulk(st, K_layers, block_table, seq_lens, n_req: int,
                    max_fin: int) -> int:
    """Rebuild every finalized page (first ``max_fin`` of each request) for
    every layer (reference quad_build.py:108-121)."""
    if n_req == 0 or max_fin <= 0:
        return 0
    blocks = bulk_blocks(block_table, seq_lens, n_req, st.page, max_fin)
    summarize_pages(st, K_layers, blocks)
    return len(K_layers) * int(blocks.numel())


def delta_blocks(block_table, seq_lens, n_req: int, page: int, max_fin: int):
    """Blocks of every finalized page p < min(seq_len // page, max_fin) of
    the first n_req requests, -1 elsewhere (device ops)."""
    sl = seq_lens[:n_req].to(torch.int64)
    fin = (sl // page).clamp_(max=max_fin)
    bt = block_table[:n_req, :max_fin].to(torch.int64)
    p = torch.arange(max_fin, device=bt.device)[None, :]
    return torch.where(p < fin[:, None], bt, -1).reshape(-1).to(torch.int32)


def quad_build_delta(st, K_layers, block_table, seq_lens, n_req: int,
                     max_fin: int, chunk_pairs: int = 8192) -> int:
    """Composition-change rebuild: every finalized block whose content tag
    (leading tag channels of its page-final key) no longer matches the live
    keys in some layer is rebuilt in all layers of ``K_layers`` (reference
    quad_build.py:110-121, build.py:532-545).  One tag kernel and one
    summary launch; returns layers x stale (request, page) entries rebuilt
    (a host read, like the reference's count)."""
    if n_req == 0 or max_fin <= 0:
        return 0
    tag = getattr(st, "r8_tag", None) if hasattr(st, "r8_mu") else \
        getattr(st, "quad_tag", None)
    if tag is None:
        raise ValueError("the state has no content tags (tagw = 0)")
    arr, k0 = _layers_arg(K_layers)
    cand = delta_blocks(block_table, seq_lens, n_req, st.page, max_fin)
    stale = torch.empty_like(cand)
    count = torch.zeros(1, dtype=torch.int32, device=cand.device)
    _lib.call("amass_tag_stale", ctypes.cast(arr, ctypes.c_void_p), len(arr),
              k0.stride(0), k0.stride(1), k0.stride(2), ptr(tag), 0,
              int(tag.shape[1]), int(st.n_kv), int(tag.shape[-1]),
              int(st.page), ptr(cand), int(cand.numel()), ptr(stale),
              ptr(count), _lib.stream_of(k0.device))
    summarize_pages(st, K_layers, stale)
    return len(K_layers) * int(count.item())


r8_build_tail = quad_build_tail
r8_build_bulk = quad_build_bulk
r8_build_delta = quad_build_delta

__all__ = ["bulk_blocks", "delta_blocks", "quad_build_bulk", "quad_build_delta",
           "r8_build_delta", "quad_build_tail",
           "r8_build_bulk", "r8_build_tail", "summarize_pages", "tail_blocks"]
