"""Serving-side wiring of the mem-v / mem-kv tier: what an engine's attention
layer calls each step so that V (and K under mem-kv) lives in pinned host
memory and the device cache holds K only.

The reference leaves this as its follow-up (backend/attn.py:85-119
``_forward_mem`` sketch, backend/_runtime.py:57-71 ``_MEM_STAGEB_WIRED``,
backend/register.py:90-101 ``_patch_kv_cache_spec_k_only``, tier/README.md
FOLLOW-UP 1-3).  ``MemSession`` fills the sketch in, engine-agnostic:

  per step     begin_step   residency invalidation of rewritten pages and the
                            staging lifecycle (flush, allocate, slot map);
                            selection page parameters derived once
  per layer    write_kv     K into the K-only device cache at the engine's
                            slot mapping (mem-v), V (and K, mem-kv) into
                            staging -- every step, prefill and decode
               decode       Stage-A select -> residency plan + miss fetch ->
                            ptr-select tiered decode + merge (pure decode)
  after layers refresh      summaries of the pages that became complete

``patch_kv_cache_spec_k_only`` is the engine half that realises the VRAM
saving: the attention layer's cache spec keeps K only (``head_size_v=0``).
"""
from __future__ import annotations

import dataclasses

import torch

from . import _lib
from . import selection as S
from . import summaries as SM
from . import tier as T
from ._lib import ptr
from .attention import ensure_stage_b_buffers


class MemSession:
    """One model's mem-v (``offload_k=False``) or mem-kv tier plus its
    selection state (``scorer`` "quad", or "clse" -- the reference config's
    default -- with per-token coordinates), sized once from engine maxima.

    Device memory: the K-only cache (L, NB, 1, page, n_kv, d) (a one-block
    stand-in under mem-kv, whose K lives in the tier), quad summaries, the
    hot buffer (``hot_frac`` of ``max_pages`` slots per layer and kv-head)
    and staging.  Host: the pinned pool(s) keyed by NB."""

    def __init__(self, *, num_layers: int, num_blocks: int, n_kv: int,
                 G: int, head_dim: int, max_reqs: int, max_pages: int,
                 max_tokens: int, page: int = 16, hot_frac: float = 0.1,
                 hot_slots: int | None = None, budget: float = 0.05,
                 rank: int = 2, v_bits: int = 4, combine: str = "nrm",
                 coverage=None, offload_k: bool = False, device="cuda",
                 max_pool_gb: float = 256.0, scorer: str = "quad",
                 c_bits: int = 4, c_grain: str = "token"):
        dev = torch.device(device)
        self.device = dev
        self.L, self.NB, self.n_kv, self.G = num_layers, num_blocks, n_kv, G
        self.d, self.page, self.R, self.MP = head_dim, page, max_reqs, max_pages
        self.offload_k = offload_k
        S_ = hot_slots if hot_slots is not None else \
            max(1, int(round(hot_frac * max_pages * max_reqs)))
        self.tier = T.Tier(num_layers=num_layers, num_blocks=num_blocks,
                           n_kv=n_kv, page=page, d=head_dim, hot_slots=S_,
                           max_reqs=max_reqs, max_pages=max_pages,
                           max_tokens=max_tokens, offload_k=offload_k,
                           device=dev, max_pool_gb=max_pool_gb)
        nb_k = 1 if offload_k else num_blocks
        self.k_cache = torch.zeros((num_layers, nb_k, 1, page, n_kv, head_dim),
                                   dtype=torch.bfloat16, device=dev)
        if scorer not in ("quad", "clse"):
            raise ValueError(f"scorer must be 'quad' or 'clse', got {scorer!r}")
        self.scorer = scorer
        extra = dict(coords="lse", c_bits=c_bits, c_grain=c_grain) \
            if scorer == "clse" else {}
        self.st = S.QuadState(dev, num_layers=num_layers,
                              num_blocks=num_blocks, n_kv=n_kv, G=G,
                              head_dim=head_dim, page=page, max_reqs=max_reqs,
                              max_pages=max_pages, rank=rank, budget=budget,
                              v_bits=v_bits, combine=combine,
                              coverage=coverage, **extra)
        ensure_stage_b_buffers(self.st, dev)
        self._n_req = 0
        self._bt = self._sl = None

    # -- per step -------------------------------------------------------------
    def begin_step(self, block_table, seq_lens, query_start_loc,
                   max_query_len: int, n_tokens: int,
                   capture: bool = False) -> None:
        """Before the first layer of a step (reference tier/tier.py:86-104
        plus builder.py's once-per-step derive)."""
        self.tier.begin_step(block_table, seq_lens, query_start_loc,
                             max_query_len, n_tokens, capture=capture)
        n_req = seq_lens.shape[0]
        if n_req:
            S.derive_page_params(self.st, seq_lens, n_req)
        self._n_req, self._bt, self._sl = n_req, block_table, seq_lens

    def write_kv(self, layer: int, key, value, slot_mapping,
                 n_tokens: int) -> None:
        """This step's K (n_tokens, n_kv, d) into the K-only cache at the
        engine's slot mapping (block * page + offset, -1 skips) under mem-v,
        and V (and K under mem-kv) into staging at the tier's own slots."""
        l = int(layer)
        if not self.offload_k:
            kc = self.k_cache[l][:, 0]                 # (NB, page, n_kv, d)
            _lib.call("amass_staging_scatter", ptr(key), key.stride(0),
                      key.stride(1), 0, 0, 0, ptr(slot_mapping), ptr(kc), 0,
                      kc.stride(0), kc.stride(1), kc.stride(2), int(n_tokens),
                      self.n_kv, self.d, self.page,
                      _lib.stream_of(self.device))
        self.tier.write_kv(l, value, n_tokens,
                           key=key if self.offload_k else None)

    def decode(self, layer: int, q, out, *, scale: float) -> None:
        """Pure-decode attention of one layer into ``out[:n_req]``: Stage-A
        selection (quad or CLSE), residency step and the ptr-select tiered
        decode."""
        l, n_req = int(layer), self._n_req
        if n_req == 0:
            return
        select = S.select_pages_clse if self.scorer == "clse" else \
            S.select_pages_quad
        select(self.st, l, q, self._bt, self._sl, n_req, scale, derive=False)
        T.mem_dynamic_decode(q, self.k_cache[l], self._bt, self._sl, self.st,
                             out, self.tier, l, scale=scale)

    # -- the reference's attention-backend seam ------------------------------
    def bind_kv_caches(self, kv_caches) -> None:
        """Layer index by cache address, as the reference's
        ``_runtime.tier_layer_index`` (backend/_runtime.py:124-135): the
        engine's per-layer K-only cache tensors in layer order."""
        self._lidx = {int(t.data_ptr()): i for i, t in enumerate(kv_caches)}

    def begin_step_from_metadata(self, m) -> None:
        """The builder half of the seam: once per step with the step's
        attention metadata (reference backend/builder.py, which runs the
        tier's begin_step and derive there).  ``m`` carries block_table,
        seq_lens, query_start_loc, max_query_len and num_actual_tokens."""
        self.begin_step(m.block_table, m.seq_lens, m.query_start_loc,
                        int(m.max_query_len), int(m.num_actual_tokens))

    def forward_mem(self, layer, query, key, value, kv_cache, m, output,
                    output_scale=None, output_block_scale=None, *,
                    scale: float):
        """The attention half: the reference's ``_forward_mem(self, layer,
        query, key, value, kv_cache, m, output, output_scale,
        output_block_scale)`` (backend/attn.py:85-120) with its follow-up
        filled in.  Writes this step's K and V (staging / K-only cache) and,
        on a pure-decode step, runs the tiered decode into ``output``
        (T, H*d) or (T, H, d) and returns it.  Returns None on other steps:
        the engine's own prefill attention runs there, as in the reference
        while its flag is off."""
        lidx = self._lidx.get(int(kv_cache.data_ptr())) if \
            getattr(self, "_lidx", None) else None
        if lidx is None:
            lidx = int(getattr(layer, "layer_idx"))
        n_tok = int(m.num_actual_tokens)
        self.write_kv(lidx, key[:n_tok], value[:n_tok],
                      m.slot_mapping[:n_tok], n_tok)
        if int(m.max_query_len) != 1:
            return None
        out3 = output if output.dim() == 3 else output.view(
            output.shape[0], self.n_kv * self.G, self.d)
        self.decode(lidx, query, out3, scale=scale)
        return output

    def refresh_summaries(self, rows=None) -> int:
        """Rebuild the last complete page of every (selected) request in all
        layers (after the step's K writes; reference builder.py:366-479's
        tail refresh).  Under mem-kv the keys live in the tier, so the caller
        refreshes from its own K instead (``summaries.summarize_pages``)."""
        if self.offload_k:
            raise RuntimeError("mem-kv keeps K in the tier: summarise from "
                               "the K source with summaries.summarize_pages")
        if self._n_req == 0:
            return 0
        K_layers = [self.k_cache[l][:, 0] for l in range(self.L)]
        return SM.quad_build_tail(self.st, K_layers, self._bt, self._sl,
                                  self._n_req, rows=rows)

    # -- reporting --------------------------------------------------------------
    def vram_bytes(self) -> dict:
        """Device bytes by component, and the resident K+V cache this
        replaces."""
        t = self.tier
        kb = self.k_cache.numel() * 2
        hot = t.residency.hot.numel() * 2 * (2 if self.offload_k else 1)
        stg = t.staging.v_pool.numel() * 2 * (2 if self.offload_k else 1)
        summ = sum(x.numel() * x.element_size() for x in (
            self.st.quad_mu, self.st.mu_scale, self.st.quad_V,
            self.st.V_scale, self.st.quad_sig2))
        resident_kv = 2 * self.L * self.NB * self.page * self.n_kv * self.d * 2
        return {"k_cache": kb, "hot": hot, "staging": stg, "summaries": summ,
                "resident_kv_equivalent": resident_kv}


def patch_kv_cache_spec_k_only(attn_cls) -> None:
    """Make ``attn_cls.get_kv_cache_spec`` report a K-only full-attention
    spec (``head_size_v=0``), so the engine's block pool holds K alone and
    fits twice the blocks at the same memory budget (reference
    backend/register.py:90-101).  Only plain full-attention specs with
    symmetric K/V heads are rewritten; anything else raises, since dropping
    its V half would leave attention without V.  Apply together with
    ``MemSession`` serving V."""
    from vllm.v1.kv_cache_interface import FullAttentionSpec
    orig = attn_cls.get_kv_cache_spec
    if getattr(orig, "_amass_k_only", False):
        return

    def get_kv_cache_spec(self, *args, **kwargs):
        spec = orig(self, *args, **kwargs)
        if spec is None:
            return spec
        if type(spec) is not FullAttentionSpec:
            raise RuntimeError(f"mem tier: cannot drop V of a "
                               f"{type(spec).__name__} layer")
        hv = getattr(spec, "head_size_v", None)
        if hv not in (None, spec.head_size) or spec.sliding_window is not None:
            raise RuntimeError("mem tier: K-only spec needs symmetric K/V heads "
                               "and full attention")
        return dataclasses.replace(spec, head_size_v=0)

    get_kv_cache_spec._amass_k_only = True
    attn_cls.get_kv_cache_spec = get_kv_cache_spec


__all__ = ["MemSession", "patch_kv_cache_spec_k_only"]
