"""Stage A (page scoring + selection) -- host side of the sm_100a kernels.

Mirrors the reference's ``amass.selection`` surface for the hot path:

  QuadState                     selection/quad_state.py:36-151 (same tensors)
  derive_page_params(st, ...)   selection/select.py:48-56
  quad_score_cuda(st, ...)      selection/quad_score_cuda.py:1724-1794
  topb_select_cuda(st, n_req)   selection/select_cuda.py:370-391
  select_pages_quad(st, ...)    selection/quad_score.py:142-153

Every function launches through ``libamass_b200.so`` on the current torch
stream, allocates nothing and never synchronises (CUDA-graph capturable).
The state objects own all buffers; the reference's own ``QuadState`` works
here too since only attributes are read.

Per-(request, kv-head) coverage selection (the reference's AmassConfig
``coverage``, D1 of its graph-safe path) is available through
``select_pages_quad(..., coverage=c)`` or a state built with ``coverage=``.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr

TAGW = 8

COMBINE = {"max": 0, "nrm": 1}


class QuadState:
    """Persistent quad selection state (alloc-once, physical-block keyed,
    L-major), laid out exactly like the reference's QuadState:

      quad_mu    (L, NB, n_kv, d)      int8   mu_scale (L, NB, n_kv)     fp16
      quad_V     (L, NB, n_kv, d, rv)  int8   V_scale  (L, NB, n_kv, r)  fp16
      quad_sig2  (L, NB, n_kv, r)      fp16   quad_tag (L, NB, n_kv, 8)  bf16
      score (R, n_kv, MP) fp32, page_table (R, n_kv, MP) int32,
      page_cnt (R, n_kv) int32, n_pages / n_sel_hi / b_fix (R,) int32,
      budget64 (1,) fp64, score_h (R, n_kv, G, MP) + hmax (R, n_kv, G) (nrm).

    ``coverage`` (optional) switches selection to per-unit nucleus coverage;
    ``b_unit`` (R, n_kv) then records each unit's budget.
    """

    def __init__(self, device, *, num_layers, num_blocks, n_kv, G, head_dim,
                 page, max_reqs, max_pages, rank=2, budget=0.1,
                 sink_pages=1, window_pages=1, tagw=TAGW, v_grain="col",
                 v_bits=8, mu_bits=8, coords="none", c_bits=4,
                 c_grain="token", combine="max", coverage=None):
        if window_pages < 1:
            raise ValueError("window_pages >= 1 (the partial tail must be in "
                             "the always-attended window)")
        if v_bits not in (4, 8) or mu_bits != 8:
            raise ValueError("quad V codes are int4 or int8; mu stays int8")
        if v_bits == 4 and rank % 2:
            raise ValueError("int4 V packs two nibbles per byte: rank even")
        if combine not in COMBINE:
            raise ValueError(f"combine must be 'max' or 'nrm', got {combine!r}")
        if coords not in ("none", "lse"):
            raise ValueError(f"coords must be 'none' or 'lse', got {coords!r}")
        if coords == "lse" and c_bits == 4 and rank % 2:
            raise ValueError("int4 coords pack two nibbles per byte: rank even")
        if c_grain not in ("token", "page"):
            raise ValueError(f"c_grain must be 'token' or 'page', got {c_grain!r}")
        L, NB, D, r, MP, R = (num_layers, num_blocks, head_dim, rank,
                              max_pages, max_reqs)
        self.L, self.NB, self.n_kv, self.G, self.d = L, NB, n_kv, G, D
        self.D = D
        self.page, self.r, self.tagw = page, r, tagw
        self.max_reqs, self.max_pages = R, MP
        self.budget = float(budget)
        self.coverage = None if coverage is None else float(coverage)
        self.sink_pages, self.window_pages = int(sink_pages), int(window_pages)
        self.v_grain, self.v_bits, self.mu_bits = v_grain, int(v_bits), 8
        self.coords, self.combine = coords, combine
        self.device = device
        rv = r // 2 if v_bits == 4 else r
        kw = dict(device=device)
        self.quad_mu = torch.zeros(L, NB, n_kv, D, dtype=torch.int8, **kw)
        self.mu_scale = torch.zeros(L, NB, n_kv, dtype=torch.float16, **kw)
        self.quad_V = torch.zeros(L, NB, n_kv, D, rv, dtype=torch.int8, **kw)
        self.V_scale = torch.zeros(L, NB, n_kv, r, dtype=torch.float16, **kw)
        self.quad_sig2 = torch.zeros(L, NB, n_kv, r, dtype=torch.float16, **kw)
        self.quad_tag = torch.full((L, NB, n_kv, tagw), float("nan"),
                                   dtype=torch.bfloat16, **kw)
        self.c_bits, self.c_grain = int(c_bits), c_grain
        if coords == "lse":
            # CLSE: per-key rank-r' coordinates, their scales (per token or
            # per page) and the out-of-subspace scatter energy
            rc = r // 2 if self.c_bits == 4 else r
            self.quad_c = torch.zeros(L, NB, n_kv, page, rc, dtype=torch.int8,
                                      **kw)
            cs_shape = (L, NB, n_kv, page) if c_grain == "token" else \
                (L, NB, n_kv)
            self.c_scale = torch.zeros(cs_shape, dtype=torch.float16, **kw)
            self.quad_resid = torch.zeros(L, NB, n_kv, dtype=torch.float16,
                                          **kw)
            self.qsq = torch.zeros(R, n_kv * G, dtype=torch.float32, **kw)
        else:
            self.quad_c = self.c_scale = self.quad_resid = self.qsq = None
        self.score = torch.empty(R, n_kv, MP, dtype=torch.float32, **kw)
        self.page_table = torch.empty(R, n_kv, MP, dtype=torch.int32, **kw)
        self.page_cnt = torch.zeros(R, n_kv, dtype=torch.int32, **kw)
        if combine == "nrm":
            # rows padded to a multiple of 4 pages: 16-byte loads in the fold
            self.score_h = torch.empty(R, n_kv, G, (MP + 3) // 4 * 4,
                                       dtype=torch.float32, **kw)[..., :MP]
            # -inf: the scorer max-accumulates into it, the fold resets it
            self.hmax = torch.full((R, n_kv, G), float("-inf"),
                                   dtype=torch.float32, **kw)
        else:
            self.score_h = self.hmax = None
        self.b_unit = torch.zeros(R, n_kv, dtype=torch.int32, **kw)
        # scratch: q as two exact int8 limbs per (request, head) + its scale
        self.q8 = torch.zeros(R, n_kv * G, 2, D, dtype=torch.int8, **kw)
        self.qs = torch.zeros(R, n_kv * G, dtype=torch.float32, **kw)
        self.n_pages = torch.zeros(R, dtype=torch.int32, **kw)
        self.n_sel_hi = torch.zeros(R, dtype=torch.int32, **kw)
        self.b_fix = torch.ones(R, dtype=torch.int32, **kw)
        self.budget64 = torch.tensor([self.budget], dtype=torch.float64, **kw)

    def bytes_per_layer(self) -> int:
        ts = (self.quad_mu, self.mu_scale, self.quad_V, self.V_scale,
              self.quad_sig2, self.quad_tag)
        return sum(t[0].numel() * t.element_size() for t in ts)

    def layer_state(self, layer: int):
        return (self.quad_mu[layer], self.mu_scale[layer], self.quad_V[layer],
                self.V_scale[layer], self.quad_sig2[layer],
                self.quad_tag[layer])


# --------------------------------------------------------------------------- #
def derive_page_params(st, seq_lens, n_req: int) -> None:
    """Refresh st.{n_pages, n_sel_hi, b_fix} for this step (one launch)."""
    if n_req > st.max_reqs:
        raise ValueError(f"n_req {n_req} > max_reqs {st.max_reqs}")
    _lib.call("amass_derive_page_params", ptr(seq_lens), ptr(st.budget64),
              ptr(st.n_pages), ptr(st.n_sel_hi), ptr(st.b_fix), int(n_req),
              int(st.page), int(st.window_pages), int(st.sink_pages),
              _lib.stream_of(seq_lens.device))


def _check_q(q, st):
    if q.dtype != torch.bfloat16 or q.stride(-1) != 1:
        raise ValueError("q must be bf16 with a contiguous head_dim")


def _rank_bits(st, V):
    r = int(getattr(st, "r", V.shape[-1]))
    v_bits = int(getattr(st, "v_bits", 8 if V.shape[-1] == r else 4))
    return r, v_bits


def _prepare(st, device, write_h):
    """One-time fix-ups for a state built elsewhere (e.g. the reference's own
    QuadState, which zero-fills hmax and has no q-limb scratch); runs outside
    any graph on first use."""
    if getattr(st, "_amass_ready", False):
        return
    if write_h and st.hmax is not None and not isinstance(st, QuadState):
        st.hmax.fill_(float("-inf"))
    if getattr(st, "q8", None) is None:
        H = st.n_kv * st.G
        st.q8 = torch.zeros(st.max_reqs, H, 2, st.d, dtype=torch.int8,
                            device=device)
        st.qs = torch.zeros(st.max_reqs, H, dtype=torch.float32,
                            device=device)
    st._amass_ready = True


def _score_launch(st, layer, q, block_table, n_req, scale, write_h,
                  seq_lens=None):
    """quad scorer launch; with ``seq_lens`` the step's page parameters
    (derive_page_params) are computed in the same launches."""
    _prepare(st, q.device, write_h)
    mu, mu_s, V, V_s, sig2 = (st.quad_mu[layer], st.mu_scale[layer],
                              st.quad_V[layer], st.V_scale[layer],
                              st.quad_sig2[layer])
    r, v_bits = _rank_bits(st, V)
    _check_q(q, st)
    if seq_lens is not None:
        if n_req > st.max_reqs:
            raise ValueError(f"n_req {n_req} > max_reqs {st.max_reqs}")
        _lib.call("amass_quad_score_derive", ptr(seq_lens), ptr(st.budget64),
                  ptr(st.n_pages), ptr(st.n_sel_hi), ptr(st.b_fix),
                  int(st.window_pages), int(st.sink_pages), ptr(q),
                  q.stride(0), q.stride(1), ptr(mu), ptr(mu_s), ptr(V),
                  ptr(V_s), ptr(sig2), ptr(block_table),
                  block_table.stride(0), ptr(st.score),
                  ptr(st.score_h) if write_h else 0,
                  st.score_h.stride(2) if write_h else 0,
                  ptr(st.hmax) if write_h else 0, ptr(st.q8), ptr(st.qs),
                  float(scale), int(n_req), int(st.n_kv), int(st.G),
                  int(st.d), int(st.page), r, v_bits, int(st.max_pages),
                  1 if write_h else 0, _lib.stream_of(q.device))
        return
    _lib.call("amass_quad_score", ptr(q), q.stride(0), q.stride(1), ptr(mu),
              ptr(mu_s), ptr(V), ptr(V_s), ptr(sig2), ptr(block_table),
              block_table.stride(0), ptr(st.n_sel_hi), ptr(st.score),
              ptr(st.score_h) if write_h else 0,
              st.score_h.stride(2) if write_h else 0,
              ptr(st.hmax) if write_h else 0, ptr(st.q8), ptr(st.qs),
              float(scale), int(n_req),
              int(st.n_kv), int(st.G), int(st.d), int(st.page), r, v_bits,
              int(st.max_pages), 1 if write_h else 0,
              _lib.stream_of(q.device))


def quad_score_cuda(st, layer: int, q, block_table, seq_lens, n_req: int,
                    scale: float) -> None:
    """Drop-in for the reference ``quad_score_cuda``: writes ``st.score`` over
    the scored region (and ``st.score_h`` + the nrm fold when
    ``st.combine == "nrm"``).  ``seq_lens`` is accepted for signature parity;
    finalized pages need no token mask."""
    nrm = getattr(st, "combine", "max") == "nrm"
    _score_launch(st, layer, q, block_table, n_req, scale, nrm)
    if nrm:
        _lib.call("amass_nrm_combine", ptr(st.score_h), st.score_h.stride(2),
                  ptr(st.n_sel_hi),
                  ptr(st.hmax), ptr(st.score), int(n_req), int(st.n_kv),
                  int(st.G), int(st.max_pages), _lib.stream_of(q.device))


quad_score = quad_score_cuda


def topb_select_cuda(st, n_req: int) -> None:
    """Drop-in for the reference ``topb_select_cuda``: static top-b from
    ``st.score`` and ``st.b_fix`` into ``st.page_table`` / ``st.page_cnt``."""
    _lib.call("amass_topb_select", ptr(st.score), ptr(st.n_pages),
              ptr(st.n_sel_hi), ptr(st.b_fix), ptr(st.page_table),
              ptr(st.page_cnt), int(n_req), int(st.n_kv),
              int(st.sink_pages), int(st.max_pages),
              _lib.stream_of(st.score.device))


topb_select = topb_select_cuda


def select_pages(st, n_req: int, *, coverage=None, from_score_h=None) -> None:
    """Fused Stage-A.2: nrm fold (when the state's combine is nrm and the
    per-head scores are pending) + top-b or per-unit coverage selection."""
    nrm = getattr(st, "combine", "max") == "nrm"
    if from_score_h is None:
        from_score_h = nrm
    cov = coverage if coverage is not None else getattr(st, "coverage", None)
    b_unit = getattr(st, "b_unit", None)
    _lib.call("amass_select_pages",
              ptr(st.score_h) if from_score_h else 0,
              st.score_h.stride(2) if from_score_h else 0,
              ptr(st.hmax) if from_score_h else 0, ptr(st.score),
              ptr(st.n_pages), ptr(st.n_sel_hi), ptr(st.b_fix),
              ptr(st.page_table), ptr(st.page_cnt), ptr(b_unit), int(n_req),
              int(st.n_kv), int(st.G), int(st.sink_pages),
              int(st.max_pages), COMBINE["nrm" if nrm else "max"],
              1 if cov is not None else 0,
              float(cov) if cov is not None else 0.0,
              _lib.stream_of(st.score.device))


def select_pages_quad(st, layer: int, q, block_table, seq_lens, n_req: int,
                      scale: float, *, derive: bool = True,
                      coverage=None) -> None:
    """One-call Stage A (quad): (derive) + score + fused fold/select.
    Writes st.page_table / st.page_cnt (and st.score)."""
    nrm = getattr(st, "combine", "max") == "nrm"
    _score_launch(st, layer, q, block_table, n_req, scale, nrm,
                  seq_lens=seq_lens if derive else None)
    select_pages(st, n_req, coverage=coverage, from_score_h=nrm)


# --------------------------------------------------------------------------- #
# CLSE scorer: quad geometry + per-key coordinates + residual energy          #
# --------------------------------------------------------------------------- #
def clse_score_cuda(st, layer: int, q, block_table, seq_lens, n_req: int,
                    scale: float) -> None:
    """Drop-in for the reference ``clse_score`` / ``clse_score_cuda``
    (``selection/quad_score.py:318-374``, ``quad_score_cuda.py:1797``):
    S_g = s*mu.q_g + logsumexp_t(s * c_t . V^T q_g) + iso_g per page; writes
    ``st.score`` (combine "max") or ``st.score_h`` + ``st.hmax`` for the nrm
    fold (combine "nrm"; ``select_pages`` folds)."""
    if getattr(st, "quad_c", None) is None:
        raise ValueError("CLSE needs a state built with coords='lse'")
    nrm = getattr(st, "combine", "max") == "nrm"
    _prepare(st, q.device, nrm)
    _check_q(q, st)
    if getattr(st, "qsq", None) is None:
        st.qsq = torch.zeros(st.max_reqs, st.n_kv * st.G, dtype=torch.float32,
                             device=q.device)
    mu, mu_s, V, V_s = (st.quad_mu[layer], st.mu_scale[layer],
                        st.quad_V[layer], st.V_scale[layer])
    c, c_s, res = st.quad_c[layer], st.c_scale[layer], st.quad_resid[layer]
    _lib.call("amass_clse_score", ptr(q), q.stride(0), q.stride(1), ptr(mu),
              ptr(mu_s), ptr(V), ptr(V_s), ptr(c), ptr(c_s),
              1 if getattr(st, "c_grain", "token") == "token" else 0,
              ptr(res), ptr(block_table), block_table.stride(0),
              ptr(seq_lens), ptr(st.n_sel_hi), ptr(st.score),
              ptr(st.score_h) if nrm else 0,
              st.score_h.stride(2) if nrm else 0,
              ptr(st.hmax) if nrm else 0, ptr(st.q8), ptr(st.qs), ptr(st.qsq),
              float(scale), int(n_req), int(st.n_kv), int(st.G), int(st.d),
              int(st.page), int(st.r), int(getattr(st, "v_bits", 8)),
              int(st.c_bits), int(st.max_pages), 1 if nrm else 0,
              _lib.stream_of(q.device))


clse_score = clse_score_cuda


def select_pages_clse(st, layer: int, q, block_table, seq_lens, n_req: int,
                      scale: float, *, derive: bool = True,
                      coverage=None) -> None:
    """One-call Stage A (CLSE): (derive) + score + fused fold/select
    (reference ``selection/quad_score.py`` select_pages_clse)."""
    if derive:
        derive_page_params(st, seq_lens, n_req)
    clse_score_cuda(st, layer, q, block_table, seq_lens, n_req, scale)
    nrm = getattr(st, "combine", "max") == "nrm"
    select_pages(st, n_req, coverage=coverage, from_score_h=nrm)


# --------------------------------------------------------------------------- #
# r8 low-rank scorer                                                          #
# --------------------------------------------------------------------------- #
class R8State:
    """Persistent r8 selection state, laid out like the reference's R8State
    (``selection/state.py:35-112``):

      r8_mu (L,NB,n_kv,d) int8 + mu_scale (L,NB,n_kv) fp16
      r8_Vk (L,NB,n_kv,d,rv) int8 + Vk_scale (L,NB,n_kv,r) fp16
      r8_c  (L,NB,n_kv,page,rc) int8 + c_scale (L,NB,n_kv,page) fp16
      score / page_table / page_cnt / n_pages / n_sel_hi / b_fix / budget64.
    """

    def __init__(self, device, *, num_layers, num_blocks, n_kv, G, head_dim,
                 page, max_reqs, max_pages, rank=8, budget=0.1, sink_pages=1,
                 window_pages=1, tagw=TAGW, vk_grain="col", c_grain="page",
                 vk_bits=8, c_bits=8, mu_bits=8, coverage=None):
        if window_pages < 1:
            raise ValueError("window_pages >= 1")
        if vk_bits not in (4, 8) or c_bits not in (4, 8) or mu_bits != 8:
            raise ValueError("Vk/c codes are int4 or int8; mu stays int8")
        L, NB, D, r, MP, R = (num_layers, num_blocks, head_dim, rank,
                              max_pages, max_reqs)
        self.L, self.NB, self.n_kv, self.G, self.d, self.D = L, NB, n_kv, G, D, D
        self.page, self.r, self.tagw = page, r, tagw
        self.max_reqs, self.max_pages = R, MP
        self.budget = float(budget)
        self.coverage = None if coverage is None else float(coverage)
        self.sink_pages, self.window_pages = int(sink_pages), int(window_pages)
        self.vk_grain, self.c_grain = vk_grain, c_grain
        self.vk_bits, self.c_bits, self.mu_bits = int(vk_bits), int(c_bits), 8
        self.combine = "max"
        self.device = device
        kw = dict(device=device)
        rvk = r // 2 if vk_bits == 4 else r
        rc = r // 2 if c_bits == 4 else r
        self.r8_mu = torch.zeros(L, NB, n_kv, D, dtype=torch.int8, **kw)
        self.mu_scale = torch.zeros(L, NB, n_kv, dtype=torch.float16, **kw)
        self.r8_Vk = torch.zeros(L, NB, n_kv, D, rvk, dtype=torch.int8, **kw)
        self.Vk_scale = torch.zeros(L, NB, n_kv, r, dtype=torch.float16, **kw)
        self.r8_c = torch.zeros(L, NB, n_kv, page, rc, dtype=torch.int8, **kw)
        self.c_scale = torch.zeros(L, NB, n_kv, page, dtype=torch.float16, **kw)
        self.r8_tag = torch.full((L, NB, n_kv, tagw), float("nan"),
                                 dtype=torch.bfloat16, **kw)
        self.score = torch.empty(R, n_kv, MP, dtype=torch.float32, **kw)
        self.page_table = torch.empty(R, n_kv, MP, dtype=torch.int32, **kw)
        self.page_cnt = torch.zeros(R, n_kv, dtype=torch.int32, **kw)
        self.score_h = self.hmax = None
        self.b_unit = torch.zeros(R, n_kv, dtype=torch.int32, **kw)
        self.q8 = torch.zeros(R, n_kv * G, 2, D, dtype=torch.int8, **kw)
        self.qs = torch.zeros(R, n_kv * G, dtype=torch.float32, **kw)
        self.n_pages = torch.zeros(R, dtype=torch.int32, **kw)
        self.n_sel_hi = torch.zeros(R, dtype=torch.int32, **kw)
        self.b_fix = torch.ones(R, dtype=torch.int32, **kw)
        self.budget64 = torch.tensor([self.budget], dtype=torch.float64, **kw)

    def layer_state(self, layer: int):
        return (self.r8_mu[layer], self.mu_scale[layer], self.r8_Vk[layer],
                self.Vk_scale[layer], self.r8_c[layer], self.c_scale[layer],
                self.r8_tag[layer])


R8_AGG = {"lse": 0, "tokmax": 1}


def r8_score_cuda(st, layer: int, q, block_table, seq_lens, n_req: int,
                  scale: float, *, token_agg: str = "lse") -> None:
    """Drop-in for the reference ``r8_score_cuda`` (``selection/score_cuda.py
    :888``): writes ``st.score`` over the scored region.  ``token_agg="tokmax"``
    replaces the per-page log-sum-exp over tokens by a max."""
    _prepare(st, q.device, False)
    _check_q(q, st)
    mu, mu_s, Vk, Vk_s, c, c_s = (st.r8_mu[layer], st.mu_scale[layer],
                                  st.r8_Vk[layer], st.Vk_scale[layer],
                                  st.r8_c[layer], st.c_scale[layer])
    _lib.call("amass_r8_score", ptr(q), q.stride(0), q.stride(1), ptr(mu),
              ptr(mu_s), ptr(Vk), ptr(Vk_s), ptr(c), ptr(c_s),
              ptr(block_table), block_table.stride(0), ptr(seq_lens),
              ptr(st.n_sel_hi), ptr(st.score), ptr(st.q8), ptr(st.qs),
              float(scale), int(n_req), int(st.n_kv), int(st.G), int(st.d),
              int(st.page), int(st.r), int(getattr(st, "vk_bits", 8)),
              int(getattr(st, "c_bits", 8)), int(st.max_pages),
              R8_AGG[token_agg], _lib.stream_of(q.device))


r8_score = r8_score_cuda


def select_pages_r8(st, layer: int, q, block_table, seq_lens, n_req: int,
                    scale: float, *, derive: bool = True, coverage=None,
                    token_agg: str = "lse") -> None:
    """One-call Stage A (r8): (derive) + r8 score + top-b / coverage select
    (reference ``selection/select.py:119-130``)."""
    if derive:
        derive_page_params(st, seq_lens, n_req)
    r8_score_cuda(st, layer, q, block_table, seq_lens, n_req, scale,
                  token_agg=token_agg)
    select_pages(st, n_req, coverage=coverage, from_score_h=False)
