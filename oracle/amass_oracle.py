"""CPU oracle for the AMASS decode-time sparse paged-attention hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker the parity tests, the
``__graft_entry__.smoke()`` check and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` compare against.  The shipped product path
(``amass_kv_b200``) never imports it and has no CPU fallback.

Every function is a numpy restatement of the reference algorithm (Python +
Triton in Js-Hwang1/amass-kv, ``src/amass/...``); each docstring cites the
file:line it follows.  Pinning: ``tests/test_oracle_golden.py`` checks these
functions against golden vectors produced by the reference's own Triton kernels
(run under ``TRITON_INTERPRET=1`` on CPU by ``tests/golden/make_golden.py``).

Conventions (identical to the reference's tensors):
  q           (T, H, d)           bf16 values held as float32
  block_table (n_req, max_blocks) int32
  quad_mu     (NB, n_kv, d) int8          mu_scale (NB, n_kv) fp16
  quad_V      (NB, n_kv, d, rv) int8      V_scale  (NB, n_kv, r)  fp16
              rv = r (int8 codes) or r//2 (two signed nibbles per byte:
              low nibble = even column, high nibble = odd column)
  quad_sig2   (NB, n_kv, r) fp16
  K, V        (NB, page, n_kv, d)  bf16 values held as float32
  score       (R, n_kv, MP) fp32; page_table (R, n_kv, MP) int32 (-1 pad)
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------- #
# small helpers                                                               #
# --------------------------------------------------------------------------- #
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bf16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    u = ((u + 0x7FFF + lsb) >> 16) << 16
    out = u.astype(np.uint32).view(F32)
    return np.where(np.isnan(x), x, out).astype(F32)


def unpack_codes(codes: np.ndarray, r: int, bits: int) -> np.ndarray:
    """int8 codes (..., rv) -> signed integer codes (..., r) as float32.

    int4 packing follows ``selection/build.py:304-312`` (low nibble = column
    2j, high nibble = column 2j+1) as read back by
    ``selection/quad_score.py:75-83``."""
    c = codes.astype(np.int32)
    if bits == 8:
        return c[..., :r].astype(F32)
    lo = c & 0xF
    hi = (c >> 4) & 0xF
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty(c.shape[:-1] + (c.shape[-1] * 2,), dtype=np.int32)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out[..., :r].astype(F32)


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """Signed int codes in [-8, 7] (..., r) -> packed int8 (..., r//2)."""
    c = codes.astype(np.int32) & 0xF
    packed = c[..., 0::2] | (c[..., 1::2] << 4)
    return packed.astype(np.uint8).view(np.int8)


# --------------------------------------------------------------------------- #
# a2: derive_page_params  (selection/select.py:30-45)                         #
# --------------------------------------------------------------------------- #
def derive_page_params(seq_lens, budget: float, page: int, window: int,
                       sink: int):
    """npg = ceil(sl/page); n_sel_hi = npg - window;
    b = clamp(ceil(fp64(n_sel_hi - sink) * budget), 1, max(n_sel, 1))
    (``selection/select.py:30-45``)."""
    sl = np.asarray(seq_lens, dtype=np.int64)
    npg = (sl + page - 1) // page
    nsh = npg - window
    s = nsh - sink
    bf = np.ceil(s.astype(np.float64) * np.float64(budget)).astype(np.int64)
    b = np.minimum(np.maximum(bf, 1), np.maximum(s, 1))
    return npg.astype(np.int32), nsh.astype(np.int32), b.astype(np.int32)


# --------------------------------------------------------------------------- #
# a3: quad page score  (selection/quad_score.py:35-107)                       #
# --------------------------------------------------------------------------- #
def quad_score_h(q, mu, mu_s, V, V_s, sig2, block_table, n_sel_hi, *,
                 scale: float, page: int, G: int, r: int, v_bits: int,
                 MP: int):
    """Per-head quad score S[g] for every scored page p < n_sel_hi.

        q~   = V^T q_g                    V = V_code * V_scale (per column)
        quad = (s^2 / 2P) * sum_k sig2_k q~_k^2
        S_g  = s * mu.q_g + quad          mu = mu_code * mu_scale

    (``selection/quad_score.py:55-107``).  Returns (R, n_kv, G, MP) float32,
    NaN where no score is written (p >= n_sel_hi)."""
    n_req = block_table.shape[0]
    n_kv = mu.shape[1]
    d = mu.shape[2]
    out = np.full((n_req, n_kv, G, MP), np.nan, dtype=F32)
    coef = F32(F32(scale) * F32(scale) * F32(1.0 / (2.0 * page)))
    for rq in range(n_req):
        nsh = int(n_sel_hi[rq])
        if nsh <= 0:
            continue
        blks = block_table[rq, :nsh].astype(np.int64)
        qg = q[rq].reshape(n_kv, G, d).astype(F32)                    # (kv,G,d)
        mu_f = mu[blks].astype(F32) * mu_s[blks].astype(F32)[..., None]
        Vc = unpack_codes(V[blks], r, v_bits)                          # (P,kv,d,r)
        Vf = Vc * V_s[blks].astype(F32)[:, :, None, :]
        s2 = sig2[blks].astype(F32)                                    # (P,kv,r)
        qt = np.einsum("kgd,pkdr->pkgr", qg, Vf, dtype=F32)            # (P,kv,G,r)
        quad = np.sum(s2[:, :, None, :] * qt * qt, axis=-1, dtype=F32) * coef
        qmu = np.einsum("kgd,pkd->pkg", qg, mu_f, dtype=F32) * F32(scale)
        S = (qmu + quad).astype(F32)                                   # (P,kv,G)
        out[rq, :, :, :nsh] = S.transpose(1, 2, 0)
    return out


def combine_max(score_h, n_sel_hi):
    """kv-union group max: score = max_g S[g] (``quad_score.py:104-105``)."""
    return np.max(score_h, axis=2)


def combine_nrm(score_h, n_sel_hi):
    """nrm combine: hmax_g = max_{p<n_sel_hi} S_g[p];
    score[p] = sum_g exp(S_g[p] - hmax_g)
    (``selection/quad_score.py:276-315``)."""
    R, n_kv, G, MP = score_h.shape
    out = np.full((R, n_kv, MP), np.nan, dtype=F32)
    for rq in range(R):
        nsh = int(n_sel_hi[rq])
        if nsh <= 0:
            continue
        S = score_h[rq, :, :, :nsh]
        hm = S.max(axis=-1, keepdims=True)
        out[rq, :, :nsh] = np.sum(np.exp(S - hm), axis=1, dtype=F32)
    return out


# --------------------------------------------------------------------------- #
# a5: top-b threshold select  (selection/select.py:60-101)                    #
# --------------------------------------------------------------------------- #
def _threshold_keep(sc, n_pages, n_sel_hi, sink, b):
    """keep mask over pages [0, n_pages) for one (req, kv) unit."""
    P = max(int(n_pages), 0)
    keep = np.zeros(P, dtype=bool)
    if P == 0:
        return keep
    nsh = int(n_sel_hi)
    keep_all = (nsh - sink) <= 1
    offs = np.arange(P)
    always = (offs < sink) | (offs >= nsh)
    if keep_all:
        return np.ones(P, dtype=bool)
    sel = sc[sink:nsh]
    srt = np.sort(sel)[::-1]
    tau = srt[int(b) - 1]
    selmask = (offs >= sink) & (offs < nsh)
    sc_full = np.full(P, -np.inf, dtype=F32)
    sc_full[:nsh] = sc[:nsh]
    keep = (selmask & (sc_full >= tau)) | always
    return keep


def topb_select(score, n_pages, n_sel_hi, b_fix, *, sink: int, MP: int):
    """tau = b-th largest score over the selectable region [sink, n_sel_hi);
    keep = (selectable & score >= tau) | p < sink | p >= n_sel_hi | n_sel <= 1;
    ascending compaction, -1 pad to MP (``selection/select.py:60-101``)."""
    R, n_kv = score.shape[0], score.shape[1]
    tab = np.full((R, n_kv, MP), -1, dtype=np.int32)
    cnt = np.zeros((R, n_kv), dtype=np.int32)
    for rq in range(R):
        for kh in range(n_kv):
            keep = _threshold_keep(score[rq, kh], n_pages[rq], n_sel_hi[rq],
                                   sink, b_fix[rq])
            idx = np.nonzero(keep)[0].astype(np.int32)
            tab[rq, kh, :idx.size] = idx
            cnt[rq, kh] = idx.size
    return tab, cnt


# --------------------------------------------------------------------------- #
# a6: per-(req, kv-head) coverage (nucleus) select                            #
#     semantic source: backend/_selection_bridge.py:95-99,117-133             #
# --------------------------------------------------------------------------- #
def page_mass(score_row, n_sel_hi, combine: str):
    """Non-negative page mass over the scored region [0, n_sel_hi):
    ``nrm`` scores are already mass sums (``quad_score.py:293-315``);
    ``max`` scores are log-masses, turned into exp(score - max)."""
    s = score_row[:n_sel_hi].astype(np.float64)
    if combine == "nrm":
        return s
    return np.exp(s - s.max())


def nucleus_b(mass, sink: int, n_sel_hi: int, coverage: float) -> int:
    """Smallest b such that the top-b selectable pages (descending mass) hold
    ``coverage`` of the scored mass minus the always-kept sink share; the
    per-unit form of ``_nucleus_b`` (``_selection_bridge.py:117-133``):
    need = max(coverage - always, 0), always = sink mass / total."""
    n_sel = n_sel_hi - sink
    total = mass.sum()
    always = mass[:sink].sum()
    need = max(coverage * total - always, 0.0)
    sp = np.sort(mass[sink:n_sel_hi])[::-1]
    csum = np.cumsum(sp)
    hit = np.nonzero(csum >= need)[0]
    b = int(hit[0]) + 1 if hit.size else n_sel
    return max(1, min(b, max(n_sel, 1)))


def coverage_select(score, n_pages, n_sel_hi, *, sink: int, MP: int,
                    coverage: float, combine: str):
    """Per-(req, kv-head) nucleus b_u, then the top-b threshold rule of
    ``select.py:76-101`` with b = b_u.  Returns (page_table, page_cnt, b_u)."""
    R, n_kv = score.shape[0], score.shape[1]
    tab = np.full((R, n_kv, MP), -1, dtype=np.int32)
    cnt = np.zeros((R, n_kv), dtype=np.int32)
    bu = np.zeros((R, n_kv), dtype=np.int32)
    for rq in range(R):
        nsh = int(n_sel_hi[rq])
        for kh in range(n_kv):
            if nsh - sink <= 1:
                b = 1
            else:
                m = page_mass(score[rq, kh], nsh, combine)
                b = nucleus_b(m, sink, nsh, coverage)
            bu[rq, kh] = b
            keep = _threshold_keep(score[rq, kh], n_pages[rq], nsh, sink, b)
            idx = np.nonzero(keep)[0].astype(np.int32)
            tab[rq, kh, :idx.size] = idx
            cnt[rq, kh] = idx.size
    return tab, cnt, bu


def selection_diff_ok(tab_a, cnt_a, tab_b, cnt_b, score, tau_tol=1e-3,
                      sink=1):
    """True when selection A differs from the reference selection B only on
    pages whose reference score lies within ``tau_tol`` (relative, floor 1) of
    B's threshold -- the smallest reference score B keeps in the selectable
    region (p >= sink, finite score): the tie band the parity contract
    allows."""
    R, n_kv = cnt_a.shape
    for rq in range(R):
        for kh in range(n_kv):
            a = set(tab_a[rq, kh, :cnt_a[rq, kh]].tolist())
            b = set(tab_b[rq, kh, :cnt_b[rq, kh]].tolist())
            diff = a ^ b
            if not diff:
                continue
            sc = score[rq, kh]
            vals = [sc[p] for p in b if p >= sink and np.isfinite(sc[p])]
            tau = min(vals) if vals else 0.0
            for p in diff:
                if not (abs(float(sc[p]) - float(tau))
                        <= tau_tol * max(1.0, abs(float(tau)))):
                    return False
    return True


def coverage_diff_ok(tab, cnt, score, n_pages, n_sel_hi, *, sink, coverage,
                     combine, rel_tol=1e-3):
    """Coverage-mode acceptance: for every unit the kept selectable pages form
    a threshold set (all pages scoring >= its smallest member) whose size k is
    a valid nucleus size up to the fp tie band -- the top-(k-1) mass is below
    need*(1+rel_tol) and the top-k mass reaches need*(1-rel_tol)."""
    R, n_kv = cnt.shape
    for rq in range(R):
        nsh = int(n_sel_hi[rq])
        npg = int(n_pages[rq])
        for kh in range(n_kv):
            kept = set(tab[rq, kh, :cnt[rq, kh]].tolist())
            if nsh - sink <= 1:
                if kept != set(range(max(npg, 0))):
                    return False
                continue
            always = set(range(sink)) | set(range(nsh, npg))
            if not always <= kept:
                return False
            sel = sorted(p for p in kept if sink <= p < nsh)
            sc = score[rq, kh]
            tau = min(sc[p] for p in sel)
            if set(sel) != {p for p in range(sink, nsh) if sc[p] >= tau}:
                return False
            m = page_mass(sc, nsh, combine)
            need = max(coverage * m.sum() - m[:sink].sum(), 0.0)
            srt = np.sort(m[sink:nsh])[::-1]
            csum = np.concatenate([[0.0], np.cumsum(srt)])
            k = len(sel)
            tol = rel_tol * max(need, 1e-30)
            if not (csum[k - 1] < need + tol or k == 1):
                return False
            if not (csum[k] >= need - tol or k == nsh - sink):
                return False
    return True


# --------------------------------------------------------------------------- #
# a7: sparse paged decode over the selected pages (+ LSE merge)               #
#     attention/decode.py:145-241, attention/merge.py:30-50                   #
# --------------------------------------------------------------------------- #
def sparse_decode(q, K, V, block_table, seq_lens, page_table, page_cnt, *,
                  scale: float, G: int):
    """Exact fp32 softmax attention of each query head over the tokens of its
    kv-head's selected pages (tokens >= seq_len masked).  Split-K + LSE merge
    (``decode.py:145-241`` + ``merge.py:30-50``) is an exact re-association
    of this; an empty selection writes 0 (``merge.py:47-48``).
    Returns (n_req, H, d) float32."""
    n_req = block_table.shape[0]
    _, page, n_kv, d = K.shape
    out = np.zeros((n_req, n_kv * G, d), dtype=F32)
    for rq in range(n_req):
        sl = int(seq_lens[rq])
        for kh in range(n_kv):
            c = int(page_cnt[rq, kh])
            if c <= 0:
                continue
            pts = page_table[rq, kh, :c].astype(np.int64)
            blks = block_table[rq, pts].astype(np.int64)
            k = K[blks, :, kh, :].reshape(-1, d).astype(F32)           # (c*P, d)
            v = V[blks, :, kh, :].reshape(-1, d).astype(F32)
            tok = (pts[:, None] * page + np.arange(page)[None, :]).reshape(-1)
            qg = q[rq, kh * G:(kh + 1) * G].astype(F32)                # (G, d)
            s = (qg @ k.T).astype(F32) * F32(scale)
            s[:, tok >= sl] = -np.inf
            m = s.max(axis=1, keepdims=True)
            p = np.exp(s - m)
            l = p.sum(axis=1, keepdims=True)
            out[rq, kh * G:(kh + 1) * G] = (p @ v) / l
    return out


def dense_page_mass(q, K, block_table, seq_lens, *, scale, G, page):
    """Exact per-(req, kv, g, page) log-sum-exp masses (the bridge's
    ``pmass``, ``_selection_bridge.py:79-82``); used by the synthetic-input
    generators to calibrate planted pages."""
    n_req = block_table.shape[0]
    _, P, n_kv, d = K.shape
    outs = []
    for rq in range(n_req):
        sl = int(seq_lens[rq])
        npg = (sl + page - 1) // page
        blks = block_table[rq, :npg].astype(np.int64)
        k = K[blks].astype(F32)                                        # (npg,P,kv,d)
        qg = q[rq].reshape(n_kv, G, d).astype(F32)
        lg = np.einsum("kgd,ptkd->kgpt", qg, k, dtype=F32) * F32(scale)
        tok = np.arange(npg)[:, None] * page + np.arange(P)[None, :]
        lg = np.where(tok[None, None] < sl, lg, -np.inf)
        mx = lg.max(axis=-1, keepdims=True)
        outs.append((mx[..., 0] + np.log(np.exp(lg - mx).sum(-1))).astype(F32))
    return outs


# --------------------------------------------------------------------------- #
# a8: r8 low-rank page score  (selection/score.py:30-120)                     #
# --------------------------------------------------------------------------- #
def r8_score(q, mu, mu_s, Vk, Vk_s, c, c_s, block_table, seq_lens, n_sel_hi,
             *, scale: float, page: int, G: int, r: int, vk_bits: int,
             c_bits: int, MP: int, combine: str = "lse"):
    """S_g = s * mu.q_g + logsumexp_{t: tok < seq_len}(s * c_t . (Vk^T q_g));
    page score = max_g S_g (``selection/score.py:30-120``).

    ``combine="tokmax"`` replaces the log-sum-exp over tokens by a max (the
    variant the BASELINE C4 text describes; not the reference form)."""
    n_req = block_table.shape[0]
    n_kv, d = mu.shape[1], mu.shape[2]
    out = np.full((n_req, n_kv, MP), np.nan, dtype=F32)
    for rq in range(n_req):
        nsh = int(n_sel_hi[rq])
        if nsh <= 0:
            continue
        sl = int(seq_lens[rq])
        blks = block_table[rq, :nsh].astype(np.int64)
        qg = q[rq].reshape(n_kv, G, d).astype(F32)
        mu_f = mu[blks].astype(F32) * mu_s[blks].astype(F32)[..., None]
        Vf = unpack_codes(Vk[blks], r, vk_bits) * \
            Vk_s[blks].astype(F32)[:, :, None, :]                      # (P,kv,d,r)
        cc = unpack_codes(c[blks], r, c_bits) * \
            c_s[blks].astype(F32)[..., None]                           # (P,kv,t,r)
        qt = np.einsum("kgd,pkdr->pkgr", qg, Vf, dtype=F32)
        tok = np.einsum("pkgr,pktr->pkgt", qt, cc, dtype=F32) * F32(scale)
        tpos = np.arange(nsh)[:, None] * page + np.arange(page)[None, :]
        tok = np.where((tpos < sl)[:, None, None, :], tok, -np.inf)
        m = tok.max(axis=-1)
        if combine == "tokmax":
            agg = m
        else:
            agg = m + np.log(np.exp(tok - m[..., None]).sum(-1))
        qmu = np.einsum("kgd,pkd->pkg", qg, mu_f, dtype=F32) * F32(scale)
        S = qmu + agg
        out[rq, :, :nsh] = S.max(axis=-1).T
    return out


# --------------------------------------------------------------------------- #
# page summary build (selection/build.py:297-452, quad_build.py:37-84)        #
# --------------------------------------------------------------------------- #
def _quant_np(x, axis, bits):
    """code = round_half_even(x / s), s = max(amax(|x|)/lvl, 1e-8) in fp32
    (``build.py:297-302``)."""
    lvl = F32((1 << (bits - 1)) - 1)
    s = np.maximum(np.abs(x).max(axis=axis, keepdims=True) / lvl, F32(1e-8))
    s = s.astype(F32)
    code = np.clip(np.rint(x / s), -lvl, lvl).astype(np.int8)
    return code, s


def page_summary(Kp, r: int, *, v_bits: int = 8, v_grain: str = "col",
                 coords: str = "none", c_bits: int = 8,
                 c_grain: str = "token", tagw: int = 8):
    """Summary of finalized pages Kp (N, page, n_kv, d) (float32 holding
    bf16 values), per (page, kv-head) (``build.py:396-452`` _page_eigh +
    ``quad_build.py:56-84`` _quad_write):

        mu = mean_t K;  dc = K - mu;  Gm = dc dc^T (page x page);  eigh(Gm)
        S2r = top-r eigenvalues (ascending order, clamped >= 1e-10)
        U8 = their eigenvectors;  Vk = dc^T U8 / sqrt(S2r)        (d, r)
        c = U8 * sqrt(S2r)  (page, r);  resid = trace - sum S2r  (CLSE)

    Eigenvectors are unique up to sign; this restatement uses numpy's fp64
    eigh, so compare sign-invariant quantities.  Returns a dict of quantised
    slabs (reference layouts) and the fp32 factors."""
    N, page, n_kv, d = Kp.shape
    K = Kp.transpose(0, 2, 1, 3).astype(F32)                   # (N,kv,t,d)
    mu = K.mean(axis=2)
    dc = K - mu[:, :, None, :]
    Gm = np.einsum("nktd,nksd->nkts", dc.astype(np.float64),
                   dc.astype(np.float64))
    S2, U = np.linalg.eigh(Gm)                                 # ascending
    S2r = np.maximum(S2[..., -r:], 1e-10).astype(F32)
    U8 = U[..., -r:].astype(F32)
    S8 = np.sqrt(S2r)
    Vk = np.einsum("nktd,nktr->nkdr", dc, U8) / S8[:, :, None, :]
    out = {}
    out["mu_code"], s = _quant_np(mu, -1, 8)
    out["mu_s"] = s[..., 0].astype(np.float16)
    if v_grain == "col":
        vc, vs = _quant_np(Vk, -2, v_bits)
        vs = vs[:, :, 0, :]
    else:
        vc, vs = _quant_np(Vk, (-2, -1), v_bits)
        vs = np.broadcast_to(vs[:, :, 0, :], Vk.shape[:2] + (r,))
    out["V_code"] = pack_int4(vc) if v_bits == 4 else vc
    out["V_s"] = vs.astype(np.float16)
    out["sig2"] = S2r.astype(np.float16)
    out["tag"] = Kp[:, page - 1, :, :tagw]
    out["factors"] = dict(mu=mu, S2r=S2r, Vk=Vk, U8=U8)
    if coords != "none":
        c = U8 * S8[:, :, None, :]                             # (N,kv,t,r)
        if c_grain == "token":
            cc, cs = _quant_np(c, -1, c_bits)
            cs = cs[..., 0]                                    # (N,kv,t)
        else:
            cc, cs = _quant_np(c, (-2, -1), c_bits)
            cs = cs[..., 0, 0]                                 # (N,kv)
        out["c_code"] = pack_int4(cc) if c_bits == 4 else cc
        out["c_s"] = cs.astype(np.float16)
        trace = (K * K).sum(axis=(2, 3)) - page * (mu * mu).sum(-1)
        out["resid"] = np.maximum(trace - S2r.sum(-1), 0).astype(np.float16)
    return out


# --------------------------------------------------------------------------- #
# CLSE page score (selection/quad_score.py:156-273)                           #
# --------------------------------------------------------------------------- #
def clse_score_h(q, mu, mu_s, V, V_s, c, c_s, resid, block_table, seq_lens,
                 n_sel_hi, *, scale: float, page: int, G: int, r: int,
                 v_bits: int, c_bits: int, token_grain: bool, MP: int):
    """Per-head CLSE score S[g] for every scored page p < n_sel_hi:

        q~    = V^T q_g                       V = V_code * V_scale (per column)
        tok_t = s * c_t . q~                   c = c_code * c_scale (token or page)
        iso   = max(|q_g|^2 - |q~|^2, 0) * resid * s^2 / (2 P (d - r))
        S_g   = s * mu.q_g + logsumexp_{t: tok < seq_len} tok_t + iso

    (``selection/quad_score.py:156-273``).  Returns (R, n_kv, G, MP) float32,
    NaN where no score is written."""
    n_req = block_table.shape[0]
    n_kv, d = mu.shape[1], mu.shape[2]
    out = np.full((n_req, n_kv, G, MP), np.nan, dtype=F32)
    iso_coef = F32(scale * scale / (2.0 * page * max(d - r, 1)))
    for rq in range(n_req):
        nsh = int(n_sel_hi[rq])
        if nsh <= 0:
            continue
        sl = int(seq_lens[rq])
        blks = block_table[rq, :nsh].astype(np.int64)
        qg = q[rq].reshape(n_kv, G, d).astype(F32)
        qsq = np.sum(qg * qg, axis=-1, dtype=F32)                      # (kv,G)
        mu_f = mu[blks].astype(F32) * mu_s[blks].astype(F32)[..., None]
        Vf = unpack_codes(V[blks], r, v_bits) * \
            V_s[blks].astype(F32)[:, :, None, :]                       # (P,kv,d,r)
        cs = c_s[blks].astype(F32)
        if not token_grain:
            cs = np.broadcast_to(cs[..., None], cs.shape + (page,))
        cc = unpack_codes(c[blks], r, c_bits) * cs[..., None]           # (P,kv,t,r)
        qt = np.einsum("kgd,pkdr->pkgr", qg, Vf, dtype=F32)
        tok = np.einsum("pkgr,pktr->pkgt", qt, cc, dtype=F32) * F32(scale)
        tpos = np.arange(nsh)[:, None] * page + np.arange(page)[None, :]
        tok = np.where((tpos < sl)[:, None, None, :], tok, -np.inf)
        m = tok.max(axis=-1)
        lse = m + np.log(np.exp(tok - m[..., None]).sum(-1))
        qhsq = np.sum(qt * qt, axis=-1, dtype=F32)
        iso = np.maximum(qsq[None] - qhsq, 0) * \
            resid[blks].astype(F32)[:, :, None] * iso_coef
        qmu = np.einsum("kgd,pkd->pkg", qg, mu_f, dtype=F32) * F32(scale)
        S = (qmu + lse + iso).astype(F32)                               # (P,kv,G)
        out[rq, :, :, :nsh] = S.transpose(1, 2, 0)
    return out


# --------------------------------------------------------------------------- #
# a10/a11: exact-LRU residency plan + miss fetch                              #
#          tier/residency.py:45-139 (plan), :196-248 (fetch)                  #
# --------------------------------------------------------------------------- #
I32_MAX = 2147483647


def residency_step(page_table, page_cnt, block_table, seq_lens, *, page: int,
                   page2slot, slot2page, lru, clock: int):
    """One ``gather_plan`` call for one layer: the clock is advanced by the
    caller; hits touch lru=clock; misses of complete pages (in request, then
    page-table order) take the exact-LRU victim (min lru among slots with
    lru < clock, lowest index on ties), evicting its old page; a page already
    installed this step is deduplicated (``residency.py:45-139``).
    Mutates page2slot (n_kv, NB), slot2page (n_kv, S), lru (n_kv, S) in place
    and returns (fetch list [(kv, blk, slot)], overflow flag)."""
    n_req, n_kv = page_cnt.shape
    misses = [[[] for _ in range(n_kv)] for _ in range(n_req)]
    for rq in range(n_req):
        sl = int(seq_lens[rq])
        for kv in range(n_kv):
            for j in range(int(page_cnt[rq, kv])):
                pt = int(page_table[rq, kv, j])
                blk = int(block_table[rq, pt])
                complete = (pt + 1) * page <= sl
                if not complete:
                    continue
                slot = int(page2slot[kv, blk])
                if slot >= 0:
                    lru[kv, slot] = clock
                else:
                    misses[rq][kv].append(blk)
    flist = []
    ovf = False
    for kv in range(n_kv):
        for rq in range(n_req):
            for blk in misses[rq][kv]:
                if page2slot[kv, blk] >= 0:
                    continue
                ck = np.where(lru[kv] >= clock, I32_MAX, lru[kv])
                s = int(np.argmin(ck))
                if ck[s] == I32_MAX:
                    ovf = True
                    continue
                old = int(slot2page[kv, s])
                if old >= 0:
                    page2slot[kv, old] = -1
                page2slot[kv, blk] = s
                slot2page[kv, s] = blk
                lru[kv, s] = clock
                flist.append((kv, blk, s))
    return flist, ovf


def residency_fetch(flist, *, hot, pool, pool_valid, vbo, v_pool, layer: int):
    """Copy each installed miss page into its hot slot: from the pinned pool
    when ``pool_valid``; else from the staging pool via ``vbo`` with
    write-through to the pinned pool (and ``pool_valid`` set); else from the
    pinned pool (``residency.py:196-248``).  Bit copies.
    hot (n_kv, S, page, d); pool (L, NB, n_kv, page, d);
    pool_valid (n_kv, NB); v_pool (NV, page, n_kv, d)."""
    for kv, blk, slot in flist:
        if pool_valid[kv, blk] > 0:
            hot[kv, slot] = pool[layer, blk, kv]
        elif vbo[blk] >= 0:
            tile = v_pool[vbo[blk], :, kv, :]
            hot[kv, slot] = tile
            pool[layer, blk, kv] = tile
            pool_valid[kv, blk] = 1
        else:
            hot[kv, slot] = pool[layer, blk, kv]


def dma_plan_runs(fetch_list, fetch_cnt, pool_valid, *, layer: int, NB: int,
                  page: int, d: int, pool_base: int, hot_base: int):
    """Copy-engine runs of a fetch list (``residency.py:438-492``): per
    kv-head, installs in list order; a flushed install starts a run that
    extends while the next install's block and slot are both one more and
    its page is flushed too; staged installs are skipped (has_staged).
    fetch_list (n_kv, S, 2) = (block, slot); pool_valid (n_kv, NB).
    Returns ([(dst, src, dpitch, spitch, width, height)], has_staged)."""
    n_kv, S, _ = fetch_list.shape
    pb = page * d * 2
    runs, staged = [], False
    for kv in range(n_kv):
        m = int(fetch_cnt[kv])
        i = 0
        while i < m:
            blk, slot = (int(x) for x in fetch_list[kv, i])
            if pool_valid[kv, blk] == 0:
                staged = True
                i += 1
                continue
            run = 1
            while (i + run < m and int(fetch_list[kv, i + run, 0]) == blk + run
                   and int(fetch_list[kv, i + run, 1]) == slot + run
                   and pool_valid[kv, blk + run] != 0):
                run += 1
            runs.append((hot_base + (kv * S + slot) * pb,
                         pool_base + ((layer * NB + blk) * n_kv + kv) * pb,
                         pb, n_kv * pb, pb, run))
            i += run
    return runs, staged


def delta_stale(tag, K, block_table, seq_lens, *, page: int, max_fin: int):
    """Content-tag staleness (``selection/build.py:532-545``): the blocks of
    finalized pages p < min(seq_len // page, max_fin), in (request, page)
    order, whose stored tag (L, NB, n_kv, tagw) differs -- as floats, NaN
    always -- from the first tagw channels of the page-final key in ANY
    layer.  K (L, NB, page, n_kv, d) float."""
    tagw = tag.shape[-1]
    out = []
    for r in range(len(seq_lens)):
        for p in range(min(int(seq_lens[r]) // page, max_fin)):
            blk = int(block_table[r, p])
            cur = K[:, blk, page - 1, :, :tagw]
            with np.errstate(invalid="ignore"):
                if (cur != tag[:, blk]).any():
                    out.append(blk)
    return out


def invalidate_written(block_table, seq_lens, query_start_loc, *, page: int,
                       page2slot, slot2page, pool_valid):
    """Drop residency and pool validity of every page a request (re)wrote
    this step -- its pages (sl - ql)//page .. (sl - 1)//page -- in all layers
    and kv-heads (``residency.py:251-282``).  page2slot/pool_valid
    (L, n_kv, NB), slot2page (L, n_kv, S), mutated in place."""
    L, n_kv, _ = page2slot.shape
    for r in range(len(seq_lens)):
        sl = int(seq_lens[r])
        if sl <= 0:
            continue
        ql = int(query_start_loc[r + 1]) - int(query_start_loc[r])
        for p in range(max((sl - ql) // page, 0), (sl - 1) // page + 1):
            blk = int(block_table[r, p])
            for l in range(L):
                for kv in range(n_kv):
                    pool_valid[l, kv, blk] = 0
                    s = int(page2slot[l, kv, blk])
                    if s >= 0:
                        page2slot[l, kv, blk] = -1
                        slot2page[l, kv, s] = -1


def staging_begin_step(st, block_table, seq_lens, query_start_loc, n_tokens,
                       *, page: int, pool, pool_valid):
    """One Staging.begin_step (``tier/staging.py:312-346``, kernels
    :80-232), sequential semantics.  ``st`` holds numpy arrays vbo, vfl,
    stack, top (int), flist, fcnt (int), ovf (int), vslot, v_pool (L, NV,
    page, n_kv, d) int16, MAXF; pool (L, NB, n_kv, page, d) int16 and
    pool_valid (L, n_kv, NB) are updated in place."""
    n_req = len(seq_lens)
    sl = [int(x) for x in seq_lens]
    ql = [int(query_start_loc[r + 1] - query_start_loc[r]) for r in range(n_req)]
    st["vslot"][:n_tokens] = -1
    for r in range(n_req):                                   # vflush_clear
        if sl[r] > 0 and ql[r] > 0:
            for p in range((sl[r] - ql[r]) // page, (sl[r] - 1) // page + 1):
                st["vfl"][block_table[r, p]] = 0
    st["fcnt"] = 0                                           # collect
    for r in range(n_req):
        if sl[r] <= 0 or ql[r] <= 0:
            continue
        for p in range((sl[r] - ql[r]) // page):
            blk = int(block_table[r, p])
            vb = int(st["vbo"][blk])
            if vb < 0:
                continue
            over = False
            if st["vfl"][blk] == 0:
                st["vfl"][blk] = 1
                if st["fcnt"] < st["MAXF"]:
                    st["flist"][st["fcnt"]] = (blk, vb)
                    st["fcnt"] += 1
                else:
                    st["vfl"][blk] = 0
                    over = True
            if not over:
                old = int(st["vbo"][blk])
                st["vbo"][blk] = -1
                if old >= 0:
                    st["stack"][st["top"]] = old
                    st["top"] += 1
    L = pool.shape[0]                                        # flush copy
    for i in range(st["fcnt"]):
        blk, vb = (int(x) for x in st["flist"][i])
        for l in range(L):
            pool[l, blk] = st["v_pool"][l, vb].transpose(1, 0, 2)
            pool_valid[l, :, blk] = 1
    for r in range(n_req):                                   # valloc
        if sl[r] <= 0 or ql[r] <= 0:
            continue
        for p in range((sl[r] - ql[r]) // page, (sl[r] - 1) // page + 1):
            blk = int(block_table[r, p])
            if st["vbo"][blk] >= 0:
                continue
            if st["top"] <= 0:
                st["ovf"] = 1
                continue
            st["top"] -= 1
            st["vbo"][blk] = st["stack"][st["top"]]
    q0 = 0                                                   # vslot
    for r in range(n_req):
        if sl[r] > 0 and ql[r] > 0:
            for i in range(ql[r]):
                pos = sl[r] - ql[r] + i
                vb = int(st["vbo"][block_table[r, pos // page]])
                st["vslot"][q0 + i] = vb * page + pos % page if vb >= 0 else -1
        q0 += max(ql[r], 0)


def staging_scatter(st, layer: int, values, n_tokens: int, *, page: int):
    """Staging.scatter_kv (``tier/staging.py:51-77``): values (n_tokens,
    n_kv, d) int16 into v_pool[layer] at vslot."""
    for t in range(n_tokens):
        vs = int(st["vslot"][t])
        if vs >= 0:
            st["v_pool"][layer, vs // page, vs % page] = values[t]


def tier_decode(q, K, block_table, seq_lens, page_table, page_cnt, *, scale,
                G, hot, page2slot, vbo, v_pool, pool, layer: int):
    """mem-v ptr-select decode (``tier/decode_mem.py:78-166``): each selected
    page's V comes from the hot buffer when complete and resident, else the
    staging pool when ``vbo >= 0``, else the pinned pool; K is resident."""
    n_req = block_table.shape[0]
    NBk, page, n_kv, d = K.shape
    Vsel = np.zeros_like(K)
    for rq in range(n_req):
        sl = int(seq_lens[rq])
        for kv in range(n_kv):
            for j in range(int(page_cnt[rq, kv])):
                pt = int(page_table[rq, kv, j])
                blk = int(block_table[rq, pt])
                complete = (pt + 1) * page <= sl
                slot = int(page2slot[kv, blk])
                if complete and slot >= 0:
                    Vsel[blk, :, kv] = hot[kv, slot]
                elif vbo[blk] >= 0:
                    Vsel[blk, :, kv] = v_pool[vbo[blk], :, kv]
                else:
                    Vsel[blk, :, kv] = pool[layer, blk, kv]
    return sparse_decode(q, K, Vsel, block_table, seq_lens, page_table,
                         page_cnt, scale=scale, G=G)


# --------------------------------------------------------------------------- #
# whole hot path for one layer                                                #
# --------------------------------------------------------------------------- #
def quad_layer_step(q, mu, mu_s, V, V_s, sig2, K, Vv, block_table, seq_lens, *,
                    scale, page, G, r, v_bits, MP, sink, window, combine,
                    budget=None, coverage=None):
    """derive -> quad score (+combine) -> select -> decode, one layer."""
    npg, nsh, b = derive_page_params(seq_lens, budget if budget else 0.1,
                                     page, window, sink)
    sh = quad_score_h(q, mu, mu_s, V, V_s, sig2, block_table, nsh,
                      scale=scale, page=page, G=G, r=r, v_bits=v_bits, MP=MP)
    score = combine_nrm(sh, nsh) if combine == "nrm" else combine_max(sh, nsh)
    if budget is not None:
        tab, cnt = topb_select(score, npg, nsh, b, sink=sink, MP=MP)
    else:
        tab, cnt, _ = coverage_select(score, npg, nsh, sink=sink, MP=MP,
                                      coverage=coverage, combine=combine)
    out = sparse_decode(q, K, Vv, block_table, seq_lens, tab, cnt,
                        scale=scale, G=G)
    return dict(n_pages=npg, n_sel_hi=nsh, b_fix=b, score_h=sh, score=score,
                page_table=tab, page_cnt=cnt, out=out)


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


__all__ = [n for n in dir() if not n.startswith("_") and n not in
           ("annotations", "math", "np")]
