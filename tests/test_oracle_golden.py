"""Pin the CPU oracle against golden vectors made by the reference's own
Triton kernels (``tests/golden/make_golden.py``)."""
import numpy as np
import pytest

from oracle import amass_oracle as O
from tests.conftest import bits_to_f32, load_golden

QUAD = ["quad_c1_nrm", "quad_c1_max", "quad_d128_i4_nrm", "quad_d128_i4_max",
        "quad_d128_i4_cov", "quad_g8_i8_cov_max"]


def _quad(z):
    G, r, vb, page, MP = [int(x) for x in z["meta"]]
    kv = bits_to_f32(z["kv"])
    return dict(G=G, r=r, v_bits=vb, page=page, MP=MP,
                scale=float(z["scale"][0]), q=bits_to_f32(z["q"]),
                K=kv[:, 0], V=kv[:, 1])


@pytest.mark.parametrize("name", QUAD)
def test_derive(name):
    z = load_golden(name)
    g = _quad(z)
    npg, nsh, b = O.derive_page_params(z["seq_lens"], float(z["budget"][0]),
                                       g["page"], 1, 1)
    assert np.array_equal(npg, z["n_pages"])
    assert np.array_equal(nsh, z["n_sel_hi"])
    assert np.array_equal(b, z["b_fix"])


@pytest.mark.parametrize("name", QUAD)
def test_quad_score(name):
    z = load_golden(name)
    g = _quad(z)
    sh = O.quad_score_h(g["q"], z["mu"], z["mu_s"], z["Vq"], z["V_s"],
                        z["sig2"], z["block_table"], z["n_sel_hi"],
                        scale=g["scale"], page=g["page"], G=g["G"], r=g["r"],
                        v_bits=g["v_bits"], MP=g["MP"])
    comb = str(z["combine"][0])
    sc = O.combine_nrm(sh, z["n_sel_hi"]) if comb == "nrm" else \
        O.combine_max(sh, z["n_sel_hi"])
    for rq, n in enumerate(z["n_sel_hi"]):
        if n <= 0:
            continue
        np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                   rtol=2e-5, atol=2e-5)
        if comb == "nrm":
            np.testing.assert_allclose(sh[rq, :, :, :n],
                                       z["score_h"][rq, :, :, :n],
                                       rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("name", QUAD)
def test_select(name):
    z = load_golden(name)
    g = _quad(z)
    sc = np.where(np.isnan(z["score"]), -np.inf, z["score"]).astype(np.float32)
    if "coverage" in z:
        tab, cnt, bu = O.coverage_select(
            sc, z["n_pages"], z["n_sel_hi"], sink=1, MP=g["MP"],
            coverage=float(z["coverage"][0]), combine=str(z["combine"][0]))
        assert np.array_equal(bu, z["b_u"])
    else:
        tab, cnt = O.topb_select(sc, z["n_pages"], z["n_sel_hi"], z["b_fix"],
                                 sink=1, MP=g["MP"])
    assert np.array_equal(cnt, z["page_cnt"])
    assert np.array_equal(tab, z["page_table"])


@pytest.mark.parametrize("name", QUAD)
def test_decode(name):
    z = load_golden(name)
    g = _quad(z)
    out = O.sparse_decode(g["q"], g["K"], g["V"], z["block_table"],
                          z["seq_lens"], z["page_table"], z["page_cnt"],
                          scale=g["scale"], G=g["G"])
    # reference: bf16 output, fp16 P  ->  bf16-level agreement
    np.testing.assert_allclose(out, z["out"], atol=2e-2, rtol=1e-2)
    assert np.abs(out - z["out"]).mean() < 2e-3


@pytest.mark.parametrize("name", ["r8_i8", "r8_i4"])
def test_r8(name):
    z = load_golden(name)
    G, r, vkb, cb, page, MP, n_kv, d = [int(x) for x in z["meta"]]
    q = bits_to_f32(z["q"])
    sc = O.r8_score(q, z["mu"], z["mu_s"], z["Vk"], z["Vk_s"], z["c"],
                    z["c_s"], z["block_table"], z["seq_lens"], z["n_sel_hi"],
                    scale=float(z["scale"][0]), page=page, G=G, r=r,
                    vk_bits=vkb, c_bits=cb, MP=MP)
    for rq, n in enumerate(z["n_sel_hi"]):
        np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                   rtol=1e-4, atol=1e-4)
    scm = np.where(np.isnan(z["score"]), -np.inf, z["score"]).astype(np.float32)
    tab, cnt = O.topb_select(scm, z["n_pages"], z["n_sel_hi"], z["b_fix"],
                             sink=1, MP=MP)
    assert np.array_equal(tab, z["page_table"])
    assert np.array_equal(cnt, z["page_cnt"])


@pytest.mark.parametrize("name", ["tier_lru", "tier_overflow"])
def test_tier(name):
    z = load_golden(name)
    g = _quad(z)
    kvb = z["kv"]
    NB, page, n_kv, d = g["K"].shape
    S = int(z["hot_slots"][0])
    p2s = np.full((n_kv, NB), -1, np.int32)
    s2p = np.full((n_kv, S), -1, np.int32)
    lru = np.zeros((n_kv, S), np.int32)
    hot = np.zeros((n_kv, S, page, d), np.int16)
    pool = z["pool_init"].copy()
    valid = z["pool_valid_init"].copy()
    v_pool = z["v_pool"][0]
    vbo = z["vbo"]
    clock = 1
    for s in range(int(z["steps"][0])):
        clock += 1
        fl, ovf = O.residency_step(z[f"page_table_{s}"], z[f"page_cnt_{s}"],
                                   z["block_table"], z["seq_lens"], page=page,
                                   page2slot=p2s, slot2page=s2p, lru=lru,
                                   clock=clock)
        O.residency_fetch(fl, hot=hot, pool=pool, pool_valid=valid, vbo=vbo,
                          v_pool=v_pool, layer=0)
        assert np.array_equal(p2s, z[f"page2slot_{s}"])
        assert np.array_equal(s2p, z[f"slot2page_{s}"])
        assert np.array_equal(lru, z[f"lru_{s}"])
        assert np.array_equal(valid, z[f"pool_valid_{s}"])
        assert len(fl) == int(z[f"fetch_cnt_{s}"][0])
        assert bool(ovf) == bool(z[f"overflow_{s}"][0])
        # hot bytes equal wherever a page is resident
        for kv in range(n_kv):
            for sl_ in range(S):
                if s2p[kv, sl_] >= 0:
                    assert np.array_equal(hot[kv, sl_],
                                          z[f"hot_{s}"][kv, sl_])
        q = bits_to_f32(z[f"q_{s}"])
        out = O.tier_decode(q, g["K"], z["block_table"], z["seq_lens"],
                            z[f"page_table_{s}"], z[f"page_cnt_{s}"],
                            scale=g["scale"], G=g["G"],
                            hot=bits_to_f32(hot), page2slot=p2s, vbo=vbo,
                            v_pool=bits_to_f32(v_pool),
                            pool=bits_to_f32(pool), layer=0)
        np.testing.assert_allclose(out, z[f"out_{s}"], atol=2e-2, rtol=1e-2)
        if name == "tier_lru":
            # the tier delivers the same V bytes as the resident cache
            assert np.array_equal(z[f"out_{s}"], z[f"out_resident_{s}"])
    assert np.array_equal(pool, z["pool_final"])


def test_bf16_round():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.3, 0.0], np.float32)
    y = O.bf16_round(x)
    assert y[0] == 1.0 and y[1] == 1.0 and y[2] == 1.0078125


def test_int4_roundtrip():
    c = np.arange(-8, 8, dtype=np.int32).reshape(2, 8)
    assert np.array_equal(O.unpack_codes(O.pack_int4(c), 8, 4), c)


@pytest.mark.parametrize("name", ["quad_d128_i4_cov", "quad_g8_i8_cov_max"])
def test_coverage_acceptance_accepts_golden(name):
    """The coverage acceptance rule used by the GPU tests accepts the
    reference-built coverage selection itself."""
    z = load_golden(name)
    sc = np.where(np.isnan(z["score"]), -np.inf, z["score"]).astype(np.float32)
    assert O.coverage_diff_ok(z["page_table"], z["page_cnt"], sc, z["n_pages"],
                              z["n_sel_hi"], sink=1,
                              coverage=float(z["coverage"][0]),
                              combine=str(z["combine"][0]))


def test_selection_tie_band():
    """A swap of two pages whose scores differ by < 1e-3 of the threshold is
    accepted; a swap across a real gap is rejected."""
    sc = np.array([[[9.0, 5.0, 3.0000, 3.0004, 1.0, np.nan]]], np.float32)
    ref = np.array([[[0, 1, 3, 5, -1, -1]]], np.int32)
    tie = np.array([[[0, 1, 2, 5, -1, -1]]], np.int32)
    gap = np.array([[[0, 1, 4, 5, -1, -1]]], np.int32)
    cnt = np.array([[4]], np.int32)
    assert O.selection_diff_ok(tie, cnt, ref, cnt, sc)
    assert not O.selection_diff_ok(gap, cnt, ref, cnt, sc)


def test_invalidate_written():
    z = load_golden("tier_invalidate")
    p2s = z["page2slot_init"].copy()
    s2p = z["slot2page_init"].copy()
    valid = z["pool_valid_init"].copy()
    O.invalidate_written(z["block_table"], z["seq_lens"],
                         z["query_start_loc"], page=int(z["page"][0]),
                         page2slot=p2s, slot2page=s2p, pool_valid=valid)
    assert np.array_equal(p2s, z["page2slot"])
    assert np.array_equal(s2p, z["slot2page"])
    assert np.array_equal(valid, z["pool_valid"])


CLSE = ["clse_i4_tok_nrm", "clse_i8_page_max", "clse_r4_i8_tok_max"]


def clse_h(z):
    g = _quad(z)
    c_bits, tok = [int(x) for x in z["cmeta"]]
    return O.clse_score_h(g["q"], z["mu"], z["mu_s"], z["Vq"], z["V_s"],
                          z["c"], z["c_s"], z["resid"], z["block_table"],
                          z["seq_lens"], z["n_sel_hi"], scale=g["scale"],
                          page=g["page"], G=g["G"], r=g["r"],
                          v_bits=g["v_bits"], c_bits=c_bits,
                          token_grain=bool(tok), MP=g["MP"])


@pytest.mark.parametrize("name", CLSE)
def test_clse_score(name):
    """The CLSE restatement against the reference's own clse_score
    (block-sweep kernel at r'=2, generic kernel at r'=4)."""
    z = load_golden(name)
    sh = clse_h(z)
    comb = str(z["combine"][0])
    nsh = z["n_sel_hi"]
    if comb == "nrm":
        for rq in range(sh.shape[0]):
            n = int(nsh[rq])
            np.testing.assert_allclose(sh[rq, :, :, :n],
                                       z["score_h"][rq, :, :, :n],
                                       rtol=2e-4, atol=2e-4)
        sc = O.combine_nrm(sh, nsh)
    else:
        sc = O.combine_max(sh, nsh)
    for rq in range(sh.shape[0]):
        n = int(nsh[rq])
        np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                   rtol=2e-4, atol=2e-4)
    # the reference's top-b of its own scores is the threshold rule
    MP = int(z["meta"][4])
    scm = np.where(np.isnan(z["score"]), -np.inf, z["score"]).astype(np.float32)
    tab, cnt = O.topb_select(scm, z["n_pages"], z["n_sel_hi"], z["b_fix"],
                             sink=1, MP=MP)
    assert np.array_equal(tab, z["page_table"])
    assert np.array_equal(cnt, z["page_cnt"])


def _tail_pages(z):
    L, NB, n_kv, d, r, vb, cb, ctok, lse = [int(x) for x in z["meta"]]
    sl = z["seq_lens"]
    fin1 = np.maximum(sl // 16 - 1, 0)
    blocks = z["block_table"][np.arange(len(sl)), fin1]
    return (L, NB, n_kv, d, r, vb, cb, ctok, lse), blocks


def _deq_cols(code, s, r, bits):
    """(..., d, rv) codes + (..., r) scales -> (..., d, r) float32"""
    return O.unpack_codes(code, r, bits) * s.astype(np.float32)[..., None, :]


def check_summary(z, got, l, blocks):
    """Sign-invariant comparison of one layer's built summaries (``got``:
    dict of the build's slabs for that layer) with the reference's."""
    (L, NB, n_kv, d, r, vb, cb, ctok, lse), _ = _tail_pages(z)
    for b in blocks:
        assert np.abs(got["mu"][b].astype(int) - z["mu"][l, b].astype(int)).max() <= 1
        np.testing.assert_allclose(got["mu_s"][b].astype(np.float32),
                                   z["mu_s"][l, b].astype(np.float32), rtol=2e-3)
        np.testing.assert_allclose(got["sig2"][b].astype(np.float32),
                                   z["sig2"][l, b].astype(np.float32),
                                   rtol=5e-3, atol=1e-2)
        vr = _deq_cols(z["V"][l, b], z["V_s"][l, b], r, vb)       # (kv,d,r)
        vg = _deq_cols(got["V"][b], got["V_s"][b], r, vb)
        sgn = np.sign((vr * vg).sum(axis=1, keepdims=True))
        lvl = 7.0 if vb == 4 else 127.0
        tol = 1.5 * z["V_s"][l, b].astype(np.float32).max() + 1e-3
        assert np.abs(vr - sgn * vg).max() <= tol, (l, b)
        assert np.array_equal(got["tag"][b], z["tag"][l, b])
        if lse:
            cr = O.unpack_codes(z["c"][l, b], r, cb).astype(np.float32)
            cg = O.unpack_codes(got["c"][b], r, cb).astype(np.float32)
            csr = z["c_s"][l, b].astype(np.float32)
            csg = got["c_s"][b].astype(np.float32)
            if not ctok:
                csr, csg = csr[..., None], csg[..., None]
            cr, cg = cr * csr[..., None], cg * csg[..., None]      # (kv,t,r)
            sgc = np.sign((cr * cg).sum(axis=1, keepdims=True))
            assert np.abs(cr - sgc * cg).max() <= 1.5 * csr.max() + 1e-3
            np.testing.assert_allclose(got["resid"][b].astype(np.float32),
                                       z["resid"][l, b].astype(np.float32),
                                       rtol=5e-3, atol=5e-2)


@pytest.mark.parametrize("name", ["build_quad_i4", "build_clse_i8"])
def test_page_summary_vs_reference_build(name):
    z = load_golden(name)
    meta, blocks = _tail_pages(z)
    L, NB, n_kv, d, r, vb, cb, ctok, lse = meta
    K = bits_to_f32(z["K"])                                       # (L,NB,t,kv,d)
    for l in range(L):
        s = O.page_summary(K[l][blocks], r, v_bits=vb,
                           coords="lse" if lse else "none", c_bits=cb,
                           c_grain="token" if ctok else "page")
        got = {"mu": {}, "mu_s": {}, "sig2": {}, "V": {}, "V_s": {},
               "tag": {}, "c": {}, "c_s": {}, "resid": {}}
        for i, b in enumerate(blocks):
            got["mu"][b] = s["mu_code"][i]
            got["mu_s"][b] = s["mu_s"][i]
            got["sig2"][b] = s["sig2"][i]
            got["V"][b] = s["V_code"][i]
            got["V_s"][b] = s["V_s"][i]
            got["tag"][b] = (s["tag"][i].view(np.uint32) >> 16).astype(np.uint16).view(np.int16)
            if lse:
                got["c"][b] = s["c_code"][i]
                got["c_s"][b] = s["c_s"][i]
                got["resid"][b] = s["resid"][i]
        check_summary(z, got, l, blocks)


def test_staging_lifecycle_vs_reference():
    z = load_golden("tier_staging")
    L, NB, n_kv, d, page, NV, MAXF, steps = [int(x) for x in z["meta"]]
    st = dict(vbo=np.full(NB, -1, np.int32), vfl=np.zeros(NB, np.int32),
              stack=np.arange(NV, dtype=np.int32), top=NV,
              flist=np.zeros((MAXF, 2), np.int32), fcnt=0, ovf=0,
              vslot=np.full(64, -1, np.int64),
              v_pool=np.zeros((L, NV, page, n_kv, d), np.int16), MAXF=MAXF)
    pool = np.zeros((L, NB, n_kv, page, d), np.int16)
    valid = np.zeros((L, n_kv, NB), np.int8)
    bt = z["block_table"]
    for s in range(steps):
        sl, ql = z["steps_sl"][s], z["steps_ql"][s]
        qsl = np.concatenate([[0], np.cumsum(ql)])
        n_tok = int(qsl[-1])
        O.staging_begin_step(st, bt, sl, qsl, n_tok, page=page, pool=pool,
                             pool_valid=valid)
        vals = z[f"vals_{s}"]
        for l in range(L):
            O.staging_scatter(st, l, vals[l], n_tok, page=page)
        assert np.array_equal(st["vbo"], z[f"vbo_{s}"]), s
        assert np.array_equal(st["vfl"], z[f"vfl_{s}"]), s
        assert st["top"] == int(z[f"top_{s}"][0]), s
        assert np.array_equal(st["stack"][:st["top"]],
                              z[f"stack_{s}"][:st["top"]]), s
        assert st["fcnt"] == int(z[f"fcnt_{s}"][0]), s
        assert np.array_equal(st["flist"][:st["fcnt"]],
                              z[f"flist_{s}"][:st["fcnt"]]), s
        assert np.array_equal(st["vslot"][:n_tok], z[f"vslot_{s}"]), s
        assert np.array_equal(pool, z[f"pool_{s}"]), s
        assert np.array_equal(valid, z[f"valid_{s}"]), s
        assert np.array_equal(st["v_pool"], z[f"vpool_{s}"]), s
        assert st["ovf"] == int(z[f"ovf_{s}"][0]), s


def test_delta_stale_vs_reference():
    z = load_golden("build_delta_tags")
    K = bits_to_f32(z["K"])
    tag = bits_to_f32(z["tag"])
    got = O.delta_stale(tag, K, z["block_table"], z["seq_lens"], page=16,
                        max_fin=int(z["max_fin"][0]))
    assert got == z["stale"].tolist()
