"""GPU parity of the CLSE scorer (quad geometry + per-key coordinates +
residual energy) against the reference's clse_score goldens and the oracle.

Bars: per-head / combined scores within 1e-3 (abs, or rel above 1) -- the
q.code products are exact integer MMAs on a 15-bit two-limb q, the token
log-sum-exp and iso term are fp32; selections identical except pages within
1e-3 of the threshold."""
import numpy as np
import pytest
import torch

from amass_kv_b200 import selection as S
from amass_kv_b200.attention import ensure_stage_b_buffers
from amass_kv_b200.selection import QuadState
from amass_kv_b200.workloads import make_clse_case
from oracle import amass_oracle as O
from tests.conftest import bits_to_f32, load_golden

pytestmark = pytest.mark.gpu
CLSE = ["clse_i4_tok_nrm", "clse_i8_page_max", "clse_r4_i8_tok_max"]
TOL = 1e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _state(dev, *, NB, n_kv, G, d, n_req, MP, r, v_bits, c_bits, c_grain,
           combine, budget, coverage=None):
    st = QuadState(dev, num_layers=1, num_blocks=NB, n_kv=n_kv, G=G,
                   head_dim=d, page=16, max_reqs=n_req, max_pages=MP, rank=r,
                   budget=budget, v_bits=v_bits, combine=combine,
                   coords="lse", c_bits=c_bits, c_grain=c_grain,
                   coverage=coverage)
    ensure_stage_b_buffers(st, dev, 128)
    return st


def _fill(st, mu, mu_s, Vq, V_s, sig2, c, c_s, resid):
    for t, x in ((st.quad_mu, mu), (st.mu_scale, mu_s), (st.quad_V, Vq),
                 (st.V_scale, V_s), (st.quad_sig2, sig2), (st.quad_c, c),
                 (st.c_scale, c_s), (st.quad_resid, resid)):
        t[0].copy_(torch.from_numpy(np.ascontiguousarray(x)))


@pytest.mark.parametrize("name", CLSE)
def test_clse_matches_reference(name, dev):
    z = load_golden(name)
    G, r, vb, page, MP = [int(x) for x in z["meta"]]
    c_bits, tok = [int(x) for x in z["cmeta"]]
    comb = str(z["combine"][0])
    kv = z["kv"]
    NB, n_kv, d = kv.shape[0], kv.shape[3], kv.shape[4]
    n_req = z["block_table"].shape[0]
    st = _state(dev, NB=NB, n_kv=n_kv, G=G, d=d, n_req=n_req, MP=MP, r=r,
                v_bits=vb, c_bits=c_bits, c_grain="token" if tok else "page",
                combine=comb, budget=float(z["budget"][0]))
    _fill(st, z["mu"], z["mu_s"], z["Vq"], z["V_s"], z["sig2"], z["c"],
          z["c_s"], z["resid"])
    q = torch.from_numpy(z["q"]).view(torch.bfloat16).to(dev)
    bt = torch.from_numpy(z["block_table"]).to(dev)
    sl = torch.from_numpy(z["seq_lens"]).to(dev)
    st.score.fill_(float("nan"))
    if comb == "nrm":
        st.score_h.fill_(float("nan"))
        S.derive_page_params(st, sl, n_req)
        S.clse_score_cuda(st, 0, q, bt, sl, n_req, float(z["scale"][0]))
        torch.cuda.synchronize()
        sh = st.score_h.cpu().numpy()
        for rq in range(n_req):
            n = int(z["n_sel_hi"][rq])
            np.testing.assert_allclose(sh[rq, :, :, :n],
                                       z["score_h"][rq, :, :, :n],
                                       rtol=TOL, atol=TOL)
        S.select_pages(st, n_req, from_score_h=True)
    else:
        S.select_pages_clse(st, 0, q, bt, sl, n_req, float(z["scale"][0]))
    torch.cuda.synchronize()
    sc = st.score.cpu().numpy()
    for rq in range(n_req):
        n = int(z["n_sel_hi"][rq])
        np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                   rtol=TOL, atol=TOL)
    ref = np.where(np.isnan(z["score"]), -np.inf, z["score"])
    assert O.selection_diff_ok(st.page_table.cpu().numpy(),
                               st.page_cnt.cpu().numpy(), z["page_table"],
                               z["page_cnt"], ref)


@pytest.mark.parametrize("seed,d,r,v_bits,c_bits,c_grain,combine,G", [
    (11, 128, 2, 4, 4, "token", "nrm", 4),
    (12, 128, 2, 4, 8, "page", "max", 4),
    (13, 64, 8, 8, 8, "token", "nrm", 4),
    (14, 128, 2, 4, 4, "token", "nrm", 2),   # token split, two head slots idle
    (15, 128, 4, 4, 8, "token", "max", 3),   # rank 4, int8 codes (4-byte rows)
    (16, 64, 4, 4, 4, "page", "nrm", 8),     # G = 8: per-lane-head form
])
def test_clse_random_vs_oracle(seed, d, r, v_bits, c_bits, c_grain, combine,
                               G, dev):
    cs = make_clse_case(seed, n_req=5, n_kv=4, G=G, d=d,
                        ctxs=(3000, 1700, 16, 260, 900), r=r, v_bits=v_bits,
                        c_bits=c_bits, c_grain=c_grain)
    x = cs.extra
    NB = cs.K.shape[0]
    st = _state(dev, NB=NB, n_kv=4, G=G, d=d, n_req=5, MP=cs.MP, r=r,
                v_bits=v_bits, c_bits=c_bits, c_grain=c_grain,
                combine=combine, budget=0.1)
    _fill(st, cs.mu, cs.mu_s, cs.Vq, cs.V_s, cs.sig2, x["c"], x["c_s"],
          x["resid"])
    q = torch.from_numpy(cs.q).to(dev).to(torch.bfloat16)
    bt = torch.from_numpy(cs.block_table).to(dev)
    sl = torch.from_numpy(cs.seq_lens).to(dev)
    S.select_pages_clse(st, 0, q, bt, sl, 5, cs.scale)
    torch.cuda.synchronize()
    nsh = st.n_sel_hi.cpu().numpy()
    sh = O.clse_score_h(cs.q, cs.mu, cs.mu_s, cs.Vq, cs.V_s, x["c"], x["c_s"],
                        x["resid"], cs.block_table, cs.seq_lens, nsh,
                        scale=cs.scale, page=16, G=G, r=r, v_bits=v_bits,
                        c_bits=c_bits, token_grain=c_grain == "token",
                        MP=cs.MP)
    ref = O.combine_nrm(sh, nsh) if combine == "nrm" else O.combine_max(sh, nsh)
    sc = st.score.cpu().numpy()
    for rq in range(5):
        n = int(nsh[rq])
        np.testing.assert_allclose(sc[rq, :, :n], ref[rq, :, :n], rtol=TOL,
                                   atol=TOL)
    npg, _, b = O.derive_page_params(cs.seq_lens, 0.1, 16, 1, 1)
    refm = np.where(np.isnan(ref), -np.inf, ref).astype(np.float32)
    tab, cnt = O.topb_select(refm, npg, nsh, b, sink=1, MP=cs.MP)
    assert O.selection_diff_ok(st.page_table.cpu().numpy(),
                               st.page_cnt.cpu().numpy(), tab, cnt, refm)
