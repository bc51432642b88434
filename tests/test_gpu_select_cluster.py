"""Top-b selection at batch sizes and unit lengths that pick each
CTA-per-unit form (a thread-block cluster of 8, 4 or 2 CTAs per unit for few
units longer than 4096 pages, one CTA otherwise), on the plain score input and on the folded per-head (nrm) input,
against the oracle's threshold rule.  Random continuous scores (no ties):
tables and counts must match exactly; the folded scores within 1e-5."""
import numpy as np
import pytest
import torch

from amass_kv_b200 import selection as S
from oracle import amass_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("n_req", [2, 12, 25, 80])     # 16 / 96 / 200 / 640 units
@pytest.mark.parametrize("fold", [False, True])
@pytest.mark.parametrize("MP", [1024, 5000])
def test_topb_cluster_forms_vs_oracle(dev, n_req, fold, MP):
    rng = np.random.default_rng(100 + n_req + 7 * fold + MP)
    n_kv, G, page = 8, 4, 16
    ctxs = rng.integers(1, MP * page + 1, n_req).astype(np.int32)
    ctxs[0] = MP * page                                 # a full-length unit
    if n_req > 2:
        ctxs[1] = 20                                    # keep-all unit
    st = S.QuadState(dev, num_layers=1, num_blocks=1, n_kv=n_kv, G=G,
                     head_dim=128, page=page, max_reqs=n_req, max_pages=MP,
                     rank=2, budget=0.05, v_bits=4,
                     combine="nrm" if fold else "max")
    sl = torch.from_numpy(ctxs).to(dev)
    S.derive_page_params(st, sl, n_req)
    nsh = st.n_sel_hi.cpu().numpy()
    npg = st.n_pages.cpu().numpy()
    b = st.b_fix.cpu().numpy()
    if fold:
        sh = rng.standard_normal((n_req, n_kv, G, MP)).astype(np.float32) * 3
        for rq in range(n_req):
            sh[rq, :, :, max(nsh[rq], 0):] = 0.0
        st.score_h[..., :MP].copy_(torch.from_numpy(sh))
        st.hmax.copy_(torch.from_numpy(
            np.stack([sh[rq, :, :, :max(nsh[rq], 1)].max(-1)
                      for rq in range(n_req)]).astype(np.float32)))
        ref_sc = O.combine_nrm(sh, nsh)
        S.select_pages(st, n_req, from_score_h=True)
    else:
        ref_sc = rng.standard_normal((n_req, n_kv, MP)).astype(np.float32)
        st.score.copy_(torch.from_numpy(ref_sc))
        S.topb_select_cuda(st, n_req)
    torch.cuda.synchronize()
    ref_sc = np.where(np.isnan(ref_sc), -np.inf, ref_sc).astype(np.float32)
    if fold:
        got = st.score.cpu().numpy()
        for rq in range(n_req):
            n = int(nsh[rq])
            if n > 0:
                np.testing.assert_allclose(got[rq, :, :n], ref_sc[rq, :, :n],
                                           rtol=1e-5, atol=1e-6)
        ref_sc = np.where(np.isfinite(ref_sc), got, -np.inf)  # GPU keys
    tab, cnt = O.topb_select(ref_sc, npg, nsh, b, sink=1, MP=MP)
    assert np.array_equal(st.page_cnt.cpu().numpy(), cnt)
    assert np.array_equal(st.page_table.cpu().numpy(), tab)
    if fold:
        assert bool(torch.isinf(st.hmax).all())            # reset for the next call
