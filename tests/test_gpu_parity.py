"""GPU parity: the sm_100a kernels (through the C ABI) against the golden
vectors from the reference's kernels and against the CPU oracle.

Bars (from the hot-path contract):
  * scores: within 1e-4 (abs, or rel above 1) of the reference's fp32
    scores -- the scorer's q.code products are exact integer MMAs on a
    15-bit two-limb form of q, so |dS| stays near max|q|/32512 of the score
    scale (<= 5e-5 on the fixtures);
  * selections: identical except pages whose score is within 1e-3 of the
    threshold (tie band);
  * attention output: max-abs 2e-2 and rel 1e-2 of an fp32 computation over
    the same pages (bf16 tolerance).
"""
import numpy as np
import pytest
import torch

from amass_kv_b200 import attention as A
from amass_kv_b200 import selection as S
from amass_kv_b200.workloads import make_quad_case
from oracle import amass_oracle as O
from tests.conftest import load_golden
from tests.gpu_helpers import DevCase

pytestmark = pytest.mark.gpu

QUAD = ["quad_c1_nrm", "quad_c1_max", "quad_d128_i4_nrm", "quad_d128_i4_max",
        "quad_d128_i4_cov", "quad_g8_i8_cov_max"]
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _scored(z, arr):
    """compare only the scored region [0, n_sel_hi) per request"""
    return [(rq, int(n)) for rq, n in enumerate(z["n_sel_hi"]) if n > 0]


@pytest.mark.parametrize("name", QUAD)
def test_derive_and_score_contract(name, dev):
    z = load_golden(name)
    c = DevCase.from_golden(z, dev)
    st = c.st
    S.derive_page_params(st, c.sl, c.n_req)
    S.quad_score_cuda(st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
    torch.cuda.synchronize()
    assert np.array_equal(st.n_pages.cpu().numpy(), z["n_pages"])
    assert np.array_equal(st.n_sel_hi.cpu().numpy(), z["n_sel_hi"])
    assert np.array_equal(st.b_fix.cpu().numpy(), z["b_fix"])
    sc = st.score.cpu().numpy()
    for rq, n in _scored(z, sc):
        np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                   rtol=1e-4, atol=1e-4)
    if "score_h" in z:
        sh = st.score_h.cpu().numpy()
        for rq, n in _scored(z, sh):
            np.testing.assert_allclose(sh[rq, :, :, :n],
                                       z["score_h"][rq, :, :, :n],
                                       rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("name", QUAD)
def test_select_and_decode(name, dev):
    z = load_golden(name)
    cov = float(z["coverage"][0]) if "coverage" in z else None
    c = DevCase.from_golden(z, dev, coverage=cov)
    st = c.st
    S.select_pages_quad(st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
    A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, st, c.out,
                                       A.ResidentVSource(c.kv), scale=c.scale)
    torch.cuda.synchronize()
    # the page parameters derived inside the scorer's launches
    assert np.array_equal(st.n_pages.cpu().numpy(), z["n_pages"])
    assert np.array_equal(st.n_sel_hi.cpu().numpy(), z["n_sel_hi"])
    assert np.array_equal(st.b_fix.cpu().numpy(), z["b_fix"])
    tab = st.page_table.cpu().numpy()
    cnt = st.page_cnt.cpu().numpy()
    ref_sc = np.where(np.isnan(z["score"]), -np.inf, z["score"])
    if cov is None:
        assert O.selection_diff_ok(tab, cnt, z["page_table"], z["page_cnt"],
                                   ref_sc), (cnt, z["page_cnt"])
    else:
        assert O.coverage_diff_ok(tab, cnt, ref_sc, z["n_pages"],
                                  z["n_sel_hi"], sink=1, coverage=cov,
                                  combine=str(z["combine"][0])), \
            (cnt, z["page_cnt"])
    # structural: ascending, -1 padded
    for rq in range(cnt.shape[0]):
        for kh in range(cnt.shape[1]):
            row = tab[rq, kh]
            n = cnt[rq, kh]
            assert np.all(np.diff(row[:n]) > 0)
            assert np.all(row[n:] == -1)
    # decode against the oracle over the SAME pages, and the golden output
    h = c.host()
    ref = O.sparse_decode(h["q"], h["K"], h["V"], z["block_table"],
                          z["seq_lens"], tab, cnt, scale=c.scale,
                          G=int(z["meta"][0]))
    out = c.out.float().cpu().numpy()
    np.testing.assert_allclose(out, ref, atol=ATOL, rtol=RTOL)
    if np.array_equal(cnt, z["page_cnt"]) and np.array_equal(tab,
                                                              z["page_table"]):
        np.testing.assert_allclose(out, z["out"], atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", ["quad_d128_i4_cov", "quad_g8_i8_cov_max"])
def test_coverage_budget_per_unit(name, dev):
    z = load_golden(name)
    c = DevCase.from_golden(z, dev, coverage=float(z["coverage"][0]))
    S.select_pages_quad(c.st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
    torch.cuda.synchronize()
    bu = c.st.b_unit.cpu().numpy()
    nsh = z["n_sel_hi"]
    for rq in range(bu.shape[0]):
        if nsh[rq] - 1 <= 1:
            continue
        # b_u within the tie band: equal unless neighbouring masses tie
        assert abs(int(bu[rq, 0]) - int(z["b_u"][rq, 0])) <= 1
        assert abs(int(bu[rq, 1]) - int(z["b_u"][rq, 1])) <= 1


def test_topb_contract_matches_golden_exactly(dev):
    """topb_select_cuda on the reference's own scores reproduces the
    reference table bit for bit (same fp32 keys -> same threshold)."""
    z = load_golden("quad_d128_i4_max")
    c = DevCase.from_golden(z, dev)
    st = c.st
    S.derive_page_params(st, c.sl, c.n_req)
    st.score.copy_(torch.from_numpy(np.nan_to_num(z["score"], nan=0.0)))
    S.topb_select_cuda(st, c.n_req)
    torch.cuda.synchronize()
    assert np.array_equal(st.page_cnt.cpu().numpy(), z["page_cnt"])
    assert np.array_equal(st.page_table.cpu().numpy(), z["page_table"])


@pytest.mark.parametrize("seed,combine,v_bits,G,cov", [
    (11, "nrm", 4, 4, None), (12, "max", 8, 4, None), (13, "nrm", 4, 8, 0.95),
    (14, "max", 4, 4, 0.9)])
def test_random_vs_oracle(seed, combine, v_bits, G, cov, dev):
    """Mid-size ragged batches (Llama geometry slice) against the oracle."""
    rng = np.random.default_rng(seed)
    ctxs = tuple(int(x) for x in rng.integers(1, 6000, size=6))
    case = make_quad_case(seed, n_req=6, n_kv=4, G=G, d=128, ctxs=ctxs, r=2,
                          v_bits=v_bits, heavy=5, shift=3.0,
                          outlier_frac=0.02)
    c = DevCase.from_case(case, dev, budget=0.05, combine=combine,
                          coverage=cov)
    st = c.st
    S.select_pages_quad(st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
    A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, st, c.out,
                                       scale=c.scale)
    torch.cuda.synchronize()
    res = O.quad_layer_step(case.q, case.mu, case.mu_s, case.Vq, case.V_s,
                            case.sig2, case.K, case.V, case.block_table,
                            case.seq_lens, scale=case.scale, page=16, G=G,
                            r=2, v_bits=v_bits, MP=case.MP, sink=1, window=1,
                            combine=combine,
                            budget=None if cov else 0.05, coverage=cov)
    sc = st.score.cpu().numpy()
    for rq, n in enumerate(res["n_sel_hi"]):
        if n > 0:
            np.testing.assert_allclose(sc[rq, :, :n], res["score"][rq, :, :n],
                                       rtol=1e-4, atol=1e-4)
    tab = st.page_table.cpu().numpy()
    cnt = st.page_cnt.cpu().numpy()
    ref_sc = np.where(np.isnan(res["score"]), -np.inf, res["score"])
    if cov is None:
        assert O.selection_diff_ok(tab, cnt, res["page_table"],
                                   res["page_cnt"], ref_sc)
    else:
        assert O.coverage_diff_ok(tab, cnt, ref_sc, res["n_pages"],
                                  res["n_sel_hi"], sink=1, coverage=cov,
                                  combine=combine)
    out = c.out.float().cpu().numpy()
    ref = O.sparse_decode(case.q, case.K, case.V, case.block_table,
                          case.seq_lens, tab, cnt, scale=case.scale, G=G)
    np.testing.assert_allclose(out, ref, atol=ATOL, rtol=RTOL)


def test_decode_dense_budget_full_matches_torch(dev):
    """budget 1.0 keeps every page: the sparse decode must equal dense
    attention (fp32 torch on the same device) -- a size-independent check."""
    rng = np.random.default_rng(5)
    ctxs = tuple(int(x) for x in rng.integers(100, 3000, size=5))
    case = make_quad_case(21, n_req=5, n_kv=8, G=4, d=128, ctxs=ctxs, r=2,
                          v_bits=4, heavy=2)
    c = DevCase.from_case(case, dev, budget=1.0, combine="max")
    st = c.st
    S.select_pages_quad(st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
    A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, st, c.out,
                                       scale=c.scale)
    torch.cuda.synchronize()
    npg = st.n_pages.cpu().numpy()
    assert np.array_equal(st.page_cnt.cpu().numpy(),
                          np.repeat(npg[:, None], 8, axis=1))
    K, V = c.kv[:, 0].float(), c.kv[:, 1].float()
    for rq in range(c.n_req):
        L = int(case.seq_lens[rq])
        blks = c.bt[rq, :int(npg[rq])].long()
        k = K[blks].reshape(-1, 8, 128)[:L]
        v = V[blks].reshape(-1, 8, 128)[:L]
        qg = c.q[rq].float().view(8, 4, 128)
        s = torch.einsum("kgd,tkd->kgt", qg, k) * c.scale
        o = torch.einsum("kgt,tkd->kgd", torch.softmax(s, -1), v).reshape(32, 128)
        torch.testing.assert_close(c.out[rq].float(), o, atol=ATOL, rtol=RTOL)


def test_empty_and_padded_rows(dev):
    """seq_len 0 rows select nothing and write zeros, never NaN."""
    z = load_golden("quad_d128_i4_nrm")
    c = DevCase.from_golden(z, dev)
    c.out.fill_(float("nan"))
    S.select_pages_quad(c.st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
    A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, c.st, c.out,
                                       scale=c.scale)
    torch.cuda.synchronize()
    out = c.out.float().cpu().numpy()
    assert np.all(out[4] == 0)
    assert np.isfinite(out).all()
