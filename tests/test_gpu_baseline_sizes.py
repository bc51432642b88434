"""GPU parity at the BASELINE configurations' real sizes, against the CPU
oracle on the same seeded inputs.

  C2  batch 1, context 32768 (2048 pages), Llama-3.1-8B geometry, 2%
      outlier channels x8, planted heavy pages, quad r'=2 int4-V nrm,
      per-head coverage 0.95;
  C3  a sample of the ragged batch: 4 requests including one of 65536 tokens
      (4096 pages), budget 0.05, nrm;
  C4  the r8 scorer at context 65536 (LSE and token-max), budget 0.05;
  C5  the mem-v tier at Llama-3.1-70B geometry (G=8): one 131072-token
      request (8192 pages) and one of 32768, a hot buffer of 10% of the
      pool, three decode steps of drifting selections through
      mem_dynamic_decode, the residency state compared with the oracle's
      exact-LRU trace after every step.

Bars: scores within 1e-4 (abs, or rel above 1); selections identical except
pages within 1e-3 of the threshold (coverage: a valid nucleus size within
the 1e-3 mass band); attention max-abs 2e-2 / rel 1e-2 of fp32 over the same
pages; residency maps, LRU clocks, fetched bytes bit-exact; the tiered
decode bitwise equal to the resident decode.  Reference semantics:
selection/quad_score.py:35-107, selection/select.py:60-101,
backend/_selection_bridge.py:117-133, selection/score.py:30-120,
tier/residency.py:45-139, tier/decode_mem.py:225-274."""
import numpy as np
import pytest
import torch

from amass_kv_b200 import attention as A
from amass_kv_b200 import selection as S
from amass_kv_b200 import tier as T
from amass_kv_b200.workloads import make_quad_case, make_r8_case
from oracle import amass_oracle as O
from tests.gpu_helpers import DevCase

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _check_quad(case, c, G, combine, budget, coverage):
    st = c.st
    tab = st.page_table.cpu().numpy()
    cnt = st.page_cnt.cpu().numpy()
    npg, nsh, b = O.derive_page_params(case.seq_lens, budget or 0.1, 16, 1, 1)
    sh = O.quad_score_h(case.q, case.mu, case.mu_s, case.Vq, case.V_s,
                        case.sig2, case.block_table, nsh, scale=case.scale,
                        page=16, G=G, r=case.r, v_bits=case.v_bits,
                        MP=case.MP)
    score = O.combine_nrm(sh, nsh) if combine == "nrm" else \
        O.combine_max(sh, nsh)
    sc = st.score.cpu().numpy()
    for rq, n in enumerate(nsh):
        if n > 0:
            np.testing.assert_allclose(sc[rq, :, :n], score[rq, :, :n],
                                       rtol=1e-4, atol=1e-4)
    ref_sc = np.where(np.isnan(score), -np.inf, score)
    if coverage is None:
        otab, ocnt = O.topb_select(ref_sc, npg, nsh, b, sink=1, MP=case.MP)
        assert O.selection_diff_ok(tab, cnt, otab, ocnt, ref_sc)
    else:
        assert O.coverage_diff_ok(tab, cnt, ref_sc, npg, nsh, sink=1,
                                  coverage=coverage, combine=combine)
    out = c.out.float().cpu().numpy()
    ref = O.sparse_decode(case.q, case.K, case.V, case.block_table,
                          case.seq_lens, tab, cnt, scale=case.scale, G=G)
    np.testing.assert_allclose(out, ref, atol=ATOL, rtol=RTOL)
    return tab, cnt


def test_c2_coverage_32k(dev):
    case = make_quad_case(202, n_req=1, n_kv=8, G=4, d=128, ctxs=(32768,),
                          r=2, v_bits=4, heavy=102, shift=3.0,
                          outlier_frac=0.02)
    c = DevCase.from_case(case, dev, budget=0.05, combine="nrm",
                          coverage=0.95)
    S.select_pages_quad(c.st, 0, c.q, c.bt, c.sl, 1, c.scale)
    A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, c.st, c.out,
                                       scale=c.scale)
    torch.cuda.synchronize()
    tab, cnt = _check_quad(case, c, 4, "nrm", None, 0.95)
    assert cnt.min() > 102          # coverage 0.95 keeps more than the plant


def test_c3_sample_with_64k_request(dev):
    ctxs = (65536, 4096, 21000, 40000)
    case = make_quad_case(303, n_req=4, n_kv=8, G=4, d=128, ctxs=ctxs, r=2,
                          v_bits=4, heavy=8, shift=3.0)
    c = DevCase.from_case(case, dev, budget=0.05, combine="nrm")
    S.select_pages_quad(c.st, 0, c.q, c.bt, c.sl, 4, c.scale)
    A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, c.st, c.out,
                                       scale=c.scale)
    torch.cuda.synchronize()
    tab, cnt = _check_quad(case, c, 4, "nrm", 0.05, None)
    # 4095 scored pages, b = ceil(0.05 * 4094) = 205, plus sink and window
    assert cnt[0].min() >= 207


@pytest.mark.parametrize("agg", ["lse", "tokmax"])
def test_c4_r8_64k(dev, agg):
    cs = make_r8_case(404, n_req=2, n_kv=8, G=4, d=128, ctxs=(65536, 65536),
                      r=8, vk_bits=8, c_bits=8)
    n_req, MP = 2, cs.MP
    NB = cs.mu.shape[0]
    st = S.R8State(dev, num_layers=1, num_blocks=NB, n_kv=8, G=4,
                   head_dim=128, page=16, max_reqs=n_req, max_pages=MP, rank=8,
                   budget=0.05, vk_bits=8, c_bits=8)
    for dst, src in ((st.r8_mu, cs.mu), (st.mu_scale, cs.mu_s),
                     (st.r8_Vk, cs.Vk), (st.Vk_scale, cs.Vk_s),
                     (st.r8_c, cs.c), (st.c_scale, cs.c_s)):
        dst[0].copy_(torch.from_numpy(np.ascontiguousarray(src)))
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    q = t(cs.q).to(torch.bfloat16)
    bt, sl = t(cs.block_table), t(cs.seq_lens)
    S.select_pages_r8(st, 0, q, bt, sl, n_req, cs.scale, token_agg=agg)
    torch.cuda.synchronize()
    npg, nsh, b = O.derive_page_params(cs.seq_lens, 0.05, 16, 1, 1)
    ref = O.r8_score(cs.q, cs.mu, cs.mu_s, cs.Vk, cs.Vk_s, cs.c, cs.c_s,
                     cs.block_table, cs.seq_lens, nsh, scale=cs.scale,
                     page=16, G=4, r=8, vk_bits=8, c_bits=8, MP=MP,
                     combine=agg)
    sc = st.score.cpu().numpy()
    for rq, n in enumerate(nsh):
        np.testing.assert_allclose(sc[rq, :, :n], ref[rq, :, :n], rtol=1e-4,
                                   atol=1e-4)
    refm = np.where(np.isnan(ref), -np.inf, ref)
    tab, cnt = O.topb_select(refm, npg, nsh, b, sink=1, MP=MP)
    assert O.selection_diff_ok(st.page_table.cpu().numpy(),
                               st.page_cnt.cpu().numpy(), tab, cnt, refm)


def test_c5_tier_128k_g8(dev):
    """Three decode steps of the mem-v tier at C5 geometry with drifting
    selections (5% budget + sink + window per unit, a third of the pages
    kept from the previous step), every page flushed to the pinned pool."""
    rng = np.random.default_rng(505)
    n_kv, G, d, page = 8, 8, 128, 16
    ctx = np.array([131072, 32768], np.int32)
    npg = -(-ctx // page)
    NB = int(npg.sum()) + 16
    MP = int(npg.max())
    perm = rng.permutation(NB)
    bt = np.zeros((2, MP), np.int32)
    o = 0
    for r in range(2):
        bt[r, :npg[r]] = perm[o:o + npg[r]]
        o += npg[r]
    S_hot = int(round(0.10 * NB))
    L, layer = 1, 0
    tier = T.Tier(num_layers=L, num_blocks=NB, n_kv=n_kv, page=page, d=d,
                  hot_slots=S_hot, max_reqs=2, max_pages=MP, n_vslots=4,
                  device=dev)
    r5 = tier.residency
    gd = torch.Generator(device=dev).manual_seed(7)
    kv = torch.randn((NB, 2, page, n_kv, d), generator=gd, device=dev).to(
        torch.bfloat16)
    tier.pool.host[layer].copy_(kv[:, 1].permute(0, 2, 1, 3).cpu())
    r5.pool_valid.fill_(1)
    kv_k = kv[:, :1].contiguous()
    st = S.QuadState(dev, num_layers=1, num_blocks=1, n_kv=n_kv, G=G,
                     head_dim=d, page=page, max_reqs=2, max_pages=MP, rank=2,
                     budget=0.05, v_bits=4, combine="nrm")
    A.ensure_stage_b_buffers(st, dev, 128)
    btd = torch.from_numpy(bt).to(dev)
    sld = torch.from_numpy(ctx).to(dev)
    Kh = kv[:, 0].float().cpu().numpy()
    Vh = kv[:, 1].float().cpu().numpy()
    o_p2s = np.full((n_kv, NB), -1, np.int32)
    o_s2p = np.full((n_kv, S_hot), -1, np.int32)
    o_lru = np.zeros((n_kv, S_hot), np.int32)
    prev = None
    for s in range(3):
        tab = np.full((2, n_kv, MP), -1, np.int32)
        cnt = np.zeros((2, n_kv), np.int32)
        for r in range(2):
            n = int(npg[r])
            b = int(np.ceil(0.05 * (n - 2)))
            for k in range(n_kv):
                keep = set()
                if prev is not None:
                    old = prev[r, k][prev[r, k] >= 0]
                    keep = set(rng.choice(old, len(old) // 3,
                                          replace=False).tolist())
                fresh = rng.choice(np.arange(1, n - 1), b, replace=False)
                pages = sorted(keep | set(fresh.tolist()) | {0, n - 1})
                tab[r, k, :len(pages)] = pages
                cnt[r, k] = len(pages)
        prev = tab
        st.page_table.copy_(torch.from_numpy(tab))
        st.page_cnt.copy_(torch.from_numpy(cnt))
        q = torch.randn((2, n_kv * G, d), generator=gd, device=dev).to(
            torch.bfloat16)
        out = torch.zeros_like(q)
        T.mem_dynamic_decode(q, kv_k, btd, sld, st, out, tier, layer,
                             scale=d ** -0.5)
        res = torch.zeros_like(q)
        A.sparse_paged_decode_batched_cuda(q, kv, btd, sld, st, res,
                                           scale=d ** -0.5)
        torch.cuda.synchronize()
        fl, ovf = O.residency_step(tab, cnt, bt, ctx, page=page,
                                   page2slot=o_p2s, slot2page=o_s2p,
                                   lru=o_lru, clock=s + 2)
        assert not ovf
        assert np.array_equal(r5.page2slot[layer].cpu().numpy(), o_p2s), s
        assert np.array_equal(r5.slot2page[layer].cpu().numpy(), o_s2p), s
        assert np.array_equal(r5.lru_clock[layer].cpu().numpy(), o_lru), s
        assert int(r5.fetch_cnt.sum()) == len(fl), s
        # every resident slot holds its page's true V bytes
        hot = r5.hot[layer].view(torch.int16).cpu().numpy()
        v16 = kv[:, 1].contiguous().view(torch.int16).cpu().numpy()
        for kvh in range(n_kv):
            slots = np.nonzero(o_s2p[kvh] >= 0)[0]
            assert np.array_equal(hot[kvh, slots],
                                  v16[o_s2p[kvh, slots], :, kvh]), (s, kvh)
        assert torch.equal(out, res), s
        ref = O.sparse_decode(q.float().cpu().numpy(), Kh, Vh, bt, ctx, tab,
                              cnt, scale=d ** -0.5, G=G)
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=ATOL,
                                   rtol=RTOL)
