"""GPU parity of the split-K decode's work split: the flat page list of all
units is cut into equal warp runs, and a run that crosses units writes one
partial per unit.  These cases drive that cut hard -- arbitrary page tables
(not from a selection), empty units, units holding every page, the
smallest legal split (2) and large run floors -- and compare the output
with the CPU oracle's fp32 attention over the same pages (max-abs 2e-2,
rel 1e-2).  Reference semantics: attention/decode.py:145-241 and
attention/merge.py:30-50 (any cut of a unit's pages is an exact
re-association of its softmax; an empty unit writes zeros)."""
import numpy as np
import pytest
import torch

from amass_kv_b200 import attention as A
from amass_kv_b200.workloads import make_quad_case
from oracle import amass_oracle as O
from tests.gpu_helpers import DevCase

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _random_tables(rng, npg, n_kv, MP, mode):
    R = len(npg)
    tab = np.full((R, n_kv, MP), -1, dtype=np.int32)
    cnt = np.zeros((R, n_kv), dtype=np.int32)
    for r in range(R):
        for k in range(n_kv):
            n = int(npg[r])
            if mode == "all":
                c = n
            elif mode == "empty_mix":
                c = 0 if rng.random() < 0.4 else int(rng.integers(1, n + 1))
            else:
                c = int(rng.integers(1, n + 1))
            pages = np.sort(rng.choice(n, size=c, replace=False))
            tab[r, k, :c] = pages
            cnt[r, k] = c
    return tab, cnt


@pytest.mark.parametrize("seed,ctxs,split,pps_min,mode", [
    (1, (3000, 17, 900, 5000, 16, 2222), 2, 1, "random"),
    (2, (3000, 17, 900, 5000, 16, 2222), 3, 8, "empty_mix"),
    (3, (6000, 4100, 33), 128, 8, "all"),
    (4, (6000, 4100, 33), 5, 64, "all"),
    (5, (700,) * 9, 16, 200, "random"),
    (6, (1,), 2, 1, "all"),
])
def test_decode_runs_vs_oracle(dev, seed, ctxs, split, pps_min, mode):
    rng = np.random.default_rng(seed)
    n_kv, G, d = 8, 4, 128
    case = make_quad_case(seed, n_req=len(ctxs), n_kv=n_kv, G=G, d=d,
                          ctxs=ctxs, r=2, v_bits=4, heavy=0)
    c = DevCase.from_case(case, dev, budget=0.1, combine="max", split=split)
    npg = -(-np.asarray(ctxs) // 16)
    tab, cnt = _random_tables(rng, npg, n_kv, case.MP, mode)
    c.st.page_table.copy_(torch.from_numpy(tab))
    c.st.page_cnt.copy_(torch.from_numpy(cnt))
    c.out.fill_(float("nan"))
    A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, c.st, c.out,
                                       scale=c.scale, pps_min=pps_min)
    torch.cuda.synchronize()
    want = O.sparse_decode(case.q, case.K, case.V, case.block_table,
                           case.seq_lens, tab, cnt, scale=case.scale, G=G)
    got = c.out.float().cpu().numpy()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)
    # empty units write exact zeros
    for r in range(len(ctxs)):
        for k in range(n_kv):
            if cnt[r, k] == 0:
                assert np.all(got[r, k * G:(k + 1) * G] == 0)


def test_decode_split_below_two_is_rejected(dev):
    case = make_quad_case(9, n_req=2, n_kv=8, G=4, d=128, ctxs=(300, 200),
                          r=2, v_bits=4, heavy=0)
    c = DevCase.from_case(case, dev, budget=0.1, combine="max", split=1)
    with pytest.raises(RuntimeError):
        A.sparse_paged_decode_batched_cuda(c.q, c.kv, c.bt, c.sl, c.st,
                                           c.out, scale=c.scale)
