"""The pipelined quad scorer (producer warp + bulk copies into a shared-memory
ring, eight consumer warps) against the register-pipelined scorer: both run
the same integer-MMA math and epilogue, so scores, per-head scores, the
per-head maxima and the selected pages must be bitwise equal; the pipelined
scores also stay within 1e-4 of the oracle.  Ragged batches cover requests
with no scored page, partial last tiles and both q-limb forms (the limb
launch below 32 requests, the in-scorer split from 32 up).  The device fault
word of the bounded barrier waits must stay 0.
Reference: selection/quad_score.py:55-107 (score), quad_score_cuda.py:
1724-1794 (entry point)."""
import ctypes

import numpy as np
import pytest
import torch

from amass_kv_b200 import _lib
from amass_kv_b200 import selection as S
from amass_kv_b200.workloads import make_quad_case
from oracle import amass_oracle as O
from tests.gpu_helpers import DevCase

pytestmark = pytest.mark.gpu


def _status(clear=0):
    f = ctypes.c_int(-1)
    n = ctypes.c_longlong(-1)
    _lib.call("amass_quad_pipeline_status", ctypes.addressof(f),
              ctypes.addressof(n), clear)
    return f.value, n.value


def _run(case, dev, combine, mode, pack=1):
    lib = _lib.load()
    prev = lib.amass_quad_pipeline(mode)
    prev_pack = lib.amass_quad_pack(pack)
    try:
        c = DevCase.from_case(case, dev, budget=0.1, combine=combine)
        S.select_pages_quad(c.st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
        torch.cuda.synchronize()
    finally:
        lib.amass_quad_pipeline(prev)
        lib.amass_quad_pack(prev_pack)
    st = c.st
    return dict(nsh=st.n_sel_hi.cpu().numpy(), score=st.score.cpu().numpy(),
                score_h=(st.score_h.cpu().numpy() if st.score_h is not None
                         else None),
                pages=st.page_table.cpu().numpy(),
                cnt=st.page_cnt.cpu().numpy())


@pytest.mark.parametrize("n_req", [9, 40])
@pytest.mark.parametrize("combine", ["max", "nrm"])
@pytest.mark.parametrize("geom", [(2, 4), (1, 8)])
def test_pipelined_scorer_bitwise(n_req, combine, geom):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    r, vb = geom
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(100 + n_req + r)
    ctxs = [int(x) for x in rng.integers(17, 2400, n_req)]
    ctxs[0], ctxs[1] = 20, 16 * 37 + 5           # no scored page; ragged tile
    case = make_quad_case(41 + n_req, n_req=n_req, n_kv=8, G=4, d=128,
                          ctxs=tuple(ctxs), r=r, v_bits=vb, heavy=2)
    _status(clear=1)
    pipe = _run(case, dev, combine, 2)
    fault, launches = _status()
    assert fault == 0
    assert launches == 1, "the pipelined scorer did not serve this geometry"
    reg = _run(case, dev, combine, 0)
    assert _status()[1] == 1
    assert np.array_equal(pipe["nsh"], reg["nsh"])
    nsh = pipe["nsh"]
    for rq in range(n_req):
        n = int(nsh[rq])
        if n <= 0:
            continue
        if combine == "nrm":
            assert np.array_equal(pipe["score_h"][rq, ..., :n],
                                  reg["score_h"][rq, ..., :n]), rq
        assert np.array_equal(pipe["score"][rq, :, :n],
                              reg["score"][rq, :, :n]), rq
    assert np.array_equal(pipe["cnt"], reg["cnt"])
    for rq in range(n_req):
        for kv in range(8):
            k = int(pipe["cnt"][rq, kv])
            assert np.array_equal(pipe["pages"][rq, kv, :k],
                                  reg["pages"][rq, kv, :k]), (rq, kv)
    want = O.quad_score_h(case.q, case.mu, case.mu_s, case.Vq, case.V_s,
                          case.sig2, case.block_table, nsh, scale=case.scale,
                          page=16, G=4, r=r, v_bits=vb, MP=case.MP)
    for rq in range(n_req):
        n = int(nsh[rq])
        if n <= 0:
            continue
        w = want[rq, :, :, :n]
        if combine == "nrm":
            np.testing.assert_allclose(pipe["score_h"][rq, ..., :n], w,
                                       rtol=1e-4, atol=1e-4)
        else:
            np.testing.assert_allclose(pipe["score"][rq, :, :n],
                                       w.max(axis=1), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("G", [4, 3, 2, 1])
@pytest.mark.parametrize("n_req", [9, 40])
def test_packed_limbs_bitwise(G, n_req):
    """Packed limbs (G <= 4: hi and lo limbs in one MMA's 8 columns, lane
    quads c and c ^ 2 swapping half their sums; per-head maxima folded once
    per request run) against the pipelined scorer's two-limb form: per-head
    scores, page maxima and the selected pages bitwise equal, for every G the
    packed form serves, both q-limb forms, both combines."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(300 + G + n_req)
    ctxs = [int(x) for x in rng.integers(17, 2400, n_req)]
    ctxs[0] = 16 * 21 + 3                        # ragged last tile
    case = make_quad_case(91 + G + n_req, n_req=n_req, n_kv=8, G=G, d=128,
                          ctxs=tuple(ctxs), r=2, v_bits=4, heavy=2)
    for combine in ("nrm", "max"):
        _status(clear=1)
        two = _run(case, dev, combine, 2, pack=0)
        pk = _run(case, dev, combine, 2, pack=1)
        nsh = pk["nsh"]
        for rq in range(n_req):
            n = int(nsh[rq])
            if n <= 0:
                continue
            if combine == "nrm":
                assert np.array_equal(pk["score_h"][rq, ..., :n],
                                      two["score_h"][rq, ..., :n]), rq
            assert np.array_equal(pk["score"][rq, :, :n],
                                  two["score"][rq, :, :n]), rq
        assert np.array_equal(pk["cnt"], two["cnt"])
        assert np.array_equal(pk["pages"], two["pages"])
        assert _status() == (0, 2)


def test_pipelined_scorer_large_request_table():
    """1200 short requests: the request table (prefix and page counts) in
    shared memory beside the ring, most CTAs crossing many request
    boundaries; scores equal the register-pipelined scorer's."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(7)
    n_req = 1200
    ctxs = tuple(int(x) for x in rng.integers(17, 120, n_req))
    case = make_quad_case(77, n_req=n_req, n_kv=8, G=4, d=128, ctxs=ctxs,
                          r=2, v_bits=4, heavy=1)
    _status(clear=1)
    wide = _run(case, dev, "nrm", 2)
    assert _status() == (0, 1)
    reg = _run(case, dev, "nrm", 0)
    nsh = wide["nsh"]
    for rq in range(n_req):
        n = int(nsh[rq])
        if n > 0:
            assert np.array_equal(wide["score_h"][rq, ..., :n],
                                  reg["score_h"][rq, ..., :n]), rq
