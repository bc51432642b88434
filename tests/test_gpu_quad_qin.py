"""The quad scorer splits q into its two int8 limbs inside the score launch
for batches of 32 requests or more, and in a separate limb launch below
that.  Both forms must give the same limbs, so the scores of a request are
bitwise equal whichever batch it is scored in: a 36-request batch (in-scorer
split) against the same requests scored as four 9-request batches (limb
launch), for max (score) and nrm (score_h + hmax) combine; the derived page
parameters equal too, and the whole batch stays within 1e-4 of the oracle.
Reference recipe: selection/quad_score_cuda.py:36-49 (two-limb int8 q)."""
import types

import numpy as np
import pytest
import torch

from amass_kv_b200 import selection as S
from amass_kv_b200.workloads import make_quad_case
from oracle import amass_oracle as O
from tests.gpu_helpers import DevCase

pytestmark = pytest.mark.gpu


def _sub(case, idx):
    """The case restricted to requests idx (same pool and summaries)."""
    c = types.SimpleNamespace(**vars(case))
    c.q = case.q[idx]
    c.block_table = np.ascontiguousarray(case.block_table[idx])
    c.seq_lens = np.ascontiguousarray(case.seq_lens[idx])
    return c


@pytest.mark.parametrize("combine", ["max", "nrm"])
def test_in_scorer_limbs_equal_limb_launch(combine):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(5)
    ctxs = tuple(int(x) for x in rng.integers(17, 1600, 36))
    case = make_quad_case(31, n_req=36, n_kv=2, G=4, d=128, ctxs=ctxs, r=2,
                          v_bits=4, heavy=2)
    full = DevCase.from_case(case, dev, budget=0.1, combine=combine)
    S.select_pages_quad(full.st, 0, full.q, full.bt, full.sl, full.n_req,
                        full.scale)
    torch.cuda.synchronize()
    nsh = full.st.n_sel_hi.cpu().numpy()
    key = "score_h" if combine == "nrm" else "score"
    got = getattr(full.st, key).cpu().numpy()
    for part in range(4):
        idx = np.arange(9 * part, 9 * part + 9)
        sub = DevCase.from_case(_sub(case, idx), dev, budget=0.1,
                                combine=combine)
        S.select_pages_quad(sub.st, 0, sub.q, sub.bt, sub.sl, sub.n_req,
                            sub.scale)
        torch.cuda.synchronize()
        assert np.array_equal(sub.st.n_sel_hi.cpu().numpy(), nsh[idx])
        assert np.array_equal(sub.st.b_fix.cpu().numpy(),
                              full.st.b_fix.cpu().numpy()[idx])
        ref = sub.st.score_h.cpu().numpy() if combine == "nrm" else \
            sub.st.score.cpu().numpy()
        for j, rq in enumerate(idx):
            n = int(nsh[rq])
            if n > 0:
                assert np.array_equal(got[rq, ..., :n], ref[j, ..., :n]), \
                    f"request {rq}: {key} differs between the two limb forms"
    # and the whole batch against the oracle's fp32 per-head scores (1e-4)
    want = O.quad_score_h(case.q, case.mu, case.mu_s, case.Vq, case.V_s,
                          case.sig2, case.block_table, nsh, scale=case.scale,
                          page=16, G=4, r=2, v_bits=4, MP=case.MP)
    for rq in range(36):
        n = int(nsh[rq])
        if n <= 0:
            continue
        w = want[rq, :, :, :n]
        g = got[rq, :, :, :n] if combine == "nrm" else got[rq, :, :n]
        if combine == "max":
            w = w.max(axis=1)
        np.testing.assert_allclose(g, w, rtol=1e-4, atol=1e-4)
