"""Drop-in through the reference's own state layout: this build's Stage A
and Stage B entry points run on stand-ins that carry exactly the attributes
of the reference's QuadState / R8State (recorded from the reference's own
constructors, tests/golden/ref_states.json) -- zero-filled hmax, unpadded
per-head score rows, no q-limb scratch, no split-K partials -- filled from
the golden vectors the reference's kernels produced, and must reproduce
those goldens (scores within 1e-4, selections up to the 1e-3 tie band,
outputs within bf16 tolerance).  The calls are the ones the reference's
runtime makes (backend/_runtime.py:183-263): select_pages_quad /
select_pages_r8, ensure_stage_b_buffers, sparse_paged_decode_batched_cuda."""
import numpy as np
import pytest
import torch

from amass_kv_b200 import attention as A
from amass_kv_b200 import selection as S
from oracle import amass_oracle as O
from tests import refstate
from tests.conftest import bits_to_f32, load_golden

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_quad_on_reference_state_layout(dev):
    z = load_golden("quad_d128_i4_nrm")
    st = refstate.build("QuadState", dev)
    for name, key in (("quad_mu", "mu"), ("mu_scale", "mu_s"),
                      ("quad_V", "Vq"), ("V_scale", "V_s"),
                      ("quad_sig2", "sig2")):
        getattr(st, name)[0].copy_(_t(z[key], dev))
    assert st.score_h.stride(2) % 4 != 0        # unpadded rows, as the reference
    q = _t(z["q"], dev).view(torch.bfloat16)
    kv = _t(z["kv"], dev).view(torch.bfloat16)
    bt, sl = _t(z["block_table"], dev), _t(z["seq_lens"], dev)
    n_req, scale = bt.shape[0], float(z["scale"][0])
    S.select_pages_quad(st, 0, q, bt, sl, n_req, scale)
    A.ensure_stage_b_buffers(st, dev)
    out = torch.zeros(q.shape, dtype=torch.bfloat16, device=dev)
    A.sparse_paged_decode_batched_cuda(q, kv, bt, sl, st, out, scale=scale)
    torch.cuda.synchronize()
    sc = st.score.cpu().numpy()
    for rq, n in enumerate(z["n_sel_hi"]):
        if n > 0:
            np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                       rtol=1e-4, atol=1e-4)
    tab, cnt = st.page_table.cpu().numpy(), st.page_cnt.cpu().numpy()
    ref_sc = np.where(np.isnan(z["score"]), -np.inf, z["score"])
    assert O.selection_diff_ok(tab, cnt, z["page_table"], z["page_cnt"],
                               ref_sc)
    kvf = bits_to_f32(z["kv"])
    want = O.sparse_decode(bits_to_f32(z["q"]), kvf[:, 0], kvf[:, 1],
                           z["block_table"], z["seq_lens"], tab, cnt,
                           scale=scale, G=int(z["meta"][0]))
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=ATOL,
                               rtol=RTOL)
    if np.array_equal(cnt, z["page_cnt"]) and np.array_equal(
            tab, z["page_table"]):
        np.testing.assert_allclose(out.float().cpu().numpy(), z["out"],
                                   atol=ATOL, rtol=RTOL)
    # hmax is left at -inf for the next step (the fold consumed it)
    assert torch.isinf(st.hmax).all() and (st.hmax < 0).all()


def test_r8_on_reference_state_layout(dev):
    z = load_golden("r8_i8")
    st = refstate.build("R8State", dev)
    for name, key in (("r8_mu", "mu"), ("mu_scale", "mu_s"), ("r8_Vk", "Vk"),
                      ("Vk_scale", "Vk_s"), ("r8_c", "c"),
                      ("c_scale", "c_s")):
        getattr(st, name)[0].copy_(_t(z[key], dev))
    q = _t(z["q"], dev).view(torch.bfloat16)
    bt, sl = _t(z["block_table"], dev), _t(z["seq_lens"], dev)
    S.select_pages_r8(st, 0, q, bt, sl, bt.shape[0], float(z["scale"][0]))
    torch.cuda.synchronize()
    sc = st.score.cpu().numpy()
    for rq, n in enumerate(z["n_sel_hi"]):
        np.testing.assert_allclose(sc[rq, :, :n], z["score"][rq, :, :n],
                                   rtol=1e-4, atol=1e-4)
    ref = np.where(np.isnan(z["score"]), -np.inf, z["score"])
    assert O.selection_diff_ok(st.page_table.cpu().numpy(),
                               st.page_cnt.cpu().numpy(), z["page_table"],
                               z["page_cnt"], ref)
