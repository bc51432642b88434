"""The recorded attribute contract of the reference's state objects
(tests/golden/ref_states.json) against this build's own state classes, and,
when the reference checkout is given in AMASS_REF_SRC, against the live
reference constructors.  CPU only."""
import os
import sys

import numpy as np
import pytest
import torch

from amass_kv_b200 import selection as S
from tests import refstate
from tests.conftest import GOLDEN


def _ours(kind):
    if kind == "QuadState":
        z = np.load(os.path.join(GOLDEN, "quad_d128_i4_nrm.npz"))
        G, r, vb, page, MP = [int(x) for x in z["meta"]]
        return S.QuadState("cpu", num_layers=1, num_blocks=z["mu"].shape[0],
                           n_kv=z["mu"].shape[1], G=G,
                           head_dim=z["mu"].shape[2], page=page,
                           max_reqs=z["block_table"].shape[0], max_pages=MP,
                           rank=r, budget=float(z["budget"][0]), v_bits=vb,
                           combine=str(z["combine"][0]))
    z = np.load(os.path.join(GOLDEN, "r8_i8.npz"))
    G, r, vkb, cb, page, MP, n_kv, d = [int(x) for x in z["meta"]]
    return S.R8State("cpu", num_layers=1, num_blocks=z["mu"].shape[0],
                     n_kv=n_kv, G=G, head_dim=d, page=page,
                     max_reqs=z["block_table"].shape[0], max_pages=MP,
                     rank=r, budget=float(z["budget"][0]), vk_bits=vkb,
                     c_bits=cb)


@pytest.mark.parametrize("kind", ["QuadState", "R8State"])
def test_own_state_is_a_superset_of_the_reference_contract(kind):
    """Every reference attribute exists on this build's state with the same
    shape and dtype (strides may differ: the per-head score rows here are
    padded to 16-byte multiples; every kernel takes the strides) and the same
    plain values."""
    spec = refstate.load_contract()[kind]
    ours = _ours(kind)
    for name, d in spec.items():
        assert hasattr(ours, name), name
        v = getattr(ours, name)
        if "tensor" in d:
            assert isinstance(v, torch.Tensor), name
            assert list(v.shape) == d["tensor"]["shape"], name
            assert str(v.dtype).replace("torch.", "") == d["tensor"]["dtype"], name
        elif d["value"] != "device":
            assert v == d["value"], (name, v, d["value"])


@pytest.mark.parametrize("kind", ["QuadState", "R8State"])
def test_stand_in_matches_the_contract(kind):
    st = refstate.build(kind, "cpu")
    spec = refstate.load_contract()[kind]
    assert set(vars(st)) == set(spec)
    assert not hasattr(st, "q8") and not hasattr(st, "m_part")


def test_fixture_matches_the_live_reference(tmp_path):
    ref = os.environ.get("AMASS_REF_SRC")
    if not ref or not os.path.isdir(ref):
        pytest.skip("AMASS_REF_SRC (the reference checkout's src/) not set")
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, here)
    import make_refstate_fixture as M
    sys.path.insert(0, ref)
    from amass.selection.quad_state import QuadState
    z = np.load(os.path.join(GOLDEN, "quad_d128_i4_nrm.npz"))
    G, r, vb, page, MP = [int(x) for x in z["meta"]]
    qs = QuadState("cpu", num_layers=1, num_blocks=z["mu"].shape[0],
                   n_kv=z["mu"].shape[1], G=G, head_dim=z["mu"].shape[2],
                   page=page, max_reqs=z["block_table"].shape[0],
                   max_pages=MP, rank=r, budget=float(z["budget"][0]),
                   v_bits=vb, combine=str(z["combine"][0]))
    assert M.describe(qs) == refstate.load_contract()["QuadState"]
