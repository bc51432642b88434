"""Record the attribute contract of the REFERENCE's own state objects.

    AMASS_REF_SRC=<reference checkout>/src python tests/golden/make_refstate_fixture.py

Constructs the reference's ``QuadState`` (selection/quad_state.py:36-151,
nrm combine, for the geometry of the ``quad_d128_i4_nrm`` golden case) and
``R8State`` (selection/state.py:35-112, for ``r8_i8``) on the CPU and writes,
for every attribute, its tensor shape, dtype, strides and initial fill (or
its plain value) to ``tests/golden/ref_states.json``.  The GPU drop-in test
builds stand-ins carrying exactly these attributes -- nothing this build's
own state classes add -- and runs this build's entry points on them.  The
fixture is committed; nothing at test time reads the reference tree.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _fill(t: torch.Tensor):
    if t.numel() == 0:
        return "empty"
    f = t.float()
    if torch.isnan(f).all():
        return "nan"
    if (f == 0).all():
        return "zeros"
    if (f == 1).all():
        return "ones"
    return None                     # torch.empty or data: unspecified


def describe(st) -> dict:
    out = {}
    for k, v in sorted(vars(st).items()):
        if isinstance(v, torch.Tensor):
            d = {"shape": list(v.shape), "dtype": str(v.dtype).replace(
                "torch.", ""), "stride": list(v.stride())}
            fill = _fill(v)
            if fill is not None:
                d["fill"] = fill
            if v.numel() == 1 and fill is None:
                d["value"] = float(v.item())
            out[k] = {"tensor": d}
        elif v is None or isinstance(v, (int, float, str, bool)):
            out[k] = {"value": v}
        elif isinstance(v, torch.device):
            out[k] = {"value": "device"}
    return out


def main():
    ref = os.environ.get("AMASS_REF_SRC")
    if not ref:
        sys.exit("set AMASS_REF_SRC to the reference checkout's src/ directory")
    sys.path.insert(0, ref)
    from amass.selection.quad_state import QuadState
    from amass.selection.state import R8State

    zq = np.load(os.path.join(HERE, "quad_d128_i4_nrm.npz"))
    G, r, vb, page, MP = [int(x) for x in zq["meta"]]
    NB, n_kv = zq["mu"].shape[0], zq["mu"].shape[1]
    n_req, d = zq["block_table"].shape[0], zq["mu"].shape[2]
    qs = QuadState("cpu", num_layers=1, num_blocks=NB, n_kv=n_kv, G=G,
                   head_dim=d, page=page, max_reqs=n_req, max_pages=MP,
                   rank=r, budget=float(zq["budget"][0]), v_bits=vb,
                   combine=str(zq["combine"][0]))
    zr = np.load(os.path.join(HERE, "r8_i8.npz"))
    G8, r8, vkb, cb, page8, MP8, n_kv8, d8 = [int(x) for x in zr["meta"]]
    rs = R8State("cpu", num_layers=1, num_blocks=zr["mu"].shape[0],
                 n_kv=n_kv8, G=G8, head_dim=d8, page=page8,
                 max_reqs=zr["block_table"].shape[0], max_pages=MP8, rank=r8,
                 budget=float(zr["budget"][0]), vk_bits=vkb, c_bits=cb)
    doc = {"_about": "attributes of the reference's QuadState "
                     "(selection/quad_state.py:36-151) for the golden "
                     "quad_d128_i4_nrm geometry and of its R8State "
                     "(selection/state.py:35-112) for r8_i8, recorded by "
                     "tests/golden/make_refstate_fixture.py",
           "QuadState": describe(qs), "R8State": describe(rs)}
    with open(os.path.join(HERE, "ref_states.json"), "w") as fh:
        json.dump(doc, fh, indent=1, sort_keys=True)
    print("wrote", os.path.join(HERE, "ref_states.json"))


if __name__ == "__main__":
    main()
