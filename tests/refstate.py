"""Stand-ins for the reference's own state objects, built only from the
attribute contract recorded in tests/golden/ref_states.json (shapes, dtypes,
strides, initial fills and plain values of the reference's QuadState and
R8State).  A stand-in carries none of the attributes this build's own state
classes add (q-limb scratch, per-unit budgets, padded per-head score rows,
split-K partials): whatever this build's entry points need beyond the
reference's contract they must add themselves, as a drop-in would."""
import json
import os

import torch

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                       "ref_states.json")
_DT = {"int8": torch.int8, "int32": torch.int32, "float16": torch.float16,
       "bfloat16": torch.bfloat16, "float32": torch.float32,
       "float64": torch.float64}


def load_contract():
    with open(FIXTURE) as fh:
        return json.load(fh)


class RefLikeState:
    """Attributes exactly as the reference's constructor leaves them."""


def build(kind: str, device) -> RefLikeState:
    spec = load_contract()[kind]
    st = RefLikeState()
    for name, d in spec.items():
        if "tensor" in d:
            t = d["tensor"]
            fill = t.get("fill")
            x = torch.empty_strided(t["shape"], t["stride"],
                                    dtype=_DT[t["dtype"]], device=device)
            if fill == "zeros":
                x.zero_()
            elif fill == "ones":
                x.fill_(1)
            elif fill == "nan":
                x.fill_(float("nan"))
            elif "value" in t:
                x.fill_(t["value"])
            setattr(st, name, x)
        elif d["value"] == "device":
            setattr(st, name, device)
        else:
            setattr(st, name, d["value"])
    return st
