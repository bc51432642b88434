"""The C ABI library builds for sm_100a, loads, and exports every symbol the
header declares (no compute calls: this runs without a GPU)."""
import ctypes
import os
import re

from tests.conftest import ROOT


def _header_symbols():
    txt = open(os.path.join(ROOT, "include", "amass_b200.h")).read()
    return sorted(set(re.findall(r"\b(amass_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_header_symbols():
    from amass_kv_b200 import _lib
    from amass_kv_b200.build import build
    build()
    lib = ctypes.CDLL(_lib.LIB_PATH)
    syms = _header_symbols()
    assert syms, "no declarations found"
    for s in syms:
        assert hasattr(lib, s), f"missing export {s}"
    # the ctypes binding covers the header exactly
    assert sorted(_lib.exported_symbols()) == syms


def test_status_strings():
    from amass_kv_b200 import _lib
    _lib.load()
    assert _lib.status_string(0) == "ok"
    assert "argument" in _lib.status_string(1)


def test_arg_validation_without_gpu():
    """Argument checks run before any launch, so they work on a CPU box."""
    from amass_kv_b200 import _lib
    lib = _lib.load()
    # n_req < 0 -> AMASS_ERR_ARG
    assert lib.amass_derive_page_params(0, 0, 0, 0, 0, -1, 16, 1, 1, 0) == 1
    # n_req == 0 -> no-op success
    assert lib.amass_derive_page_params(0, 0, 0, 0, 0, 0, 16, 1, 1, 0) == 0
    # unsupported geometry (G > 8) on the quad scorer
    one = ctypes.c_void_p(16)
    rc = lib.amass_quad_score(one, 512, 128, one, one, one, one, one, one, 64,
                              one, one, 0, 0, 0, one, one, ctypes.c_float(0.1), 1,
                              1, 16, 128, 16, 2, 4, 64, 0, 0)
    assert rc == 2
