"""ctypes binding of libamass_b200.so (the C ABI declared in
include/amass_b200.h).

The library is the only compute path: if it is missing or fails to load, every
entry point raises -- there is no CPU or Triton fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libamass_b200.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_U = ctypes.c_uint64


class DmaRun(ctypes.Structure):
    """AmassDmaRun: one copy-engine copy (rows of a strided 2-D copy)."""
    _fields_ = [("dst", ctypes.c_uint64), ("src", ctypes.c_uint64),
                ("dst_k", ctypes.c_uint64), ("src_k", ctypes.c_uint64),
                ("dpitch", ctypes.c_int64), ("spitch", ctypes.c_int64),
                ("width", ctypes.c_int64), ("height", ctypes.c_int64)]


# name -> argtypes (restype is int status for every compute entry point)
_SIGS = {
    "amass_init": [],
    "amass_version": [],
    "amass_derive_page_params": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "amass_quad_score": [_P, _L, _L, _P, _P, _P, _P, _P, _P, _L, _P, _P, _P,
                         _L, _P, _P, _P, _F, _I, _I, _I, _I, _I, _I, _I, _I,
                         _I, _P],
    "amass_quad_score_derive": [_P, _P, _P, _P, _P, _I, _I, _P, _L, _L, _P,
                                _P, _P, _P, _P, _P, _L, _P, _P, _L, _P, _P,
                                _P, _F, _I, _I, _I, _I, _I, _I, _I, _I, _I,
                                _P],
    "amass_quad_pipeline": [_I],
    "amass_quad_pack": [_I],
    "amass_quad_pipeline_status": [_P, _P, _I],
    "amass_r8_score": [_P, _L, _L, _P, _P, _P, _P, _P, _P, _P, _L, _P, _P, _P,
                       _P, _P, _F, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P],
    "amass_clse_score": [_P, _L, _L, _P, _P, _P, _P, _P, _P, _I, _P, _P, _L,
                         _P, _P, _P, _P, _L, _P, _P, _P, _P, _F, _I, _I, _I,
                         _I, _I, _I, _I, _I, _I, _I, _P],
    "amass_summarize_pages": [_P, _I, _L, _L, _L, _P, _I, _I, _I, _I, _I, _I,
                              _I, _P, _P, _P, _P, _I, _I, _P, _P, _I, _P, _P,
                              _I, _I, _P, _P],
    "amass_tag_stale": [_P, _I, _L, _L, _L, _P, _I, _I, _I, _I, _I, _P, _I,
                        _P, _P, _P],
    "amass_nrm_combine": [_P, _L, _P, _P, _P, _I, _I, _I, _I, _P],
    "amass_topb_select": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "amass_select_pages": [_P, _L, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I,
                           _I, _I, _I, _I, _I, _F, _P],
    "amass_sparse_decode": [_P, _L, _L, _P, _L, _L, _L, _P, _L, _L, _L, _P,
                            _L, _P, _P, _P, _P, _P, _P, _I, _I, _P, _L, _L,
                            _F, _I, _I, _I, _I, _I, _I, _P],
    "amass_sparse_decode_noalloc": [_P, _L, _L, _P, _L, _L, _L, _P, _L, _L,
                                    _L, _P, _L, _P, _P, _P, _I, _I, _P, _L,
                                    _L, _F, _I, _I, _I, _I, _I, _I, _P],
    "amass_sparse_decode_gather": [_P, _L, _L, _P, _L, _L, _L, _P, _L, _L,
                                   _L, _P, _L, _P, _P, _P, _P, _P, _P, _I,
                                   _I, _P, _I, _I, _L, _L, _F, _I, _I, _I,
                                   _I, _I, _I, _P],
    "amass_peer_barrier": [_P, _I, _I, _P, _P, _P],
    "amass_staging_begin_step": [_P, _L, _P, _P, _I, _I, _I, _P, _P, _P, _P,
                                 _P, _P, _P, _P, _I, _P, _P, _L, _L, _L, _L,
                                 _P, _P, _P, _I, _I, _I, _I, _I, _P, _I,
                                 _P],
    "amass_staging_scatter": [_P, _L, _L, _P, _L, _L, _P, _P, _P, _L, _L, _L,
                              _I, _I, _I, _I, _P],
    "amass_host_device_pointer": [_P, _P],
    "amass_tier_plan_capacity": [_I],
    "amass_tier_plan": [_P, _P, _P, _L, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                        _I, _I, _I, _I, _I, _I, _P],
    "amass_tier_fetch": [_P, _P, _P, _P, _P, _P, _P, _L, _L, _L, _P, _P, _P,
                         _I, _I, _I, _I, _I, _I, _P],
    "amass_tier_fetch_staged": [_P, _P, _P, _P, _P, _P, _P, _L, _L, _L, _P,
                                _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "amass_tier_dma_plan": [_P, _P, _P, _I, _I, _I, _I, _I, _I, _U, _U, _U,
                            _U, _P, _I, _P, _P],
    "amass_dma_issue": [_P, _I, _P],
    "amass_tier_invalidate": [_P, _L, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I,
                              _I, _P],
    "amass_tier_decode": [_P, _L, _L, _P, _L, _L, _L, _P, _P, _P, _P, _L, _L,
                          _L, _P, _P, _P, _P, _P, _I, _I, _I, _P, _L, _P, _P, _P,
                          _P, _P, _P, _I, _I, _P, _L, _L, _F, _I, _I, _I, _I,
                          _I, _I, _P],
    "amass_tier_decode_install": [_P, _L, _L, _P, _L, _L, _L, _P, _P, _P, _P,
                                  _L, _L, _L, _P, _P, _P, _P, _P, _P, _I, _I,
                                  _I, _P, _L, _P, _P, _P, _P, _P, _P, _I, _I,
                                  _P, _L, _L, _F, _I, _I, _I, _I, _I, _I, _P],
}

_lib = None
_lock = threading.Lock()


def exported_symbols():
    """Every C entry point this binding declares (tests check the .so)."""
    return sorted(list(_SIGS) + ["amass_status_string",
                                 "amass_sparse_decode_noalloc_capacity"])


def load():
    """Load the library once; raise loudly if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libamass_b200.so not found at {LIB_PATH}; build it with "
                "`python -m amass_kv_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        lib.amass_sparse_decode_noalloc_capacity.argtypes = []
        lib.amass_sparse_decode_noalloc_capacity.restype = ctypes.c_size_t
        lib.amass_status_string.argtypes = [ctypes.c_int]
        lib.amass_status_string.restype = ctypes.c_char_p
        _lib = lib
        return lib


def status_string(rc: int) -> str:
    return load().amass_status_string(rc).decode()


def call(name: str, *args) -> None:
    """Invoke a C entry point; raise RuntimeError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name} failed: {status_string(rc)} (status {rc})")


def ptr(t) -> int:
    """Device address of a tensor (0 for None)."""
    return 0 if t is None else t.data_ptr()


def stream_of(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
