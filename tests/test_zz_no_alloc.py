"""The allocation-free decode entry point against the regular one.

amass_sparse_decode_noalloc serves callers that cannot allocate device
memory (a plugin living inside another runtime's memory pool, a serving loop
that must not touch the allocator): its split-K partials sit in a fixed
device array inside the library.  This test calls both entry points through
the C ABI on the same selection and checks that the outputs are bitwise
equal (both run the same kernels with the same split; only the partials'
home differs), on two calls in a row (the second call sees the first
call's leftovers in the shared array), and checks the regular call against
the CPU oracle's fp32 decode over the same pages.  The file is named to be
collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from amass_kv_b200 import _lib
from amass_kv_b200 import selection as S
from amass_kv_b200.attention import split_kv
from amass_kv_b200.workloads import make_quad_case
from oracle import amass_oracle as O
from tests.gpu_helpers import DevCase

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2
SPLIT = 16


def _decode_args(c, out, split, pps_min):
    k, v = split_kv(c.kv)
    P = _lib.ptr
    st = c.st
    head = [P(c.q), c.q.stride(0), c.q.stride(1), P(k), k.stride(0),
            k.stride(1), k.stride(2), P(v), v.stride(0), v.stride(1),
            v.stride(2), P(c.bt), c.bt.stride(0), P(st.page_table),
            P(st.page_cnt), P(c.sl)]
    tail = [P(out), out.stride(0), out.stride(1), ctypes.c_float(c.scale),
            c.n_req, st.n_kv, st.G, st.d, 16, st.max_pages,
            _lib.stream_of(c.q.device)]
    return head, tail


@pytest.mark.parametrize("seed", [31, 32])
def test_noalloc_matches_regular_decode_twice(seed):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    rng = np.random.default_rng(seed)
    ctxs = tuple(int(x) for x in rng.integers(40, 5000, size=6))
    case = make_quad_case(seed, n_req=6, n_kv=8, G=4, d=128, ctxs=ctxs, r=2,
                          v_bits=4, heavy=4, shift=3.0)
    c = DevCase.from_case(case, dev, budget=0.1, combine="nrm", split=SPLIT)
    S.select_pages_quad(c.st, 0, c.q, c.bt, c.sl, c.n_req, c.scale)
    need = c.n_req * 8 * SPLIT * 4 * (128 + 2)
    assert need <= lib.amass_sparse_decode_noalloc_capacity()

    ref = torch.zeros_like(c.out)
    head, tail = _decode_args(c, ref, SPLIT, 4)
    st = c.st
    rc = lib.amass_sparse_decode(*head, _lib.ptr(st.m_part),
                                 _lib.ptr(st.l_part), _lib.ptr(st.acc_part),
                                 SPLIT, 4, *tail)
    assert rc == 0, _lib.status_string(rc)
    torch.cuda.synchronize()
    tab = st.page_table.cpu().numpy()
    cnt = st.page_cnt.cpu().numpy()
    want = O.sparse_decode(case.q, case.K, case.V, case.block_table,
                           case.seq_lens, tab, cnt, scale=case.scale, G=4)
    np.testing.assert_allclose(ref.float().cpu().numpy(), want, atol=ATOL,
                               rtol=RTOL)
    for _ in range(2):
        out = torch.full_like(c.out, float("nan"))
        head, tail = _decode_args(c, out, SPLIT, 4)
        rc = lib.amass_sparse_decode_noalloc(*head, SPLIT, 4, *tail)
        assert rc == 0, _lib.status_string(rc)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_noalloc_rejects_oversize_request():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    one = ctypes.c_void_p(256)
    # 4096 requests x 8 heads x split 128 x G 4 x 130 floats >> capacity
    rc = lib.amass_sparse_decode_noalloc(
        one, 4096, 128, one, 64, 64, 64, one, 64, 64, 64, one, 64, one, one,
        one, 128, 4, one, 4096, 128, ctypes.c_float(0.1), 4096, 8, 4, 128,
        16, 64, 0)
    assert rc == 3
