"""The copy-engine run planner (a host function of the C ABI, so it runs
without a GPU) against the oracle's restatement of the reference's run
coalescing: identical runs, in order, and the staged flag."""
import ctypes

import numpy as np
import pytest

from amass_kv_b200 import _lib
from oracle import amass_oracle as O


def _plan(fl, fc, pv, *, layer, NB, page, d, pool_base, hot_base, cap=None,
          k_bases=(0, 0)):
    n_kv, S, _ = fl.shape
    cap = cap if cap is not None else max(1, int(fc.sum()))
    runs = (_lib.DmaRun * cap)()
    n, st = ctypes.c_int(0), ctypes.c_int(0)
    fl = np.ascontiguousarray(fl, np.int32)
    fc = np.ascontiguousarray(fc, np.int32)
    pv = np.ascontiguousarray(pv, np.int8)
    rc = _lib.load().amass_tier_dma_plan(
        fl.ctypes.data, fc.ctypes.data, pv.ctypes.data, layer, NB, n_kv, S,
        page, d, pool_base, hot_base, k_bases[0], k_bases[1],
        ctypes.cast(runs, ctypes.c_void_p), cap, ctypes.byref(n),
        ctypes.byref(st))
    return rc, list(runs)[:n.value], bool(st.value)


@pytest.mark.parametrize("seed", range(6))
def test_dma_plan_matches_oracle(seed):
    rng = np.random.default_rng(seed)
    n_kv, S, NB, page, d, layer = 4, 64, 200, 16, 128, 1
    fl = np.zeros((n_kv, S, 2), np.int32)
    fc = rng.integers(0, S + 1, n_kv).astype(np.int32)
    for kv in range(n_kv):
        # runs of consecutive (block, slot) broken at random points
        blk, slot = int(rng.integers(0, 50)), int(rng.integers(0, 8))
        slots = rng.permutation(S)
        for e in range(fc[kv]):
            if rng.random() < 0.2:
                blk = int(rng.integers(0, NB - S))
            fl[kv, e] = (blk % NB, slots[e] if seed % 2 else (slot + e) % S)
            blk += 1
    pv = (rng.random((n_kv, NB)) > 0.1).astype(np.int8)
    pool_base, hot_base = 1 << 40, 1 << 36
    rc, runs, staged = _plan(fl, fc, pv, layer=layer, NB=NB, page=page, d=d,
                             pool_base=pool_base, hot_base=hot_base)
    assert rc == 0
    exp, exp_staged = O.dma_plan_runs(fl, fc, pv, layer=layer, NB=NB,
                                      page=page, d=d, pool_base=pool_base,
                                      hot_base=hot_base)
    got = [(r.dst, r.src, r.dpitch, r.spitch, r.width, r.height) for r in runs]
    assert got == exp
    assert staged == exp_staged
    assert all(r.dst_k == 0 and r.src_k == 0 for r in runs)


def test_dma_plan_k_tier_and_limits():
    n_kv, S, NB, page, d = 1, 8, 16, 16, 64
    fl = np.zeros((n_kv, S, 2), np.int32)
    fl[0, :4] = [(3, 0), (4, 1), (5, 2), (9, 3)]
    fc = np.array([4], np.int32)
    pv = np.ones((n_kv, NB), np.int8)
    rc, runs, staged = _plan(fl, fc, pv, layer=0, NB=NB, page=page, d=d,
                             pool_base=4096, hot_base=8192,
                             k_bases=(1 << 20, 1 << 24))
    assert rc == 0 and not staged
    assert [r.height for r in runs] == [3, 1]
    pb = page * d * 2
    assert runs[0].src_k == (1 << 20) + 3 * pb
    assert runs[0].dst_k == (1 << 24)
    # too small a run buffer -> capacity error
    rc, _, _ = _plan(fl, fc, pv, layer=0, NB=NB, page=page, d=d,
                     pool_base=4096, hot_base=8192, cap=1)
    assert rc == 3
    # out-of-range block -> argument error
    fl[0, 1, 0] = NB
    rc, _, _ = _plan(fl, fc, pv, layer=0, NB=NB, page=page, d=d,
                     pool_base=4096, hot_base=8192)
    assert rc == 1
