"""Failure detection without a GPU fault: the cross-GPU barrier's bounded
wait.  One process, one GPU: the "peer" flag array is a second local buffer
that nothing writes, so the wait for that rank runs out; the kernel records
the missing rank in the error word and returns (no trap), the host reads the
status, and the context stays usable.  A peer that already arrived passes."""
import ctypes
import time

import pytest
import torch

from amass_kv_b200 import _lib
from amass_kv_b200._lib import ptr

pytestmark = pytest.mark.gpu


def _barrier(flags_me, flags_peer, epoch, err):
    arr = (ctypes.c_void_p * 2)(flags_me.data_ptr(), flags_peer.data_ptr())
    _lib.call("amass_peer_barrier", ctypes.cast(arr, ctypes.c_void_p), 2, 0,
              ptr(epoch), ptr(err), _lib.stream_of(flags_me.device))


def test_barrier_wait_times_out_with_status():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    i32 = dict(dtype=torch.int32, device=dev)
    flags_me, flags_peer = torch.zeros(2, **i32), torch.zeros(2, **i32)
    epoch, err = torch.zeros(1, **i32), torch.zeros(1, **i32)
    t0 = time.time()
    _barrier(flags_me, flags_peer, epoch, err)
    torch.cuda.synchronize(dev)
    waited = time.time() - t0
    assert int(err.item()) == 2            # 1 + the rank that never arrived
    assert int(epoch.item()) == 1
    assert int(flags_peer[0].item()) == 1  # our arrival reached the peer
    assert int(flags_me[0].item()) == 1
    assert waited < 30
    # the context is still usable
    x = torch.arange(1000, device=dev, dtype=torch.float32)
    assert float(x.sum().item()) == 499500.0


def test_barrier_passes_when_peer_arrived():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    i32 = dict(dtype=torch.int32, device=dev)
    flags_me, flags_peer = torch.zeros(2, **i32), torch.zeros(2, **i32)
    flags_me[1] = 7                         # the peer's arrival for epochs <= 7
    epoch, err = torch.zeros(1, **i32), torch.zeros(1, **i32)
    for _ in range(3):
        _barrier(flags_me, flags_peer, epoch, err)
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    assert int(epoch.item()) == 3
    assert int(flags_peer[0].item()) == 3
