"""Host logic of the multi-GPU layouts (CPU; gloo process groups)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from amass_kv_b200 import sharding as SH


def test_lpt_partition_covers_and_balances():
    rng = np.random.default_rng(0)
    costs = rng.lognormal(0, 1, 64)
    for world in (1, 2, 4, 8):
        parts = SH.lpt_partition(costs, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        loads = [costs[p].sum() for p in parts]
        # LPT bound: makespan <= (4/3 - 1/(3m)) OPT, OPT >= max(mean, max)
        opt_lb = max(costs.sum() / world, costs.max())
        assert max(loads) <= (4 / 3 - 1 / (3 * world)) * opt_lb + 1e-9 or \
            max(loads) <= costs.max() + 1e-9


def test_lpt_partition_small_exact():
    assert SH.lpt_partition([5, 4, 3, 3, 3], 2) == [[0, 3], [1, 2, 4]]


def test_kv_head_range():
    assert [SH.kv_head_range(8, 4, r) for r in range(4)] == \
        [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        SH.kv_head_range(8, 3, 0)


def test_request_bytes_formula():
    b = SH.request_bytes([4096, 17], n_kv=8, page=16, budget=0.05, b_sum=266,
                         d=128, G=4)
    npg = 256
    nsh = npg - 1
    kept = int(np.ceil((nsh - 1) * 0.05)) + 2
    want = 8 * nsh * 266 + 4 * nsh + 8 * kept * 2 * 16 * 128 * 2 + \
        8 * 4 * 128 * 4
    assert b[0] == want
    # 2 pages: nothing selectable, both pages kept
    assert b[1] == 8 * 1 * 266 + 4 + 8 * 2 * 8192 + 8 * 4 * 128 * 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gather_worker(rank, world, port, T, H, d, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = SH.HeadGather(T, H, d, mode="nccl")
        Hl = H // world
        loc = torch.arange(T * Hl * d, dtype=torch.float32).view(T, Hl, d)
        g.local.copy_((loc + 1000 * rank).to(torch.bfloat16))
        out = g.all_gather().float()
        ok = True
        for r in range(world):
            want = (loc + 1000 * r).to(torch.bfloat16).float()
            ok &= bool(torch.equal(out[:, r * Hl:(r + 1) * Hl], want))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_gather_places_every_rank_slice(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker,
                         args=(r, world, port, 3, 8, 4, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(res[r] for r in range(world)), res
