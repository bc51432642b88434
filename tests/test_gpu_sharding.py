"""Multi-GPU layouts on B200s: the kv-head-sharded decode (merge kernel that
stores into every rank's output over NVLink + peer barrier, and the NCCL
all-gather variant) places every rank's rows bit for bit as that rank's own
decode of its heads, and matches the single-GPU decode of all heads within
bf16 tolerance.
World 1 runs on one GPU; worlds 2 and 4 run when that many GPUs are
visible."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _state(dev, b, n_kv, G, lo, hi, n_req, MP):
    from amass_kv_b200.attention import ensure_stage_b_buffers
    from amass_kv_b200.selection import QuadState
    st = QuadState(dev, num_layers=1, num_blocks=1, n_kv=hi - lo, G=G,
                   head_dim=128, page=16, max_reqs=n_req, max_pages=MP,
                   rank=2, budget=0.05, v_bits=4, combine="nrm")
    st.quad_mu = b["quad_mu"][:, :, lo:hi].contiguous()
    st.mu_scale = b["mu_scale"][:, :, lo:hi].contiguous()
    st.quad_V = b["quad_V"][:, :, lo:hi].contiguous()
    st.V_scale = b["V_scale"][:, :, lo:hi].contiguous()
    st.quad_sig2 = b["quad_sig2"][:, :, lo:hi].contiguous()
    ensure_stage_b_buffers(st, dev, 128)
    return st


def _select(st, q, bt, sl, n_req, scale):
    from amass_kv_b200 import selection as S
    S.derive_page_params(st, sl, n_req)
    S._score_launch(st, 0, q, bt, n_req, scale, True)
    S.select_pages(st, n_req, from_score_h=True)


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist
    from amass_kv_b200 import attention as A
    from amass_kv_b200 import sharding as SH
    from amass_kv_b200.workloads import make_quad_case_gpu
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=dev)
    try:
        n_req, n_kv, G, d = 5, 8, 4, 128
        ctxs = [3000, 700, 33, 16, 12000]
        b = make_quad_case_gpu(dev, seed=11, ctxs=ctxs, n_kv=n_kv, G=G, d=d,
                               r=2, v_bits=4, layers=1)
        kv, bt, sl = b["kv_cache"][0], b["block_table"], b["seq_lens"]
        qf = b["q"][0]
        MP = b["MP"]
        scale = d ** -0.5
        # single-GPU reference over all heads
        st = _state(dev, b, n_kv, G, 0, n_kv, n_req, MP)
        _select(st, qf, bt, sl, n_req, scale)
        ref = torch.zeros_like(qf)
        A.sparse_paged_decode_batched_cuda(qf, kv, bt, sl, st, ref,
                                           scale=scale)
        # this rank's kv heads
        lo, hi = SH.kv_head_range(n_kv, world, rank)
        st_l = _state(dev, b, n_kv, G, lo, hi, n_req, MP)
        q_l = qf[:, lo * G:hi * G].contiguous()
        kv_l = kv[:, :, :, lo:hi].contiguous()
        _select(st_l, q_l, bt, sl, n_req, scale)
        g = SH.HeadGather(n_req, n_kv * G, d, device=dev, mode=mode)
        outs = []
        for _ in range(3):                    # both p2p buffers, then reuse
            o = SH.sparse_paged_decode_kvsharded(q_l, kv_l, bt, sl, st_l, g,
                                                 scale=scale)
            torch.cuda.synchronize()
            outs.append(o.clone())
        if mode == "p2p":
            g.check()
        # every rank's rows equal that rank's own decode of its heads, bit
        # for bit (the same kernels on the same per-rank batch), computed
        # here for all ranks' head ranges
        exp = torch.zeros_like(qf)
        for rr in range(world):
            lo2, hi2 = SH.kv_head_range(n_kv, world, rr)
            st2 = _state(dev, b, n_kv, G, lo2, hi2, n_req, MP)
            q2 = qf[:, lo2 * G:hi2 * G].contiguous()
            _select(st2, q2, bt, sl, n_req, scale)
            o2 = torch.zeros_like(q2)
            A.sparse_paged_decode_batched_cuda(
                q2, kv[:, :, :, lo2:hi2].contiguous(), bt, sl, st2, o2,
                scale=scale)
            exp[:, lo2 * G:hi2 * G] = o2
        torch.cuda.synchronize()
        ok = all(bool(torch.equal(o, exp)) for o in outs)
        # and the all-heads decode within bf16 tolerance (the split-K cut
        # of a unit depends on the batch's total pages, so fp32 sums
        # associate differently)
        err = float((outs[-1].float() - ref.float()).abs().max())
        ok = ok and torch.allclose(outs[-1].float(), ref.float(), atol=2e-2,
                                   rtol=1e-2)
        q.put((rank, ok, err))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, repr(e)))
    finally:
        dist.destroy_process_group()


def _run(world, mode):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, ok, info = q.get(timeout=300)
        res[r] = (ok, info)
    for p in procs:
        p.join(timeout=120)
    assert all(v[0] for v in res.values()), res


@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_kvsharded_world1(mode):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _run(1, mode)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_kvsharded_multi_gpu(world, mode):
    _run(world, mode)
