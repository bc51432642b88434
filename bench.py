"""Benchmark: the AMASS sparse-decode hot path, one layer-step per step.

Workload (BASELINE C3): ragged continuous-batching decode, Llama-3.1-8B
attention geometry (32 query / 8 KV heads, head_dim 128, bf16 KV, page 16),
batch 64 with contexts drawn log-uniformly from 4K to 64K tokens, block
tables drawn from one shared random page pool, fixed budget 5% of pages,
quad summaries r'=2 with int4 V and the nrm GQA combine (the AmassConfig
defaults).  A step = derive + quad score + nrm fold/top-b select + split-K
decode + merge for one layer.  Steps rotate over `--layers` independent layer
slabs (each ~0.5 GB of algorithmic traffic) so the working set is far larger
than the 126 MB L2: no explicit flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Multi-GPU (torchrun, one process per GPU): every rank runs its own C3 batch
(sequence sharding of independent requests, no collective on the data path);
`value` is the max over ranks of the per-step device time ("scaling": weak).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse decode µs/layer/step & HBM TB/s frac, B=64 ctx=32K " \
         "Llama-8B geometry"
UNIT = "us/layer/step"
N_REQ, N_KV, G, D, PAGE = 64, 8, 4, 128, 16
RANK_Q, V_BITS, BUDGET, COMBINE = 2, 4, 0.05, "nrm"
B_SUM = D + 2 + D * RANK_Q // 2 + 2 * RANK_Q + 2 * RANK_Q     # 266 B


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            pk = json.load(fh)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic_table():
    """Per-launch DRAM traffic of each kernel from the committed ncu summary
    (profiles/traffic.json), scaled by the launch's algorithmic bytes."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as fh:
            return json.load(fh)
    except Exception:
        return {}


# --------------------------------------------------------------------------- #
# clocks during the timed region (NVML polling thread)                        #
# --------------------------------------------------------------------------- #
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, index):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(
                self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(
                    self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(
                    nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                break
            time.sleep(0.002)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._nv is not None:
            self._t.join()

    def summary(self):
        reasons = [n for b, n in _REASONS.items() if self.reasons & b and
                   n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples
                else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


# --------------------------------------------------------------------------- #
# the hot path over one layer (public API)                                    #
# --------------------------------------------------------------------------- #
class Batch:
    def __init__(self, dev, seed, layers):
        import torch
        from amass_kv_b200.attention import ensure_stage_b_buffers
        from amass_kv_b200.selection import QuadState
        from amass_kv_b200.workloads import c3_contexts, make_quad_case_gpu
        self.ctxs = c3_contexts(seed, N_REQ)
        b = make_quad_case_gpu(dev, seed=seed, ctxs=self.ctxs, n_kv=N_KV, G=G,
                               d=D, page=PAGE, r=RANK_Q, v_bits=V_BITS,
                               layers=layers)
        self.kv, self.q = b["kv_cache"], b["q"]
        self.bt, self.sl = b["block_table"], b["seq_lens"]
        self.MP, self.NB, self.layers = b["MP"], b["NB"], layers
        st = QuadState(dev, num_layers=1, num_blocks=1, n_kv=N_KV, G=G,
                       head_dim=D, page=PAGE, max_reqs=N_REQ, max_pages=self.MP,
                       rank=RANK_Q, budget=BUDGET, v_bits=V_BITS,
                       combine=COMBINE)
        # point the state's slabs at the generated multi-layer summaries
        st.quad_mu, st.mu_scale = b["quad_mu"], b["mu_scale"]
        st.quad_V, st.V_scale, st.quad_sig2 = (b["quad_V"], b["V_scale"],
                                               b["quad_sig2"])
        ensure_stage_b_buffers(st, dev, 128)
        self.st = st
        self.scale = 1.0 / math.sqrt(D)
        self.out = torch.empty(N_REQ, N_KV * G, D, dtype=torch.bfloat16,
                               device=dev)
        # derive, q-limbs, score, select, decode, merge
        self.launches_per_step = 6
        self.pps_min = None

    def stage(self, layer, k, q=None):
        """Stage k of the layer-step: 0 = derive + quad score, 1 = nrm fold +
        top-b select, 2 = split-K decode + merge."""
        from amass_kv_b200 import attention as A
        from amass_kv_b200 import selection as S
        st, l = self.st, layer
        q = self.q[l] if q is None else q
        nrm = COMBINE == "nrm"
        if k == 0:
            S.derive_page_params(st, self.sl, N_REQ)
            S._score_launch(st, l, q, self.bt, N_REQ, self.scale, nrm)
        elif k == 1:
            S.select_pages(st, N_REQ, from_score_h=nrm)
        else:
            A.sparse_paged_decode_batched_cuda(q, self.kv[l], self.bt, self.sl,
                                               st, self.out, scale=self.scale,
                                               pps_min=self.pps_min)

    def step(self, layer, q=None):
        for k in range(3):
            self.stage(layer, k, q)

    def algorithmic_bytes(self, layer):
        """Per-layer-step algorithmic bytes (summaries + block-table entries +
        selected K/V pages + q/out) and the per-kernel split."""
        self.step(layer)
        import torch
        torch.cuda.synchronize()
        nsh = np.maximum(self.st.n_sel_hi.cpu().numpy().astype(np.int64), 0)
        cnt = self.st.page_cnt.cpu().numpy().astype(np.int64)
        qo = N_REQ * N_KV * G * D * 2
        score_b = int((N_KV * nsh * B_SUM + 4 * nsh).sum()) + qo // 2
        kv_b = int(cnt.sum()) * 2 * PAGE * D * 2
        decode_b = kv_b + qo
        return dict(score=score_b, decode=decode_b,
                    total=score_b + kv_b + qo, pages=int(cnt.sum()),
                    mean_ctx=float(np.mean(self.ctxs)))


def run_gpu(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from amass_kv_b200 import _lib
    _lib.load()
    batch = Batch(dev, seed=1000 + rank, layers=args.layers)
    batch.pps_min = args.pps_min
    L = args.layers
    alg = [batch.algorithmic_bytes(l) for l in range(L)]

    # ---- CUDA-graph the per-layer step (the serving configuration) --------
    graphs = []
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for l in range(L):
            batch.step(l)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    if not args.no_graph:
        for l in range(L):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                batch.step(l)
            graphs.append(g)
        torch.cuda.synchronize()

    def one(i):
        if graphs:
            graphs[i % L].replay()
        else:
            batch.step(i % L)

    for i in range(args.warmup):
        one(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
        enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for i in range(args.steps):
            one(i)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / args.steps

    # ---- per-stage device time: each stage of a layer-step captured as its
    # own CUDA graph; graphs replayed back to back with events between them
    # on the launching stream (no host gaps inside the measured intervals) --
    stage_graphs = []
    for l in range(L):
        gs = []
        for k in range(3):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                batch.stage(l, k)
            gs.append(g)
        stage_graphs.append(gs)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)]
          for _ in range(args.steps)]
    for i in range(args.warmup):
        for g in stage_graphs[i % L]:
            g.replay()
    for i in range(args.steps):
        gs = stage_graphs[i % L]
        ev[i][0].record()
        for k in range(3):
            gs[k].replay()
            ev[i][k + 1].record()
    torch.cuda.synchronize()
    t_score = np.mean([e[0].elapsed_time(e[1]) for e in ev])
    t_select = np.mean([e[1].elapsed_time(e[2]) for e in ev])
    t_decode = np.mean([e[2].elapsed_time(e[3]) for e in ev])

    # ---- e2e through the public API with host buffers --------------------
    qh = torch.empty((L,) + tuple(batch.q.shape[1:]), dtype=torch.bfloat16,
                     pin_memory=True)
    qh.copy_(batch.q.cpu())
    slh = batch.sl.cpu().pin_memory()
    outh = torch.empty(tuple(batch.out.shape), dtype=torch.bfloat16,
                       pin_memory=True)
    qd = torch.empty_like(batch.q[0])
    h2d = qd.numel() * 2 + slh.numel() * 4
    d2h = outh.numel() * 2
    for i in range(args.warmup):
        qd.copy_(qh[i % L], non_blocking=True)
        batch.sl.copy_(slh, non_blocking=True)
        batch.step(i % L, q=qd)
        outh.copy_(batch.out, non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
        enable_timing=True)
    x0.record()
    for i in range(args.steps):
        qd.copy_(qh[i % L], non_blocking=True)
        batch.sl.copy_(slh, non_blocking=True)
        batch.step(i % L, q=qd)
        outh.copy_(batch.out, non_blocking=True)
    x1.record()
    torch.cuda.synchronize()
    e2e_ms = x0.elapsed_time(x1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    if rank == 0:
        peak, peak_kind = _peaks()
        a_score = np.mean([a["score"] for a in alg])
        a_decode = np.mean([a["decode"] for a in alg])
        a_total = np.mean([a["total"] for a in alg])
        kernels = {"derive+quad_score": (t_score, a_score),
                   "select": (t_select, 0.0),
                   "sparse_decode+merge": (t_decode, a_decode)}
        dom = max(kernels, key=lambda k: kernels[k][0])
        if kernels[dom][1] == 0:
            dom = "sparse_decode+merge"
        t_dom, b_dom = kernels[dom]
        ach = b_dom / (t_dom * 1e-3) / 1e9
        tr = _traffic_table().get(dom)
        traffic = None
        if tr:
            traffic = float(tr["bytes_per_alg_byte"]) * b_dom
        step_gbs = a_total / (ms_step * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(ms_step * 1e3, 2), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE C3 shapes)",
            "config": {
                "workload": "C3: ragged B=64 decode, ctx log-uniform 4K-64K "
                            f"(realized mean {alg[0]['mean_ctx']:.0f}), "
                            "Llama-3.1-8B attn (32q/8kv, d128, bf16, page 16),"
                            " quad r'=2 int4-V nrm, budget 0.05",
                "batch_per_gpu": N_REQ, "requests_per_step": N_REQ * world,
                "parallelism": f"sequence-sharded x{world}" if world > 1
                else "single GPU",
                "l2": f"inputs larger than L2: {L} layer slabs rotated "
                      f"(~{a_total / 1e6:.0f} MB algorithmic bytes each)",
                "cuda_graph": not args.no_graph,
                "selected_pages_per_step": alg[0]["pages"],
            },
            "step_roofline": {"bound": "hbm", "achieved": round(step_gbs, 1),
                              "peak": peak, "unit": "GB/s",
                              "frac": round(step_gbs / peak, 4),
                              "alg_bytes": int(a_total),
                              "peak_kind": peak_kind},
            "roofline": {"kernel": dom, "bound": "hbm",
                         "achieved": round(ach, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(ach / peak, 4),
                         "traffic": traffic, "alg_bytes": int(b_dom),
                         "peak_kind": peak_kind},
            "kernel_us": {k: round(v[0] * 1e3, 2) for k, v in kernels.items()},
            "e2e": {"value": round(e2e_ms / args.steps * 1e3, 2), "unit": UNIT,
                    "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": batch.launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(batch.ctxs)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# --------------------------------------------------------------------------- #
# CPU baseline: the oracle restatement of the reference algorithm             #
# --------------------------------------------------------------------------- #
def _oracle_worker(conn, ctx, seed):
    """Owns one request of the batch: builds it once, then runs the oracle
    layer-step (derive, quad score, nrm fold, top-b, decode) per request."""
    from amass_kv_b200.workloads import make_quad_case
    from oracle import amass_oracle as O
    case = make_quad_case(seed, n_req=1, n_kv=N_KV, G=G, d=D, ctxs=(ctx,),
                          r=RANK_Q, v_bits=V_BITS, heavy=4, shift=3.0)
    conn.send("ready")
    while conn.recv() == "go":
        t0 = time.perf_counter()
        O.quad_layer_step(case.q, case.mu, case.mu_s, case.Vq, case.V_s,
                          case.sig2, case.K, case.V, case.block_table,
                          case.seq_lens, scale=case.scale, page=PAGE, G=G,
                          r=RANK_Q, v_bits=V_BITS, MP=case.MP, sink=1,
                          window=1, combine=COMBINE, budget=BUDGET)
        conn.send(time.perf_counter() - t0)


class OraclePool:
    """`procs` worker processes, each pinned to one sampled request."""

    def __init__(self, ctxs, procs):
        import multiprocessing as mp
        cx = mp.get_context("spawn")
        self.sample = [int(c) for c in ctxs[:procs]]
        self.scale = float(np.sum(ctxs)) / float(np.sum(self.sample))
        self.conns, self.procs = [], []
        for i, c in enumerate(self.sample):
            a, b = cx.Pipe()
            p = cx.Process(target=_oracle_worker, args=(b, c, 77 + i),
                           daemon=True)
            p.start()
            self.conns.append(a)
            self.procs.append(p)
        for c in self.conns:
            assert c.recv() == "ready"

    def round(self):
        """One parallel layer-step over the sample; returns (wall s, value
        scaled to the whole batch in us/layer/step)."""
        t0 = time.perf_counter()
        for c in self.conns:
            c.send("go")
        for c in self.conns:
            c.recv()
        wall = time.perf_counter() - t0
        return wall, wall * self.scale * 1e6

    def close(self):
        for c in self.conns:
            c.send("stop")
        for p in self.procs:
            p.join(timeout=10)


def _n_procs():
    return max(1, min(os.cpu_count() or 1, 16))


def cpu_baseline(ctxs, rounds=3):
    procs = _n_procs()
    pool = OraclePool(ctxs, procs)
    try:
        pool.round()
        vals = [pool.round()[1] for _ in range(rounds)]
    finally:
        pool.close()
    return {"value": round(float(np.mean(vals)), 1), "unit": UNIT,
            "cores": procs, "kind": "port",
            "sample": f"{procs} of {len(ctxs)} requests (ctx "
                      f"{sum(pool.sample)} of {int(np.sum(ctxs))} tokens), one "
                      f"oracle process each, wall time x{pool.scale:.2f} "
                      f"(token ratio)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from amass_kv_b200.workloads import c3_contexts
    ctxs = c3_contexts(1000, N_REQ)
    procs = _n_procs()
    pool = OraclePool(ctxs, procs)
    try:
        for _ in range(args.warmup):
            pool.round()
        vals = [pool.round()[1] for _ in range(args.steps)]
    finally:
        pool.close()
    v = float(np.mean(vals))
    sample = (f"{procs} of {N_REQ} requests per step (ctx {sum(pool.sample)} "
              f"of {int(np.sum(ctxs))} tokens), one oracle process each, wall "
              f"time x{pool.scale:.2f} (token ratio)")
    line = {"metric": METRIC, "value": round(v, 1), "unit": UNIT,
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(v / 1e3, 3), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE C3 shapes)",
            "impl": "reference",
            "config": {"workload": "C3 (as the GPU arm); CPU oracle port of "
                       "the reference algorithm"},
            "cpu_baseline": {"value": round(v, 1), "unit": UNIT,
                             "cores": procs, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 1), "unit": UNIT,
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--impl", default="amass_b200",
                    choices=["amass_b200", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pps-min", type=int, default=None,
                    help="decode pages-per-chunk floor (default: by batch)")
    ap.add_argument("--requests", type=int, default=N_REQ,
                    help="batch size per GPU (64 = BASELINE C3; smaller only "
                         "for profiling captures)")
    args = ap.parse_args()
    globals()["N_REQ"] = args.requests
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
