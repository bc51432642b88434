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

Timing: `--repeats` back-to-back loops of exactly K graph-replayed steps,
CUDA events on the launching stream, the max over ranks per loop, the median
loop reported.  At N=1 the line also carries `parity` (the CPU oracle run on
layer 0 of the timed inputs, every request, compared with the GPU's pages and
output), the timed `cpu_baseline` of that oracle run, and `ctx32k` (every
context 32768 tokens).

Multi-GPU (torchrun, one process per GPU): the one 64-request batch is split
across the ranks by LPT on per-request algorithmic bytes (sequence sharding:
requests are independent, no collective on the data path; "scaling":
"strong"), with per-rank bytes and times; `layouts` adds the weak form (every
rank the full batch) and the kv-head-sharded form with its output gather.
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
SPLIT = 128                 # split-K partial slots per (request, kv-head)
QUAD_QIN_REQ = 32           # quad scorer splits q itself from this batch size
                            # (kQuadQinReq in csrc/quad_score.cu)
RANK_Q, V_BITS, BUDGET, COMBINE = 2, 4, 0.05, "nrm"
SCORER = "quad"                     # --scorer: quad (headline) or clse

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
    """Polls the SM clock and the clock-event reasons of the GPU behind
    torch device `device` (looked up by PCI bus id, so CUDA_VISIBLE_DEVICES
    renumbering cannot point it at another GPU); read-only NVML queries."""

    def __init__(self, device):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._lock = threading.Lock()
        try:
            import pynvml
            import torch
            props = torch.cuda.get_device_properties(device)
            bus = (f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:"
                   f"{props.pci_device_id:02x}.0")
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(
                self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def sample(self) -> bool:
        """One reading (also called from the launching thread between timed
        loops, where the sampler thread may not get the GIL while the host
        queues graph replays)."""
        nv = self._nv
        if nv is None:
            return False
        try:
            mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
            rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
        except Exception:
            return False
        with self._lock:
            self.samples.append(mhz)
            self.reasons |= rs
        return True

    def _run(self):
        while not self._stop.is_set():
            if not self.sample():
                break
            time.sleep(0.001)

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
    """One C3-shaped decode batch resident in HBM (``layers`` independent
    layer slabs) with its QuadState and Stage-B buffers.  ``ctxs`` is the
    batch's context lengths (default: the C3 draw of ``seed``)."""

    def __init__(self, dev, seed, layers, n_kv=None, gather=None, ctxs=None):
        import torch
        from amass_kv_b200.attention import ensure_stage_b_buffers
        from amass_kv_b200.selection import QuadState
        from amass_kv_b200.workloads import c3_contexts, make_quad_case_gpu
        n_kv = n_kv or N_KV
        self.n_kv, self.gather = n_kv, gather
        self.ctxs = np.asarray(c3_contexts(seed, N_REQ) if ctxs is None
                               else ctxs, dtype=np.int64)
        self.n_req = n_req = len(self.ctxs)
        b = make_quad_case_gpu(dev, seed=seed, ctxs=self.ctxs, n_kv=n_kv, G=G,
                               d=D, page=PAGE, r=RANK_Q, v_bits=V_BITS,
                               layers=layers)
        self.kv, self.q = b["kv_cache"], b["q"]
        self.bt, self.sl = b["block_table"], b["seq_lens"]
        self.MP, self.NB, self.layers = b["MP"], b["NB"], layers
        st = QuadState(dev, num_layers=1, num_blocks=1, n_kv=n_kv, G=G,
                       head_dim=D, page=PAGE, max_reqs=n_req, max_pages=self.MP,
                       rank=RANK_Q, budget=BUDGET, v_bits=V_BITS,
                       combine=COMBINE)
        # point the state's slabs at the generated multi-layer summaries
        st.quad_mu, st.mu_scale = b["quad_mu"], b["mu_scale"]
        st.quad_V, st.V_scale, st.quad_sig2 = (b["quad_V"], b["V_scale"],
                                               b["quad_sig2"])
        self.clse = SCORER == "clse"
        if self.clse:
            # CLSE extras of the same blocks: int4 rank-2 token coordinates
            # (one byte per token), per-token fp16 scales, residual energy
            gd = torch.Generator(device=dev).manual_seed(seed + 7)
            Lx, NBx = b["quad_mu"].shape[0], b["quad_mu"].shape[1]
            st.quad_c = torch.randint(-128, 128, (Lx, NBx, n_kv, PAGE, 1),
                                      generator=gd, device=dev,
                                      dtype=torch.int8)
            st.c_scale = (torch.rand((Lx, NBx, n_kv, PAGE), generator=gd,
                                     device=dev) * 0.05 + 0.01).half()
            st.quad_resid = (torch.rand((Lx, NBx, n_kv), generator=gd,
                                        device=dev) * 50 + 10).half()
            st.c_bits, st.c_grain = 4, "token"
        ensure_stage_b_buffers(st, dev, SPLIT)
        self.st = st
        self.scale = 1.0 / math.sqrt(D)
        self.out = torch.empty(n_req, n_kv * G, D, dtype=torch.bfloat16,
                               device=dev)
        # stage 0 = derive + score, 1 = nrm fold + select, 2 = split-K
        # decode + merge
        self.stages = (0, 1, 2)
        self.stage_names = {0: "derive+quad_score", 1: "select",
                            2: "sparse_decode+merge"}
        # quad: score (q limbs and derive inside it from 32 requests up,
        # else a q-limb launch before it), select, decode, merge; CLSE:
        # derive, q-limbs, score, select, decode, merge
        self.launches_per_step = 6 if self.clse else \
            (4 if n_req >= QUAD_QIN_REQ else 5)
        self.pps_min = None

    def stage(self, layer, k, q=None):
        """Stage k of the layer-step: 0 = derive + quad score, 1 = nrm fold +
        top-b select, 2 = split-K decode + merge."""
        from amass_kv_b200 import attention as A
        from amass_kv_b200 import selection as S
        st, l, n = self.st, layer, self.n_req
        q = self.q[l] if q is None else q
        nrm = COMBINE == "nrm"
        if k == 0:
            if self.clse:
                S.derive_page_params(st, self.sl, n)
                S.clse_score_cuda(st, l, q, self.bt, self.sl, n, self.scale)
            else:
                S._score_launch(st, l, q, self.bt, n, self.scale, nrm,
                                seq_lens=self.sl)
        elif k == 1:
            S.select_pages(st, n, from_score_h=nrm)
        elif self.gather is not None:
            from amass_kv_b200 import sharding as SH
            self.out_full = SH.sparse_paged_decode_kvsharded(
                q, self.kv[l], self.bt, self.sl, st, self.gather,
                scale=self.scale, pps_min=self.pps_min)
        else:
            A.sparse_paged_decode_batched_cuda(q, self.kv[l], self.bt, self.sl,
                                               st, self.out, scale=self.scale,
                                               pps_min=self.pps_min)

    def step(self, layer, q=None):
        for k in self.stages:
            self.stage(layer, k, q)

    def algorithmic_bytes(self, layer):
        """Per-layer-step algorithmic bytes (summaries + block-table entries +
        selected K/V pages + q/out) and the per-kernel split."""
        self.step(layer)
        import torch
        torch.cuda.synchronize()
        nsh = np.maximum(self.st.n_sel_hi.cpu().numpy().astype(np.int64), 0)
        cnt = self.st.page_cnt.cpu().numpy().astype(np.int64)
        qo = self.n_req * self.n_kv * G * D * 2
        b_sum = B_SUM + (PAGE * 1 + 2 * PAGE + 2 if self.clse else 0)
        score_b = int((self.n_kv * nsh * b_sum + 4 * nsh).sum()) + qo // 2
        kv_b = int(cnt.sum()) * 2 * PAGE * D * 2
        decode_b = kv_b + qo
        return dict(score=score_b, decode=decode_b,
                    total=score_b + kv_b + qo, pages=int(cnt.sum()),
                    mean_ctx=float(np.mean(self.ctxs)))

    def capture(self, cap_mode, stages=None):
        """One CUDA graph per layer of the given stages (eager warm-up of every
        layer on a side stream first: kernel attributes are set outside
        capture)."""
        import torch
        stages = self.stages if stages is None else stages
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for l in range(self.layers):
                for k in stages:
                    self.stage(l, k)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graphs = []
        for l in range(self.layers):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode=cap_mode):
                for k in stages:
                    self.stage(l, k)
            graphs.append(g)
        torch.cuda.synchronize()
        return graphs


def _timed_repeats(run_one, steps, repeats, world, dev, clk_index=None):
    """`repeats` back-to-back timed loops of exactly `steps` steps each (CUDA
    events on the launching stream, barrier + synchronize around the whole
    region); returns (per-repeat ms/step as the max over ranks, clock
    summary or None)."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(repeats)]
    clk = ClockSampler(dev) if clk_index is not None else None
    if clk is not None:
        clk.__enter__()
    i = 0
    for e0, e1 in ev:
        e0.record()
        for _ in range(steps):
            run_one(i)
            i += 1
        e1.record()
        if clk is not None:
            clk.sample()      # between loops: outside every timed interval
    if clk is not None:
        # wait with the GIL released so the sampler thread runs while the
        # queued steps execute
        while not ev[-1][1].query():
            time.sleep(0.0005)
    torch.cuda.synchronize()
    if clk is not None:
        clk.__exit__(None, None, None)
    ms = torch.tensor([e0.elapsed_time(e1) / steps for e0, e1 in ev],
                      dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
    return ms.cpu().tolist(), (clk.summary() if clk is not None else None)


def _stage_times(batch, cap_mode, steps, warmup):
    """Per-stage device time: each stage of a layer-step captured as its own
    CUDA graph, graphs replayed back to back with events between them on the
    launching stream (no host gaps inside the measured intervals); and the
    marginal cost of each stage inside the whole step (prefix graphs of the
    first 1, 2, ... stages).  Returns {stage: ms} twice."""
    import torch
    L, ks = batch.layers, batch.stages
    nk = len(ks)
    stage_graphs = [[None] * nk for _ in range(L)]
    for l in range(L):
        for j, k in enumerate(ks):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode=cap_mode):
                batch.stage(l, k)
            stage_graphs[l][j] = g
    prefix = [batch.capture(cap_mode, stages=ks[:j + 1]) for j in range(nk)]
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)]
          for _ in range(steps)]
    for i in range(warmup):
        for g in stage_graphs[i % L]:
            g.replay()
    for i in range(steps):
        gs = stage_graphs[i % L]
        ev[i][0].record()
        for j in range(nk):
            gs[j].replay()
            ev[i][j + 1].record()
    torch.cuda.synchronize()
    iso = {k: float(np.mean([e[j].elapsed_time(e[j + 1]) for e in ev]))
           for j, k in enumerate(ks)}
    pref = []
    for gs in prefix:
        for i in range(warmup):
            gs[i % L].replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
            enable_timing=True)
        e0.record()
        for i in range(steps):
            gs[i % L].replay()
        e1.record()
        torch.cuda.synchronize()
        pref.append(e0.elapsed_time(e1) / steps)
    marg = {k: pref[j] - (pref[j - 1] if j else 0.0) for j, k in enumerate(ks)}
    return iso, marg


def _measure_c3(batch, args, world, dev, cap_mode, clocks=False):
    """Graph-replayed layer-steps of `batch`: median (over repeats) of the
    max-over-ranks ms/step, all repeats, clocks."""
    import torch
    graphs = batch.capture(cap_mode)
    L = batch.layers

    def one(i):
        graphs[i % L].replay()

    for i in range(args.warmup):
        one(i)
    reps, clk = _timed_repeats(one, args.steps, args.repeats, world, dev,
                               clk_index=dev if clocks else None)
    del graphs
    torch.cuda.synchronize()
    return float(statistics.median(reps)), reps, clk


def _roofline(batch, alg, t_stage_ms, peak, peak_kind):
    """The dominant stage's algorithmic bytes over its live time."""
    a_score = np.mean([a["score"] for a in alg])
    a_decode = np.mean([a["decode"] for a in alg])
    bytes_of = {0: a_score, 1: 0.0, 2: a_decode}
    kernels = {batch.stage_names[k]: (t_stage_ms[k], bytes_of[k])
               for k in batch.stages}
    dom = max(kernels, key=lambda k: kernels[k][0])
    if kernels[dom][1] == 0:
        dom = "sparse_decode+merge"
    t_dom, b_dom = kernels[dom]
    ach = b_dom / (t_dom * 1e-3) / 1e9
    tr = _traffic_table().get(dom)
    traffic = float(tr["bytes_per_alg_byte"]) * b_dom if tr else None
    return kernels, {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                     "traffic": traffic, "alg_bytes": int(b_dom),
                     "peak_kind": peak_kind}


def _e2e(batch, args, world, dev):
    """The public serving API (pipeline.StepPipeline) with pinned host
    buffers: every step uploads q + seq_lens and downloads the output."""
    import torch
    import torch.distributed as dist
    from amass_kv_b200.pipeline import StepPipeline
    L = batch.layers
    qh = torch.empty((L,) + tuple(batch.q.shape[1:]), dtype=torch.bfloat16,
                     pin_memory=True)
    qh.copy_(batch.q.cpu())
    slh = batch.sl.cpu().pin_memory()
    outh = torch.empty(tuple(batch.out.shape), dtype=torch.bfloat16,
                       pin_memory=True)
    h2d = qh[0].numel() * 2 + slh.numel() * 4
    d2h = outh.numel() * 2
    pipe = StepPipeline(batch.st, [batch.kv[l] for l in range(L)], batch.bt,
                        n_req=batch.n_req, scale=batch.scale,
                        q_shape=tuple(batch.q.shape[1:]), device=dev,
                        scorer="clse" if batch.clse else "quad")
    for i in range(args.warmup):
        pipe.submit(i % L, qh[i % L], slh, outh)
    pipe.synchronize()
    if world > 1:
        dist.barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
        enable_timing=True)
    x0.record()
    pipe.h2d.wait_stream(torch.cuda.current_stream())
    for i in range(args.steps):
        pipe.submit(i % L, qh[i % L], slh, outh)
    torch.cuda.current_stream().wait_stream(pipe.d2h)
    x1.record()
    torch.cuda.synchronize()
    ms = x0.elapsed_time(x1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": round(ms / args.steps * 1e3, 2), "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}


def _kv_layout(args, world, rank, dev):
    """KV-head-sharded layout of the same 64-request batch: rank g owns
    n_kv/world kv heads of every request, the merge kernel stores each
    merged row into every rank's output over NVLink (p2p) or NCCL gathers.
    Returns the max-over-ranks step time and, per rank, the stage times
    with the gather and with a local-only output (their difference is the
    exchange's cost)."""
    import torch
    import torch.distributed as dist
    from amass_kv_b200 import sharding as SH
    gather = SH.HeadGather(N_REQ, N_KV * G, D, device=dev, mode=args.gather)
    cap = "thread_local" if args.gather == "nccl" else "global"
    batch = Batch(dev, seed=1000, layers=args.layers, n_kv=N_KV // world,
                  gather=gather)
    batch.pps_min = args.pps_min
    alg = [batch.algorithmic_bytes(l) for l in range(batch.layers)]
    med, reps, _ = _measure_c3(batch, args, world, dev, cap)
    iso_g, _ = _stage_times(batch, cap, args.steps, args.warmup)
    batch.gather = None                       # local output only
    iso_l, _ = _stage_times(batch, cap, args.steps, args.warmup)
    mine = {"rank": rank, "kv_heads": N_KV // world,
            "alg_bytes": int(np.mean([a["total"] for a in alg])),
            "decode_merge_gather_us": round(iso_g[2] * 1e3, 2),
            "decode_merge_local_us": round(iso_l[2] * 1e3, 2),
            "stage_us": {batch.stage_names[k]: round(v * 1e3, 2)
                         for k, v in iso_g.items()}}
    per = [None] * world
    dist.all_gather_object(per, mine)
    res = {"value": round(med * 1e3, 2), "unit": UNIT,
           "gather": args.gather, "repeats_us": [round(x * 1e3, 2)
                                                 for x in reps],
           "per_rank": per,
           "gather_us_rank_max": round(max(p["decode_merge_gather_us"] -
                                           p["decode_merge_local_us"]
                                           for p in per), 2)}
    del batch
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return res


def run_gpu(args):
    import torch
    import torch.distributed as dist
    from amass_kv_b200 import sharding as SH
    from amass_kv_b200.workloads import c3_contexts
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from amass_kv_b200 import _lib
    _lib.load()
    peak, peak_kind = _peaks()

    # ---- the C3 batch, partitioned across the ranks by sequence (LPT on
    # per-request algorithmic bytes): strong scaling, no collective -------
    ctxs = np.asarray(c3_contexts(1000, N_REQ), dtype=np.int64)
    costs = SH.request_bytes(ctxs, n_kv=N_KV, page=PAGE, budget=BUDGET,
                             b_sum=B_SUM, d=D, G=G)
    parts = SH.lpt_partition(costs, world)
    mine = parts[rank]
    batch = Batch(dev, seed=1000 + (rank if world > 1 else 0),
                  layers=args.layers, ctxs=ctxs[mine])
    batch.pps_min = args.pps_min
    L = batch.layers
    alg = [batch.algorithmic_bytes(l) for l in range(L)]
    med, reps, clk = _measure_c3(batch, args, world, dev, "global",
                                 clocks=True)
    iso, marg = _stage_times(batch, "global", args.steps, args.warmup)
    # this rank's own median step time (not max-over-ranks): limiter view
    own = med if world == 1 else _measure_c3(batch, args, 1, dev,
                                             "global")[0]
    e2e = _e2e(batch, args, world, dev)
    kernels, roof = _roofline(batch, alg, iso, peak, peak_kind)
    a_total = float(np.mean([a["total"] for a in alg]))
    rank_info = {"rank": rank, "requests": len(mine),
                 "ctx_tokens": int(ctxs[mine].sum()),
                 "alg_bytes": int(a_total), "own_us": round(own * 1e3, 2),
                 "stage_us": {batch.stage_names[k]: round(v * 1e3, 2)
                              for k, v in iso.items()}}
    per_rank = [rank_info]
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, rank_info)
    tot_bytes = sum(p["alg_bytes"] for p in per_rank)
    job_gbs = tot_bytes / (med * 1e-3) / 1e9

    launches = batch_launches(batch, args)
    import ctypes
    n_pipe = ctypes.c_longlong(0)
    _lib.call("amass_quad_pipeline_status", None, ctypes.addressof(n_pipe), 0)
    quad_kernel = ("quad_score_pipe_kernel (bulk-copy ring)" if n_pipe.value
                   else "quad_score_kernel (register pipeline)")
    names = dict(batch.stage_names)
    parity = cpu = None
    ctx32 = score_layout = None
    if world == 1:
        if not args.no_cpu_baseline:
            parity, cpu = _oracle_check(batch)
        if not args.no_ctx32k:
            ctx32 = _ctx32k(args, dev, peak, peak_kind)
        if not args.no_score_layout and not batch.clse:
            score_layout = _score_layout(batch, args, peak)
    # secondary layouts at N > 1: the same batch replicated on every rank
    # (weak scaling, identical per-rank work) and the kv-head-sharded form
    layouts = None
    if world > 1 and not args.no_layouts:
        del batch
        torch.cuda.empty_cache()
        wb = Batch(dev, seed=1000, layers=args.layers)
        wb.pps_min = args.pps_min
        w_alg = float(np.mean([wb.algorithmic_bytes(l)["total"]
                               for l in range(wb.layers)]))
        w_med, w_reps, _ = _measure_c3(wb, args, world, dev, "global")
        del wb
        torch.cuda.empty_cache()
        layouts = {
            "seq_weak": {"value": round(w_med * 1e3, 2), "unit": UNIT,
                         "note": "every rank the full 64-request C3 batch "
                                 "(same seed: identical per-rank work)",
                         "requests_per_step": N_REQ * world,
                         "job_gbs": round(world * w_alg / (w_med * 1e-3)
                                          / 1e9, 1)},
            "kv": _kv_layout(args, world, rank, dev),
        }

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(med * 1e3, 2), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(med, 5), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE C3 shapes)",
            "config": {
                "workload": "C3: ragged B=64 decode, ctx log-uniform 4K-64K "
                            f"(realized mean {float(np.mean(ctxs)):.0f}), "
                            "Llama-3.1-8B attn (32q/8kv, d128, bf16, page 16),"
                            + (" clse r'=2 int4-V int4 token coords nrm"
                               if SCORER == "clse" else " quad r'=2 int4-V nrm")
                            + ", budget 0.05",
                "requests_per_step": N_REQ,
                "parallelism": (f"sequence-sharded x{world} (one 64-request "
                                "batch split by LPT on per-request bytes)"
                                if world > 1 else "single GPU"),
                "l2": f"inputs larger than L2: {L} layer slabs rotated "
                      f"(~{a_total / 1e6:.0f} MB algorithmic bytes each on "
                      "rank 0)",
                "cuda_graph": True,
                "timing": f"median of {args.repeats} timed loops of "
                          f"{args.steps} steps (max over ranks per loop)",
                "selected_pages_per_step": int(alg[0]["pages"]),
                "quad_scorer": None if SCORER == "clse" else quad_kernel,
            },
            "repeats_us": [round(x * 1e3, 2) for x in reps],
            "step_roofline": {"bound": "hbm", "achieved": round(job_gbs, 1),
                              "peak": round(peak * world, 1), "unit": "GB/s",
                              "frac": round(job_gbs / (peak * world), 4),
                              "alg_bytes": int(tot_bytes),
                              "peak_kind": peak_kind,
                              "note": "all ranks' algorithmic bytes / the "
                                      "max-over-ranks step time / (N x peak)"},
            "roofline": roof,
            "kernel_us": {k: round(v[0] * 1e3, 2) for k, v in kernels.items()},
            "marginal_us": {names[k]: round(v * 1e3, 2)
                            for k, v in marg.items()},
            "per_rank": per_rank,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk,
        }
        if world > 1:
            lim = max(per_rank, key=lambda p: p["own_us"])
            line["limiter"] = {
                "rank": lim["rank"], "own_us": lim["own_us"],
                "stage": max(lim["stage_us"], key=lim["stage_us"].get),
                "bytes_imbalance": round(max(p["alg_bytes"] for p in per_rank)
                                         / (tot_bytes / world), 4)}
        if layouts:
            line["layouts"] = layouts
        if ctx32 is not None:
            line["ctx32k"] = ctx32
        if score_layout is not None:
            line["score_layout"] = score_layout
        if parity is not None:
            line["parity"] = parity
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
        if parity is not None and not parity["ok"]:
            sys.stderr.write("PARITY MISS against the CPU oracle\n")
            sys.stdout.flush()
            os._exit(3)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


def _score_layout(batch, args, peak):
    """What bounds the quad scorer: the batch's scoring stage (derive + quad
    score) timed on its own with the batch's block table (each request's
    blocks drawn from one random permutation of the pool, as a long-running
    paged cache leaves them) and again with each request's blocks contiguous
    in the same pool.  Same requests, pages and bytes; only the addresses of
    the 1 KB per-block summary rows change.  Device time, CUDA graphs."""
    import torch
    n = batch.n_req
    npg = [(int(c) + PAGE - 1) // PAGE for c in batch.ctxs]
    contig = torch.zeros_like(batch.bt)
    o = 0
    for i, m in enumerate(npg):
        contig[i, :m] = torch.arange(o, o + m, dtype=torch.int32,
                                     device=contig.device)
        o += m
    sb = float(np.mean([batch.algorithmic_bytes(l)["score"]
                        for l in range(batch.layers)]))
    orig = batch.bt
    out = {}
    try:
        for name, bt in (("random", orig), ("contiguous", contig)):
            batch.bt = bt
            gs = batch.capture("global", stages=(0,))
            for i in range(args.warmup):
                gs[i % batch.layers].replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(args.steps):
                gs[i % batch.layers].replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / args.steps * 1e3
            out[name] = {"us": round(us, 2),
                         "gbs": round(sb / (us * 1e-6) / 1e9, 1),
                         "frac": round(sb / (us * 1e-6) / 1e9 / peak, 4)}
            del gs
    finally:
        batch.bt = orig
    out["score_bytes"] = int(sb)
    out["note"] = ("derive + quad score of the timed batch, block table as "
                   "timed (random) vs each request's blocks contiguous; same "
                   "pages and bytes")
    return out


def batch_launches(batch, args):
    return batch.launches_per_step * args.steps * args.repeats


def _ctx32k(args, dev, peak, peak_kind):
    """The metric's literal shape: 64 requests, every context 32768 tokens
    (2048 pages), same geometry and budget; device time only."""
    import torch
    layers = 2                     # 2 x ~0.7 GB algorithmic: far above L2
    b = Batch(dev, seed=1032, layers=layers, ctxs=[32768] * N_REQ)
    b.pps_min = args.pps_min
    alg = float(np.mean([b.algorithmic_bytes(l)["total"]
                         for l in range(layers)]))
    med, reps, _ = _measure_c3(b, args, 1, dev, "global")
    del b
    torch.cuda.empty_cache()
    gbs = alg / (med * 1e-3) / 1e9
    return {"value": round(med * 1e3, 2), "unit": UNIT,
            "config": "B=64, every ctx 32768, otherwise as the headline",
            "step_roofline": {"achieved": round(gbs, 1), "peak": peak,
                              "frac": round(gbs / peak, 4),
                              "alg_bytes": int(alg), "peak_kind": peak_kind}}


# --------------------------------------------------------------------------- #
# CPU side: the oracle restatement of the reference algorithm, run on the     #
# GPU arm's own inputs (the parity check and the timed CPU baseline)          #
# --------------------------------------------------------------------------- #
_POOL_REQS = None     # per-request host inputs, inherited by forked workers


def host_requests(batch, layer=0):
    """Per-request numpy inputs of `batch` (layer `layer`) in the oracle's
    conventions, each request with its own blocks renumbered 0..npg-1:
    q (H, d) f32; K, V as bf16 bits (npg, page, n_kv, d) uint16; the quad
    summaries of those blocks; seq_len."""
    import torch
    reqs = []
    kv, st = batch.kv[layer], batch.st
    for r in range(batch.n_req):
        sl = int(batch.ctxs[r])
        npg = -(-sl // PAGE)
        blk = batch.bt[r, :npg].long()
        kvr = kv.index_select(0, blk).view(torch.int16).cpu().numpy()
        reqs.append(dict(
            r=r, sl=sl, npg=npg,
            q=batch.q[layer][r].float().cpu().numpy(),
            K=kvr[:, 0].view(np.uint16), V=kvr[:, 1].view(np.uint16),
            mu=st.quad_mu[layer].index_select(0, blk).cpu().numpy(),
            mu_s=st.mu_scale[layer].index_select(0, blk).cpu().numpy(),
            Vq=st.quad_V[layer].index_select(0, blk).cpu().numpy(),
            V_s=st.V_scale[layer].index_select(0, blk).cpu().numpy(),
            sig2=st.quad_sig2[layer].index_select(0, blk).cpu().numpy()))
    return reqs


def _bits_f32(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def _oracle_worker(conn, owned):
    """Forked worker: owns requests `owned` of the inherited _POOL_REQS and
    runs the oracle layer-step (derive, quad score, nrm fold, top-b, decode)
    on them per "go"; "check" also returns the oracle's decode over the GPU's
    page tables."""
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(1)
    except Exception:
        pass
    from oracle import amass_oracle as O
    mine = []
    for i in owned:
        x = dict(_POOL_REQS[i])
        x["K"], x["V"] = _bits_f32(x["K"]), _bits_f32(x["V"])
        x["bt"] = np.arange(x["npg"], dtype=np.int32)[None]
        x["sla"] = np.array([x["sl"]], dtype=np.int32)
        mine.append(x)
    conn.send("ready")

    def step(x):
        return O.quad_layer_step(
            x["q"][None], x["mu"], x["mu_s"], x["Vq"], x["V_s"], x["sig2"],
            x["K"], x["V"], x["bt"], x["sla"], scale=1.0 / math.sqrt(D),
            page=PAGE, G=G, r=RANK_Q, v_bits=V_BITS, MP=x["npg"], sink=1,
            window=1, combine=COMBINE, budget=BUDGET)

    while True:
        msg = conn.recv()
        if msg == "stop":
            break
        if msg == "go":
            t0 = time.perf_counter()
            for x in mine:
                step(x)
            conn.send(time.perf_counter() - t0)
        elif msg[0] == "check":
            gpu = msg[1]
            res = {}
            for x in mine:
                o = step(x)
                tab, cnt = gpu[x["r"]]
                od = O.sparse_decode(x["q"][None], x["K"], x["V"], x["bt"],
                                     x["sla"], tab[None], cnt[None],
                                     scale=1.0 / math.sqrt(D), G=G)
                res[x["r"]] = (o["page_table"][0], o["page_cnt"][0],
                               o["score"][0], od[0])
            conn.send(res)


class OraclePool:
    """Forked CPU workers over the whole batch: requests assigned by LPT on
    context length, one process per host core used.  Every round runs every
    request of the batch once (no sampling, no extrapolation)."""

    def __init__(self, reqs, procs):
        import multiprocessing as mp
        global _POOL_REQS
        _POOL_REQS = reqs
        from amass_kv_b200.sharding import lpt_partition
        procs = max(1, min(procs, len(reqs)))
        self.parts = [p for p in lpt_partition([x["sl"] for x in reqs], procs)
                      if p]
        self.procs_n = len(self.parts)
        cx = mp.get_context("fork")
        self.conns, self.procs = [], []
        for owned in self.parts:
            a, b = cx.Pipe()
            p = cx.Process(target=_oracle_worker, args=(b, owned), daemon=True)
            p.start()
            self.conns.append(a)
            self.procs.append(p)
        for c in self.conns:
            assert c.recv() == "ready"
        _POOL_REQS = None

    def round(self):
        """One parallel layer-step over the whole batch; wall seconds."""
        t0 = time.perf_counter()
        for c in self.conns:
            c.send("go")
        for c in self.conns:
            c.recv()
        return time.perf_counter() - t0

    def check(self, gpu_tabs):
        for c in self.conns:
            c.send(("check", gpu_tabs))
        res = {}
        for c in self.conns:
            res.update(c.recv())
        return res

    def close(self):
        for c in self.conns:
            c.send("stop")
        for p in self.procs:
            p.join(timeout=30)


def _n_procs():
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except Exception:
        return max(1, os.cpu_count() or 1)


def _oracle_check(batch, rounds=2):
    """Runs the oracle on the GPU arm's own layer-0 inputs for every request
    of the batch: times `rounds` whole-batch layer-steps (the cpu_baseline)
    and checks the GPU's selection (identical up to the 1e-3 threshold tie
    band) and output (max-abs 2e-2 / rel 1e-2 of the fp32 decode over the
    GPU's pages)."""
    import torch
    from oracle import amass_oracle as O
    batch.step(0)
    torch.cuda.synchronize()
    tab = batch.st.page_table.cpu().numpy()
    cnt = batch.st.page_cnt.cpu().numpy()
    out = batch.out.float().cpu().numpy()
    reqs = host_requests(batch, 0)
    pool = OraclePool(reqs, _n_procs())
    del reqs
    try:
        pool.round()                                   # warm-up
        walls = [pool.round() for _ in range(rounds)]
        gpu_tabs = {r: (tab[r][:, :-(-int(batch.ctxs[r]) // PAGE)], cnt[r])
                    for r in range(batch.n_req)}
        res = pool.check(gpu_tabs)
    finally:
        pool.close()
    sel_ok, out_ok, worst = True, True, 0.0
    bad = []
    for r in range(batch.n_req):
        otab, ocnt, osc, od = res[r]
        npg = otab.shape[-1]
        sc = np.where(np.isnan(osc), -np.inf, osc)
        s_ok = O.selection_diff_ok(tab[r][None, :, :npg], cnt[r][None],
                                   otab[None], ocnt[None], sc[None])
        err = np.abs(out[r] - od)
        o_ok = bool(np.all(err <= 2e-2 + 1e-2 * np.abs(od)))
        worst = max(worst, float(err.max()))
        if not (s_ok and o_ok):
            bad.append(r)
        sel_ok &= s_ok
        out_ok &= o_ok
    parity = {"ok": bool(sel_ok and out_ok), "requests_checked": batch.n_req,
              "selection_ok": bool(sel_ok), "output_ok": bool(out_ok),
              "max_abs_err": round(worst, 5), "bad_requests": bad[:8],
              "bar": "pages identical except ties within 1e-3 of the "
                     "threshold; output max-abs 2e-2 + rel 1e-2 of the fp32 "
                     "oracle decode over the GPU's pages",
              "inputs": "layer 0 of the timed batch, copied from HBM"}
    cpu = {"value": round(float(np.mean(walls)) * 1e6, 1), "unit": UNIT,
           "cores": pool.procs_n, "kind": "port",
           "sample": f"the whole {batch.n_req}-request batch (layer 0 of the "
                     f"timed inputs) per layer-step, {pool.procs_n} forked "
                     f"oracle processes (LPT by context), mean of {rounds} "
                     "timed rounds after one warm-up"}
    return parity, cpu


def run_reference(args):
    """The reference arm: the reference algorithm's CPU restatement (the
    oracle port) on the box's host cores over the whole C3 batch each step,
    on exactly the GPU arm's N=1 inputs (generated on the GPU the same way,
    copied to host before any timing)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    batch = Batch(dev, seed=1000, layers=args.layers)
    reqs = host_requests(batch, 0)
    n_req, mean_ctx = batch.n_req, float(np.mean(batch.ctxs))
    del batch
    torch.cuda.empty_cache()
    pool = OraclePool(reqs, _n_procs())
    del reqs
    try:
        for _ in range(args.warmup):
            pool.round()
        walls = [pool.round() for _ in range(args.steps)]
    finally:
        pool.close()
    v = float(np.mean(walls)) * 1e6
    sample = (f"the whole {n_req}-request batch every step (no sampling), "
              f"{pool.procs_n} forked oracle processes (LPT by context)")
    line = {"metric": METRIC, "value": round(v, 1), "unit": UNIT,
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(v / 1e3, 3), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE C3 shapes)",
            "impl": "reference",
            "config": {"workload": "C3 as the GPU arm at N=1 (realized mean "
                       f"ctx {mean_ctx:.0f}); the CPU oracle port of the "
                       "reference algorithm on the identical inputs",
                       "timed_region_s": round(float(np.sum(walls)), 2)},
            "cpu_baseline": {"value": round(v, 1), "unit": UNIT,
                             "cores": pool.procs_n, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 1), "unit": UNIT,
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)

# --------------------------------------------------------------------------- #
# C5: mem-v tiered decode (V in the pinned host pool, exact-LRU hot buffer)  #
# --------------------------------------------------------------------------- #
C5_REQ, C5_KV, C5_G = 16, 8, 8


def run_c5(args):
    """BASELINE C5: Llama-3.1-70B attention (64 q / 8 kv heads, d 128), B=16,
    contexts uniform on [32K, 128K], V of every page in the pinned mapped host
    pool, K and summaries in HBM, hot buffer of 10% of the pages per kv-head
    (capped at 8192 slots), budget 0.05, q rotating slowly so the selection
    drifts.  A step = derive + quad score + select + residency plan + miss
    fetch + ptr-select decode + merge for one layer; it is timed stage by
    stage (CUDA graphs, events between them) after `--warmup` steps that
    bring the hot buffer to its steady hit rate."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from amass_kv_b200 import attention as A
    from amass_kv_b200 import selection as S
    from amass_kv_b200 import tier as T
    from amass_kv_b200.attention import ensure_stage_b_buffers
    from amass_kv_b200.selection import QuadState
    from amass_kv_b200.workloads import make_quad_case_gpu
    n5 = args.batch or C5_REQ
    rng = np.random.default_rng(5000 + rank)
    ctxs = rng.integers(32768, 131072 + 1, n5)
    b = make_quad_case_gpu(dev, seed=5000 + rank, ctxs=ctxs, n_kv=C5_KV,
                           G=C5_G, d=D, page=PAGE, r=RANK_Q, v_bits=V_BITS,
                           layers=1)
    NB, MP = b["NB"], b["MP"]
    kv, bt, sl = b["kv_cache"][0], b["block_table"], b["seq_lens"]
    st = QuadState(dev, num_layers=1, num_blocks=1, n_kv=C5_KV, G=C5_G,
                   head_dim=D, page=PAGE, max_reqs=n5, max_pages=MP,
                   rank=RANK_Q, budget=BUDGET, v_bits=V_BITS, combine=COMBINE)
    st.quad_mu, st.mu_scale = b["quad_mu"], b["mu_scale"]
    st.quad_V, st.V_scale, st.quad_sig2 = (b["quad_V"], b["V_scale"],
                                           b["quad_sig2"])
    ensure_stage_b_buffers(st, dev, SPLIT)
    hot_slots = min(8192, max(1, int(round(0.10 * NB))))
    n_vslots = 2 * n5
    tier = T.Tier(num_layers=1, num_blocks=NB, n_kv=C5_KV, page=PAGE, d=D,
                  hot_slots=hot_slots, max_reqs=n5, max_pages=MP,
                  n_vslots=n_vslots, device=dev)
    # every page flushed to the pinned pool; the resident V half stays only
    # for the resident-decode comparison
    vt = kv[:, 1].permute(0, 2, 1, 3).contiguous()
    tier.pool.host[0].copy_(vt.cpu())
    del vt
    tier.residency.pool_valid.fill_(1)
    kv_k_only = kv[:, :1]                     # K-only (nb, 1, page, kv, d)
    scale = 1.0 / math.sqrt(D)
    q0 = b["q"][0].float()
    q1 = torch.randn_like(q0)
    qbuf = torch.empty_like(b["q"][0])
    out = torch.empty_like(qbuf)
    out_res = torch.empty_like(qbuf)

    def set_q(i):
        th = 0.02 * i
        qbuf.copy_((q0 * math.cos(th) + q1 * math.sin(th)).to(torch.bfloat16))

    r5 = tier.residency

    def stage(k):
        if k == 0:
            S._score_launch(st, 0, qbuf, bt, n5, scale, COMBINE == "nrm",
                            seq_lens=sl)
        elif k == 1:
            S.select_pages(st, n5, from_score_h=COMBINE == "nrm")
        elif k == 2:
            r5.gather_plan(0, st.page_table, st.page_cnt, bt, sl, n5)
        elif k == 3:
            r5.gather_fetch(0, tier.staging, tier.pool.dev_view)
        elif k == 4:
            T.mem_decode_ptrsel(qbuf, kv_k_only, bt, sl, st, out, tier, 0,
                                scale=scale, entry_slots=r5.miss_pages)
        elif k == 5:
            A.sparse_paged_decode_batched_cuda(qbuf, kv, bt, sl, st, out_res,
                                               scale=scale)
        else:
            # the product path (mem_dynamic_decode, fetch="kernel"): the
            # decode fetches the plan's installs itself
            T.mem_decode_ptrsel(qbuf, kv_k_only, bt, sl, st, out, tier, 0,
                                scale=scale, entry_slots=r5.miss_pages,
                                install=True)

    # path A (product): score, select, plan, decode-with-install, and the
    # resident decode of the same pages for the equality check; path B:
    # score, select, plan, separate fetch, decode
    paths = {"install": (0, 1, 2, 6), "separate_fetch": (0, 1, 2, 3, 4)}
    set_q(0)
    for k in range(7):                   # eager first use (attributes)
        stage(k)
    torch.cuda.synchronize()
    graphs = {}
    for k in range(7):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            stage(k)
        graphs[k] = g
    g_path = {}
    for name, ks in paths.items():
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for k in ks:
                stage(k)
        g_path[name] = g
    torch.cuda.synchronize()
    page_bytes = PAGE * D * 2
    warm = max(args.warmup, 10)
    steps = max(args.steps, 20) if args.steps else 20
    qi = [0]

    def next_q():
        qi[0] += 1
        set_q(qi[0])

    res = {}
    misses, selected, equal = [], [], True
    with ClockSampler(dev) as clk:
        for name, ks in paths.items():
            stage_ks = ks + (5,)
            for _ in range(warm):
                next_q()
                for k in ks:
                    graphs[k].replay()
            torch.cuda.synchronize()
            ev = [[torch.cuda.Event(enable_timing=True)
                   for _ in range(len(stage_ks) + 1)] for _ in range(steps)]
            for i in range(steps):
                next_q()
                ev[i][0].record()
                for j, k in enumerate(stage_ks):
                    graphs[k].replay()
                    ev[i][j + 1].record()
                torch.cuda.synchronize()
                if name == "install":
                    misses.append(int(r5.fetch_cnt.sum()))
                    selected.append(int(st.page_cnt.sum()))
                equal = equal and bool(torch.equal(out, out_res))
            t = np.array([[e[j].elapsed_time(e[j + 1])
                           for j in range(len(stage_ks))] for e in ev]) * 1e3
            # whole-step graph, continuing the residency state
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
                enable_timing=True)
            full = []
            for i in range(steps):
                next_q()
                e0.record()
                g_path[name].replay()
                e1.record()
                torch.cuda.synchronize()
                full.append(e0.elapsed_time(e1) * 1e3)
            res[name] = (float(np.median(full)), dict(zip(stage_ks,
                                                          t.mean(0))))
    tier_step = res["install"][0]
    if world > 1:
        x = torch.tensor([tier_step], device=dev)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        tier_step = float(x.item())
    names = {0: "derive+score", 1: "select", 2: "residency_plan",
             3: "miss_fetch", 4: "tiered_decode+merge",
             5: "resident_decode+merge",
             6: "tiered_decode+merge_with_fetch"}
    miss_b = float(np.mean(misses)) * page_bytes
    t_sep_fetch = res["separate_fetch"][1][3]
    link_fetch = miss_b / (t_sep_fetch * 1e-6) / 1e9 if miss_b else 0.0
    peaks = _host_link_peaks(tier, r5, dev)
    # DRAM-tier roofline of the install decode: its HBM bytes (K tiles and
    # hot V tiles of the selected pages, q/out) at the HBM peak plus the miss
    # bytes at the measured host-link peak
    hbm, kind = _peaks()
    sel_pages = float(np.mean(selected))
    miss_pages = float(np.mean(misses))
    hbm_bytes = sel_pages * page_bytes * 2 - miss_pages * page_bytes + \
        n5 * C5_KV * C5_G * D * 4
    t_roof = hbm_bytes / (hbm * 1e9) + miss_b / (peaks["uva_read_gbs"] * 1e9)
    t_inst = res["install"][1][6] * 1e-6
    wp = _c5_write_path(T, tier, kv, bt, sl, n5, NB, MP)
    wp["begin_step_us_one_cta_walk"] = _c5_write_path(
        T, tier, kv, bt, sl, n5, NB, MP, cand_cap=0)["begin_step_us_per_step"]
    n_pages_tot = NB
    kb = n_pages_tot * C5_KV * page_bytes
    summ = n_pages_tot * C5_KV * B_SUM
    hot_b = C5_KV * hot_slots * page_bytes
    stg_b = n_vslots * C5_KV * page_bytes
    saved = 1.0 - (kb + summ + hot_b + stg_b) / (2 * kb + summ)
    # mem-kv: K tiered too (reference tier/tier.py:70-84 offload_k); the same
    # batch and selection through a second tier whose pinned pools hold K and
    # V, whole step score -> select -> plan -> decode with install
    del tier, r5
    torch.cuda.empty_cache()
    tkv = T.Tier(num_layers=1, num_blocks=NB, n_kv=C5_KV, page=PAGE, d=D,
                 hot_slots=hot_slots, max_reqs=n5, max_pages=MP,
                 n_vslots=n_vslots, offload_k=True, device=dev)
    tkv.pool.host[0].copy_(kv[:, 1].permute(0, 2, 1, 3).cpu())
    tkv.pool_k.host[0].copy_(kv[:, 0].permute(0, 2, 1, 3).cpu())
    tkv.residency.pool_valid.fill_(1)
    rkv = tkv.residency

    def kv_step():
        stage(0)
        stage(1)
        rkv.gather_plan(0, st.page_table, st.page_cnt, bt, sl, n5)
        T.mem_decode_ptrsel(qbuf, kv, bt, sl, st, out, tkv, 0, scale=scale,
                            entry_slots=rkv.miss_pages, install=True)

    set_q(0)
    kv_step()
    torch.cuda.synchronize()
    gkv = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gkv):
        kv_step()
    for _ in range(warm):
        next_q()
        gkv.replay()
    torch.cuda.synchronize()
    kv_full, kv_eq, kv_miss, kv_sel = [], True, [], []
    for i in range(steps):
        next_q()
        e0.record()
        gkv.replay()
        e1.record()
        torch.cuda.synchronize()
        kv_full.append(e0.elapsed_time(e1) * 1e3)
        kv_miss.append(int(rkv.fetch_cnt.sum()))
        kv_sel.append(int(st.page_cnt.sum()))
        graphs[5].replay()
        torch.cuda.synchronize()
        kv_eq = kv_eq and bool(torch.equal(out, out_res))
    saved_kv = 1.0 - (summ + 2 * hot_b + 2 * stg_b) / (2 * kb + summ)
    mem_kv = {"value": round(float(np.median(kv_full)), 2), "unit": UNIT,
              "vram_saved_frac": round(saved_kv, 4),
              "hit_rate": round(1.0 - float(np.sum(kv_miss)) /
                                max(1, float(np.sum(kv_sel))), 4),
              "miss_pages_per_step": round(float(np.mean(kv_miss)), 1),
              "tiered_equals_resident": kv_eq,
              "note": "K and V in pinned host pools, hot K and V slots; "
                      "vram_saved = 1 - (summaries + hot K/V + staging K/V)"
                      " / (K + V + summaries)"}
    del gkv, tkv, rkv
    if rank == 0:
        hbm, kind = _peaks()
        line = {
            "metric": "mem-v tiered sparse decode us/layer/step (C5)",
            "value": round(float(tier_step), 2), "unit": UNIT,
            "n_gpus": world, "steps": steps, "warmup": warm,
            "higher_is_better": False, "scaling": "weak", "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE C5 shapes)",
            "config": {"workload": "C5: B=16, ctx U(32K,128K) (realized mean "
                       f"{float(np.mean(ctxs)):.0f}), Llama-3.1-70B attn "
                       "(64q/8kv, d128), V in pinned host pool, hot = 10% of "
                       f"pages ({hot_slots} slots/kv-head), budget 0.05, "
                       "quad r'=2 int4-V nrm, q rotating 0.02 rad/step",
                       "NB": NB},
            "stage_us": {"note": "per-stage graphs (sum differs from the "
                                 "whole-step value by graph boundaries)",
                         **{names[k]: round(float(v), 2)
                            for k, v in res["install"][1].items()}},
            "separate_fetch_path": {
                "value": round(res["separate_fetch"][0], 2),
                "stage_us": {names[k]: round(float(v), 2)
                             for k, v in res["separate_fetch"][1].items()}},
            "dram_tier_roofline": {
                "kernel": "tiered_decode+merge_with_fetch",
                "hbm_bytes": int(hbm_bytes), "miss_bytes": int(miss_b),
                "roofline_us": round(t_roof * 1e6, 2),
                "achieved_us": round(t_inst * 1e6, 2),
                "frac": round(t_roof / t_inst, 4),
                "formula": "hbm_bytes / hbm_peak + miss_bytes / uva_read_gbs"},
            "host_link": {**peaks,
                          "separate_fetch_gbs": round(link_fetch, 2)},
            "write_path": wp,
            "hit_rate": round(1.0 - float(np.sum(misses)) /
                              max(1, float(np.sum(selected))), 4),
            "miss_pages_per_step": round(float(np.mean(misses)), 1),
            "selected_pages_per_step": round(float(np.mean(selected)), 1),
            "vram_saved_frac": round(saved, 4),
            "tiered_equals_resident": equal,
            "mem_kv": mem_kv,
            "hbm_peak_gbs": hbm, "peak_kind": kind,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _host_link_peaks(tier, r5, dev):
    """Host-link peaks on this box: a 256 MiB pinned -> device copy (copy
    engine) and the tier's UVA fetch kernel reading every hot slot's page
    from the pinned pool at once (the kernel that serves misses).  Leaves the
    residency maps untouched; the hot buffer is overwritten, so this runs
    after the timed steps."""
    import torch
    src = torch.empty(256 << 20, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(2):
        dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
        enable_timing=True)
    e0.record()
    for _ in range(5):
        dst.copy_(src, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    h2d = 5 * src.numel() / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del src, dst
    # synthetic full fetch: slot s of head k <- block s (every entry flushed)
    fl, fc = r5.fetch_list.clone(), r5.fetch_cnt.clone()
    S = r5.S
    ar = torch.arange(S, dtype=torch.int32, device=dev)
    r5.fetch_list[:, :S, 0] = ar % r5.NB
    r5.fetch_list[:, :S, 1] = ar
    r5.fetch_cnt.fill_(S)
    valid = r5.pool_valid.clone()
    r5.pool_valid.fill_(1)
    r5.gather_fetch(0, tier.staging, tier.pool.dev_view)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(3):
        r5.gather_fetch(0, tier.staging, tier.pool.dev_view)
    e1.record()
    torch.cuda.synchronize()
    nbytes = 3 * r5.n_kv * S * r5.page * r5.d * 2
    uva = nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9
    r5.fetch_list.copy_(fl)
    r5.fetch_cnt.copy_(fc)
    r5.pool_valid.copy_(valid)
    return {"h2d_copy_gbs": round(h2d, 2), "uva_read_gbs": round(uva, 2),
            "how": "256 MiB pinned->device copy; tier fetch kernel reading "
                   "every hot slot's page (n_kv x S pages) over UVA"}


def _c5_write_path(T, tier, kv, bt, sl, n5, NB, MP, n_steps=64,
                   cand_cap=4096):
    """The tier's write path at C5: a separate Staging replays the last
    ``n_steps`` decode steps of every request (one prefill step that writes
    each request's partial page, then one token per request per step) with
    the true V bytes, so every flush rewrites the bytes the pinned pool
    already holds.  Times begin_step (once per step, all layers' flushes; one
    layer here) and scatter_kv (once per layer) as CUDA graphs."""
    import torch
    dev = kv.device
    n_kv, d = kv.shape[3], kv.shape[4]
    stg = T.Staging(num_layers=1, num_blocks=NB, n_kv=n_kv, page=PAGE, d=d,
                    max_reqs=n5, max_pages=MP, max_tokens=n5 * PAGE,
                    device=dev, cand_cap=cand_cap)
    valid = torch.zeros((1, n_kv, NB), dtype=torch.int8, device=dev)
    pool = tier.pool.dev_view
    sl64 = sl[:n5].to(torch.int64)
    start = sl64 - n_steps
    ps = (start // PAGE) * PAGE
    btl = bt[:n5].to(torch.int64)

    def v_at(r_idx, pos):
        blk = btl[r_idx, pos // PAGE]
        return kv[blk, 1, pos % PAGE]                      # (n, n_kv, d)

    # prefill step: positions [ps, start) of every request
    qlp = (start - ps).to(torch.int32)
    qslp = torch.zeros(n5 + 1, dtype=torch.int32, device=dev)
    qslp[1:] = torch.cumsum(qlp, 0)
    r_idx = torch.repeat_interleave(torch.arange(n5, device=dev),
                                    qlp.to(torch.int64))
    pos = ps[r_idx] + (torch.arange(r_idx.numel(), device=dev)
                       - qslp[:-1].to(torch.int64)[r_idx])
    n_tok = int(r_idx.numel())
    stg.begin_step(bt, start.to(torch.int32), qslp, max(int(qlp.max()), 1),
                   n_tok, pool=pool, pool_valid=valid)
    if n_tok:
        stg.scatter_kv(0, None, v_at(r_idx, pos).contiguous(), n_tok)
    # decode timeline: graphs over fixed buffers
    sl_g = start.to(torch.int32) + 1
    qsl_g = torch.arange(n5 + 1, dtype=torch.int32, device=dev)
    ar = torch.arange(n5, device=dev)
    vals = torch.stack([v_at(ar, start + i) for i in range(n_steps)])
    val_g = torch.empty_like(vals[0])
    torch.cuda.synchronize()
    stg.begin_step(bt, sl_g, qsl_g, 1, n5, pool=pool, pool_valid=valid)
    val_g.copy_(vals[0])
    stg.scatter_kv(0, None, val_g, n5)
    g_bs, g_sc = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_bs):
        stg.begin_step(bt, sl_g, qsl_g, 1, n5, pool=pool, pool_valid=valid)
    with torch.cuda.graph(g_sc):
        stg.scatter_kv(0, None, val_g, n5)
    t_bs, t_sc, flushes = [], [], 0
    for i in range(1, n_steps):
        sl_g.copy_((start + i + 1).to(torch.int32))
        val_g.copy_(vals[i])
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record()
        g_bs.replay()
        e[1].record()
        g_sc.replay()
        e[2].record()
        torch.cuda.synchronize()
        t_bs.append(e[0].elapsed_time(e[1]) * 1e3)
        t_sc.append(e[1].elapsed_time(e[2]) * 1e3)
        flushes += int(stg.flush_cnt.item())
    stg.assert_free_partition()
    if int(stg.overflow.item()):
        raise RuntimeError("write path: staging overflow at C5")
    return {"begin_step_us_per_step": round(float(np.mean(t_bs[2:])), 2),
            "scatter_us_per_layer": round(float(np.mean(t_sc[2:])), 2),
            "flushed_pages_per_step": round(flushes / (n_steps - 1), 2),
            "context_pages_walked_per_step": int((sl64 // PAGE).sum()),
            "staging_blocks": stg.NV}


# --------------------------------------------------------------------------- #
# C2 (B=1 coverage) and C4 (r8 scorer + Jaccard vs quad): secondary lines     #
# --------------------------------------------------------------------------- #
def run_select_workload(args):
    """C2: Llama-3.1-8B geometry, batch 1, context 32768, 2% outlier
    channels x8, 5% planted pages carrying 90% of the exact softmax mass,
    quad r'=2 int4-V nrm summaries built from the keys, per-head coverage
    0.95.  C4: batch 32, context 65536, r8 scorer (per-head rank-8 basis,
    int8 coordinates with one scale per (block, head), token-max page
    score), coverage 0.95, and the quad selection of the same inputs for the
    Jaccard overlap.  A step = derive + score + coverage select + decode +
    merge of one layer, CUDA-graph replayed; per-stage graphs give the
    split."""
    import torch
    from amass_kv_b200 import attention as A
    from amass_kv_b200 import selection as S
    from amass_kv_b200.attention import ensure_stage_b_buffers
    from amass_kv_b200.selection import QuadState, R8State
    from amass_kv_b200.workloads import make_planted_gpu
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    c4 = args.workload == "c4"
    ctxs = [65536] * (args.batch or 32) if c4 else [32768] * (args.batch or 1)
    b = make_planted_gpu(dev, seed=2024 + (4 if c4 else 2), ctxs=ctxs,
                         n_kv=N_KV, G=G, d=D, page=PAGE, heavy_frac=0.05,
                         target_mass=0.9, outlier_frac=0.0 if c4 else 0.02,
                         r_quad=RANK_Q, v_bits=V_BITS, r8=8, c_bits=8)
    n_req, MP = len(ctxs), b["MP"]
    kv, q, bt, sl = b["kv_cache"], b["q"], b["block_table"], b["seq_lens"]
    scale = 1.0 / math.sqrt(D)
    cov = 0.95
    stq = QuadState(dev, num_layers=1, num_blocks=1, n_kv=N_KV, G=G,
                    head_dim=D, page=PAGE, max_reqs=n_req, max_pages=MP,
                    rank=RANK_Q, budget=BUDGET, v_bits=V_BITS, combine=COMBINE,
                    coverage=cov)
    stq.quad_mu, stq.mu_scale = b["quad_mu"], b["mu_scale"]
    stq.quad_V, stq.V_scale, stq.quad_sig2 = (b["quad_V"], b["V_scale"],
                                              b["quad_sig2"])
    ensure_stage_b_buffers(stq, dev, SPLIT)
    out = torch.empty_like(q)
    st = stq
    if c4:
        st8 = R8State(dev, num_layers=1, num_blocks=1, n_kv=N_KV, G=G,
                      head_dim=D, page=PAGE, max_reqs=n_req, max_pages=MP,
                      rank=8, budget=BUDGET, coverage=cov, vk_bits=8, c_bits=8,
                      c_grain="tensor")
        st8.r8_mu, st8.mu_scale = b["r8_mu"], b["mu_scale"]
        st8.r8_Vk, st8.Vk_scale = b["r8_Vk"], b["Vk_scale"]
        st8.r8_c, st8.c_scale = b["r8_c"], b["c_scale"]
        ensure_stage_b_buffers(st8, dev, SPLIT)
        st = st8

    def stage(k, which=None):
        s_ = which or st
        if k == 0:
            S.derive_page_params(s_, sl, n_req)
            if s_ is stq:
                S._score_launch(s_, 0, q, bt, n_req, scale, COMBINE == "nrm")
            else:
                S.r8_score_cuda(s_, 0, q, bt, sl, n_req, scale,
                                token_agg="tokmax")
        elif k == 1:
            S.select_pages(s_, n_req, coverage=cov,
                           from_score_h=(s_ is stq and COMBINE == "nrm"))
        else:
            A.sparse_paged_decode_batched_cuda(q, kv, bt, sl, s_, out,
                                               scale=scale,
                                               pps_min=args.pps_min)

    for k in range(3):
        stage(k)
    torch.cuda.synchronize()
    full = torch.cuda.CUDAGraph()
    with torch.cuda.graph(full):
        for k in range(3):
            stage(k)
    parts = []
    for k in range(3):
        g_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_):
            stage(k)
        parts.append(g_)
    torch.cuda.synchronize()
    steps, warm = args.steps, max(args.warmup, 3)
    for _ in range(warm):
        full.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
        enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record()
        for _ in range(steps):
            full.replay()
        e1.record()
        torch.cuda.synchronize()
    us_step = e0.elapsed_time(e1) / steps * 1e3
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)]
          for _ in range(steps)]
    for i in range(steps):
        ev[i][0].record()
        for k in range(3):
            parts[k].replay()
            ev[i][k + 1].record()
    torch.cuda.synchronize()
    t = np.array([[e[k].elapsed_time(e[k + 1]) for k in range(3)]
                  for e in ev]).mean(0) * 1e3
    cnt = st.page_cnt.cpu().numpy().astype(np.int64)
    nsh = np.maximum(st.n_sel_hi.cpu().numpy().astype(np.int64), 0)
    b_sum = (D + 2 + D * 8 + 16 + PAGE * 8 + 2 * PAGE) if c4 else B_SUM
    alg = int((N_KV * nsh * b_sum + 4 * nsh).sum()) + int(cnt.sum()) * 2 * \
        PAGE * D * 2 + n_req * N_KV * G * D * 4
    hbm, kind = _peaks()
    line = {
        "metric": ("r8 scorer + coverage sparse decode us/layer/step (C4)"
                   if c4 else "coverage sparse decode us/layer/step (C2)"),
        "value": round(us_step, 2), "unit": UNIT, "n_gpus": 1,
        "steps": steps, "warmup": warm, "higher_is_better": False,
        "dtype": "bf16", "data": "synthetic (seeded; BASELINE C4 shapes)"
        if c4 else "synthetic (seeded; BASELINE C2 shapes)",
        "config": {"workload": (
            "C4: B=32, ctx 65536, Llama-3.1-8B attn, r8 (rank 8 per-head "
            "basis, int8 coords, one scale per (block, head), token-max), "
            "coverage 0.95" if c4 else
            "C2: B=1, ctx 32768, Llama-3.1-8B attn, 2% outlier channels x8, "
            "quad r'=2 int4-V nrm from the keys, coverage 0.95"),
            "planted_heavy_frac": 0.05,
            "planted_mass": round(b["planted_mass"], 4)},
        "stage_us": {"derive+score": round(float(t[0]), 2),
                     "coverage_select": round(float(t[1]), 2),
                     "sparse_decode+merge": round(float(t[2]), 2)},
        "selected_pages_per_step": int(cnt.sum()),
        "mean_pages_per_unit": round(float(cnt.mean()), 1),
        "step_roofline": {"bound": "hbm", "alg_bytes": alg,
                          "achieved": round(alg / (us_step * 1e-6) / 1e9, 1),
                          "peak": hbm, "unit": "GB/s",
                          "frac": round(alg / (us_step * 1e-6) / 1e9 / hbm, 4),
                          "peak_kind": kind},
        "clocks": clk.summary(),
    }
    # planted recall: share of planted (request, kv, page) kept
    tab = st.page_table.cpu().numpy()
    planted = b["planted"].cpu().numpy()
    hit = tot = 0
    for r in range(n_req):
        for k in range(N_KV):
            sel = set(tab[r, k, :cnt[r, k]].tolist())
            pp = np.nonzero(planted[r, k])[0]
            tot += len(pp)
            hit += sum(1 for p in pp if p in sel)
    line["planted_recall"] = round(hit / max(tot, 1), 4)
    if c4:
        # quad selection of the same inputs (coverage 0.95) vs r8's
        for k in range(2):
            stage(k, stq)
        torch.cuda.synchronize()
        tq = stq.page_table.cpu().numpy()
        cq = stq.page_cnt.cpu().numpy()
        jac = []
        for r in range(n_req):
            for k in range(N_KV):
                a_ = set(tab[r, k, :cnt[r, k]].tolist())
                b_ = set(tq[r, k, :cq[r, k]].tolist())
                jac.append(len(a_ & b_) / max(len(a_ | b_), 1))
        line["jaccard_r8_vs_quad"] = round(float(np.mean(jac)), 4)
        line["quad_selected_pages"] = int(cq.sum())
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- #
# summary build (page finalize): the C3 batch, Llama-3.1-8B's 32 layers       #
# --------------------------------------------------------------------------- #
def run_build(args):
    """Timing of the page-finalize summary build at the C3 batch: the tail
    rebuild (every request's last finalized page, all 32 layers, one launch)
    and the bulk build of every finalized page of one layer (the prefill
    case), quad r'=2 int4-V; CUDA events around CUDA-graph replays."""
    import torch
    from amass_kv_b200 import summaries as SU
    from amass_kv_b200.selection import QuadState
    from amass_kv_b200.workloads import c3_contexts
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    L = 32
    ctxs = c3_contexts(1000, N_REQ)
    npg = [(int(c) + PAGE - 1) // PAGE for c in ctxs]
    NB = sum(npg) + 64
    MP = max(npg)
    g = torch.Generator(device="cpu").manual_seed(3)
    perm = torch.randperm(NB, generator=g).to(torch.int32)
    bt = torch.zeros(N_REQ, MP, dtype=torch.int32)
    o = 0
    for i, n in enumerate(npg):
        bt[i, :n] = perm[o:o + n]
        o += n
    bt = bt.to(dev)
    sl = torch.as_tensor(np.asarray(ctxs), dtype=torch.int32, device=dev)
    # one shared random key cache viewed as 32 layers (summaries depend only
    # on the page bytes; distinct layers would only cost memory)
    K = torch.randn((NB, PAGE, N_KV, D), device=dev).to(torch.bfloat16)
    st = QuadState(dev, num_layers=L, num_blocks=NB, n_kv=N_KV, G=G,
                   head_dim=D, page=PAGE, max_reqs=N_REQ, max_pages=MP,
                   rank=RANK_Q, budget=BUDGET, v_bits=V_BITS, combine=COMBINE)
    Ks = [K] * L
    stb = QuadState(dev, num_layers=1, num_blocks=NB, n_kv=N_KV, G=G,
                    head_dim=D, page=PAGE, max_reqs=N_REQ, max_pages=MP,
                    rank=RANK_Q, budget=BUDGET, v_bits=V_BITS, combine=COMBINE)
    res = {}
    for name, fn in (("tail_all_layers", lambda: SU.quad_build_tail(
                          st, Ks, bt, sl, N_REQ)),
                     ("bulk_one_layer", lambda: SU.quad_build_bulk(
                          stb, [K], bt, sl, N_REQ, MP))):
        fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
            enable_timing=True)
        n = max(args.steps // 10, 5)
        e0.record()
        for _ in range(n):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        res[name] = round(e0.elapsed_time(e1) / n * 1e3, 2)
    fin = sum(int(c) // PAGE for c in ctxs)
    line = {"metric": "page summary build us (C3 batch)",
            "value": res["tail_all_layers"], "unit": "us/finalize-step",
            "higher_is_better": False, "dtype": "f32 (eigh), int8/int4 out",
            "data": "synthetic (seeded; BASELINE C3 shapes)",
            "config": {"workload": "quad r'=2 int4-V summaries; tail = last "
                       "finalized page of 64 requests x 8 kv-heads x 32 "
                       f"layers ({N_REQ * N_KV * L} page-heads); bulk = all "
                       f"{fin} finalized pages x 8 kv-heads of one layer"},
            "bulk_one_layer_us": res["bulk_one_layer"],
            "page_heads_per_s_bulk": round(fin * N_KV / (res["bulk_one_layer"]
                                                         * 1e-6), 0)}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--impl", default="amass_b200",
                    choices=["amass_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pps-min", type=int, default=None,
                    help="decode pages-per-chunk floor (default: by batch)")
    ap.add_argument("--scorer", default="quad", choices=["quad", "clse"],
                    help="Stage-A scorer of the c3 step: quad (the headline) "
                         "or clse (the reference config's default score)")
    ap.add_argument("--repeats", type=int, default=None,
                    help="timed loops of --steps steps (median reported; "
                         "default: enough for about 1000 steps, 5..50)")
    ap.add_argument("--no-ctx32k", action="store_true",
                    help="skip the all-32K-context secondary measurement")
    ap.add_argument("--quad-pipe", type=int, default=1, choices=[0, 1, 2],
                    help="quad scorer choice (amass_quad_pipeline): 1 the "
                         "library default, 2 pipelined wherever it applies, "
                         "0 register-pipelined for every call")
    ap.add_argument("--quad-pack", type=int, default=1, choices=[0, 1],
                    help="pipelined scorer limb form (amass_quad_pack): 1 "
                         "packed limbs for G <= 4 (library default), 0 the "
                         "two-limb form")
    ap.add_argument("--no-score-layout", action="store_true",
                    help="skip the scorer's contiguous-block-table timing")
    ap.add_argument("--no-layouts", action="store_true",
                    help="N > 1: skip the weak and kv-head-sharded layouts")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="kv mode output exchange: merge kernel stores to "
                         "every rank over NVLink, or NCCL all-gather")
    ap.add_argument("--workload", default="c3",
                    choices=["c3", "c2", "c4", "c5", "build"],
                    help="c3 = the headline resident decode (default); c2 = "
                         "batch-1 coverage; c4 = r8 scorer + Jaccard vs quad; "
                         "c5 = the mem-v tiered decode")
    ap.add_argument("--batch", type=int, default=None,
                    help="batch size of the c2/c4/c5 workloads (default: the "
                         "config's; smaller only for profiling captures)")
    ap.add_argument("--split", type=int, default=SPLIT,
                    help="split-K partial slots per unit (the decode's run "
                         "floor is ceil(max pages / (split - 1)))")
    ap.add_argument("--requests", type=int, default=N_REQ,
                    help="batch size per GPU (64 = BASELINE C3; smaller only "
                         "for profiling captures)")
    args = ap.parse_args()
    globals()["N_REQ"] = args.requests
    globals()["SPLIT"] = args.split
    globals()["SCORER"] = args.scorer
    args.warmup = max(args.warmup, 3)
    if args.repeats is None:
        args.repeats = max(5, min(50, 1000 // max(args.steps, 1)))
    if args.impl == "reference":
        run_reference(args)
        return
    if args.quad_pipe != 1:
        from amass_kv_b200 import _lib
        _lib.load().amass_quad_pipeline(args.quad_pipe)
    if args.quad_pack != 1:
        from amass_kv_b200 import _lib
        _lib.load().amass_quad_pack(args.quad_pack)
    if args.workload == "c5":
        run_c5(args)
    elif args.workload in ("c2", "c4"):
        run_select_workload(args)
    elif args.workload == "build":
        run_build(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
