"""mem-v / mem-kv DRAM tier -- host side of the sm_100a tier kernels.

Mirrors the reference's ``amass.tier`` surface for the decode hot path:

  MappedHostVPool          tier/pool.py:104-151
  Staging (V/K pools+vbo)  tier/staging.py:235-310 (buffers only)
  Residency                tier/residency.py:281-575
  Tier                     tier/tier.py:37-180 (step / bytes_report)
  mem_decode_ptrsel        tier/decode_mem.py:169-222
  mem_dynamic_decode       tier/decode_mem.py:225-274

V (and K under mem-kv) of every page lives in a pinned, device-mapped host
pool (L, NB, n_kv, page, d); each (layer, kv-head) keeps a VRAM hot buffer of
S page slots filled by exact LRU; pages written this step and not yet flushed
sit in the VRAM staging pool addressed by ``vbo``.  Every step of one layer is
three launches: plan (hits/misses/victims), fetch (host link -> hot), and the
ptr-select decode that reads each page from hot | staging | pinned.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from ._lib import ptr
from .attention import ensure_stage_b_buffers, pps_min_for, split_kv

_FETCH_MODES = ("kernel", "dma", "off")


def host_device_pointer(host_tensor: torch.Tensor) -> int:
    """Device address of a pinned host tensor (UVA zero-copy); raises if the
    memory is not pinned and mapped (reference tier/pool.py:65-80)."""
    if not host_tensor.is_pinned():
        raise ValueError("pool tensor must be pinned (pin_memory=True)")
    dev = ctypes.c_void_p(0)
    _lib.call("amass_host_device_pointer", ctypes.c_void_p(host_tensor.data_ptr()),
              ctypes.byref(dev))
    return int(dev.value)


class DevPtrTensor:
    """A device address without a torch.Tensor wrapper (``data_ptr()``,
    ``dtype``, ``shape``) -- the pinned pool's device view."""

    __slots__ = ("_ptr", "dtype", "device", "shape")

    def __init__(self, p: int, dtype, device, shape=()):
        self._ptr, self.dtype, self.device, self.shape = int(p), dtype, device, shape

    def data_ptr(self) -> int:
        return self._ptr


def gpu_local_cpus(device) -> list | None:
    """CPUs of the NUMA node nearest ``device`` (NVML's CPU affinity of the
    GPU, looked up by PCI bus id so CUDA_VISIBLE_DEVICES renumbering does not
    matter), or None when NVML is unavailable.  Read-only NVML queries."""
    try:
        import pynvml
    except ImportError:
        return None
    props = torch.cuda.get_device_properties(device)
    bus = (f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:"
           f"{props.pci_device_id:02x}.0")
    try:
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            n = (os.cpu_count() + 63) // 64
            words = pynvml.nvmlDeviceGetCpuAffinity(h, n)
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        return None
    cpus = [64 * i + b for i, w in enumerate(words) for b in range(64)
            if (int(w) >> b) & 1]
    return cpus or None


class _cpu_affinity:
    """Run the body on ``cpus`` (first-touch placement of host pages on
    their NUMA node), then restore the caller's affinity."""

    def __init__(self, cpus):
        self.cpus = cpus

    def __enter__(self):
        self.old = None
        if self.cpus and hasattr(os, "sched_setaffinity"):
            self.old = os.sched_getaffinity(0)
            allowed = set(self.cpus) & self.old
            if allowed:
                os.sched_setaffinity(0, allowed)
                # one writer thread: pool threads keep their own affinity
                self.threads = torch.get_num_threads()
                torch.set_num_threads(1)
            else:
                self.old = None
        return self

    def __exit__(self, *exc):
        if self.old is not None:
            torch.set_num_threads(self.threads)
            os.sched_setaffinity(0, self.old)
        return False


class MappedHostVPool:
    """Pinned host pool (L, NB, n_kv, page, d) + its device view.  The page of
    (layer, block, kv-head) starts at element ((l*NB + blk)*n_kv + kv)*page*d
    (reference tier/pool.py:104-147)."""

    def __init__(self, *, num_layers: int, num_blocks: int, n_kv: int,
                 page: int, d: int, dtype=torch.bfloat16, device=None,
                 max_pool_gb: float = 256.0, numa_local: bool = True):
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"pool dtype must be bf16/fp16, got {dtype}")
        self.L, self.NB, self.n_kv = num_layers, num_blocks, n_kv
        self.page, self.d, self.dtype = page, d, dtype
        pool_bytes = num_layers * num_blocks * n_kv * page * d * 2
        if pool_bytes > max_pool_gb * (1 << 30):
            raise RuntimeError(
                f"pinned V pool would be {pool_bytes / 2**30:.1f} GiB "
                f"(> max_pool_gb={max_pool_gb}); reduce num_blocks or raise "
                "max_pool_gb (host DRAM, not VRAM)")
        dev = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        # pages are placed where they are first written: zero the pool from
        # the CPUs next to this GPU, so its host-link reads stay on-node
        self.numa_cpus = gpu_local_cpus(dev) if numa_local else None
        with _cpu_affinity(self.numa_cpus):
            self.host = torch.empty((num_layers, num_blocks, n_kv, page, d),
                                    dtype=dtype, pin_memory=True)
            self.host.zero_()
        self.dev_view = DevPtrTensor(host_device_pointer(self.host),
                                     torch.int16, dev, tuple(self.host.shape))
        self.pool_gib = pool_bytes / 2**30
        self.device = dev

    def page_offset(self, layer: int, blk: int, kv: int) -> int:
        return ((layer * self.NB + blk) * self.n_kv + kv) * self.page * self.d

    def vram_note(self) -> str:
        return (f"host_pool={self.pool_gib:.2f}GiB (DRAM, keyed by NB={self.NB}; "
                "VRAM hot/staging bounded to the working set)")


class Staging:
    """VRAM staging pools for pages written but not yet flushed, and their
    per-step lifecycle (reference tier/staging.py:235-520).

    v_pool (L, NV, page, n_kv, d) [+ k_pool under mem-kv]; vbo (NB,) = staging
    block of an engine block or -1; v_flushed (NB,) latch; a free stack of
    staging blocks (v_free_stack, v_free_top); v_slot_mapping (max_tokens,)
    int64; the per-step flush list (max_flush, 2) + flush_cnt; overflow latch.
    NV defaults to the working-set bound 2*ceil(max_tokens/page) + 4*max_reqs
    (reference :251-274); ``n_vslots`` is accepted as a synonym of v_blocks."""

    def __init__(self, *, num_layers: int, num_blocks: int, n_kv: int,
                 page: int, d: int, max_reqs: int = 1, max_pages: int = 1,
                 max_tokens: int = 1, dtype=torch.bfloat16, device="cuda",
                 v_blocks: int | None = None, max_flush: int | None = None,
                 offload_k: bool = False, n_vslots: int | None = None,
                 cand_cap: int = 4096):
        self.L, self.NB, self.n_kv = num_layers, num_blocks, n_kv
        self.page, self.d = page, d
        self.R, self.MP, self.max_tokens = max_reqs, max_pages, max_tokens
        self.offload_k = offload_k
        dev = torch.device(device)
        self.device = dev
        chunk_pages = (max_tokens + page - 1) // page
        if v_blocks is None:
            v_blocks = n_vslots
        if v_blocks is None or v_blocks <= 0:
            v_blocks = 2 * chunk_pages + 4 * max_reqs
        if max_flush is None or max_flush <= 0:
            max_flush = chunk_pages + 2 * max_reqs + 64
        self.NV, self.MAXF, self.chunk_pages = v_blocks, max_flush, chunk_pages
        i32 = torch.int32
        self.v_pool = torch.zeros((num_layers, v_blocks, page, n_kv, d),
                                  dtype=dtype, device=dev)
        self.k_pool = torch.zeros_like(self.v_pool) if offload_k else None
        self.vbo = torch.full((num_blocks,), -1, dtype=i32, device=dev)
        self.v_flushed = torch.zeros((num_blocks,), dtype=i32, device=dev)
        self.v_free_stack = torch.arange(v_blocks, dtype=i32, device=dev)
        self.v_free_top = torch.full((1,), v_blocks, dtype=i32, device=dev)
        self.v_slot_mapping = torch.full((max(max_tokens, 1),), -1,
                                         dtype=torch.int64, device=dev)
        self.flush_list = torch.zeros((max_flush, 2), dtype=i32, device=dev)
        self.flush_cnt = torch.zeros((1,), dtype=i32, device=dev)
        self.overflow = torch.zeros((1,), dtype=i32, device=dev)
        # scratch of the collect pre-pass (count + staged complete pages)
        self.cand_cap = max(0, min(int(cand_cap), 4096))
        self.cand = torch.zeros((1 + self.cand_cap,), dtype=i32, device=dev)
        pools = self.v_pool.numel() * (2 if offload_k else 1)
        self.vpool_gib = pools * self.v_pool.element_size() / 2**30

    # the ordered per-step lifecycle (outside or inside a graph: no sync)
    def begin_step(self, block_table, seq_lens, query_start_loc,
                   max_query_len: int, n_tokens: int, pool, pool_valid,
                   capture: bool = False, poolk=None) -> None:
        """Reset this step's slots; clear the flushed latch of rewritten
        pages; collect + free complete staged pages; copy them to the pinned
        pool (pool_valid = 1); allocate staging blocks for this step's pages;
        fill v_slot_mapping (reference staging.py:312-346).  ``pool`` /
        ``poolk`` are the pinned pools' device views."""
        if n_tokens > self.v_slot_mapping.numel():
            raise RuntimeError(f"{n_tokens} tokens > v_slot_mapping capacity "
                               f"{self.v_slot_mapping.numel()}")
        n_req = seq_lens.shape[0]
        if capture:
            self.v_slot_mapping[:n_tokens].fill_(-1)
            return
        vp = self.v_pool
        has_k = self.k_pool is not None
        _lib.call("amass_staging_begin_step", ptr(block_table),
                  block_table.stride(0), ptr(seq_lens), ptr(query_start_loc),
                  int(n_req), int(n_tokens), int(max_query_len),
                  ptr(self.v_slot_mapping), ptr(self.vbo), ptr(self.v_flushed),
                  ptr(self.v_free_stack), ptr(self.v_free_top),
                  ptr(self.flush_list), ptr(self.flush_cnt),
                  ptr(self.overflow), self.MAXF, ptr(vp),
                  ptr(self.k_pool) if has_k else 0, vp.stride(0),
                  vp.stride(1), vp.stride(2), vp.stride(3), pool.data_ptr(),
                  poolk.data_ptr() if has_k else 0, ptr(pool_valid), self.L,
                  self.NB, self.n_kv, self.d, self.page, ptr(self.cand),
                  self.cand_cap, _lib.stream_of(self.device))

    def scatter_kv(self, lidx: int, key, value, n_tokens: int) -> None:
        """Write path: this step's V (and K under mem-kv) (n_tokens, n_kv, d)
        into layer ``lidx``'s staging pool(s) at v_slot_mapping (reference
        staging.py:348-367)."""
        vp = self.v_pool[lidx]
        has_k = self.k_pool is not None
        kp = self.k_pool[lidx] if has_k else None
        _lib.call("amass_staging_scatter", ptr(value), value.stride(0),
                  value.stride(1), ptr(key) if has_k else 0,
                  key.stride(0) if has_k else 0, key.stride(1) if has_k else 0,
                  ptr(self.v_slot_mapping), ptr(vp), ptr(kp) if has_k else 0,
                  vp.stride(0), vp.stride(1), vp.stride(2), int(n_tokens),
                  self.n_kv, self.d, self.page, _lib.stream_of(self.device))

    # invariant checks (host sync; debug)
    def assert_free_partition(self) -> None:
        """Assigned (vbo >= 0) and free (v_free_stack[:top]) staging blocks
        partition [0, NV) (reference staging.py:454-470)."""
        top = int(self.v_free_top.item())
        if not 0 <= top <= self.NV:
            raise AssertionError(f"free_top={top} out of [0, {self.NV}]")
        assigned = self.vbo[self.vbo >= 0]
        free = self.v_free_stack[:top]
        both = torch.cat([assigned, free])
        if both.numel() != self.NV or int(torch.unique(both).numel()) != self.NV:
            raise AssertionError("staging blocks: assigned + free do not "
                                 f"partition [0, {self.NV})")

    def assert_no_lost_v(self, block_table, seq_lens, query_start_loc,
                         pool_valid) -> None:
        """Every complete page written by earlier steps is staged or flushed
        in every layer and kv-head (reference staging.py:472-486)."""
        sl = seq_lens.tolist()
        qsl = query_start_loc.tolist()
        vbo = self.vbo.cpu()
        pv = pool_valid.cpu()
        for r in range(len(sl)):
            ql = qsl[r + 1] - qsl[r]
            if sl[r] <= 0 or ql <= 0:
                continue
            for p in range((sl[r] - ql) // self.page):
                blk = int(block_table[r, p])
                if int(vbo[blk]) < 0 and not bool((pv[:, :, blk] == 1).all()):
                    raise AssertionError(f"request {r} block {blk}: complete "
                                         "page neither staged nor flushed")

    def assert_capacity(self) -> None:
        floor = self.chunk_pages + self.R
        if self.NV < floor:
            raise AssertionError(f"v_blocks NV={self.NV} < floor {floor}")

    def bytes_report(self) -> str:
        return f"v_pool={self.vpool_gib:.3f}GiB (NV={self.NV} blocks)"


class CopyEngine:
    """Copy-engine transport on dedicated side streams, double-buffered so a
    prefetch for step N+1 does not queue behind step N's (reference
    tier/dma.py:77-140).  ``memcpy_async`` is one contiguous copy,
    ``memcpy_2d_async`` a strided 2-D copy (one coalesced run); both go
    through the library's ``amass_dma_issue``.  The reference's scattered
    one-call batch copy is not provided: this build's fetch is the kernel
    (graph-capturable) or these run copies."""

    def __init__(self, n_buffers: int = 2, device=None):
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        self.streams = [torch.cuda.Stream(self.device)
                        for _ in range(n_buffers)]
        self.events = [torch.cuda.Event() for _ in range(n_buffers)]
        self._i = 0
        self.has_batch = False

    def next_stream(self):
        s = self.streams[self._i]
        self._i = (self._i + 1) % len(self.streams)
        return s

    def issue(self, runs, stream) -> None:
        if len(runs):
            _lib.call("amass_dma_issue", ctypes.cast(runs, ctypes.c_void_p),
                      len(runs), stream.cuda_stream)

    def memcpy_async(self, dst_ptr: int, src_ptr: int, nbytes: int,
                     stream) -> None:
        self.issue((_lib.DmaRun * 1)(_lib.DmaRun(dst_ptr, src_ptr, 0, 0,
                                                 nbytes, nbytes, nbytes, 1)),
                   stream)

    def memcpy_2d_async(self, dst_ptr: int, dpitch: int, src_ptr: int,
                        spitch: int, width_bytes: int, height: int,
                        stream) -> None:
        self.issue((_lib.DmaRun * 1)(_lib.DmaRun(dst_ptr, src_ptr, 0, 0,
                                                 dpitch, spitch, width_bytes,
                                                 height)), stream)

    def memcpy_batch(self, *args, **kwargs) -> None:
        raise RuntimeError("the scattered one-call batch copy is not part of "
                           "this build; use the kernel fetch or run copies")

    def record(self, stream):
        ev = (self.events[self.streams.index(stream)]
              if stream in self.streams else torch.cuda.Event())
        ev.record(stream)
        return ev


class Residency:
    """Exact-LRU hot-buffer residency of every (layer, kv-head)
    (reference tier/residency.py:281-348).

    State (device, allocated once): hot (L, n_kv, S, page, d) [+ hot_k under
    mem-kv], page2slot (L, n_kv, NB), slot2page / lru_clock (L, n_kv, S),
    pool_valid (L, n_kv, NB) int8, clock int32[2] (clock, CTA ticket; starts
    at 1 like the reference), overflow (1,), and per-call scratch
    fetch_list (n_kv, S, 2) / fetch_cnt (n_kv,) / miss_pages (R, n_kv, MP)."""

    def __init__(self, *, num_layers: int, num_blocks: int, n_kv: int,
                 hot_slots: int, page: int, d: int, max_reqs: int,
                 max_pages: int, dtype=torch.bfloat16, device="cuda",
                 offload_k: bool = False):
        self.L, self.NB, self.n_kv = num_layers, num_blocks, n_kv
        self.S, self.page, self.d = hot_slots, page, d
        self.R, self.MP = max_reqs, max_pages
        self.dtype, self.offload_k = dtype, offload_k
        dev = torch.device(device)
        self.device = dev
        i32, i8 = torch.int32, torch.int8
        self.hot = torch.zeros((num_layers, n_kv, hot_slots, page, d),
                               dtype=dtype, device=dev)
        self.hot_i16 = self.hot.view(torch.int16)
        self.hot_k = torch.zeros_like(self.hot) if offload_k else None
        self.hot_k_i16 = self.hot_k.view(torch.int16) if offload_k else None
        self.page2slot = torch.full((num_layers, n_kv, num_blocks), -1,
                                    dtype=i32, device=dev)
        self.slot2page = torch.full((num_layers, n_kv, hot_slots), -1,
                                    dtype=i32, device=dev)
        self.lru_clock = torch.zeros((num_layers, n_kv, hot_slots), dtype=i32,
                                     device=dev)
        self.pool_valid = torch.zeros((num_layers, n_kv, num_blocks),
                                      dtype=i8, device=dev)
        self.clock = torch.tensor([1, 0], dtype=i32, device=dev)
        self.overflow = torch.zeros((1,), dtype=i32, device=dev)
        self.fetch_list = torch.zeros((n_kv, hot_slots, 2), dtype=i32,
                                      device=dev)
        self.fetch_cnt = torch.zeros((n_kv,), dtype=i32, device=dev)
        self.miss_pages = torch.zeros((max_reqs, n_kv, max_pages), dtype=i32,
                                      device=dev)
        self.plan_capacity = _lib.load().amass_tier_plan_capacity(hot_slots)
        if self.plan_capacity <= 0:
            raise ValueError(f"hot_slots={hot_slots} outside (0, 8192]")
        elem = self.hot.element_size()
        hot_n = self.hot.numel() * (2 if offload_k else 1)
        self.hot_gib = hot_n * elem / 2**30
        self.maps_gib = sum(t.numel() * t.element_size() for t in (
            self.page2slot, self.slot2page, self.lru_clock, self.pool_valid,
            self.fetch_list, self.fetch_cnt, self.miss_pages)) / 2**30

    # -- per step ------------------------------------------------------------
    def invalidate_written(self, block_table, seq_lens, query_start_loc) -> None:
        """Drop residency and pool validity of every page (re)written this
        step, all layers (reference residency.py:352-367)."""
        n_req = seq_lens.shape[0]
        _lib.call("amass_tier_invalidate", ptr(block_table),
                  block_table.stride(0), ptr(seq_lens), ptr(query_start_loc),
                  ptr(self.page2slot), ptr(self.slot2page),
                  ptr(self.pool_valid), int(n_req), self.L, self.n_kv,
                  self.NB, self.S, self.page, _lib.stream_of(self.device))

    def gather_plan(self, layer, page_table, page_cnt, block_table, seq_lens,
                    n_req) -> None:
        """Hits touch the LRU, misses take exact-LRU victims (clock advances
        by one); the installed misses land in fetch_list/fetch_cnt
        (reference residency.py:385-407)."""
        l = int(layer)
        if page_table.shape[-1] > self.MP or n_req > self.R:
            raise ValueError(f"selection ({n_req} requests x "
                             f"{page_table.shape[-1]} pages) exceeds the "
                             f"residency's max_reqs={self.R} / "
                             f"max_pages={self.MP}")
        _lib.call("amass_tier_plan", ptr(page_table), ptr(page_cnt),
                  ptr(block_table), block_table.stride(0), ptr(seq_lens),
                  ptr(self.page2slot[l]), ptr(self.slot2page[l]),
                  ptr(self.lru_clock[l]), ptr(self.clock), ptr(self.overflow),
                  ptr(self.fetch_list), ptr(self.fetch_cnt),
                  ptr(self.miss_pages), int(n_req),
                  self.n_kv, int(page_table.shape[-1]), self.page, self.NB,
                  self.S, _lib.stream_of(self.device))

    def gather_fetch(self, layer, staging, pool, n_req=None, stream=None,
                     poolk=None) -> None:
        """Copy the planned misses into their hot slots: pinned pool when
        flushed, else staging with write-through (reference residency.py:
        409-436).  ``pool``/``poolk`` are device views (``dev_view``)."""
        st = (stream.cuda_stream if stream is not None
              else _lib.stream_of(self.device))
        self._fetch("amass_tier_fetch", layer, staging, pool, poolk, st)

    def _fetch(self, entry, layer, staging, pool, poolk, st) -> None:
        l = int(layer)
        vp = staging.v_pool[l]
        has_k = self.hot_k_i16 is not None
        if has_k and (poolk is None or staging.k_pool is None):
            raise ValueError("mem-kv residency needs poolk and staging.k_pool")
        kp = staging.k_pool[l] if has_k else None
        _lib.call(entry, ptr(self.fetch_list), ptr(self.fetch_cnt),
                  ptr(self.hot_i16[l]), pool.data_ptr(), ptr(self.pool_valid[l]),
                  ptr(staging.vbo), ptr(vp), vp.stride(0), vp.stride(1),
                  vp.stride(2), ptr(self.hot_k_i16[l]) if has_k else 0,
                  poolk.data_ptr() if has_k else 0, ptr(kp) if has_k else 0,
                  l, self.NB, self.n_kv, self.S, self.page, self.d, st)

    def gather_fetch_staged(self, layer, staging, pool, n_req=None,
                            poolk=None) -> None:
        """The kernel fetch restricted to installs whose page is not flushed
        (the ones the copy-engine plan leaves out): the device half of the
        copy-engine fetch (reference residency.py:
        527-548)."""
        self._fetch("amass_tier_fetch_staged", layer, staging, pool, poolk,
                    _lib.stream_of(self.device))

    def build_dma_plan(self, layer, pool, n_req=None, poolk=None):
        """Copy-engine plan of the last gather_plan's flushed installs (host:
        reads fetch_list / fetch_cnt / pool_valid back, a device sync):
        (runs, has_staged), runs a ctypes array of DmaRun.  Each run is one
        strided 2-D copy of contiguous blocks into contiguous hot slots of
        one kv-head (reference residency.py:438-492).  For a prefetch, build
        during the previous step."""
        l = int(layer)
        fl = self.fetch_list.cpu().contiguous()
        fc = self.fetch_cnt.cpu().contiguous()
        pv = self.pool_valid[l].cpu().contiguous()
        cap = max(1, int(fc.sum()))
        runs = (_lib.DmaRun * cap)()
        n = ctypes.c_int(0)
        staged = ctypes.c_int(0)
        has_k = self.hot_k_i16 is not None
        if has_k and poolk is None:
            raise ValueError("mem-kv residency needs poolk")
        _lib.call("amass_tier_dma_plan", fl.data_ptr(), fc.data_ptr(),
                  pv.data_ptr(), l, self.NB, self.n_kv, self.S, self.page,
                  self.d, pool.data_ptr(), self.hot_i16[l].data_ptr(),
                  poolk.data_ptr() if has_k else 0,
                  self.hot_k_i16[l].data_ptr() if has_k else 0,
                  ctypes.cast(runs, ctypes.c_void_p), cap, ctypes.byref(n),
                  ctypes.byref(staged))
        return (_lib.DmaRun * n.value).from_buffer(runs), bool(staged.value)

    def issue_dma_plan(self, runs, copy_engine, stream) -> None:
        """Issue a built plan on ``stream`` (copy engines only; reference
        residency.py:494-509)."""
        copy_engine.issue(runs, stream)

    def gather_fetch_dma(self, layer, staging, pool, n_req, copy_engine,
                         poolk=None, stream=None):
        """Copy-engine fetch (build + issue): flushed installs by the copy
        engines on a side stream, unflushed installs by the kernel on the
        current stream.  Returns the side stream's event (reference
        residency.py:511-525)."""
        stream = stream if stream is not None else copy_engine.next_stream()
        runs, has_staged = self.build_dma_plan(layer, pool, n_req, poolk)
        # victim slots may still be read by work queued before the plan
        stream.wait_stream(torch.cuda.current_stream(self.device))
        self.issue_dma_plan(runs, copy_engine, stream)
        ev = copy_engine.record(stream)
        if has_staged:
            self.gather_fetch_staged(layer, staging, pool, n_req, poolk)
        return ev

    def gather(self, layer, page_table, page_cnt, block_table, seq_lens,
               n_req, staging, pool, poolk=None) -> None:
        """plan + fetch (reference residency.py:369-383)."""
        self.gather_plan(layer, page_table, page_cnt, block_table, seq_lens,
                         n_req)
        self.gather_fetch(layer, staging, pool, n_req, poolk=poolk)

    # -- debug / reporting (host sync) ---------------------------------------
    def assert_maps_inverse(self, layer: int | None = None) -> None:
        """page2slot and slot2page are mutual inverses (reference
        residency.py:550-572)."""
        layers = range(self.L) if layer is None else [layer]
        for l in layers:
            p2s, s2p = self.page2slot[l].cpu(), self.slot2page[l].cpu()
            for kv in range(self.n_kv):
                for s, blk in enumerate(s2p[kv].tolist()):
                    if blk >= 0 and int(p2s[kv, blk]) != s:
                        raise AssertionError(
                            f"slot2page[{l},{kv},{s}]={blk} but page2slot="
                            f"{int(p2s[kv, blk])}")
                res = (p2s[kv] >= 0).nonzero().flatten().tolist()
                for blk in res:
                    s = int(p2s[kv, blk])
                    if int(s2p[kv, s]) != blk:
                        raise AssertionError(
                            f"page2slot[{l},{kv},{blk}]={s} but slot2page="
                            f"{int(s2p[kv, s])}")

    def misses_last_call(self) -> int:
        return int(self.fetch_cnt.sum())

    def bytes_report(self) -> str:
        return (f"hot={self.hot_gib:.3f}GiB maps={self.maps_gib:.4f}GiB "
                f"(S={self.S} slots x {self.n_kv} kv x {self.L} layers)")


class Tier:
    """pool (+ pool_k) + staging + residency (reference tier/tier.py:37-180)."""

    def __init__(self, *, num_layers: int, num_blocks: int, n_kv: int,
                 page: int, d: int, hot_slots: int, max_reqs: int,
                 max_pages: int, n_vslots: int | None = None,
                 offload_k: bool = False, dtype=torch.bfloat16, device="cuda",
                 max_pool_gb: float = 256.0, max_tokens: int | None = None,
                 v_blocks: int | None = None):
        kw = dict(num_layers=num_layers, num_blocks=num_blocks, n_kv=n_kv,
                  page=page, d=d)
        self.offload_k = offload_k
        self.pool = MappedHostVPool(**kw, dtype=dtype, device=device,
                                    max_pool_gb=max_pool_gb)
        self.pool_k = (MappedHostVPool(**kw, dtype=dtype, device=device,
                                       max_pool_gb=max_pool_gb)
                       if offload_k else None)
        self.staging = Staging(**kw, max_reqs=max_reqs, max_pages=max_pages,
                               max_tokens=max_tokens or max_reqs,
                               v_blocks=v_blocks or n_vslots, dtype=dtype,
                               device=device, offload_k=offload_k)
        self.residency = Residency(**kw, hot_slots=hot_slots,
                                   max_reqs=max_reqs, max_pages=max_pages,
                                   dtype=dtype, device=device,
                                   offload_k=offload_k)

    @classmethod
    def from_config(cls, cfg, *, num_layers, num_blocks, n_kv, page, d,
                    max_reqs, max_pages, n_vslots, device="cuda"):
        """Hot slots = cfg.hot_frac of max_pages (at least 1), mem-kv when
        cfg.mem_mode == "mem-kv" (reference tier/tier.py:70-84)."""
        frac = float(getattr(cfg, "hot_frac", 0.1))
        S = max(1, int(round(frac * max_pages)))
        return cls(num_layers=num_layers, num_blocks=num_blocks, n_kv=n_kv,
                   page=page, d=d, hot_slots=S, max_reqs=max_reqs,
                   max_pages=max_pages, n_vslots=n_vslots,
                   offload_k=getattr(cfg, "mem_mode", "mem-v") == "mem-kv",
                   device=device,
                   max_pool_gb=float(getattr(cfg, "max_pool_gb", 256.0)))

    def begin_step(self, block_table, seq_lens, query_start_loc,
                   max_query_len: int, n_tokens: int,
                   capture: bool = False) -> None:
        """Residency invalidation of the rewritten pages, then the staging
        lifecycle (reference tier/tier.py:86-104); capture batches mutate
        nothing."""
        if not capture:
            self.residency.invalidate_written(block_table, seq_lens,
                                              query_start_loc)
        self.staging.begin_step(block_table, seq_lens, query_start_loc,
                                max_query_len, n_tokens, self.pool.dev_view,
                                self.residency.pool_valid, capture=capture,
                                poolk=self.pool_k.dev_view if self.pool_k
                                else None)

    def write_kv(self, lidx, value, n_tokens, key=None) -> None:
        """In-graph write path: this step's V (and K, mem-kv) into staging
        (reference tier/tier.py:125-130)."""
        self.staging.scatter_kv(lidx, key, value, n_tokens)

    def assert_invariants(self, block_table, seq_lens, query_start_loc) -> None:
        if int(self.staging.overflow.item()) != 0:
            raise AssertionError("staging free stack underflowed")
        self.staging.assert_free_partition()
        self.residency.assert_maps_inverse()
        self.staging.assert_no_lost_v(block_table, seq_lens, query_start_loc,
                                      self.residency.pool_valid)

    def step(self, lidx, page_table, page_cnt, block_table, seq_lens,
             n_req) -> None:
        self.residency.gather(lidx, page_table, page_cnt, block_table,
                              seq_lens, n_req, self.staging,
                              self.pool.dev_view,
                              poolk=self.pool_k.dev_view if self.pool_k
                              else None)

    @property
    def copy_engine(self) -> CopyEngine:
        """Lazily created double-buffered copy engine (reference
        tier/tier.py:144-152)."""
        ce = getattr(self, "_copy_engine", None)
        if ce is None:
            ce = CopyEngine(device=self.residency.device)
            self._copy_engine = ce
        return ce

    def step_dma(self, lidx, page_table, page_cnt, block_table, seq_lens,
                 n_req, wait: bool = True):
        """``step`` with the flushed misses moved by the copy engines: plan
        on the device, build the runs on the host (a sync), issue them on a
        side stream that first waits for the current stream; staged misses
        go to the kernel.  Returns the side stream's event; ``wait`` makes
        the current stream wait on it (reference tier/tier.py:154-169)."""
        self.residency.gather_plan(lidx, page_table, page_cnt, block_table,
                                   seq_lens, n_req)
        ev = self.residency.gather_fetch_dma(
            lidx, self.staging, self.pool.dev_view, n_req, self.copy_engine,
            poolk=self.pool_k.dev_view if self.pool_k else None)
        if wait:
            torch.cuda.current_stream(self.residency.device).wait_event(ev)
        return ev

    def bytes_report(self) -> str:
        return (f"{self.pool.vram_note()}; {self.residency.bytes_report()}; "
                f"staging={self.staging.v_pool.numel() * 2 / 2**30:.3f}GiB")


def mem_decode_ptrsel(q, kv_cache, block_table, seq_lens, st, out, tier,
                      lidx: int, *, scale=None, pps_min=None,
                      entry_slots=None, install: bool = False) -> None:
    """ptr-select tiered split-K decode + merge into ``out[:n_req]`` (bf16):
    per page V (and K under mem-kv) from hot | staging | pinned
    (reference tier/decode_mem.py:169-222).  Bitwise equal to the resident
    decode on the same bytes.  ``entry_slots``: the residency's
    ``miss_pages`` right after its plan for this same selection (hits then
    skip the page2slot lookup), else None.  ``install`` (needs
    ``entry_slots``): the plan's fetch is done here instead of by
    ``gather_fetch`` -- each page the plan installed is read from staging or
    the pinned pool and written into its hot slot (written through to the
    pinned pool when it was staged and unflushed), so each miss crosses the
    host link once and the separate fetch launch goes away."""
    if scale is None:
        # the state's softmax scale, else 1/sqrt(head_dim)
        scale = getattr(st, "scale", None) or q.shape[-1] ** -0.5
    n_req = seq_lens.shape[0]
    r5, stg = tier.residency, tier.staging
    l = int(lidx)
    if getattr(st, "m_part", None) is None:
        ensure_stage_b_buffers(st, q.device)
    if pps_min is None:
        pps_min = pps_min_for(n_req)
    vp = stg.v_pool[l]
    if tier.offload_k:
        kres, skb, skt, skh = None, 0, 0, 0
        stg_k = stg.k_pool[l]
        pool_k = tier.pool_k.dev_view.data_ptr()
    else:
        kres, _ = split_kv(kv_cache)
        skb, skt, skh = kres.stride(0), kres.stride(1), kres.stride(2)
        stg_k = None
        pool_k = 0
    if q.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("q and out must be bf16")
    if install and entry_slots is None:
        raise ValueError("install needs the plan's entry_slots")
    fn = "amass_tier_decode_install" if install else "amass_tier_decode"
    pv = (ptr(r5.pool_valid[l]),) if install else ()
    _lib.call(fn, ptr(q), q.stride(0), q.stride(1),
              ptr(kres), skb, skt, skh,
              ptr(r5.hot[l]), ptr(r5.hot_k[l]) if tier.offload_k else 0,
              ptr(vp), ptr(stg_k), vp.stride(0), vp.stride(1), vp.stride(2),
              tier.pool.dev_view.data_ptr(), pool_k, *pv,
              ptr(r5.page2slot[l]), ptr(stg.vbo), ptr(entry_slots), l, r5.NB,
              r5.S,
              ptr(block_table), block_table.stride(0), ptr(st.page_table),
              ptr(st.page_cnt), ptr(seq_lens), ptr(st.m_part), ptr(st.l_part),
              ptr(st.acc_part), int(st.split), int(pps_min), ptr(out),
              out.stride(0), out.stride(1), float(scale), int(n_req),
              r5.n_kv, int(st.G), r5.d, r5.page, int(st.max_pages),
              _lib.stream_of(q.device))


def mem_dynamic_decode(q, kv_cache, block_table, seq_lens, st, out, tier,
                       lidx: int, *, scale=None, fetch: str = "kernel",
                       impl: str = "ptrsel") -> None:
    """One layer of the tiered decode: residency step (plan + fetch) of the
    layer's selection, then the ptr-select decode (reference
    tier/decode_mem.py:225-274).  ``fetch="off"`` decodes from the current
    residency without a step; ``fetch="dma"`` moves the flushed misses with
    the copy engines (host-planned runs, a host sync).  The reference's
    ``impl`` variants are one decode path here."""
    if fetch not in _FETCH_MODES:
        raise ValueError(f"fetch must be one of {_FETCH_MODES}, got {fetch!r}")
    if impl not in ("ptrsel", "cuda"):
        raise ValueError(f"impl must be 'ptrsel' (or its alias 'cuda'), got {impl!r}")
    n_req = seq_lens.shape[0]
    es = None
    if fetch == "kernel":
        r5 = tier.residency
        if st.page_table.shape[-1] == r5.MP:
            # plan, then the decode fetches the installed misses itself
            r5.gather_plan(lidx, st.page_table, st.page_cnt, block_table,
                           seq_lens, n_req)
            mem_decode_ptrsel(q, kv_cache, block_table, seq_lens, st, out,
                              tier, lidx, scale=scale,
                              entry_slots=r5.miss_pages, install=True)
            return
        tier.step(lidx, st.page_table, st.page_cnt, block_table, seq_lens,
                  n_req)
    elif fetch == "dma":
        tier.step_dma(lidx, st.page_table, st.page_cnt, block_table, seq_lens,
                      n_req, wait=True)
        if st.page_table.shape[-1] == tier.residency.MP:
            es = tier.residency.miss_pages
    mem_decode_ptrsel(q, kv_cache, block_table, seq_lens, st, out, tier, lidx,
                      scale=scale, entry_slots=es)


__all__ = ["CopyEngine", "DevPtrTensor", "MappedHostVPool", "Residency", "Staging", "Tier",
           "host_device_pointer", "mem_decode_ptrsel", "mem_dynamic_decode"]
