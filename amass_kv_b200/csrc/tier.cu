// mem-v / mem-kv DRAM tier on sm_100a: exact-LRU hot-buffer residency plan,
// the miss fetch from the pinned, device-mapped host pool, and the
// invalidation of rewritten pages (reference tier/residency.py:45-282).
//
// Plan semantics (per layer; residency.py:45-139, gather_plan :385-407):
//   clk = clock + 1, and the call leaves clock = clk.  For every
//   (request, kv-head) unit and every selected COMPLETE page: a resident page
//   (page2slot >= 0) is a hit and its slot is touched (lru = clk); otherwise
//   it is a miss.  Per kv-head, misses are taken in (request, page-table)
//   order; a page already installed this call is skipped (dedup); each
//   remaining miss takes the slot with the smallest (lru, slot index) among
//   slots with lru < clk (exact LRU), evicts that slot's old page, installs
//   the miss (lru = clk) and is appended to the fetch list.  With no eligible
//   slot left the miss stays non-resident and the overflow flag is set (the
//   decode then reads that page from the staging or pinned pool).
//
// Parallel form.  The reference walks the misses one at a time.  Here one CTA
// per kv-head (1) touches hits and lists its misses in order in shared
// memory, (2) dedups them with an atomicMin claim on page2slot (the first
// occurrence wins), (3) sorts the slots by (lru, index) with a bitonic sort,
// ineligible slots last, and (4) gives the k-th unique miss the k-th sorted
// slot.  This picks the same victims as the sequential walk: an install makes
// its slot ineligible, so the k-th install of the walk takes the k-th
// smallest eligible key, and evicted pages are never misses of the same call.
#include <algorithm>

#include "common.cuh"

namespace amass {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kPlanMaxSlots = 8192;
constexpr size_t kPlanSmem = 200 * 1024;

struct PlanArgs {
  const int32_t* tab;     // (R, n_kv, MP)
  const int32_t* cnt;     // (R, n_kv)
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* sl;
  int32_t* p2s;           // (n_kv, NB)   this layer
  int32_t* s2p;           // (n_kv, S)
  int32_t* lru;           // (n_kv, S)
  int32_t* clock;         // [0] clock, [1] CTA ticket (0 between calls)
  int32_t* overflow;      // (1,)
  int32_t* flist;         // (n_kv, S, 2): (blk, slot)
  int32_t* fcnt;          // (n_kv,)
  int n_req, n_kv, MP, page, NB, S, max_miss;
};

// Ordered block-wide append of one flag per thread: returns this thread's
// position (meaningful when flag) and advances *base by the block total.
AMASS_DEV int block_append(bool flag, int* wcnt, int* base) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned bal = __ballot_sync(0xffffffffu, flag);
  if (lane == 0) wcnt[warp] = __popc(bal);
  __syncthreads();
  int off = *base, tot = 0;
#pragma unroll 4
  for (int w = 0; w < kPlanWarps; ++w) {
    const int c = wcnt[w];
    off += w < warp ? c : 0;
    tot += c;
  }
  const int pos = off + __popc(bal & ((1u << lane) - 1u));
  __syncthreads();
  if (threadIdx.x == 0) *base += tot;
  __syncthreads();
  return pos;
}

__global__ void __launch_bounds__(kPlanThreads)
tier_plan_kernel(PlanArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  extern __shared__ __align__(16) uint8_t smem[];
  int S2 = 1;
  while (S2 < a.S) S2 <<= 1;
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem);   // S2 (lru, slot) keys
  int* mblk = reinterpret_cast<int*>(keys + S2);        // misses, in order
  __shared__ int wcnt[kPlanWarps];
  __shared__ int nmiss, nuniq, neligible, dropped;
  const int kv = blockIdx.x;
  const int clk = a.clock[0] + 1;
  int32_t* p2s = a.p2s + (int64_t)kv * a.NB;
  int32_t* s2p = a.s2p + (int64_t)kv * a.S;
  int32_t* lru = a.lru + (int64_t)kv * a.S;
  if (threadIdx.x == 0) { nmiss = 0; nuniq = 0; dropped = 0; }
  __syncthreads();

  // (1) hits touch their slot; misses of complete pages are listed in
  //     (request, page-table) order
  for (int r = 0; r < a.n_req; ++r) {
    const int c = a.cnt[(int64_t)r * a.n_kv + kv];
    const int sl = a.sl[r];
    const int32_t* tr = a.tab + ((int64_t)r * a.n_kv + kv) * a.MP;
    const int32_t* btr = a.bt + (int64_t)r * a.bt_stride;
    for (int j0 = 0; j0 < c; j0 += kPlanThreads) {
      const int j = j0 + threadIdx.x;
      bool miss = false;
      int blk = 0;
      if (j < c) {
        const int pt = tr[j];
        if ((pt + 1) * a.page <= sl) {
          blk = btr[pt];
          const int slot = p2s[blk];
          if (slot >= 0) lru[slot] = clk;
          else miss = true;
        }
      }
      const int pos = block_append(miss, wcnt, &nmiss);
      if (miss) {
        if (pos < a.max_miss) mblk[pos] = blk;
        else dropped = 1;
      }
    }
  }
  __syncthreads();
  const int M = min(nmiss, a.max_miss);
  // (2) dedup: the first occurrence of a block claims page2slot
  for (int i = threadIdx.x; i < M; i += kPlanThreads)
    atomicMin(&p2s[mblk[i]], INT_MIN + i);
  // (3) slot keys: (lru biased to unsigned, index); slots touched this call
  //     get the top band and sort last
  for (int s = threadIdx.x; s < S2; s += kPlanThreads) {
    uint64_t k = ~0ull;
    if (s < a.S) {
      const int l = lru[s];
      const uint32_t hi = l >= clk ? 0xffffffffu
                                   : (uint32_t)l ^ 0x80000000u;
      k = ((uint64_t)hi << 32) | (uint32_t)s;
    }
    keys[s] = k;
  }
  __syncthreads();
  for (int size = 2; size <= S2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < S2 / 2; i += kPlanThreads) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t x = keys[lo], y = keys[hi];
        if ((x > y) == up) { keys[lo] = y; keys[hi] = x; }
      }
      __syncthreads();
    }
  }
  // eligible slots = keys below the top band (sorted: binary search)
  if (threadIdx.x == 0) {
    int lo = 0, hi = a.S;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((uint32_t)(keys[mid] >> 32) != 0xffffffffu) lo = mid + 1; else hi = mid;
    }
    neligible = lo;
  }
  __syncthreads();
  // (4) install: the k-th unique miss takes the k-th eligible slot.  A later
  //     duplicate of an installed block reads a slot (>= 0), not its claim.
  const int E = neligible;
  int32_t* fl = a.flist + (int64_t)kv * a.S * 2;
  for (int i0 = 0; i0 < M; i0 += kPlanThreads) {
    const int i = i0 + threadIdx.x;
    int blk = 0;
    bool u = false;
    if (i < M) {
      blk = mblk[i];
      u = p2s[blk] == INT_MIN + i;
    }
    const int k = block_append(u, wcnt, &nuniq);
    if (u) {
      if (k >= E) {
        p2s[blk] = -1;
        dropped = 1;
      } else {
        const int slot = (int)(keys[k] & 0xffffffffu);
        const int old = s2p[slot];
        if (old >= 0) p2s[old] = -1;
        p2s[blk] = slot;
        s2p[slot] = blk;
        lru[slot] = clk;
        fl[2 * k] = blk;
        fl[2 * k + 1] = slot;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    a.fcnt[kv] = min(nuniq, E);
    if (dropped) atomicExch(a.overflow, 1);
    // the last CTA to finish commits the advanced clock; every CTA read the
    // clock before taking its ticket
    __threadfence();
    const int t = atomicAdd(&a.clock[1], 1);
    if (t == (int)gridDim.x - 1) {
      a.clock[0] = clk;
      a.clock[1] = 0;
    }
  }
}

struct FetchArgs {
  const int32_t* flist;   // (n_kv, S, 2)
  const int32_t* fcnt;    // (n_kv,)
  int16_t* hot;           // (n_kv, S, page, d) this layer
  int16_t* pool;          // pinned (L, NB, n_kv, page, d), device view
  int8_t* valid;          // (n_kv, NB) this layer
  const int32_t* vbo;     // (NB,)
  const int16_t* vpool;   // staging, this layer (NV, page, n_kv, d) strided
  int64_t svb, svt, svh;
  int16_t* hot_k;         // mem-kv K tier (all null under mem-v)
  int16_t* pool_k;
  const int16_t* kpool;
  int layer, NB, n_kv, S;
};

// One warp copies one (16 x D) tile of 16-bit elements: all loads first
// (PER 16-byte loads per lane in flight, which the host link's latency
// needs), then all stores.  dst rows are contiguous; src rows are src_rs
// elements apart.  Bit copies.
template <int D>
AMASS_DEV void copy_tile(int16_t* dst, const int16_t* src, int64_t src_rs,
                         int lane) {
  constexpr int kPerRow = D / 8;
  constexpr int PER = 16 * kPerRow / 32;
  uint4 v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    const int row = e / kPerRow, ch = e % kPerRow;
    v[i] = __ldcv(reinterpret_cast<const uint4*>(src + row * src_rs + ch * 8));
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    const int row = e / kPerRow, ch = e % kPerRow;
    *reinterpret_cast<uint4*>(dst + (int64_t)row * D + ch * 8) = v[i];
  }
}

// Fetch of the installed misses (reference residency.py:196-248): pinned pool
// when flushed (pool_valid), else the staging pool with write-through to the
// pinned pool and pool_valid = 1, else the pinned pool.  One warp per entry.
template <int D>
__global__ void __launch_bounds__(256)
tier_fetch_kernel(FetchArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  constexpr int64_t kTile = 16 * D;
  const int total = a.n_kv * a.S;
  for (int i = gw; i < total; i += nw) {
    const int kv = i / a.S, e = i - kv * a.S;
    if (e >= a.fcnt[kv]) continue;
    const int blk = a.flist[2 * (int64_t)i], slot = a.flist[2 * (int64_t)i + 1];
    const int64_t hot_off = ((int64_t)kv * a.S + slot) * kTile;
    const int64_t pool_off =
        (((int64_t)a.layer * a.NB + blk) * a.n_kv + kv) * kTile;
    const bool vld = a.valid[(int64_t)kv * a.NB + blk] > 0;
    const int vb = a.vbo[blk];
    if (vld || vb < 0) {
      copy_tile<D>(a.hot + hot_off, a.pool + pool_off, D, lane);
      if (a.hot_k) copy_tile<D>(a.hot_k + hot_off, a.pool_k + pool_off, D, lane);
    } else {
      const int16_t* src = a.vpool + vb * a.svb + kv * a.svh;
      copy_tile<D>(a.hot + hot_off, src, a.svt, lane);
      copy_tile<D>(a.pool + pool_off, src, a.svt, lane);
      if (a.hot_k) {
        const int16_t* ks = a.kpool + vb * a.svb + kv * a.svh;
        copy_tile<D>(a.hot_k + hot_off, ks, a.svt, lane);
        copy_tile<D>(a.pool_k + pool_off, ks, a.svt, lane);
      }
      if (lane == 0) a.valid[(int64_t)kv * a.NB + blk] = 1;
    }
  }
}

struct InvalArgs {
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* sl;
  const int32_t* qsl;     // (R+1,) query start locations
  int32_t* p2s;           // (L, n_kv, NB)
  int32_t* s2p;           // (L, n_kv, S)
  int8_t* valid;          // (L, n_kv, NB)
  int n_req, L, n_kv, NB, S, page;
};

// Drop residency and pool validity of every page (re)written this step, in
// all layers and kv-heads (reference residency.py:251-282).  One thread per
// (layer, kv-head, request) walks the pages of the request's new tokens.
__global__ void tier_invalidate_kernel(InvalArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)a.L * a.n_kv * a.n_req;
  if (t >= total) return;
  const int r = (int)(t % a.n_req);
  const int64_t lk = t / a.n_req;            // layer * n_kv + kv
  const int sl = a.sl[r];
  if (sl <= 0) return;
  const int ql = a.qsl[r + 1] - a.qsl[r];
  const int p0 = (sl - ql) / a.page, p1 = (sl - 1) / a.page;
  for (int p = max(p0, 0); p <= p1; ++p) {
    const int blk = a.bt[(int64_t)r * a.bt_stride + p];
    const int64_t row = lk * a.NB + blk;
    a.valid[row] = 0;
    const int slot = a.p2s[row];
    if (slot >= 0) {
      a.p2s[row] = -1;
      a.s2p[lk * a.S + slot] = -1;
    }
  }
}

}  // namespace
}  // namespace amass

extern "C" int amass_tier_plan_capacity(int hot_slots) {
  if (hot_slots <= 0 || hot_slots > amass::kPlanMaxSlots) return 0;
  int S2 = 1;
  while (S2 < hot_slots) S2 <<= 1;
  const long long room = (long long)amass::kPlanSmem - 8LL * S2;
  return room > 0 ? (int)(room / 4) : 0;
}

extern "C" int amass_tier_plan(const int32_t* page_table,
                               const int32_t* page_cnt,
                               const int32_t* block_table, int64_t bt_stride,
                               const int32_t* seq_lens, int32_t* page2slot,
                               int32_t* slot2page, int32_t* lru_clock,
                               int32_t* clock, int32_t* overflow,
                               int32_t* fetch_list, int32_t* fetch_cnt,
                               int n_req, int n_kv, int max_pages, int page,
                               int num_blocks, int hot_slots, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || max_pages <= 0 || num_blocks <= 0 ||
      hot_slots <= 0 || page <= 0)
    return AMASS_ERR_ARG;
  if (!page_table || !page_cnt || !block_table || !seq_lens || !page2slot ||
      !slot2page || !lru_clock || !clock || !overflow || !fetch_list ||
      !fetch_cnt)
    return AMASS_ERR_ARG;
  if (hot_slots > kPlanMaxSlots) return AMASS_ERR_UNSUPPORTED;
  int S2 = 1;
  while (S2 < hot_slots) S2 <<= 1;
  const int max_miss = amass_tier_plan_capacity(hot_slots);
  const size_t smem = (size_t)S2 * 8 + (size_t)max_miss * 4;
  PlanArgs a;
  a.tab = page_table; a.cnt = page_cnt; a.bt = block_table;
  a.bt_stride = bt_stride; a.sl = seq_lens; a.p2s = page2slot;
  a.s2p = slot2page; a.lru = lru_clock; a.clock = clock; a.overflow = overflow;
  a.flist = fetch_list; a.fcnt = fetch_cnt; a.n_req = n_req; a.n_kv = n_kv;
  a.MP = max_pages; a.page = page; a.NB = num_blocks; a.S = hot_slots;
  a.max_miss = max_miss;
  static int configured = 0;
  if (!configured) {
    cudaFuncSetAttribute(tier_plan_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kPlanSmem);
    configured = 1;
  }
  if (int rc = launch_pdl(tier_plan_kernel, dim3(n_kv), dim3(kPlanThreads),
                          smem, static_cast<cudaStream_t>(stream), a))
    return rc;
  return launch_status();
}

extern "C" int amass_tier_fetch(const int32_t* fetch_list,
                                const int32_t* fetch_cnt, void* hot,
                                void* pool_dev, int8_t* pool_valid,
                                const int32_t* vbo, const void* v_pool,
                                int64_t svb, int64_t svt, int64_t svh,
                                void* hot_k, void* pool_k_dev,
                                const void* k_pool, int layer, int num_blocks,
                                int n_kv, int hot_slots, int page, int head_dim,
                                void* stream) {
  using namespace amass;
  if (!fetch_list || !fetch_cnt || !hot || !pool_dev || !pool_valid || !vbo ||
      !v_pool || num_blocks <= 0 || n_kv <= 0 || hot_slots <= 0 || layer < 0)
    return AMASS_ERR_ARG;
  if ((hot_k != nullptr) != (pool_k_dev != nullptr) ||
      (hot_k != nullptr) != (k_pool != nullptr))
    return AMASS_ERR_ARG;
  if (page != 16) return AMASS_ERR_UNSUPPORTED;
  // 16-byte copies: every base and stride in whole 8-element pieces
  const uintptr_t al = reinterpret_cast<uintptr_t>(hot) |
                       reinterpret_cast<uintptr_t>(pool_dev) |
                       reinterpret_cast<uintptr_t>(v_pool) |
                       reinterpret_cast<uintptr_t>(hot_k) |
                       reinterpret_cast<uintptr_t>(pool_k_dev) |
                       reinterpret_cast<uintptr_t>(k_pool);
  if ((al & 15) || (svb % 8) || (svt % 8) || (svh % 8)) return AMASS_ERR_ARG;
  FetchArgs a;
  a.flist = fetch_list; a.fcnt = fetch_cnt;
  a.hot = static_cast<int16_t*>(hot); a.pool = static_cast<int16_t*>(pool_dev);
  a.valid = pool_valid; a.vbo = vbo;
  a.vpool = static_cast<const int16_t*>(v_pool);
  a.svb = svb; a.svt = svt; a.svh = svh;
  a.hot_k = static_cast<int16_t*>(hot_k);
  a.pool_k = static_cast<int16_t*>(pool_k_dev);
  a.kpool = static_cast<const int16_t*>(k_pool);
  a.layer = layer; a.NB = num_blocks; a.n_kv = n_kv; a.S = hot_slots;
  const long long warps = (long long)n_kv * hot_slots;
  const int grid = (int)std::min<long long>((warps + 7) / 8, num_sms() * 8LL);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  if (head_dim == 128)
    rc = launch_pdl(tier_fetch_kernel<128>, dim3(grid), dim3(256), 0, st, a);
  else if (head_dim == 64)
    rc = launch_pdl(tier_fetch_kernel<64>, dim3(grid), dim3(256), 0, st, a);
  else
    return AMASS_ERR_UNSUPPORTED;
  if (rc) return rc;
  return launch_status();
}

extern "C" int amass_tier_invalidate(const int32_t* block_table,
                                     int64_t bt_stride,
                                     const int32_t* seq_lens,
                                     const int32_t* query_start_loc,
                                     int32_t* page2slot, int32_t* slot2page,
                                     int8_t* pool_valid, int n_req,
                                     int num_layers, int n_kv, int num_blocks,
                                     int hot_slots, int page, void* stream) {
  using namespace amass;
  if (n_req < 0 || num_layers <= 0 || n_kv <= 0 || num_blocks <= 0 ||
      hot_slots <= 0 || page <= 0)
    return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!block_table || !seq_lens || !query_start_loc || !page2slot ||
      !slot2page || !pool_valid)
    return AMASS_ERR_ARG;
  InvalArgs a;
  a.bt = block_table; a.bt_stride = bt_stride; a.sl = seq_lens;
  a.qsl = query_start_loc; a.p2s = page2slot; a.s2p = slot2page;
  a.valid = pool_valid; a.n_req = n_req; a.L = num_layers; a.n_kv = n_kv;
  a.NB = num_blocks; a.S = hot_slots; a.page = page;
  const long long total = (long long)num_layers * n_kv * n_req;
  if (int rc = launch_pdl(tier_invalidate_kernel,
                          dim3((unsigned)((total + 127) / 128)), dim3(128), 0,
                          static_cast<cudaStream_t>(stream), a))
    return rc;
  return launch_status();
}

extern "C" int amass_host_device_pointer(void* host, void** dev) {
  if (!host || !dev) return AMASS_ERR_ARG;
  return cudaHostGetDevicePointer(dev, host, 0) == cudaSuccess ? AMASS_OK
                                                               : AMASS_ERR_CUDA;
}
