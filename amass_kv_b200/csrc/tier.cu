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
// Parallel form.  The reference walks the misses one at a time.  Here a
// classification kernel over the whole GPU touches the hits and marks the
// misses entry by entry (the gathers behind it are random and would
// serialise on one SM), then one CTA per kv-head (1) lists its misses in
// order in shared memory (each thread reads a contiguous range of the
// flattened (request, page-table entry) list; one block scan orders them),
// (2) dedups them with an atomicMin claim on page2slot (the first occurrence
// wins), (3) finds the `take` = min(unique misses, eligible slots) smallest
// (lru, index) keys: a radix select on the lru clock gives the take-th
// smallest value T, the fewer-than-take slots with lru < T are sorted, and
// slots with lru == T follow in index order, and (4) gives the k-th unique
// miss the k-th victim.  This picks the same victims as the sequential walk:
// an install makes its slot ineligible, so the k-th install of the walk takes
// the k-th smallest eligible key, and evicted pages are never misses of the
// same call.
#include <algorithm>
#include <climits>

#include "common.cuh"

namespace amass {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kPlanMaxSlots = 8192;
constexpr int kPlanMaxReq = 4096;
constexpr int kPer = 4;                 // entries per thread per round
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
  int32_t* mpage;         // (R, n_kv, MP): miss block | -(hit slot + 2) | -1
  int n_req, n_kv, MP, page, NB, S, max_miss;
};

// Block-wide exclusive scan of one int per thread (kPlanThreads threads);
// *total receives the block sum.  Ends with a barrier, so wtot can be reused.
AMASS_DEV int block_scan_excl(int v, int* wtot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wtot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int x = wtot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += t;
    }
    wtot[lane] = x;
  }
  __syncthreads();
  const int base = warp ? wtot[warp - 1] : 0;
  *total = wtot[kPlanWarps - 1];
  __syncthreads();
  return base + incl - v;
}

// Hit/miss classification of every selected entry (reference
// residency.py:45-82), spread over the whole GPU: the gathers it needs
// (page table -> block table -> page2slot) are random, and one SM's L1 would
// serialise them.  One warp per chunk of 32*kClsPer consecutive entries of a
// (request, kv-head) unit; a hit touches its slot (lru = clock + 1).
// mpage[entry] = block (>= 0) for a miss of a complete page, -(slot + 2) for
// a hit (its slot cannot be evicted by this call: it now holds the newest
// clock), -1 for a page that is not complete.
constexpr int kClsPer = 4;
constexpr int kClsChunk = 32 * kClsPer;

__global__ void __launch_bounds__(256)
tier_classify_kernel(PlanArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int chunks = (a.MP + kClsChunk - 1) / kClsChunk;
  const int items = a.n_req * a.n_kv * chunks;
  const int clk = a.clock[0] + 1;
  for (int it = gw; it < items; it += nw) {
    const int u = it / chunks, ch = it - u * chunks;
    const int c = __ldg(a.cnt + u);
    const int j0 = ch * kClsChunk + lane * kClsPer;
    if (ch * kClsChunk >= c) continue;
    const int r = u / a.n_kv, kv = u - r * a.n_kv;
    const int sl = __ldg(a.sl + r);
    const int32_t* tr = a.tab + (int64_t)u * a.MP;
    const int32_t* br = a.bt + (int64_t)r * a.bt_stride;
    int32_t* p2s = a.p2s + (int64_t)kv * a.NB;
    int pt[kClsPer], bk[kClsPer], slot[kClsPer];
#pragma unroll
    for (int i = 0; i < kClsPer; ++i)
      pt[i] = j0 + i < c ? __ldg(tr + j0 + i) : -1;
#pragma unroll
    for (int i = 0; i < kClsPer; ++i) {
      const bool comp = pt[i] >= 0 && (pt[i] + 1) * a.page <= sl;
      bk[i] = comp ? __ldg(br + pt[i]) : -1;
    }
#pragma unroll
    for (int i = 0; i < kClsPer; ++i) slot[i] = bk[i] >= 0 ? p2s[bk[i]] : -1;
#pragma unroll
    for (int i = 0; i < kClsPer; ++i) {
      if (j0 + i >= c) continue;
      const bool hit = bk[i] >= 0 && slot[i] >= 0;
      if (hit) a.lru[(int64_t)kv * a.S + slot[i]] = clk;
      a.mpage[(int64_t)u * a.MP + j0 + i] =
          hit ? -(slot[i] + 2) : (bk[i] >= 0 ? bk[i] : -1);
    }
  }
}

// Dynamic shared memory of the plan kernel: request offsets, the sort keys of
// the victims older than the threshold clock, the ordered victim slots, a copy
// of the lru clocks and the ordered miss list.
struct PlanSmem {
  int* reqoff;       // kPlanMaxReq + 1
  uint64_t* keys;    // S2
  int* victim;       // S
  int* lru;          // S: this kv-head's lru clocks after the hit touches
  int* mblk;         // max_miss
};

AMASS_DEV PlanSmem plan_smem(uint8_t* base, int S, int S2) {
  PlanSmem p;
  p.keys = reinterpret_cast<uint64_t*>(base);
  p.reqoff = reinterpret_cast<int*>(p.keys + S2);
  p.victim = p.reqoff + kPlanMaxReq + 1;
  p.lru = p.victim + S;
  p.mblk = p.lru + S;
  return p;
}

__global__ void __launch_bounds__(kPlanThreads)
tier_plan_kernel(PlanArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  extern __shared__ __align__(16) uint8_t smem[];
  int S2 = 1;
  while (S2 < a.S) S2 <<= 1;
  const PlanSmem sm = plan_smem(smem, a.S, S2);
  __shared__ int wtot[kPlanWarps];
  __shared__ unsigned wred[kPlanWarps], wred2[kPlanWarps], wred3[kPlanWarps];
  __shared__ int hist[2048];
  __shared__ int sel_bin, sel_below, nT, dropped;
  const int tid = threadIdx.x;
  const int kv = blockIdx.x;
  const int clk = a.clock[0] + 1;
  int32_t* p2s = a.p2s + (int64_t)kv * a.NB;
  int32_t* s2p = a.s2p + (int64_t)kv * a.S;
  int32_t* lru = a.lru + (int64_t)kv * a.S;
  if (tid == 0) { dropped = 0; nT = 0; }

  // ---- request offsets of this kv-head's selected pages ------------------
  int total;
  {
    const int per = (a.n_req + kPlanThreads - 1) / kPlanThreads;
    const int r0 = tid * per, r1 = min(r0 + per, a.n_req);
    int loc = 0;
    for (int r = r0; r < r1; ++r) loc += a.cnt[(int64_t)r * a.n_kv + kv];
    int run = block_scan_excl(loc, wtot, &total);
    for (int r = r0; r < r1; ++r) {
      sm.reqoff[r] = run;
      run += a.cnt[(int64_t)r * a.n_kv + kv];
    }
    if (tid == 0) sm.reqoff[a.n_req] = total;
    __syncthreads();
  }
  // ---- (1) misses in (request, entry) order: each thread reads kPer
  //      consecutive entries of the classified list; one block scan per
  //      round orders the appends.  (Hits were touched by the classifier.)
  int mtot = 0;
  for (int base = 0; base < total; base += kPlanThreads * kPer) {
    const int f0 = base + tid * kPer;
    int blk[kPer];
    int nm = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) blk[i] = -1;
    if (f0 < total) {
      int lo = 0, hi = a.n_req - 1;          // last r with reqoff[r] <= f0
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sm.reqoff[mid] <= f0) lo = mid; else hi = mid - 1;
      }
      int r = lo;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int f = f0 + i;
        if (f < total) {
          while (f >= sm.reqoff[r + 1]) ++r;
          blk[i] = a.mpage[((int64_t)r * a.n_kv + kv) * a.MP + (f - sm.reqoff[r])];
          if (blk[i] >= 0) ++nm; else blk[i] = -1;
        }
      }
    }
    int rtot;
    int pos = mtot + block_scan_excl(nm, wtot, &rtot);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (blk[i] < 0) continue;
      if (pos < a.max_miss) sm.mblk[pos] = blk[i];
      else dropped = 1;
      ++pos;
    }
    mtot += rtot;
  }
  __syncthreads();
  const int M = min(mtot, a.max_miss);
  // ---- (2) dedup: the first occurrence of a block claims page2slot -------
  for (int i = tid; i < M; i += kPlanThreads)
    atomicMin(&p2s[sm.mblk[i]], INT_MIN + i);
  __syncthreads();
  const int mper = (M + kPlanThreads - 1) / kPlanThreads;
  const int i0 = min(tid * mper, M), i1 = min(i0 + mper, M);
  int nu = 0;
  for (int i = i0; i < i1; ++i) {
    const int blk = sm.mblk[i];
    if (p2s[blk] == INT_MIN + i) ++nu;
    else sm.mblk[i] = blk | INT_MIN;                  // duplicate
  }
  int U;
  const int ubase = block_scan_excl(nu, wtot, &U);

  // ---- (3) victims: the `take` smallest (lru, slot) among slots with
  //      lru < clk, in order.  Radix-select the take-th smallest lru T
  //      (11-bit digits of lru - min), sort the fewer-than-take slots with
  //      lru < T, then append slots with lru == T in index order. ---------
  unsigned vmin = 0xffffffffu, vmax = 0u, ne = 0u;
  for (int s = tid; s < a.S; s += kPlanThreads) {
    const int l = lru[s];
    sm.lru[s] = l;
    if (l < clk) {
      const unsigned u = (unsigned)l ^ 0x80000000u;
      vmin = min(vmin, u);
      vmax = max(vmax, u);
      ++ne;
    }
  }
  {
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      vmin = min(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
      vmax = max(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
      ne += __shfl_xor_sync(0xffffffffu, ne, o);
    }
    if (lane == 0) { wred[warp] = vmin; wred2[warp] = vmax; wred3[warp] = ne; }
    __syncthreads();
    if (warp == 0) {
      vmin = wred[lane]; vmax = wred2[lane]; ne = wred3[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        vmin = min(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
        vmax = max(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
        ne += __shfl_xor_sync(0xffffffffu, ne, o);
      }
      if (lane == 0) { wred[0] = vmin; wred2[0] = vmax; wred3[0] = ne; }
    }
    __syncthreads();
    vmin = wred[0]; vmax = wred2[0]; ne = wred3[0];
  }
  const int E = (int)ne;
  const int take = min(U, E);
  if (take > 0) {
    const unsigned range = vmax - vmin;
    const int nbits = range ? 32 - __clz(range) : 0;
    unsigned prefix = 0, pmask = 0;
    int need = take, below = 0;
    for (int shift = nbits > 0 ? ((nbits + 10) / 11 - 1) * 11 : -1; shift >= 0;
         shift -= 11) {
      for (int b = tid; b < 2048; b += kPlanThreads) hist[b] = 0;
      __syncthreads();
      for (int s = tid; s < a.S; s += kPlanThreads) {
        const int l = sm.lru[s];
        const unsigned v = ((unsigned)l ^ 0x80000000u) - vmin;
        if (l < clk && (v & pmask) == prefix)
          atomicAdd(&hist[(v >> shift) & 2047], 1);
      }
      __syncthreads();
      const int h0 = hist[2 * tid], h1 = hist[2 * tid + 1];
      int tot;
      const int ex = block_scan_excl(h0 + h1, wtot, &tot);
      if (ex < need && need <= ex + h0) { sel_bin = 2 * tid; sel_below = ex; }
      else if (ex + h0 < need && need <= ex + h0 + h1) {
        sel_bin = 2 * tid + 1; sel_below = ex + h0;
      }
      __syncthreads();
      prefix |= (unsigned)sel_bin << shift;
      pmask |= 2047u << shift;
      need -= sel_below;
      below += sel_below;
      __syncthreads();
    }
    const unsigned T = vmin + prefix;           // biased lru of the threshold
    const int c = below;                        // slots with lru < T
    // keys of the slots older than T (unordered), then sorted
    int P2 = 1;
    while (P2 < c) P2 <<= 1;
    if (c > 0) {
      if (tid == 0) nT = 0;
      __syncthreads();
      for (int s = tid; s < a.S; s += kPlanThreads) {
        const int l = sm.lru[s];
        const unsigned u = (unsigned)l ^ 0x80000000u;
        if (l < clk && u < T) {
          const int k = atomicAdd(&nT, 1);
          sm.keys[k] = ((uint64_t)u << 32) | (uint32_t)s;
        }
      }
      __syncthreads();
      for (int k = c + tid; k < P2; k += kPlanThreads) sm.keys[k] = ~0ull;
      __syncthreads();
      for (int size = 2; size <= P2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int i = tid; i < P2 / 2; i += kPlanThreads) {
            const int lo = 2 * i - (i & (stride - 1));
            const int hi = lo + stride;
            const bool up = (lo & size) == 0;
            const uint64_t x = sm.keys[lo], y = sm.keys[hi];
            if ((x > y) == up) { sm.keys[lo] = y; sm.keys[hi] = x; }
          }
          __syncthreads();
        }
      }
      for (int k = tid; k < c; k += kPlanThreads)
        sm.victim[k] = (int)(sm.keys[k] & 0xffffffffu);
    }
    // slots with lru == T in index order fill victims [c, take): each
    // thread scans a contiguous run of slots, one block scan orders them
    {
      const int sper = (a.S + kPlanThreads - 1) / kPlanThreads;
      const int s0 = min(tid * sper, a.S), s1 = min(s0 + sper, a.S);
      int ne2 = 0;
      for (int s = s0; s < s1; ++s) {
        const int l = sm.lru[s];
        ne2 += (l < clk && ((unsigned)l ^ 0x80000000u) == T) ? 1 : 0;
      }
      int got;
      int pos = c + block_scan_excl(ne2, wtot, &got);
      for (int s = s0; s < s1 && pos < take; ++s) {
        const int l = sm.lru[s];
        if (l < clk && ((unsigned)l ^ 0x80000000u) == T) sm.victim[pos++] = s;
      }
    }
    __syncthreads();
  }
  // ---- (4) install: the k-th unique miss takes victim k -----------------
  int32_t* fl = a.flist + (int64_t)kv * a.S * 2;
  int k = ubase;
  for (int i = i0; i < i1; ++i) {
    const int blk = sm.mblk[i];
    if (blk < 0) continue;                       // duplicate
    if (k >= take) {
      p2s[blk] = -1;
      dropped = 1;
    } else {
      const int slot = sm.victim[k];
      const int old = s2p[slot];
      if (old >= 0) p2s[old] = -1;
      p2s[blk] = slot;
      s2p[slot] = blk;
      lru[slot] = clk;
      fl[2 * k] = blk;
      fl[2 * k + 1] = slot;
    }
    ++k;
  }
  __syncthreads();
  if (tid == 0) {
    a.fcnt[kv] = take;
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
  int staged_only;        // copy only the installs whose page is not flushed
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
    if (a.staged_only && vld) continue;
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
  const long long room = (long long)amass::kPlanSmem - 8LL * S2 -
                         8LL * hot_slots - 4LL * (amass::kPlanMaxReq + 1);
  return room > 0 ? (int)(room / 4) : 0;
}

extern "C" int amass_tier_plan(const int32_t* page_table,
                               const int32_t* page_cnt,
                               const int32_t* block_table, int64_t bt_stride,
                               const int32_t* seq_lens, int32_t* page2slot,
                               int32_t* slot2page, int32_t* lru_clock,
                               int32_t* clock, int32_t* overflow,
                               int32_t* fetch_list, int32_t* fetch_cnt,
                               int32_t* miss_pages, int n_req, int n_kv,
                               int max_pages, int page, int num_blocks,
                               int hot_slots, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || max_pages <= 0 || num_blocks <= 0 ||
      hot_slots <= 0 || page <= 0)
    return AMASS_ERR_ARG;
  if (!page_table || !page_cnt || !block_table || !seq_lens || !page2slot ||
      !slot2page || !lru_clock || !clock || !overflow || !fetch_list ||
      !fetch_cnt || !miss_pages)
    return AMASS_ERR_ARG;
  if (hot_slots > kPlanMaxSlots || n_req > kPlanMaxReq)
    return AMASS_ERR_UNSUPPORTED;
  int S2 = 1;
  while (S2 < hot_slots) S2 <<= 1;
  const int max_miss = amass_tier_plan_capacity(hot_slots);
  const size_t smem = (size_t)S2 * 8 + (size_t)hot_slots * 8 +
                      (size_t)(kPlanMaxReq + 1) * 4 + (size_t)max_miss * 4;
  PlanArgs a{};
  a.tab = page_table; a.cnt = page_cnt; a.bt = block_table;
  a.bt_stride = bt_stride; a.sl = seq_lens; a.p2s = page2slot;
  a.s2p = slot2page; a.lru = lru_clock; a.clock = clock; a.overflow = overflow;
  a.flist = fetch_list; a.fcnt = fetch_cnt; a.n_req = n_req; a.n_kv = n_kv;
  a.MP = max_pages; a.page = page; a.NB = num_blocks; a.S = hot_slots;
  a.max_miss = max_miss;
  a.mpage = miss_pages;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    const int chunks = (max_pages + kClsChunk - 1) / kClsChunk;
    const long long warps = (long long)n_req * n_kv * chunks;
    // an empty batch still runs the plan (the clock advances, as in the
    // reference's gather_plan): one idle classify CTA
    const int grid = (int)std::max<long long>(
        1, std::min<long long>((warps + 7) / 8, num_sms() * 8LL));
    if (int rc = launch_pdl(tier_classify_kernel, dim3(grid), dim3(256), 0, st,
                            a))
      return rc;
  }
  static unsigned long long configured = 0;
  if (first_on_device(configured)) {
    cudaFuncSetAttribute(tier_plan_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kPlanSmem);
  }
  if (int rc = launch_pdl(tier_plan_kernel, dim3(n_kv), dim3(kPlanThreads),
                          smem, st, a))
    return rc;
  return launch_status();
}

namespace amass {
namespace {
int tier_fetch_impl(const int32_t* fetch_list, const int32_t* fetch_cnt,
                    void* hot, void* pool_dev, int8_t* pool_valid,
                    const int32_t* vbo, const void* v_pool, int64_t svb,
                    int64_t svt, int64_t svh, void* hot_k, void* pool_k_dev,
                    const void* k_pool, int layer, int num_blocks, int n_kv,
                    int hot_slots, int page, int head_dim, void* stream,
                    bool staged_only) {
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
  FetchArgs a{};
  a.flist = fetch_list; a.fcnt = fetch_cnt;
  a.hot = static_cast<int16_t*>(hot); a.pool = static_cast<int16_t*>(pool_dev);
  a.valid = pool_valid; a.vbo = vbo;
  a.vpool = static_cast<const int16_t*>(v_pool);
  a.svb = svb; a.svt = svt; a.svh = svh;
  a.hot_k = static_cast<int16_t*>(hot_k);
  a.pool_k = static_cast<int16_t*>(pool_k_dev);
  a.kpool = static_cast<const int16_t*>(k_pool);
  a.layer = layer; a.NB = num_blocks; a.n_kv = n_kv; a.S = hot_slots;
  a.staged_only = staged_only ? 1 : 0;
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
}  // namespace
}  // namespace amass

extern "C" int amass_tier_fetch(const int32_t* fetch_list,
                                const int32_t* fetch_cnt, void* hot,
                                void* pool_dev, int8_t* pool_valid,
                                const int32_t* vbo, const void* v_pool,
                                int64_t svb, int64_t svt, int64_t svh,
                                void* hot_k, void* pool_k_dev,
                                const void* k_pool, int layer, int num_blocks,
                                int n_kv, int hot_slots, int page, int head_dim,
                                void* stream) {
  return amass::tier_fetch_impl(fetch_list, fetch_cnt, hot, pool_dev,
                                pool_valid, vbo, v_pool, svb, svt, svh, hot_k,
                                pool_k_dev, k_pool, layer, num_blocks, n_kv,
                                hot_slots, page, head_dim, stream, false);
}

extern "C" int amass_tier_fetch_staged(
    const int32_t* fetch_list, const int32_t* fetch_cnt, void* hot,
    void* pool_dev, int8_t* pool_valid, const int32_t* vbo, const void* v_pool,
    int64_t svb, int64_t svt, int64_t svh, void* hot_k, void* pool_k_dev,
    const void* k_pool, int layer, int num_blocks, int n_kv, int hot_slots,
    int page, int head_dim, void* stream) {
  return amass::tier_fetch_impl(fetch_list, fetch_cnt, hot, pool_dev,
                                pool_valid, vbo, v_pool, svb, svt, svh, hot_k,
                                pool_k_dev, k_pool, layer, num_blocks, n_kv,
                                hot_slots, page, head_dim, stream, true);
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
  InvalArgs a{};
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

// ===========================================================================
// Staging lifecycle of the tier's write side (reference tier/staging.py:
// 51-232, begin_step :312-346, scatter_kv :348-367).  Under mem-v the V of
// the tokens written each step lands in a bounded VRAM staging pool
// v_pool (L, NV, page, n_kv, d); once a page is complete its V is flushed to
// the pinned pool and the staging block recycled through a free stack.
// begin_step runs, in this order (flush-before-reuse):
//   1. v_slot_mapping[:n_tokens] = -1
//   2. vflush_clear  pages written this step lose their flushed latch
//   3. collect       complete pages written by earlier steps that hold a
//                    staging block: claim the flushed latch (first claim
//                    enters the flush list (blk, vb), at most max_flush) and
//                    free the staging block (pushed on the free stack)
//   4. flush copy    v_pool[l, vb] -> pinned pool[l, blk] for every layer and
//                    kv-head, pool_valid = 1 (bit copies)
//   5. valloc        a staging block for every page written this step that
//                    has none (pop the free stack; underflow sets overflow)
//   6. vslot         v_slot_mapping[token] = vb * page + pos % page, or -1
// Requests with seq_len <= 0 or no new tokens are skipped throughout.
// ===========================================================================
namespace amass {
namespace {

struct StgArgs {
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* sl;
  const int32_t* qsl;     // (n_req + 1,)
  int n_req, n_tokens, page;
  int64_t* vslot;         // (max_tokens,)
  int32_t* vbo;           // (NB,)
  int32_t* vfl;           // (NB,) flushed latch
  int32_t* stack;         // (NV,)
  int32_t* top;           // (1,)
  int32_t* flist;         // (MAXF, 2)
  int32_t* fcnt;          // (1,)
  int32_t* ovf;           // (1,)
  int MAXF;
  const int16_t* vpool;   // (L, NV, page, n_kv, d) at svl/svb/svt/svh
  const int16_t* kpool;   // mem-kv (or null)
  int64_t svl, svb, svt, svh;
  int16_t* pool;          // pinned (L, NB, n_kv, page, d) device view
  int16_t* poolk;
  int8_t* valid;          // (L, n_kv, NB)
  int L, NB, n_kv;
  int32_t* cand;          // [0] = count, [1..cap] = keys r * bt_stride + p
  int cand_cap;           // 0: collect walks every complete page itself
};

AMASS_DEV void req_span(const StgArgs& a, int r, int& sl, int& ql) {
  sl = a.sl[r];
  ql = a.qsl[r + 1] - a.qsl[r];
}

__global__ void stg_vflush_clear_kernel(StgArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int r = blockIdx.x;
  int sl, ql;
  req_span(a, r, sl, ql);
  if (r == 0 && threadIdx.x == 0 && a.cand) a.cand[0] = 0;
  if (sl <= 0 || ql <= 0) return;
  const int p0 = (sl - ql) / a.page, p1 = (sl - 1) / a.page;
  for (int p = p0 + (int)threadIdx.x; p <= p1; p += blockDim.x)
    a.vfl[a.bt[(int64_t)r * a.bt_stride + p]] = 0;
}

// Whole-GPU pre-pass of collect: the complete settled pages whose block is
// staged (vbo >= 0) -- a handful among all context pages -- appended in any
// order as keys r * bt_stride + p.  grid (x, n_req).
__global__ void __launch_bounds__(256) stg_cand_kernel(StgArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int r = blockIdx.y;
  int sl, ql;
  req_span(a, r, sl, ql);
  if (sl <= 0 || ql <= 0) return;
  const int np_ctx = (sl - ql) / a.page;
  const int64_t row = (int64_t)r * a.bt_stride;
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < np_ctx;
       p += gridDim.x * blockDim.x) {
    const int blk = __ldg(a.bt + row + p);
    if (a.vbo[blk] >= 0) {
      const int i = atomicAdd(a.cand, 1);
      if (i < a.cand_cap) a.cand[1 + i] = (int)(row + p);
    }
  }
}

constexpr int kStgThreads = 1024;

// Block-wide exclusive scan of a 0/1 flag (kStgThreads threads); *tot gets
// the block count.  Ends with a barrier.
AMASS_DEV int stg_scan(int v, int* wsum, int* tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned bal = __ballot_sync(0xffffffffu, v != 0);
  if (lane == 0) wsum[warp] = __popc(bal);
  __syncthreads();
  int off = 0, t = 0;
  for (int w = 0; w < kStgThreads / 32; ++w) {
    off += w < warp ? wsum[w] : 0;
    t += wsum[w];
  }
  __syncthreads();
  *tot = t;
  return off + __popc(bal & ((1u << lane) - 1u));
}

constexpr int kStgCandCap = 4096;

// One ordered chunk of collect: thread t holds the t-th page of the chunk
// (vb < 0: nothing to do).  A staged page whose latch was clear enters the
// flush list (past max_flush the latch is undone and the page stays staged);
// every staged page that leaves staging frees its block onto the stack.  The
// two block scans keep list slots and pushes in chunk order.
AMASS_DEV void stg_collect_chunk(const StgArgs& a, int blk, int vb, int* wsum,
                                 int& s_fcnt, int& s_top) {
  int fl = 1;
  if (vb >= 0) fl = atomicExch(a.vfl + blk, 1);
  const bool act = vb >= 0;
  const bool nw = act && fl == 0;
  int nnew;
  const int i = s_fcnt + stg_scan(nw, wsum, &nnew);
  const bool ok = nw && i < a.MAXF;
  if (ok) {
    a.flist[2 * i] = blk;
    a.flist[2 * i + 1] = vb;
  }
  const bool over = nw && !ok;
  if (over) a.vfl[blk] = 0;
  int old = -1;
  if (act && !over) old = atomicExch(a.vbo + blk, -1);
  const bool dofree = old >= 0;
  int nfree;
  const int j = s_top + stg_scan(dofree, wsum, &nfree);
  if (dofree) a.stack[j] = old;
  if (threadIdx.x == 0) {
    s_fcnt = min(s_fcnt + nnew, a.MAXF);
    s_top += nfree;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kStgThreads)
stg_collect_kernel(StgArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ int wsum[kStgThreads / 32];
  __shared__ int s_fcnt, s_top;
  __shared__ int keys[kStgCandCap];
  if (threadIdx.x == 0) { s_fcnt = 0; s_top = *a.top; }
  const int ncand = a.cand_cap > 0 ? *a.cand : 0;
  __syncthreads();
  if (a.cand_cap > 0 && ncand <= a.cand_cap) {
    // ascending keys = (request, page) order: bitonic sort in shared memory
    int n2 = 1;
    while (n2 < ncand) n2 <<= 1;
    for (int i = threadIdx.x; i < n2; i += kStgThreads)
      keys[i] = i < ncand ? a.cand[1 + i] : INT_MAX;
    __syncthreads();
    for (int k = 2; k <= n2; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < n2; i += kStgThreads) {
          const int x = i ^ j;
          if (x > i) {
            const int u = keys[i], w = keys[x];
            if (((i & k) == 0) == (u > w)) { keys[i] = w; keys[x] = u; }
          }
        }
        __syncthreads();
      }
    for (int c0 = 0; c0 < ncand; c0 += kStgThreads) {
      const int c = c0 + threadIdx.x;
      int blk = 0, vb = -1;
      if (c < ncand) {
        blk = a.bt[keys[c]];
        vb = a.vbo[blk];
      }
      stg_collect_chunk(a, blk, vb, wsum, s_fcnt, s_top);
    }
  } else {
    for (int r = 0; r < a.n_req; ++r) {
    int sl, ql;
    req_span(a, r, sl, ql);
    if (sl <= 0 || ql <= 0) continue;
      const int np_ctx = (sl - ql) / a.page;
      for (int p0 = 0; p0 < np_ctx; p0 += kStgThreads) {
        const int p = p0 + threadIdx.x;
        int blk = 0, vb = -1;
        if (p < np_ctx) {
          blk = a.bt[(int64_t)r * a.bt_stride + p];
          vb = a.vbo[blk];
        }
        stg_collect_chunk(a, blk, vb, wsum, s_fcnt, s_top);
      }
    }
  }
  if (threadIdx.x == 0) {
    *a.fcnt = s_fcnt;
    *a.top = s_top;
  }
}

// one warp per (flush entry, layer, kv-head) tile
template <int D>
__global__ void __launch_bounds__(256)
stg_flush_copy_kernel(StgArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int n = min(*a.fcnt, a.MAXF);
  const int total = n * a.L * a.n_kv;
  constexpr int64_t kTile = 16 * D;
  for (int it = gw; it < total; it += nw) {
    const int e = it / (a.L * a.n_kv);
    const int rem = it - e * a.L * a.n_kv;
    const int l = rem / a.n_kv, kv = rem - l * a.n_kv;
    const int64_t blk = a.flist[2 * e], vb = a.flist[2 * e + 1];
    const int64_t src = l * a.svl + vb * a.svb + kv * a.svh;
    const int64_t dst = (((int64_t)l * a.NB + blk) * a.n_kv + kv) * kTile;
    copy_tile<D>(a.pool + dst, a.vpool + src, a.svt, lane);
    if (a.kpool) copy_tile<D>(a.poolk + dst, a.kpool + src, a.svt, lane);
    if (lane == 0) a.valid[((int64_t)l * a.n_kv + kv) * a.NB + blk] = 1;
  }
}

// Block-wide exclusive scan of an int (kStgThreads threads); *tot gets the
// block sum.  Ends with a barrier.
AMASS_DEV int stg_scan_int(int v, int* wsum, int* tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  int off = 0, t = 0;
  for (int w = 0; w < kStgThreads / 32; ++w) {
    off += w < warp ? wsum[w] : 0;
    t += wsum[w];
  }
  __syncthreads();
  *tot = t;
  return off + x - v;
}

// Staging blocks for the pages written this step, in (request, page) order
// off the LIFO free stack: the k-th page without a block takes
// stack[top - 1 - k]; pages past the stack's depth set the overflow latch.
// One CTA; the written pages of up to 1024 requests are flattened and their
// (block table, vbo) loads issued together.  (A block written by two
// requests in one step -- not a valid engine state -- would get two blocks.)
__global__ void __launch_bounds__(kStgThreads) stg_valloc_kernel(StgArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ int wsum[kStgThreads / 32];
  __shared__ int offs[kStgThreads + 1], p0s[kStgThreads];
  __shared__ int s_top, s_ovf;
  const int tid = threadIdx.x;
  if (tid == 0) { s_top = *a.top; s_ovf = 0; }
  for (int r0 = 0; r0 < a.n_req; r0 += kStgThreads) {
    int c = 0, p0 = 0;
    if (r0 + tid < a.n_req) {
      int sl, ql;
      req_span(a, r0 + tid, sl, ql);
      if (sl > 0 && ql > 0) {
        p0 = (sl - ql) / a.page;
        c = (sl - 1) / a.page - p0 + 1;
      }
    }
    int tot;
    const int ex = stg_scan_int(c, wsum, &tot);
    offs[tid] = ex;
    p0s[tid] = p0;
    if (tid == 0) offs[kStgThreads] = tot;
    __syncthreads();
    for (int e0 = 0; e0 < tot; e0 += kStgThreads) {
      const int e = e0 + tid;
      int blk = 0;
      bool need = false;
      if (e < tot) {
        int lo = 0, hi = kStgThreads;          // offs[lo] <= e < offs[hi]
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (offs[mid] <= e) lo = mid; else hi = mid;
        }
        const int64_t row = (int64_t)(r0 + lo) * a.bt_stride;
        blk = a.bt[row + p0s[lo] + (e - offs[lo])];
        need = a.vbo[blk] < 0;
      }
      const int top0 = s_top;
      int nneed;
      const int k = stg_scan(need, wsum, &nneed);
      if (need) {
        const int idx = top0 - 1 - k;
        if (idx >= 0) a.vbo[blk] = a.stack[idx];
        else s_ovf = 1;
      }
      if (tid == 0) s_top = max(top0 - nneed, 0);
      __syncthreads();
    }
    __syncthreads();
  }
  if (tid == 0) {
    *a.top = s_top;
    if (s_ovf) *a.ovf = 1;
  }
}

__global__ void stg_vslot_kernel(StgArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int r = blockIdx.y;
  int sl, ql;
  req_span(a, r, sl, ql);
  if (sl <= 0 || ql <= 0) return;
  const int q0 = a.qsl[r];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ql;
       i += gridDim.x * blockDim.x) {
    const int pos = sl - ql + i;
    const int blk = a.bt[(int64_t)r * a.bt_stride + pos / a.page];
    const int vb = a.vbo[blk];
    a.vslot[q0 + i] = vb >= 0 ? (int64_t)vb * a.page + pos % a.page : -1;
  }
}

struct ScatArgs {
  const int16_t* v;       // (n_tokens, n_kv, d) at svt/svh
  const int16_t* k;       // mem-kv (or null)
  int64_t vt, vh, kt, kh;
  const int64_t* vslot;
  int16_t* vp;            // this layer (NV, page, n_kv, d) at pb/pt/ph
  int16_t* kp;
  int64_t pb, pt, ph;
  int n_tokens, n_kv, d, page;
};

// one warp per token: its n_kv rows of d 16-bit values, 16-byte pieces
__global__ void __launch_bounds__(256) stg_scatter_kernel(ScatArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= a.n_tokens) return;
  const int64_t vs = a.vslot[t];
  if (vs < 0) return;
  const int64_t vb = vs / a.page, off = vs % a.page;
  const int per = a.d / 8;
  for (int e = lane; e < a.n_kv * per; e += 32) {
    const int kv = e / per, ch = e - kv * per;
    const int64_t dst = vb * a.pb + off * a.pt + kv * a.ph + ch * 8;
    *reinterpret_cast<uint4*>(a.vp + dst) =
        *reinterpret_cast<const uint4*>(a.v + t * a.vt + kv * a.vh + ch * 8);
    if (a.k)
      *reinterpret_cast<uint4*>(a.kp + dst) =
          *reinterpret_cast<const uint4*>(a.k + t * a.kt + kv * a.kh + ch * 8);
  }
}

}  // namespace
}  // namespace amass

extern "C" int amass_staging_begin_step(
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* query_start_loc, int n_req, int n_tokens, int max_query_len,
    int64_t* v_slot_mapping, int32_t* vbo, int32_t* v_flushed,
    int32_t* free_stack, int32_t* free_top, int32_t* flush_list,
    int32_t* flush_cnt, int32_t* overflow, int max_flush, const void* v_pool,
    const void* k_pool, int64_t svl, int64_t svb, int64_t svt, int64_t svh,
    void* pool_dev, void* pool_k_dev, int8_t* pool_valid, int num_layers,
    int num_blocks, int n_kv, int head_dim, int page, int32_t* cand,
    int cand_cap, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_tokens < 0 || num_layers <= 0 || num_blocks <= 0 ||
      n_kv <= 0 || max_flush <= 0 || cand_cap < 0 || (cand_cap > 0 && !cand))
    return AMASS_ERR_ARG;
  if (!v_slot_mapping || !vbo || !v_flushed || !free_stack || !free_top ||
      !flush_list || !flush_cnt || !overflow || !v_pool || !pool_dev ||
      !pool_valid || (n_req > 0 && (!block_table || !seq_lens || !query_start_loc)))
    return AMASS_ERR_ARG;
  if ((k_pool != nullptr) != (pool_k_dev != nullptr)) return AMASS_ERR_ARG;
  if (page != 16 || (head_dim != 64 && head_dim != 128)) return AMASS_ERR_UNSUPPORTED;
  const uintptr_t al = reinterpret_cast<uintptr_t>(v_pool) |
                       reinterpret_cast<uintptr_t>(k_pool) |
                       reinterpret_cast<uintptr_t>(pool_dev) |
                       reinterpret_cast<uintptr_t>(pool_k_dev);
  if ((al & 15) || (svl % 8) || (svb % 8) || (svt % 8) || (svh % 8))
    return AMASS_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_tokens > 0 &&
      cudaMemsetAsync(v_slot_mapping, 0xff, sizeof(int64_t) * n_tokens, st) !=
          cudaSuccess)
    return AMASS_ERR_CUDA;
  if (n_req == 0) return AMASS_OK;
  StgArgs a{};
  a.bt = block_table; a.bt_stride = bt_stride; a.sl = seq_lens;
  a.qsl = query_start_loc; a.n_req = n_req; a.n_tokens = n_tokens;
  a.page = page; a.vslot = v_slot_mapping; a.vbo = vbo; a.vfl = v_flushed;
  a.stack = free_stack; a.top = free_top; a.flist = flush_list;
  a.fcnt = flush_cnt; a.ovf = overflow; a.MAXF = max_flush;
  a.vpool = static_cast<const int16_t*>(v_pool);
  a.kpool = static_cast<const int16_t*>(k_pool);
  a.svl = svl; a.svb = svb; a.svt = svt; a.svh = svh;
  a.pool = static_cast<int16_t*>(pool_dev);
  a.poolk = static_cast<int16_t*>(pool_k_dev);
  a.valid = pool_valid; a.L = num_layers; a.NB = num_blocks; a.n_kv = n_kv;
  // keys must fit int32; otherwise collect walks the pages itself
  const bool use_cand = cand_cap > 0 && (int64_t)n_req * bt_stride < INT_MAX;
  a.cand = use_cand ? cand : nullptr;
  a.cand_cap = use_cand ? std::min(cand_cap, kStgCandCap) : 0;
  int rc;
  if ((rc = launch_pdl(stg_vflush_clear_kernel, dim3(n_req), dim3(32), 0, st, a))) return rc;
  if (use_cand) {
    const int gx = (int)std::min<int64_t>((bt_stride + 255) / 256, 64);
    if ((rc = launch_pdl(stg_cand_kernel, dim3(gx, n_req), dim3(256), 0, st, a)))
      return rc;
  }
  if ((rc = launch_pdl(stg_collect_kernel, dim3(1), dim3(kStgThreads), 0, st, a))) return rc;
  {
    const long long warps = (long long)max_flush * num_layers * n_kv;
    const int grid = (int)std::min<long long>((warps + 7) / 8, num_sms() * 8LL);
    rc = head_dim == 128
             ? launch_pdl(stg_flush_copy_kernel<128>, dim3(grid), dim3(256), 0, st, a)
             : launch_pdl(stg_flush_copy_kernel<64>, dim3(grid), dim3(256), 0, st, a);
    if (rc) return rc;
  }
  if ((rc = launch_pdl(stg_valloc_kernel, dim3(1), dim3(kStgThreads), 0, st, a))) return rc;
  {
    const int bx = std::max(1, std::min((max_query_len + 127) / 128, 64));
    if ((rc = launch_pdl(stg_vslot_kernel, dim3(bx, n_req), dim3(128), 0, st, a)))
      return rc;
  }
  return launch_status();
}

extern "C" int amass_staging_scatter(const void* value, int64_t v_st,
                                     int64_t v_sh, const void* key,
                                     int64_t k_st, int64_t k_sh,
                                     const int64_t* v_slot_mapping,
                                     void* v_pool_layer, void* k_pool_layer,
                                     int64_t pb, int64_t pt, int64_t ph,
                                     int n_tokens, int n_kv, int head_dim,
                                     int page, void* stream) {
  using namespace amass;
  if (n_tokens < 0 || n_kv <= 0 || head_dim <= 0 || page <= 0) return AMASS_ERR_ARG;
  if (n_tokens == 0) return AMASS_OK;
  if (!value || !v_slot_mapping || !v_pool_layer) return AMASS_ERR_ARG;
  if ((key != nullptr) != (k_pool_layer != nullptr)) return AMASS_ERR_ARG;
  const uintptr_t al = reinterpret_cast<uintptr_t>(value) |
                       reinterpret_cast<uintptr_t>(key) |
                       reinterpret_cast<uintptr_t>(v_pool_layer) |
                       reinterpret_cast<uintptr_t>(k_pool_layer);
  if ((al & 15) || (head_dim % 8) || (v_st % 8) || (v_sh % 8) ||
      (key && ((k_st % 8) || (k_sh % 8))) || (pb % 8) || (pt % 8) || (ph % 8))
    return AMASS_ERR_ARG;
  ScatArgs a{};
  a.v = static_cast<const int16_t*>(value);
  a.k = static_cast<const int16_t*>(key);
  a.vt = v_st; a.vh = v_sh; a.kt = k_st; a.kh = k_sh;
  a.vslot = v_slot_mapping;
  a.vp = static_cast<int16_t*>(v_pool_layer);
  a.kp = static_cast<int16_t*>(k_pool_layer);
  a.pb = pb; a.pt = pt; a.ph = ph;
  a.n_tokens = n_tokens; a.n_kv = n_kv; a.d = head_dim; a.page = page;
  if (int rc = launch_pdl(stg_scatter_kernel, dim3((n_tokens + 7) / 8), dim3(256),
                          0, static_cast<cudaStream_t>(stream), a))
    return rc;
  return launch_status();
}
