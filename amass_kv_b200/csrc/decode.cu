// Stage B on sm_100a: split-K sparse paged decode over the selected pages
// with a log-sum-exp merge (reference attention/decode.py:128-241,
// attention/merge.py:21-50).
//
// Work decomposition.  The selected pages of all (request, kv-head) units,
// units in order, form one flat list of P pages.  A persistent grid of 4-warp
// CTAs cuts it into equal contiguous runs, one per warp (each CTA first scans
// the per-unit page counts into shared memory), so a ragged batch balances
// across the SMs to within one page.  A run that crosses a unit boundary
// writes one (m, l, acc) partial per unit it touches; the partials of a unit
// are the consecutive runs that cover it.  Each warp streams its pages
// through its own NST-deep cp.async ring in shared memory (16-byte copies
// into an XOR-swizzled [token][d] tile, zero-filled beyond seq_len); the ring
// runs across unit boundaries.  (The reference cuts each unit into
// pps = max(ceil(cnt/split), PPS_MIN)-page chunks, decode.py:154-160; any
// cut is an exact re-association of the same softmax.)
//
// Per page a warp computes the transposed products: S^T = K Q^T
// (m16n8k16 bf16 MMAs, rows = the 16 tokens from ldmatrix, cols = the G query
// heads of the group), an online softmax per head in the log2 domain, and
// O^T += V^T P^T (V^T via ldmatrix.trans, P^T moved into the B operand with
// movmatrix) -- D/16 MMAs for each product, half of the head-major form.  A
// second kernel merges the partials of each (request, query head) and writes
// bf16 output.
#include <cstdlib>

#include "common.cuh"

namespace amass {
namespace {

// warps per CTA and cp.async ring depth per warp (head_dim 128); override
// at build time only for tuning sweeps
#ifndef AMASS_DEC_WARPS
#define AMASS_DEC_WARPS 8
#endif
#ifndef AMASS_DEC_NST
#define AMASS_DEC_NST 2
#endif
constexpr int kDecWarps = AMASS_DEC_WARPS;
constexpr int kMaxPeers = 8;
constexpr int kDecThreads = kDecWarps * 32;

struct DecArgs {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  const __nv_bfloat16* k;
  int64_t k_sb, k_st, k_sh;
  const __nv_bfloat16* v;
  int64_t v_sb, v_st, v_sh;
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* tab;
  const int32_t* cnt;
  const int32_t* sl;
  float* m_part;
  float* l_part;
  float* acc_part;
  __nv_bfloat16* out;
  int64_t o_st, o_sh;
  float scale_log2;
  int split, pps_min;
  int n_req, n_kv, G, MP, units;
  // mem-v / mem-kv tier sources (TIER kernels only): per page the V tile
  // (and the K tile when hot_k is set) comes from the hot buffer when the
  // page is complete and resident, else the staging pool when vbo >= 0,
  // else the pinned pool (reference tier/decode_mem.py:118-147)
  const __nv_bfloat16* hot_v;   // (n_kv, S, 16, D)
  const __nv_bfloat16* hot_k;   // null: K from the resident cache k
  const __nv_bfloat16* stg_v;   // (NV, 16, n_kv, D) at svb/svt/svh
  const __nv_bfloat16* stg_k;
  const __nv_bfloat16* pool_v;  // pinned (L, NB, n_kv, 16, D), device view
  const __nv_bfloat16* pool_k;
  int64_t svb, svt, svh;
  const int32_t* p2s;           // (n_kv, NB) this layer
  const int32_t* vbo;           // (NB,)
  const int32_t* eslot;         // (R, n_kv, MP) classified entries or null
  int t_layer, t_NB, t_S;
  // install mode (TIER): a page the residency plan installed this step is
  // read from its source (staging or pinned) and its tile is then written
  // into the assigned hot slot (and written through to the pinned pool when
  // it came from staging unflushed) -- the miss fetch, done by the decode
  int8_t* pvalid;               // (n_kv, NB) this layer, or null
  int install;
  int dec_warps;                // warps of the decode grid (run split)
  int merge_wph;                // merge warps per (request, head) row
  // merged rows go to n_out buffers (this GPU's `out` alone, or every
  // rank's output under kv-head sharding: peer addresses over NVLink), at
  // global head head_off + local head
  __nv_bfloat16* outs[kMaxPeers];
  int n_out, head_off;
};

// Pages per warp run: the flat list of P selected pages (units in order) is
// cut into runs of `share` pages, one per warp of the grid (nw warps), so the
// runs are balanced to within one page whatever the unit sizes; a run that
// crosses units writes one partial per unit it touches.  The floor
// ceil(cmax / (split - 1)) bounds the partials of any unit by `split`.
AMASS_DEV int range_share(int P, int cmax, int nw, int split, int pps_min) {
  int s = (P + nw - 1) / max(nw, 1);
  s = max(s, max(pps_min, 1));
  s = max(s, (cmax + split - 2) / (split - 1));
  return s;
}

template <int D>
struct Tile {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kChunks = D / 8;              // 16-byte chunks per row
  static constexpr int kTileBytes = 16 * kRowBytes;  // one K or V page tile
  static constexpr int kStageBytes = 2 * kTileBytes;
};

AMASS_DEV uint32_t swz(int row, int chunk) { return chunk ^ (row & 7); }

// one landed 16 x D tile (XOR-swizzled rows in shared memory) to a dense
// row-major tile in global memory, 16-byte stores
template <int D>
AMASS_DEV void install_tile(const uint8_t* src, uint8_t* dst, int lane) {
  using T = Tile<D>;
#pragma unroll
  for (int i = 0; i < (16 * T::kChunks) / 32; ++i) {
    const int id = lane + 32 * i;
    const int row = id / T::kChunks, ch = id % T::kChunks;
    const uint4 x = *reinterpret_cast<const uint4*>(
        src + row * T::kRowBytes + swz(row, ch) * 16);
    *reinterpret_cast<uint4*>(dst + row * T::kRowBytes + ch * 16) = x;
  }
}

template <int D, int NST, bool TIER>
__global__ void __launch_bounds__(kDecThreads)
decode_kernel(DecArgs a) {
  grid_dep_wait();     // inputs written by the previous kernel
  grid_dep_launch();
  using T = Tile<D>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;                                    // warps x NST
  // per stage: install targets (hot V, hot K, pinned V, pinned K, valid
  // flag; 0 = none), then the valid row count
  uint64_t* inst = reinterpret_cast<uint64_t*>(smem + kDecWarps * NST * T::kStageBytes);
  int* meta = reinterpret_cast<int*>(inst + kDecWarps * NST * 5);
  int* pfx = meta + kDecWarps * NST;                         // units + 1

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int U = a.units;

  // ---- page prefix over units and the largest unit (every CTA; tiny) -----
  __shared__ int wtot[kDecWarps], wmx[kDecWarps];
  {
    const int per = (U + kDecThreads - 1) / kDecThreads;
    const int u0 = threadIdx.x * per;
    int local = 0, mx = 0;
    for (int u = u0; u < min(u0 + per, U); ++u) {
      const int c = max(a.cnt[u], 0);
      local += c;
      mx = max(mx, c);
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 31) wtot[warp] = incl;
    if (lane == 0) wmx[warp] = mx;
    __syncthreads();
    int woff = 0;
    for (int w = 0; w < warp; ++w) woff += wtot[w];
    int run = woff + incl - local;
    for (int u = u0; u < min(u0 + per, U); ++u) {
      pfx[u] = run;
      run += max(a.cnt[u], 0);
    }
    if (threadIdx.x == kDecThreads - 1) pfx[U] = run;
    __syncthreads();
  }
  int cmax = 0;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) cmax = max(cmax, wmx[w]);
  const int P = pfx[U];
  const int share = range_share(P, cmax, (int)gridDim.x * kDecWarps, a.split,
                                a.pps_min);
  // ---- this warp's contiguous run [g0, g1) of the flat page list ---------
  const int w = blockIdx.x * kDecWarps + warp;
  const int g0 = (int)min((int64_t)w * share, (int64_t)P);
  const int g1 = min(g0 + share, P);
  if (g0 >= g1) return;
  // unit holding flat page f: largest u with pfx[u] <= f (and pfx[u+1] > f)
  auto unit_of = [&](int f) {
    int lo = 0, hi = U - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pfx[mid] <= f) lo = mid; else hi = mid - 1;
    }
    return lo;
  };

  uint8_t* my_stages = stages + warp * NST * T::kStageBytes;
  int* my_meta = meta + warp * NST;
  uint64_t* my_inst = inst + warp * NST * 5;

  // Index batches: lane i resolves page ib + i of this run -- page table,
  // block table and (tier) source lookups -- into the K and V tile
  // addresses and the valid row count, 32 pages per round of independent
  // loads, so the copy stream never waits on a dependent index load.
  int ib = g0;
  uint64_t bk = 0, bv = 0;
  int bvalid = 0, bkst = 0, bvst = 0;
  uint64_t bi_v = 0, bi_k = 0, bw_v = 0, bw_k = 0, bw_f = 0;   // install mode
  auto resolve = [&](int base) {
    ib = base;
    const int f = base + lane;
    if (f < g1) {
      const int u = unit_of(f);
      const int j = f - pfx[u];
      const int r = u / a.n_kv, kv = u - r * a.n_kv;
      const int pt = a.tab[(int64_t)u * a.MP + j];
      // hot slot of a classified hit (-(slot + 2)), loaded beside pt
      const int ev = (TIER && a.eslot) ? a.eslot[(int64_t)u * a.MP + j] : -1;
      const int64_t blk = a.bt[(int64_t)r * a.bt_stride + pt];
      const int seq = a.sl[r];
      bvalid = min(16, seq - pt * 16);
      const __nv_bfloat16* kp = a.k + blk * a.k_sb + kv * a.k_sh;
      const __nv_bfloat16* vp = a.v + blk * a.v_sb + kv * a.v_sh;
      int64_t kst = a.k_st, vst = a.v_st;
      bi_v = bi_k = bw_v = bw_k = bw_f = 0;
      if constexpr (TIER) {
        // one source decision per page, on the address (same bytes, so the
        // math matches the resident decode bit for bit)
        const int hslot = ev <= -2 ? -ev - 2 : a.p2s[(int64_t)kv * a.t_NB + blk];
        const bool complete = (pt + 1) * 16 <= seq;
        // install mode: a miss the plan gave a slot is not in it yet
        const bool installed = a.install && ev >= 0 && complete && hslot >= 0;
        const bool use_hot = ev <= -2 || (complete && hslot >= 0 && !installed);
        const int vb = use_hot ? -1 : a.vbo[blk];
        int64_t off;
        const __nv_bfloat16 *hv, *hk;
        if (use_hot) {
          off = ((int64_t)kv * a.t_S + hslot) * (16 * D);
          hv = a.hot_v; hk = a.hot_k; vst = D;
        } else if (vb >= 0) {
          off = vb * a.svb + kv * a.svh;
          hv = a.stg_v; hk = a.stg_k; vst = a.svt;
        } else {
          off = (((int64_t)a.t_layer * a.t_NB + blk) * a.n_kv + kv) * (16 * D);
          hv = a.pool_v; hk = a.pool_k; vst = D;
        }
        vp = hv + off;
        if (a.hot_k) { kp = hk + off; kst = vst; }
        if (installed) {
          const int64_t hoff = ((int64_t)kv * a.t_S + hslot) * (16 * D);
          bi_v = reinterpret_cast<uint64_t>(a.hot_v + hoff);
          if (a.hot_k) bi_k = reinterpret_cast<uint64_t>(a.hot_k + hoff);
          const int64_t vrow = (int64_t)kv * a.t_NB + blk;
          if (vb >= 0 && a.pvalid[vrow] == 0) {
            // staged and not flushed: write through to the pinned pool
            const int64_t poff =
                (((int64_t)a.t_layer * a.t_NB + blk) * a.n_kv + kv) * (16 * D);
            bw_v = reinterpret_cast<uint64_t>(a.pool_v + poff);
            if (a.hot_k) bw_k = reinterpret_cast<uint64_t>(a.pool_k + poff);
            bw_f = reinterpret_cast<uint64_t>(a.pvalid + vrow);
          }
        }
      }
      bk = reinterpret_cast<uint64_t>(kp);
      bv = reinterpret_cast<uint64_t>(vp);
      bkst = (int)kst;
      bvst = (int)vst;
    }
  };
  resolve(g0);
  // K/V pages are read once: first out of L2, so the page and block
  // tables, partials and the next stage's inputs stay resident
  const uint64_t pol = l2_evict_first();
  // issue cursor: flat page fi of this run
  int fi = g0;
  auto issue = [&](int slot) {
    if (fi < g1) {
      if (fi - ib >= 32) resolve(fi);
      const int k = fi - ib;
      const int valid = __shfl_sync(0xffffffffu, bvalid, k);
      const __nv_bfloat16* kp = reinterpret_cast<const __nv_bfloat16*>(
          __shfl_sync(0xffffffffu, bk, k));
      const __nv_bfloat16* vp = reinterpret_cast<const __nv_bfloat16*>(
          __shfl_sync(0xffffffffu, bv, k));
      const int kst = __shfl_sync(0xffffffffu, bkst, k);
      const int vst = __shfl_sync(0xffffffffu, bvst, k);
      if (lane == 0) my_meta[slot] = valid;
      if (TIER && a.install) {
        const uint64_t iv = __shfl_sync(0xffffffffu, bi_v, k);
        const uint64_t ik = __shfl_sync(0xffffffffu, bi_k, k);
        const uint64_t wv = __shfl_sync(0xffffffffu, bw_v, k);
        const uint64_t wk = __shfl_sync(0xffffffffu, bw_k, k);
        const uint64_t wf = __shfl_sync(0xffffffffu, bw_f, k);
        if (lane == 0) {
          uint64_t* m = my_inst + slot * 5;
          m[0] = iv; m[1] = ik; m[2] = wv; m[3] = wk; m[4] = wf;
        }
      }
      const uint32_t sbase = smem_u32(my_stages + slot * T::kStageBytes);
#pragma unroll
      for (int i = 0; i < (16 * T::kChunks) / 32; ++i) {
        const int id = lane + 32 * i;
        const int row = id / T::kChunks, ch = id % T::kChunks;
        const bool ok = row < valid;
        const uint32_t doff = row * T::kRowBytes + swz(row, ch) * 16;
        const int rr = ok ? row : 0;
        cp_async16_pol(sbase + doff, kp + rr * kst + ch * 8, ok, pol);
        cp_async16_pol(sbase + T::kTileBytes + doff, vp + rr * vst + ch * 8, ok, pol);
      }
      ++fi;
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < NST - 1; ++s) issue(s);
  int slot_c = 0, slot_i = NST - 1;

  const int g = lane >> 2, c4 = lane & 3;
  constexpr int KS = D / 16;
  int fc = g0, uc = unit_of(g0);

  while (fc < g1) {
    const int u = uc;
    const int seg_end = min(pfx[u + 1], g1);
    const int r = u / a.n_kv, kv = u - r * a.n_kv;
    // Q fragment (B operand): cols = query heads of the group
    uint32_t qa[KS][2];
    {
      const bool gv = g < a.G;
      const __nv_bfloat16* qp = a.q + (int64_t)r * a.q_st +
                                (int64_t)(kv * a.G + (gv ? g : 0)) * a.q_sh;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(qp + 16 * s + 2 * c4);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(qp + 16 * s + 8 + 2 * c4);
        qa[s][0] = gv ? w0 : 0u;
        qa[s][1] = gv ? w1 : 0u;
      }
    }
    // per thread: query heads h0 = 2*c4, h1 = 2*c4 + 1 (columns of the
    // transposed tiles); l holds this lane's partial sums until the end
    float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
    float o[D / 16][4];   // O^T fragments: rows d = 16*dt + g (+8), cols h0, h1
#pragma unroll
    for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    for (; fc < seg_end; ++fc) {
      issue(slot_i);
      slot_i = (slot_i + 1 == NST) ? 0 : slot_i + 1;
      cp_async_wait<NST - 1>();
      __syncwarp();
      const uint32_t kbase = smem_u32(my_stages + slot_c * T::kStageBytes);
      const uint32_t vbase = kbase + T::kTileBytes;
      const int valid = my_meta[slot_c];
      if (TIER && a.install) {
        const uint64_t* m = my_inst + slot_c * 5;
        if (m[0]) {
          // the page's tiles (complete pages: all 16 rows) into the hot slot
          const uint8_t* st_k = my_stages + slot_c * T::kStageBytes;
          const uint8_t* st_v = st_k + T::kTileBytes;
          install_tile<D>(st_v, reinterpret_cast<uint8_t*>(m[0]), lane);
          if (m[1]) install_tile<D>(st_k, reinterpret_cast<uint8_t*>(m[1]), lane);
          if (m[2]) install_tile<D>(st_v, reinterpret_cast<uint8_t*>(m[2]), lane);
          if (m[3]) install_tile<D>(st_k, reinterpret_cast<uint8_t*>(m[3]), lane);
          if (m[4] && lane == 0) *reinterpret_cast<int8_t*>(m[4]) = 1;
        }
      }

      // S^T = K Q^T: rows = the 16 tokens, cols = the query heads; A = K
      // from shared memory (ldmatrix), B = the q fragment; two accumulators
      // (even / odd k-steps) halve the dependent MMA chain
      float st0[4] = {0.f, 0.f, 0.f, 0.f}, st1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int mat = lane >> 3, rin = lane & 7;
        const int tok = (mat & 1) * 8 + rin;
        const int ch = 2 * ks + (mat >> 1);
        uint32_t ka[4];
        ldsm_x4(ka, kbase + tok * T::kRowBytes + swz(tok, ch) * 16);
        mma_bf16((ks & 1) ? st1 : st0, ka, qa[ks][0], qa[ks][1]);
      }
      // online softmax per head (log2 domain): this lane holds tokens g and
      // g + 8 of heads h0, h1; the column max spans the 8 lanes of equal c4
      float x[4];
      x[0] = (g < valid) ? (st0[0] + st1[0]) * a.scale_log2 : -INFINITY;
      x[1] = (g < valid) ? (st0[1] + st1[1]) * a.scale_log2 : -INFINITY;
      x[2] = (g + 8 < valid) ? (st0[2] + st1[2]) * a.scale_log2 : -INFINITY;
      x[3] = (g + 8 < valid) ? (st0[3] + st1[3]) * a.scale_log2 : -INFINITY;
      float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
      for (int o_ = 4; o_ < 32; o_ <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o_));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o_));
      }
      const float mn0 = fmaxf(m_i[0], mx0), mn1 = fmaxf(m_i[1], mx1);
      const float al0 = exp2f(m_i[0] - mn0), al1 = exp2f(m_i[1] - mn1);
      const float p0 = exp2f(x[0] - mn0), p1 = exp2f(x[1] - mn1);
      const float p2 = exp2f(x[2] - mn0), p3 = exp2f(x[3] - mn1);
      l_i[0] = l_i[0] * al0 + (p0 + p2);
      l_i[1] = l_i[1] * al1 + (p1 + p3);
      m_i[0] = mn0;
      m_i[1] = mn1;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        o[i][0] *= al0; o[i][2] *= al0;
        o[i][1] *= al1; o[i][3] *= al1;
      }
      // P^T (tokens x heads) as the B operand: each 8x8 bf16 block of the
      // C fragment transposed in registers
      const uint32_t pb0 = movmatrix_t(pack_bf2(p0, p1));
      const uint32_t pb1 = movmatrix_t(pack_bf2(p2, p3));
      // O^T += V^T P^T: A = V^T tiles (ldmatrix.trans of the V rows)
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        const int mat = lane >> 3, rin = lane & 7;
        const int tok = (mat >> 1) * 8 + rin;
        const int ch = 2 * dt + (mat & 1);
        uint32_t va[4];
        ldsm_x4_t(va, vbase + tok * T::kRowBytes + swz(tok, ch) * 16);
        mma_bf16(o[dt], va, pb0, pb1);
      }
      __syncwarp();
      slot_c = (slot_c + 1 == NST) ? 0 : slot_c + 1;
    }

    // ---- this warp's partial of unit u: slot = segment index ------------
#pragma unroll
    for (int o_ = 4; o_ < 32; o_ <<= 1) {
      l_i[0] += __shfl_xor_sync(0xffffffffu, l_i[0], o_);
      l_i[1] += __shfl_xor_sync(0xffffffffu, l_i[1], o_);
    }
    const int64_t slotp = (int64_t)u * a.split + (w - pfx[u] / share);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int hh = 2 * c4 + j;
      if (hh < a.G) {
        if (g == 0) {
          a.m_part[slotp * a.G + hh] = m_i[j];
          a.l_part[slotp * a.G + hh] = l_i[j];
        }
        float* ab = a.acc_part + (slotp * a.G + hh) * D;
#pragma unroll
        for (int dt = 0; dt < D / 16; ++dt) {
          ab[16 * dt + g] = o[dt][j];
          ab[16 * dt + g + 8] = o[dt][2 + j];
        }
      }
    }
    // next non-empty unit
    uc = u + 1;
    while (uc < U - 1 && pfx[uc + 1] <= fc) ++uc;
  }
  cp_async_wait<0>();
}

// ---- merge of the run partials (reference attention/merge.py:30-50) -------
// A 256-thread CTA merges 8 / WPH (request, query head) rows; WPH warps
// share one row's partials (partial j goes to warp j % WPH) and combine
// their (m, l, acc) through shared memory.  WPH > 1 when there are few rows
// and many partials per row (small batches): it keeps the merge from
// running on a handful of warps.
constexpr int kMergeThreads = 256;

template <int D>
__global__ void __launch_bounds__(kMergeThreads)
merge_kernel(DecArgs a) {
  // Before the wait only the unit page counts are read: they come from the
  // kernel before the decode, which had completed when the decode (which
  // waits for it first thing) let this grid start.
  constexpr int PER = D / 32;
  __shared__ float sM[8], sL[8];
  __shared__ float sacc[8][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int WPH = a.merge_wph;
  const int part = warp % WPH;
  const int H = a.n_kv * a.G;
  const int idx = blockIdx.x * (8 / WPH) + warp / WPH;  // (r, h)
  const bool live = idx < a.n_req * H;
  const int r = live ? idx / H : 0, h = live ? idx - r * H : 0;
  const int kv = h / a.G, g = h - kv * a.G;
  const int u = r * a.n_kv + kv;
  // the decode's run split, once per CTA: pages of all units and of the
  // units before this CTA's first unit (every thread's loads in flight
  // together), the largest unit; then each row adds the few units between
  __shared__ int red[3][8];
  const int H_ = a.n_kv * a.G;
  const int idx0 = blockIdx.x * (8 / WPH);
  const int u_lo = min(idx0, a.n_req * H_ - 1) / a.G;
  int tot = 0, pre = 0, cmx = 0;
  {
    constexpr int kU = 4;
    for (int v0 = threadIdx.x * kU; v0 < a.units; v0 += kMergeThreads * kU) {
      int cv[kU];
#pragma unroll
      for (int j = 0; j < kU; ++j) cv[j] = v0 + j < a.units ? max(a.cnt[v0 + j], 0) : 0;
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        tot += cv[j];
        cmx = max(cmx, cv[j]);
        if (v0 + j < u_lo) pre += cv[j];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      pre += __shfl_xor_sync(0xffffffffu, pre, o);
      tot += __shfl_xor_sync(0xffffffffu, tot, o);
      cmx = max(cmx, __shfl_xor_sync(0xffffffffu, cmx, o));
    }
    if (lane == 0) { red[0][warp] = pre; red[1][warp] = tot; red[2][warp] = cmx; }
    __syncthreads();
    pre = tot = cmx = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      pre += red[0][w];
      tot += red[1][w];
      cmx = max(cmx, red[2][w]);
    }
  }
  float acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.f;
  float Mrun = -INFINITY;
  float L = 0.f;
  const int c = live ? max(a.cnt[u], 0) : 0;
  int mine = 0;
  if (c > 0) {
    for (int v = u_lo; v < u; ++v) pre += max(a.cnt[v], 0);
    const int share = range_share(tot, cmx, a.dec_warps, a.split, a.pps_min);
    const int nact = (pre + c - 1) / share - pre / share + 1;
    mine = nact > part ? (nact - part + WPH - 1) / WPH : 0;
  }
  grid_dep_wait();     // the decode's partials
  grid_dep_launch();
  if (mine > 0) {
    const int64_t s0 = (int64_t)u * a.split;
    const float* accb = a.acc_part + (s0 * a.G + g) * D + lane * PER;
    // partials in batches of kB, every load of a batch issued before any
    // use: a round's run weights (lane = run) and its first batch of acc
    // rows travel together, one memory round trip
    constexpr int kB = 8;
    auto load_batch = [&](float2 (*xs)[PER / 2], int j0, int base, int n) {
#pragma unroll
      for (int jj = 0; jj < kB; ++jj) {
        const int j = min(j0 + jj, n - 1);              // clamped: weight 0
        const float* ap = accb + (int64_t)(part + (base + j) * WPH) * a.G * D;
#pragma unroll
        for (int i = 0; i < PER; i += 2)
          xs[jj][i / 2] = __ldcg(reinterpret_cast<const float2*>(ap + i));
      }
    };
    for (int base = 0; base < mine; base += 32) {
      const int n = min(32, mine - base);
      float2 xs[kB][PER / 2];
      load_batch(xs, 0, base, n);
      float m = -INFINITY, l = 0.f;
      if (lane < n) {
        const int64_t sl = s0 + part + (base + lane) * WPH;
        m = a.m_part[sl * a.G + g];
        l = a.l_part[sl * a.G + g];
        if (!(l > 0.f)) m = -INFINITY;
      }
      float M = m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      // runs of this round are merged relative to their own max; rounds
      // (more than 32 runs per warp) are combined by rescaling below
      const float w = (m == -INFINITY) ? 0.f : exp2f(m - M);
      float lw = w * l;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
      float racc[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) racc[i] = 0.f;
      for (int j0 = 0; j0 < n; j0 += kB) {
        if (j0 > 0) load_batch(xs, j0, base, n);
#pragma unroll
        for (int jj = 0; jj < kB; ++jj) {
          const int j = j0 + jj;
          const float wsh = __shfl_sync(0xffffffffu, w, j & 31);
          const float wj = j < n ? wsh : 0.f;
#pragma unroll
          for (int i = 0; i < PER; i += 2) {
            racc[i] += wj * xs[jj][i / 2].x;
            racc[i + 1] += wj * xs[jj][i / 2].y;
          }
        }
      }
      if (base == 0 || Mrun == -INFINITY) {
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[i] = racc[i];
        L = lw;
        Mrun = M;
      } else if (M > -INFINITY) {
        const float Mn = fmaxf(Mrun, M);
        const float so = exp2f(Mrun - Mn), sn = exp2f(M - Mn);
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[i] = acc[i] * so + racc[i] * sn;
        L = L * so + lw * sn;
        Mrun = Mn;
      }
    }
  }
  if (WPH > 1) {
    // the WPH warps of a row combine through shared memory
    if (lane == 0) { sM[warp] = Mrun; sL[warp] = L; }
#pragma unroll
    for (int i = 0; i < PER; ++i) sacc[warp][lane * PER + i] = acc[i];
    __syncthreads();
    if (part == 0) {
      float M = -INFINITY;
      for (int p = 0; p < WPH; ++p) M = fmaxf(M, sM[warp + p]);
      float Lt = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[i] = 0.f;
      for (int p = 0; p < WPH; ++p) {
        const float mp = sM[warp + p];
        const float sp = (mp == -INFINITY) ? 0.f : exp2f(mp - M);
        Lt += sp * sL[warp + p];
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[i] += sp * sacc[warp + p][lane * PER + i];
      }
      L = Lt;
    }
  }
  if (!live || part != 0) return;
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint32_t w[PER / 2];
#pragma unroll
  for (int i = 0; i < PER; i += 2) w[i / 2] = pack_bf2(acc[i] * inv, acc[i + 1] * inv);
  const int64_t off = (int64_t)r * a.o_st + (int64_t)(a.head_off + h) * a.o_sh + lane * PER;
  for (int p = 0; p < a.n_out; ++p) {
    __nv_bfloat16* op = a.outs[p] + off;
    if constexpr (PER == 4) {
      *reinterpret_cast<uint2*>(op) = make_uint2(w[0], w[1]);
    } else {
#pragma unroll
      for (int i = 0; i < PER / 2; ++i) reinterpret_cast<uint32_t*>(op)[i] = w[i];
    }
  }
}

template <int D, int NST>
size_t decode_smem(int units) {
  return (size_t)kDecWarps * NST * Tile<D>::kStageBytes +
         (size_t)kDecWarps * NST * 5 * sizeof(uint64_t) +
         (size_t)kDecWarps * NST * sizeof(int) + (size_t)(units + 1) * sizeof(int);
}

template <int D, int NST, bool TIER>
int launch_decode(const DecArgs& a, cudaStream_t st) {
  const size_t smem = decode_smem<D, NST>(a.units);
  if (smem > 220 * 1024) return AMASS_ERR_UNSUPPORTED;
  auto kern = decode_kernel<D, NST, TIER>;
  static unsigned long long configured = 0;
  if (first_on_device(configured)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         220 * 1024);
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecThreads, smem);
  if (per_sm < 1) per_sm = 1;
  const int grid = num_sms() * per_sm;
  DecArgs b = a;
  b.dec_warps = grid * kDecWarps;
  if (int rc = launch_pdl(kern, dim3(grid), dim3(kDecThreads), smem, st, b)) return rc;
  int rc = launch_status();
  if (rc) return rc;
  const int heads = a.n_req * a.n_kv * a.G;
  // warps per merged row: enough rows x warps for one 8-warp CTA per SM
  // (1 at the C3 batch of 64 requests, 8 at batch 1)
  int wph = 1;
  while (wph < 8 && (long long)heads * wph < (long long)num_sms() * 8) wph <<= 1;
  b.merge_wph = wph;
  const int hpb = 8 / wph;
  if (int rc = launch_pdl(merge_kernel<D>, dim3((heads + hpb - 1) / hpb),
                          dim3(kMergeThreads), 0, st, b))
    return rc;
  return launch_status();
}

}  // namespace
}  // namespace amass

namespace amass {
namespace {

// Resident decode into n_out output buffers (outs[0] = out for the plain
// call); rows of this call's heads land at global head head_off + h.
int resident_decode(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v, int64_t v_sb,
    int64_t v_st, int64_t v_sh, const int32_t* block_table, int64_t bt_stride,
    const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, float* m_part, float* l_part, float* acc_part,
    int split, int pps_min, void* const* outs, int n_out, int head_off,
    int64_t o_stride_t, int64_t o_stride_h, float scale, int n_req, int n_kv,
    int G, int head_dim, int page, int max_pages, void* stream) {
  void* out = n_out > 0 ? outs[0] : nullptr;
  if (n_out < 1 || n_out > kMaxPeers || head_off < 0) return AMASS_ERR_ARG;
  for (int p = 0; p < n_out; ++p)
    if (!outs[p] || (head_dim == 128 && (reinterpret_cast<uintptr_t>(outs[p]) & 7)))
      return AMASS_ERR_ARG;
  if (head_dim == 128 && ((o_stride_t % 4) || (o_stride_h % 4)))
    return AMASS_ERR_ARG;
  if (n_req < 0 || n_kv <= 0 || G <= 0 || split < 2 || pps_min <= 0 ||
      max_pages <= 0)
    return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!q || !k || !v || !block_table || !page_table || !page_cnt || !seq_lens ||
      !m_part || !l_part || !acc_part || !out)
    return AMASS_ERR_ARG;
  if (G > 8 || page != 16) return AMASS_ERR_UNSUPPORTED;
  // 16-byte cp.async rows and 4-byte q/out accesses
  if ((k_st % 8) || (k_sb % 8) || (k_sh % 8) || (v_st % 8) || (v_sb % 8) ||
      (v_sh % 8) || (reinterpret_cast<uintptr_t>(k) & 15) ||
      (reinterpret_cast<uintptr_t>(v) & 15) || (q_stride_h % 2) ||
      (q_stride_t % 2) || (o_stride_h % 2) || (o_stride_t % 2))
    return AMASS_ERR_ARG;
  DecArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_stride_t; a.q_sh = q_stride_h;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.k_sb = k_sb; a.k_st = k_st; a.k_sh = k_sh;
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.v_sb = v_sb; a.v_st = v_st; a.v_sh = v_sh;
  a.bt = block_table; a.bt_stride = bt_stride;
  a.tab = page_table; a.cnt = page_cnt; a.sl = seq_lens;
  a.m_part = m_part; a.l_part = l_part; a.acc_part = acc_part;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_st = o_stride_t; a.o_sh = o_stride_h;
  for (int p = 0; p < n_out; ++p) a.outs[p] = static_cast<__nv_bfloat16*>(outs[p]);
  a.n_out = n_out; a.head_off = head_off;
  a.scale_log2 = scale * kLog2e;
  a.split = split; a.pps_min = pps_min;
  a.n_req = n_req; a.n_kv = n_kv; a.G = G; a.MP = max_pages;
  a.units = n_req * n_kv;
  a.hot_v = a.hot_k = a.stg_v = a.stg_k = a.pool_v = a.pool_k = nullptr;
  a.svb = a.svt = a.svh = 0;
  a.p2s = a.vbo = a.eslot = nullptr;
  a.t_layer = a.t_NB = a.t_S = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) return launch_decode<128, AMASS_DEC_NST, false>(a, st);
  if (head_dim == 64) return launch_decode<64, 3, false>(a, st);
  return AMASS_ERR_UNSUPPORTED;
}

}  // namespace
}  // namespace amass

extern "C" int amass_sparse_decode(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v, int64_t v_sb,
    int64_t v_st, int64_t v_sh, const int32_t* block_table, int64_t bt_stride,
    const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, float* m_part, float* l_part, float* acc_part,
    int split, int pps_min, void* out, int64_t o_stride_t, int64_t o_stride_h,
    float scale, int n_req, int n_kv, int G, int head_dim, int page,
    int max_pages, void* stream) {
  void* outs[1] = {out};
  return amass::resident_decode(
      q, q_stride_t, q_stride_h, k, k_sb, k_st, k_sh, v, v_sb, v_st, v_sh,
      block_table, bt_stride, page_table, page_cnt, seq_lens, m_part, l_part,
      acc_part, split, pps_min, outs, 1, 0, o_stride_t, o_stride_h, scale,
      n_req, n_kv, G, head_dim, page, max_pages, stream);
}

extern "C" int amass_sparse_decode_gather(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v, int64_t v_sb,
    int64_t v_st, int64_t v_sh, const int32_t* block_table, int64_t bt_stride,
    const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, float* m_part, float* l_part, float* acc_part,
    int split, int pps_min, void* const* out_peers, int n_peers,
    int head_offset, int64_t o_stride_t, int64_t o_stride_h, float scale,
    int n_req, int n_kv, int G, int head_dim, int page, int max_pages,
    void* stream) {
  if (!out_peers) return AMASS_ERR_ARG;
  return amass::resident_decode(
      q, q_stride_t, q_stride_h, k, k_sb, k_st, k_sh, v, v_sb, v_st, v_sh,
      block_table, bt_stride, page_table, page_cnt, seq_lens, m_part, l_part,
      acc_part, split, pps_min, out_peers, n_peers, head_offset, o_stride_t,
      o_stride_h, scale, n_req, n_kv, G, head_dim, page, max_pages, stream);
}

namespace amass {
namespace {
int tier_decode_impl(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* hot_v,
    const void* hot_k, const void* stg_v, const void* stg_k, int64_t svb,
    int64_t svt, int64_t svh, const void* pool_v, const void* pool_k,
    const int32_t* page2slot, const int32_t* vbo, const int32_t* entry_slots,
    int layer, int num_blocks, int hot_slots, const int32_t* block_table,
    int64_t bt_stride, const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, float* m_part, float* l_part, float* acc_part,
    int split, int pps_min, void* out, int64_t o_stride_t, int64_t o_stride_h,
    float scale, int n_req, int n_kv, int G, int head_dim, int page,
    int max_pages, void* stream, int8_t* pool_valid, int install) {
  if (n_req < 0 || n_kv <= 0 || G <= 0 || split < 2 || pps_min <= 0 ||
      max_pages <= 0 || layer < 0 || num_blocks <= 0 || hot_slots <= 0)
    return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  const bool k_tier = hot_k != nullptr;
  if (!q || !hot_v || !stg_v || !pool_v || !page2slot || !vbo ||
      !block_table || !page_table || !page_cnt || !seq_lens || !m_part ||
      !l_part || !acc_part || !out)
    return AMASS_ERR_ARG;
  if (k_tier ? (!stg_k || !pool_k) : !k) return AMASS_ERR_ARG;
  if (G > 8 || page != 16) return AMASS_ERR_UNSUPPORTED;
  const uintptr_t al = reinterpret_cast<uintptr_t>(hot_v) |
                       reinterpret_cast<uintptr_t>(stg_v) |
                       reinterpret_cast<uintptr_t>(pool_v) |
                       reinterpret_cast<uintptr_t>(hot_k) |
                       reinterpret_cast<uintptr_t>(stg_k) |
                       reinterpret_cast<uintptr_t>(pool_k) |
                       (k_tier ? 0 : reinterpret_cast<uintptr_t>(k));
  if ((al & 15) || (svb % 8) || (svt % 8) || (svh % 8) ||
      (!k_tier && ((k_st % 8) || (k_sb % 8) || (k_sh % 8))) ||
      (q_stride_h % 2) || (q_stride_t % 2) || (o_stride_h % 2) ||
      (o_stride_t % 2))
    return AMASS_ERR_ARG;
  DecArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_stride_t; a.q_sh = q_stride_h;
  a.k = static_cast<const __nv_bfloat16*>(k_tier ? hot_k : k);
  a.k_sb = k_tier ? 0 : k_sb; a.k_st = k_tier ? head_dim : k_st;
  a.k_sh = k_tier ? 0 : k_sh;
  a.v = static_cast<const __nv_bfloat16*>(hot_v);
  a.v_sb = 0; a.v_st = head_dim; a.v_sh = 0;
  a.bt = block_table; a.bt_stride = bt_stride;
  a.tab = page_table; a.cnt = page_cnt; a.sl = seq_lens;
  a.m_part = m_part; a.l_part = l_part; a.acc_part = acc_part;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_st = o_stride_t; a.o_sh = o_stride_h;
  a.outs[0] = a.out; a.n_out = 1; a.head_off = 0;
  if (head_dim == 128 && ((o_stride_t % 4) || (o_stride_h % 4) ||
                          (reinterpret_cast<uintptr_t>(out) & 7)))
    return AMASS_ERR_ARG;
  a.scale_log2 = scale * kLog2e;
  a.split = split; a.pps_min = pps_min;
  a.n_req = n_req; a.n_kv = n_kv; a.G = G; a.MP = max_pages;
  a.units = n_req * n_kv;
  a.hot_v = static_cast<const __nv_bfloat16*>(hot_v);
  a.hot_k = static_cast<const __nv_bfloat16*>(hot_k);
  a.stg_v = static_cast<const __nv_bfloat16*>(stg_v);
  a.stg_k = static_cast<const __nv_bfloat16*>(stg_k);
  a.pool_v = static_cast<const __nv_bfloat16*>(pool_v);
  a.pool_k = static_cast<const __nv_bfloat16*>(pool_k);
  a.svb = svb; a.svt = svt; a.svh = svh;
  a.p2s = page2slot; a.vbo = vbo; a.eslot = entry_slots;
  a.t_layer = layer; a.t_NB = num_blocks; a.t_S = hot_slots;
  a.pvalid = pool_valid; a.install = install;
  if (install && (!pool_valid || !entry_slots)) return AMASS_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) return launch_decode<128, AMASS_DEC_NST, true>(a, st);
  if (head_dim == 64) return launch_decode<64, 3, true>(a, st);
  return AMASS_ERR_UNSUPPORTED;
}
}  // namespace
}  // namespace amass

extern "C" int amass_tier_decode(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* hot_v,
    const void* hot_k, const void* stg_v, const void* stg_k, int64_t svb,
    int64_t svt, int64_t svh, const void* pool_v, const void* pool_k,
    const int32_t* page2slot, const int32_t* vbo, const int32_t* entry_slots,
    int layer, int num_blocks, int hot_slots, const int32_t* block_table,
    int64_t bt_stride, const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, float* m_part, float* l_part, float* acc_part,
    int split, int pps_min, void* out, int64_t o_stride_t, int64_t o_stride_h,
    float scale, int n_req, int n_kv, int G, int head_dim, int page,
    int max_pages, void* stream) {
  return amass::tier_decode_impl(
      q, q_stride_t, q_stride_h, k, k_sb, k_st, k_sh, hot_v, hot_k, stg_v,
      stg_k, svb, svt, svh, pool_v, pool_k, page2slot, vbo, entry_slots, layer,
      num_blocks, hot_slots, block_table, bt_stride, page_table, page_cnt,
      seq_lens, m_part, l_part, acc_part, split, pps_min, out, o_stride_t,
      o_stride_h, scale, n_req, n_kv, G, head_dim, page, max_pages, stream,
      nullptr, 0);
}

extern "C" int amass_tier_decode_install(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, void* hot_v, void* hot_k,
    const void* stg_v, const void* stg_k, int64_t svb, int64_t svt,
    int64_t svh, void* pool_v, void* pool_k, int8_t* pool_valid,
    const int32_t* page2slot, const int32_t* vbo, const int32_t* entry_slots,
    int layer, int num_blocks, int hot_slots, const int32_t* block_table,
    int64_t bt_stride, const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, float* m_part, float* l_part, float* acc_part,
    int split, int pps_min, void* out, int64_t o_stride_t, int64_t o_stride_h,
    float scale, int n_req, int n_kv, int G, int head_dim, int page,
    int max_pages, void* stream) {
  return amass::tier_decode_impl(
      q, q_stride_t, q_stride_h, k, k_sb, k_st, k_sh, hot_v, hot_k, stg_v,
      stg_k, svb, svt, svh, pool_v, pool_k, page2slot, vbo, entry_slots, layer,
      num_blocks, hot_slots, block_table, bt_stride, page_table, page_cnt,
      seq_lens, m_part, l_part, acc_part, split, pps_min, out, o_stride_t,
      o_stride_h, scale, n_req, n_kv, G, head_dim, page, max_pages, stream,
      pool_valid, 1);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of amass_sparse_decode.
//
// Some callers cannot allocate device memory at all: a plugin that runs
// inside another runtime's memory pool, a host loop that must not touch the
// CUDA allocator once serving has started, or a binding with no tensor
// library to own buffers.  For them the split-K partials live in one
// file-scope device array, fixed in size, that every GPU loading this
// library keeps until the process exits.  Nothing is allocated or freed.
// ---------------------------------------------------------------------------
namespace amass {
namespace {

constexpr size_t kNoAllocFloats = size_t(4) << 20;   // 16 MiB of fp32 partials
static __device__ __align__(256) float g_decode_scratch[kNoAllocFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array for the current device; resolved once
// per device (the host-side symbol is not a device address).
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return AMASS_ERR_CUDA;
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p)
      return AMASS_ERR_CUDA;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return AMASS_OK;
}

}  // namespace
}  // namespace amass

extern "C" size_t amass_sparse_decode_noalloc_capacity(void) {
  return amass::kNoAllocFloats;
}

extern "C" int amass_sparse_decode_noalloc(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v, int64_t v_sb,
    int64_t v_st, int64_t v_sh, const int32_t* block_table, int64_t bt_stride,
    const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, int split, int pps_min, void* out,
    int64_t o_stride_t, int64_t o_stride_h, float scale, int n_req, int n_kv,
    int G, int head_dim, int page, int max_pages, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || G <= 0 || split < 2 || head_dim <= 0)
    return AMASS_ERR_ARG;
  // partial layout: m (units*split*G), l (same), acc (units*split*G*D)
  const size_t slots = (size_t)n_req * n_kv * split * G;
  const size_t need = slots * (2 + (size_t)head_dim);
  if (need > kNoAllocFloats) return AMASS_ERR_CAPACITY;
  float* base = nullptr;
  const int rc = scratch_for_current_device(&base);
  if (rc) return rc;
  return amass_sparse_decode(q, q_stride_t, q_stride_h, k, k_sb, k_st, k_sh, v,
                             v_sb, v_st, v_sh, block_table, bt_stride,
                             page_table, page_cnt, seq_lens, base,
                             base + slots, base + 2 * slots, split, pps_min,
                             out, o_stride_t, o_stride_h, scale, n_req, n_kv,
                             G, head_dim, page, max_pages, stream);
}
