// Stage A.1: the quad (Gaussian-MGF) page scorer on sm_100a.
//
// Math (reference selection/quad_score.py:55-107), per (request r, kv-head h,
// page p < n_sel_hi, query head g of the GQA group):
//     qmu_g  = mu_code . q_g            q~_{g,k} = V_code[:,k] . q_g
//     S_g    = s*mu_scale*qmu_g + s^2/(2P) * sum_k sig2_k (V_scale_k q~_{g,k})^2
//
// Work decomposition.  A work item is (16-page tile of one request, kv-head).
// The grid is persistent; warp gw owns kv-head gw % n_kv and one contiguous
// range of tiles, so the n_kv heads of a tile -- whose summary rows are
// adjacent in memory -- are read by sibling warps at the same time and share
// DRAM sectors, and a warp's q operand changes only when its range enters a
// new request.  Each warp runs a three-deep register pipeline: block-table
// reads two tiles ahead, the 16-byte summary loads one tile ahead, the
// tensor-core math on the current tile.
//
// Math on the tensor cores: the 1+rank dot products of 16 pages with the G
// query heads are integer MMAs (m16n8k32, s8 x s8 -> s32).  A = the raw int8
// summary codes (an int4 code is used as 16*code, one mask away from its
// packed byte), B = q split exactly into two int8 limbs,
// q ~= s_q * (128*hi + lo) with s_q = max|q_g| / 16256 (a prologue kernel
// writes the limbs once per call into caller scratch).  Products and sums are
// exact integers; the only rounding is the 15-bit limb form of q
// (|dq| <= max|q| / 32512).  Lane (m, c) owns pages m and m+8 and the
// contiguous head_dim slice [c*D/4, (c+1)*D/4); A and B use the same
// d <-> k-slot assignment, so code words feed the MMA without byte shuffles.
//
// With the nrm combine the kernel also max-accumulates the per-head page
// maximum into hmax[r, h, g]; the fold (nrm_combine / select_pages) consumes
// it and resets it to -inf, so the fold is a single pass.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"

namespace amass {
namespace {

constexpr int kQuadWarps = 8;
constexpr int kQuadMaxReq = 4096;

struct QuadArgs {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  const int8_t* mu;
  const __half* mus;
  const int8_t* V;
  const __half* Vs;
  const __half* sig2;
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* nsh;
  float* score;
  float* score_h;
  float* hmax;
  int8_t* q8;        // (n_req, H, 2, D): hi limb then lo limb per head
  float* qs;         // (n_req, H) limb scale
  float scale, coef;
  int n_req, n_kv, G, MP;
  int64_t SHS;       // score_h row stride (elements; >= MP)
  // r8 scorer only
  const int8_t* c;   // (NB, n_kv, page, rc) int8 per-token coordinates
  const __half* cs;  // (NB, n_kv, page) fp16 per-token scale
  const int32_t* sl; // (n_req,) seq_lens
  int page, tokmax;
  // CLSE (quad geometry + per-key coordinates) only
  const __half* resid;  // (NB, n_kv) residual scatter energy, or null
  float* qsq;           // (n_req, H) |q_g|^2 written by the q prologue
  float iso_coef;       // s^2 / (2 P (d - r))
  int ctok;             // coordinate scales per token (1) or per page (0)
  int write_h;          // per-head scores + hmax (nrm) instead of the max
  // derive_page_params folded into the q prologue (null dv_sl: not asked)
  const int32_t* dv_sl;
  const double* dv_budget;
  int32_t* dv_npg;
  int32_t* dv_nsh;
  int32_t* dv_b;
  int dv_win, dv_sink;
};

AMASS_DEV void atomic_max_float(float* addr, float v) {
  if (v >= 0.f)
    atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
  else
    atomicMin(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

AMASS_DEV void mma_s8(int* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- prologue: q -> two exact-range int8 limbs per (request, head) --------
template <int D>
__global__ void __launch_bounds__(256) q_limbs_kernel(QuadArgs a) {
  grid_dep_wait();     // inputs written by the previous kernel
  grid_dep_launch();
  if (a.dv_sl && blockIdx.x == 0) {
    // this step's page parameters for the scorer (the next launch)
    const double bud = a.dv_budget[0];
    for (int i = threadIdx.x; i < a.n_req; i += blockDim.x)
      derive_one(a.dv_sl[i], bud, a.page, a.dv_win, a.dv_sink, a.dv_npg + i,
                 a.dv_nsh + i, a.dv_b + i);
  }
  const int H = a.n_kv * a.G;
  const int idx = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (idx >= a.n_req * H) return;
  const int r = idx / H, h = idx - r * H;
  const __nv_bfloat16* qp = a.q + (int64_t)r * a.q_st + (int64_t)h * a.q_sh;
  constexpr int PER = D / 32;
  float v[PER];
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    v[i] = __bfloat162float(qp[lane * PER + i]);
    mx = fmaxf(mx, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float sq = mx > 0.f ? mx / 16256.f : 1.f;
  const float inv = 1.f / sq;
  int8_t* hi = a.q8 + (int64_t)idx * 2 * D;
  int8_t* lo = hi + D;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int qi = __float2int_rn(v[i] * inv);            // |qi| <= 16256
    const int h8 = (qi >= 0 ? qi + 64 : qi - 63) / 128;   // nearest, |h8|<=127
    hi[lane * PER + i] = (int8_t)h8;
    lo[lane * PER + i] = (int8_t)(qi - 128 * h8);         // |lo| <= 64
  }
  if (lane == 0) a.qs[idx] = sq;
  if (a.qsq) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) ss += v[i] * v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) a.qsq[idx] = ss;
  }
}

// 4 code bytes (d0..d0+3) of byte-column KB from a step's V words, RB bytes/d
template <int RB, int KB>
AMASS_DEV uint32_t gather4(const uint32_t* w) {
  if constexpr (RB == 1) {
    return w[0];
  } else if constexpr (RB == 2) {
    return __byte_perm(w[0], w[1], KB | ((2 + KB) << 4) | ((4 + KB) << 8) |
                                        ((6 + KB) << 12));
  } else {
    constexpr int B0 = KB, B1 = RB + KB, B2 = 2 * RB + KB, B3 = 3 * RB + KB;
    const uint32_t x = __byte_perm(w[B0 / 4], w[B1 / 4], (B0 & 3) | ((4 + (B1 & 3)) << 4));
    const uint32_t y = __byte_perm(w[B2 / 4], w[B3 / 4], (B2 & 3) | ((4 + (B3 & 3)) << 4));
    return __byte_perm(x, y, 0x5410);
  }
}
// column K of 4 consecutive d: int8 codes, or 16 * int4 codes
template <int R, int VB, int K>
AMASS_DEV uint32_t vcol4(const uint32_t* w) {
  if constexpr (VB == 8) {
    return gather4<R, K>(w);
  } else {
    const uint32_t x = gather4<R / 2, K / 2>(w);
    return (K & 1) ? (x & 0xF0F0F0F0u) : ((x << 4) & 0xF0F0F0F0u);
  }
}

template <int R, int VB, int K>
struct VCols {
  // wa/wb: the step's V words for rows a/b (2*RB words: d0..d0+7)
  static AMASS_DEV void run(int (*acc)[2][4], const uint32_t* wa,
                            const uint32_t* wb, const uint32_t* bh,
                            const uint32_t* bl) {
    constexpr int RB = (VB == 8) ? R : R / 2;
    uint32_t a[4];
    a[0] = vcol4<R, VB, K>(wa);
    a[1] = vcol4<R, VB, K>(wb);
    a[2] = vcol4<R, VB, K>(wa + RB);
    a[3] = vcol4<R, VB, K>(wb + RB);
    mma_s8(acc[1 + K][0], a, bh[0], bh[1]);
    mma_s8(acc[1 + K][1], a, bl[0], bl[1]);
    if constexpr (K + 1 < R) VCols<R, VB, K + 1>::run(acc, wa, wb, bh, bl);
  }
};

// Per-lane view of one item: two page rows (m, m+8) of one kv-head.
template <int D, int R, int VB>
struct Item {
  static constexpr int RB = (VB == 8) ? R : R / 2;   // V code bytes per d
  static constexpr int MU_U4 = D / 64;               // mu bytes per lane / 16
  static constexpr int V_BYTES = (D / 4) * RB;       // V bytes per lane
  static constexpr bool V_PRE = V_BYTES <= 64;       // keep V in registers
  static constexpr int V_U4 = V_PRE ? V_BYTES / 16 : 1;
  static constexpr int RW = (R + 1) / 2;             // 32-bit words / row
  int r, h, p0;
  bool va, vb;
  int rowa, rowb;               // block id, then block * n_kv + head
  uint4 mu[2][MU_U4];
  uint4 v[2][V_U4];
  __half2 mus;                  // (row a, row b)
  uint32_t vs[2][RW], s2[2][RW];  // fp16 scales, two per word
  AMASS_DEV float vsf(int half, int k) const {
    const uint32_t w = vs[half][k >> 1];
    return __half2float(__ushort_as_half((uint16_t)((k & 1) ? (w >> 16) : w)));
  }
  AMASS_DEV float s2f(int half, int k) const {
    const uint32_t w = s2[half][k >> 1];
    return __half2float(__ushort_as_half((uint16_t)((k & 1) ? (w >> 16) : w)));
  }
};

// R fp16 values at p into RW words (two per word; R odd only for R == 1)
template <int R>
AMASS_DEV void load_halves(uint32_t* w, const __half* p) {
  if constexpr (R == 1) {
    w[0] = __ldg(reinterpret_cast<const unsigned short*>(p));
  } else {
#pragma unroll
    for (int k = 0; k < R / 2; ++k)
      w[k] = __ldg(reinterpret_cast<const unsigned int*>(p) + k);
  }
}

// index phase: tile -> (request, first page), block-table reads -> rows
template <int D, int R, int VB>
AMASS_DEV void load_idx(Item<D, R, VB>& it, const QuadArgs& a,
                        const int* prefix, const int* nshs, int item,
                        int lane, int* rhint = nullptr) {
  const int t = item / a.n_kv;
  const int h = item - t * a.n_kv;
  int r;
  if (rhint) {                       // tiles ascend: walk forward from hint
    r = *rhint;
    while (prefix[r + 1] <= t) ++r;
    *rhint = r;
  } else {
    int lo = 0, hi = a.n_req - 1;    // request of tile t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
    }
    r = lo;
  }
  const int nsh = nshs[r];
  const int p0 = (t - prefix[r]) * 16;
  const int m = lane >> 2;
  const int pa = p0 + m, pb = pa + 8;
  it.r = r; it.h = h; it.p0 = p0;
  it.va = pa < nsh; it.vb = pb < nsh;
  const int32_t* btr = a.bt + (int64_t)r * a.bt_stride;
  it.rowa = it.va ? __ldg(btr + pa) : 0;    // block ids; scaled in load_data
  it.rowb = it.vb ? __ldg(btr + pb) : 0;
}

// data phase: the 16-byte summary loads of an item whose block ids are known
template <int D, int R, int VB, bool S2 = true>
AMASS_DEV void load_data(Item<D, R, VB>& it, const QuadArgs& a, int lane) {
  using I = Item<D, R, VB>;
  const int c = lane & 3;
  it.rowa = it.rowa * a.n_kv + it.h;
  it.rowb = it.rowb * a.n_kv + it.h;
  const int8_t* mua = a.mu + (int64_t)it.rowa * D + c * (D / 4);
  const int8_t* mub = a.mu + (int64_t)it.rowb * D + c * (D / 4);
#pragma unroll
  for (int i = 0; i < I::MU_U4; ++i) {
    it.mu[0][i] = ldg_nc_v4(mua + 16 * i);
    it.mu[1][i] = ldg_nc_v4(mub + 16 * i);
  }
  if constexpr (I::V_PRE) {
    const int8_t* Va = a.V + (int64_t)it.rowa * (D * I::RB) + c * I::V_BYTES;
    const int8_t* Vb = a.V + (int64_t)it.rowb * (D * I::RB) + c * I::V_BYTES;
#pragma unroll
    for (int i = 0; i < I::V_U4; ++i) {
      it.v[0][i] = ldg_nc_v4(Va + 16 * i);
      it.v[1][i] = ldg_nc_v4(Vb + 16 * i);
    }
  }
  __half2 ms;
  ms.x = a.mus[it.rowa];
  ms.y = a.mus[it.rowb];
  it.mus = ms;
  load_halves<R>(it.vs[0], a.Vs + (int64_t)it.rowa * R);
  load_halves<R>(it.vs[1], a.Vs + (int64_t)it.rowb * R);
  if constexpr (S2) {     // sig2: quad scorer only
    load_halves<R>(it.s2[0], a.sig2 + (int64_t)it.rowa * R);
    load_halves<R>(it.s2[1], a.sig2 + (int64_t)it.rowb * R);
  }
}

// q operand of one (request, kv-head): limbs for B fragments + limb scales
template <int D>
struct QFrag {
  static constexpr int KS = D / 32;
  uint32_t bh[KS][2], bl[KS][2];
  float sq[2];
};

// PK (G <= 4): packed limbs -- B column n < 4 holds the hi limb of query head
// n, column n >= 4 the lo limb of head n - 4, both in bh (bl unused), so one
// m16n8k32 forms both limb sums; lane quads c and c ^ 2 then hold the hi and
// lo sums of the same heads 2(c & 1), 2(c & 1) + 1.
template <int D, bool PK = false>
AMASS_DEV void load_qfrag(QFrag<D>& f, const QuadArgs& a, int r, int h,
                          int lane) {
  constexpr int KS = D / 32;
  const int m = lane >> 2, c = lane & 3;
  const int H = a.n_kv * a.G;
  const int hm = PK ? (m & 3) : m;           // query head of this B column
  const bool gv = hm < a.G;
  const int64_t qrow = (int64_t)r * H + h * a.G + (gv ? hm : 0);
  const int8_t* qh = a.q8 + qrow * 2 * D + c * (D / 4);
  const int8_t* ql = qh + D;
  if (PK && m >= 4) qh = ql;                 // the lo-limb columns
#pragma unroll
  for (int i = 0; i < KS / 2; ++i) {
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(qh) + i);
    f.bh[2 * i][0] = gv ? x.x : 0u; f.bh[2 * i][1] = gv ? x.y : 0u;
    f.bh[2 * i + 1][0] = gv ? x.z : 0u; f.bh[2 * i + 1][1] = gv ? x.w : 0u;
    if constexpr (!PK) {
      const uint4 y = __ldg(reinterpret_cast<const uint4*>(ql) + i);
      f.bl[2 * i][0] = gv ? y.x : 0u; f.bl[2 * i][1] = gv ? y.y : 0u;
      f.bl[2 * i + 1][0] = gv ? y.z : 0u; f.bl[2 * i + 1][1] = gv ? y.w : 0u;
    }
  }
  const int cq = PK ? (c & 1) : c;
  const int g0 = min(2 * cq, a.G - 1), g1 = min(2 * cq + 1, a.G - 1);
  const float* qsr = a.qs + (int64_t)r * H + h * a.G;
  f.sq[0] = __ldg(qsr + g0);
  f.sq[1] = __ldg(qsr + g1);
}

// The q operand straight from the bf16 query (the quad scorer's form: no
// separate limb launch).  Lane (m, c) holds query head m of kv head h (the
// A-fragment row group of this lane) over d in [c*D/4, (c+1)*D/4); the four
// lanes of a quad cover the row, so max|q| is a quad reduction.  Limbs and
// scale are the q-limb prologue's, bit for bit: s = max|q|/16256,
// qi = rn(q/s), hi = nearest(qi/128), lo = qi - 128*hi.
// PK: the packed-limb columns of load_qfrag.
template <int D, bool PK = false>
AMASS_DEV void qfrag_from_q(QFrag<D>& f, const QuadArgs& a, int r, int h,
                            int lane) {
  constexpr int SL = D / 4;                  // d values per lane
  const int m = lane >> 2, c = lane & 3;
  const int hm = PK ? (m & 3) : m;           // query head of this B column
  const bool gv = hm < a.G;
  const __nv_bfloat16* qp = a.q + (int64_t)r * a.q_st +
                            (int64_t)(h * a.G + (gv ? hm : 0)) * a.q_sh + c * SL;
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < SL; i += 8) {
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(qp + i));
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 v = __bfloat1622float2(p2[e]);
      mx = fmaxf(mx, fmaxf(fabsf(v.x), fabsf(v.y)));
    }
  }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float sq = mx > 0.f ? mx / 16256.f : 1.f;
  const float inv = 1.f / sq;
#pragma unroll
  for (int i = 0; i < SL; i += 8) {
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(qp + i));
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&x);
    uint32_t wh[2] = {0u, 0u}, wl[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float2 v2 = __bfloat1622float2(p2[e >> 1]);
      const float v = (e & 1) ? v2.y : v2.x;
      const int qi = __float2int_rn(v * inv);               // |qi| <= 16256
      const int h8 = (qi >= 0 ? qi + 64 : qi - 63) / 128;   // |h8| <= 127
      const int l8 = qi - 128 * h8;                         // |l8| <= 64
      wh[e >> 2] |= (uint32_t)(h8 & 0xff) << (8 * (e & 3));
      wl[e >> 2] |= (uint32_t)(l8 & 0xff) << (8 * (e & 3));
    }
    const int s = i / 8;                      // words 2s, 2s + 1 of the slice
    if constexpr (PK) {
      const bool lo_col = m >= 4;
      f.bh[s][0] = gv ? (lo_col ? wl[0] : wh[0]) : 0u;
      f.bh[s][1] = gv ? (lo_col ? wl[1] : wh[1]) : 0u;
    } else {
      f.bh[s][0] = gv ? wh[0] : 0u; f.bh[s][1] = gv ? wh[1] : 0u;
      f.bl[s][0] = gv ? wl[0] : 0u; f.bl[s][1] = gv ? wl[1] : 0u;
    }
  }
  // column scales: query heads 2c, 2c + 1 (the rows of lane quads 2c, 2c + 1;
  // PK: 2(c & 1), 2(c & 1) + 1)
  const int cq = PK ? (c & 1) : c;
  const int g0 = min(2 * cq, a.G - 1), g1 = min(2 * cq + 1, a.G - 1);
  f.sq[0] = __shfl_sync(0xffffffffu, sq, 4 * g0);
  f.sq[1] = __shfl_sync(0xffffffffu, sq, 4 * g1);
}

// The (1+R) x 2-limb integer dot products of one item: acc[comp][limb][4]
// (comp 0 = mu, 1+k = V column k), C-fragment layout (rows pages m, m+8;
// cols query heads 2c, 2c+1).
// Shared-memory image of one tile's V rows for items whose V slice does not
// fit the register pipeline (rank 8): row = 4 lane slices of V_BYTES + 16 B,
// so the 8 lanes of a 16-byte load phase hit 8 different bank quads.
template <int D, int R, int VB>
struct VStage {
  static constexpr int RB = (VB == 8) ? R : R / 2;
  static constexpr int V_BYTES = (D / 4) * RB;
  static constexpr int SLICE = V_BYTES + 16;
  static constexpr int ROW = 4 * SLICE;
  static constexpr int BYTES = 16 * ROW;
};

template <int D, int R, int VB>
AMASS_DEV void item_dots(const Item<D, R, VB>& it, const QFrag<D>& qf,
                         const QuadArgs& a, int lane, int (*acc)[2][4],
                         const uint8_t* vsm = nullptr) {
  using I = Item<D, R, VB>;
  constexpr int KS = D / 32;                 // m16n8k32 steps
  constexpr int RB = I::RB;
  const int c = lane & 3;
  const uint32_t (*bh)[2] = qf.bh;
  const uint32_t (*bl)[2] = qf.bl;
#pragma unroll
  for (int i = 0; i <= R; ++i)
#pragma unroll
    for (int l = 0; l < 2; ++l)
      acc[i][l][0] = acc[i][l][1] = acc[i][l][2] = acc[i][l][3] = 0;
  const uint32_t* mwa = reinterpret_cast<const uint32_t*>(it.mu[0]);
  const uint32_t* mwb = reinterpret_cast<const uint32_t*>(it.mu[1]);
#pragma unroll
  for (int s = 0; s < KS; ++s) {
    const uint32_t am[4] = {mwa[2 * s], mwb[2 * s], mwa[2 * s + 1], mwb[2 * s + 1]};
    mma_s8(acc[0][0], am, bh[s][0], bh[s][1]);
    mma_s8(acc[0][1], am, bl[s][0], bl[s][1]);
    uint32_t wva[2 * RB], wvb[2 * RB];
    if constexpr (I::V_PRE) {
      const uint32_t* va = reinterpret_cast<const uint32_t*>(it.v[0]);
      const uint32_t* vb = reinterpret_cast<const uint32_t*>(it.v[1]);
#pragma unroll
      for (int j = 0; j < 2 * RB; ++j) {
        wva[j] = va[s * 2 * RB + j];
        wvb[j] = vb[s * 2 * RB + j];
      }
    } else if (vsm) {
      using VSt = VStage<D, R, VB>;
      const int m = lane >> 2;
      const uint8_t* Va = vsm + m * VSt::ROW + c * VSt::SLICE + s * 8 * RB;
      const uint8_t* Vb = Va + 8 * VSt::ROW;
#pragma unroll
      for (int j = 0; j < 2 * RB; j += 4) {
        const uint4 x = *reinterpret_cast<const uint4*>(Va + 4 * j);
        const uint4 y = *reinterpret_cast<const uint4*>(Vb + 4 * j);
        wva[j] = x.x; wva[j + 1] = x.y; wva[j + 2] = x.z; wva[j + 3] = x.w;
        wvb[j] = y.x; wvb[j + 1] = y.y; wvb[j + 2] = y.z; wvb[j + 3] = y.w;
      }
    } else {
      const int8_t* Va = a.V + (int64_t)it.rowa * (D * RB) + c * I::V_BYTES + s * 8 * RB;
      const int8_t* Vb = a.V + (int64_t)it.rowb * (D * RB) + c * I::V_BYTES + s * 8 * RB;
#pragma unroll
      for (int j = 0; j < 2 * RB; j += 4) {
        const uint4 x = __ldg(reinterpret_cast<const uint4*>(Va) + j / 4);
        const uint4 y = __ldg(reinterpret_cast<const uint4*>(Vb) + j / 4);
        wva[j] = x.x; wva[j + 1] = x.y; wva[j + 2] = x.z; wva[j + 3] = x.w;
        wvb[j] = y.x; wvb[j + 1] = y.y; wvb[j + 2] = y.z; wvb[j + 3] = y.w;
      }
    }
    VCols<R, VB, 0>::run(acc, wva, wvb, bh[s], bl[s]);
  }

}

template <int D, int R, int VB, bool WRITE_H>
AMASS_DEV void score_item(const Item<D, R, VB>& it, const QFrag<D>& qf,
                          const QuadArgs& a, int lane) {
  const int m = lane >> 2, c = lane & 3;
  int acc[1 + R][2][4];
  item_dots(it, qf, a, lane, acc);
  // epilogue: rows pa (idx 0,1) and pb (idx 2,3); cols g = 2c, 2c+1
  const float* sq = qf.sq;
  constexpr float vdiv = (VB == 8) ? 1.f : 1.f / 16.f;
  float S[2][2];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const float mus = half ? __high2float(it.mus) : __low2float(it.mus);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int idx = 2 * half + j;
      float quad = 0.f;
#pragma unroll
      for (int k = 0; k < R; ++k) {
        const float vs = it.vsf(half, k);
        const float s2 = it.s2f(half, k);
        const float qt = (float)(128 * acc[1 + k][0][idx] + acc[1 + k][1][idx]) *
                         (sq[j] * vdiv) * vs;
        quad += s2 * qt * qt;
      }
      const float qmu = (float)(128 * acc[0][0][idx] + acc[0][1][idx]) * sq[j];
      S[half][j] = qmu * mus * a.scale + quad * a.coef;
    }
  }
  const int pa = it.p0 + m, pb = pa + 8;
  if constexpr (WRITE_H) {
    float* base = a.score_h + ((int64_t)it.r * a.n_kv + it.h) * a.G * a.SHS;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int g = 2 * c + j;
      float mx = -INFINITY;
      if (g < a.G) {
        if (it.va) { base[(int64_t)g * a.SHS + pa] = S[0][j]; mx = S[0][j]; }
        if (it.vb) { base[(int64_t)g * a.SHS + pb] = S[1][j]; mx = fmaxf(mx, S[1][j]); }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      if (m == 0 && g < a.G && mx > -INFINITY)
        atomic_max_float(a.hmax + ((int64_t)it.r * a.n_kv + it.h) * a.G + g, mx);
    }
  } else {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float mx = (2 * c < a.G) ? S[half][0] : -INFINITY;
      if (2 * c + 1 < a.G) mx = fmaxf(mx, S[half][1]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const bool pv = half ? it.vb : it.va;
      if (pv && c == 0)
        a.score[((int64_t)it.r * a.n_kv + it.h) * a.MP + (half ? pb : pa)] = mx;
    }
  }
}

// Packed-limb form of item_dots + score_item (G <= 4, qf from the PK loads):
// one m16n8k32 per (component, k-step) gives the hi-limb sums in columns 0-3
// and the lo-limb sums in columns 4-7.  Lane quads c and c ^ 2 swap half their
// sums so each lane holds both limbs of one page row (c < 2: row m, c >= 2:
// row m + 8) for heads 2(c & 1), 2(c & 1) + 1, and evaluates the same
// expressions as score_item on them: the scores are bit-identical.
template <int R, int VB, int K>
struct VColsPK {
  static AMASS_DEV void run(int (*acc)[4], const uint32_t* wa,
                            const uint32_t* wb, const uint32_t* b) {
    constexpr int RB = (VB == 8) ? R : R / 2;
    uint32_t x[4];
    x[0] = vcol4<R, VB, K>(wa);
    x[1] = vcol4<R, VB, K>(wb);
    x[2] = vcol4<R, VB, K>(wa + RB);
    x[3] = vcol4<R, VB, K>(wb + RB);
    mma_s8(acc[1 + K], x, b[0], b[1]);
    if constexpr (K + 1 < R) VColsPK<R, VB, K + 1>::run(acc, wa, wb, b);
  }
};

// WRITE_H: the per-head page maxima are kept per lane in rmx[2] (heads
// 2(c & 1), 2(c & 1) + 1) across the tiles of one request and folded into
// hmax by flush_hmax when the warp moves to another request or finishes --
// one warp reduction and one atomic per (request, head) run instead of per
// tile.  max is exact, so hmax is the same.
template <int D, int R, int VB, bool WRITE_H>
AMASS_DEV void score_item_pk(const Item<D, R, VB>& it, const QFrag<D>& qf,
                             const QuadArgs& a, int lane, float* rmx) {
  using I = Item<D, R, VB>;
  static_assert(I::V_PRE, "packed limbs: V slice in registers");
  constexpr int KS = D / 32;
  constexpr int RB = I::RB;
  const int m = lane >> 2, c = lane & 3;
  const int half = c >> 1;                   // 0: row m, 1: row m + 8
  int acc[1 + R][4];
#pragma unroll
  for (int i = 0; i <= R; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0;
  const uint32_t* mwa = reinterpret_cast<const uint32_t*>(it.mu[0]);
  const uint32_t* mwb = reinterpret_cast<const uint32_t*>(it.mu[1]);
  const uint32_t* va = reinterpret_cast<const uint32_t*>(it.v[0]);
  const uint32_t* vb = reinterpret_cast<const uint32_t*>(it.v[1]);
#pragma unroll
  for (int s = 0; s < KS; ++s) {
    const uint32_t am[4] = {mwa[2 * s], mwb[2 * s], mwa[2 * s + 1], mwb[2 * s + 1]};
    mma_s8(acc[0], am, qf.bh[s][0], qf.bh[s][1]);
    uint32_t wva[2 * RB], wvb[2 * RB];
#pragma unroll
    for (int j = 0; j < 2 * RB; ++j) {
      wva[j] = va[s * 2 * RB + j];
      wvb[j] = vb[s * 2 * RB + j];
    }
    VColsPK<R, VB, 0>::run(acc, wva, wvb, qf.bh[s]);
  }
  // hi sums of row m + 8 go to the lo lanes, lo sums of row m to the hi lanes
  int hi[1 + R][2], lo[1 + R][2];
#pragma unroll
  for (int i = 0; i <= R; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int got = __shfl_xor_sync(0xffffffffu, half ? acc[i][j] : acc[i][2 + j], 2);
      hi[i][j] = half ? got : acc[i][j];
      lo[i][j] = half ? acc[i][2 + j] : got;
    }
  const float* sq = qf.sq;
  constexpr float vdiv = (VB == 8) ? 1.f : 1.f / 16.f;
  const float mus = half ? __high2float(it.mus) : __low2float(it.mus);
  // this lane's row of scale words (selects: a runtime row index into the
  // item's arrays would put them in local memory)
  uint32_t vsw[I::RW], s2w[I::RW];
#pragma unroll
  for (int w = 0; w < I::RW; ++w) {
    vsw[w] = half ? it.vs[1][w] : it.vs[0][w];
    s2w[w] = half ? it.s2[1][w] : it.s2[0][w];
  }
  auto h16 = [](uint32_t w, int k) {
    return __half2float(__ushort_as_half((uint16_t)((k & 1) ? (w >> 16) : w)));
  };
  float S[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float quad = 0.f;
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const float vs = h16(vsw[k >> 1], k);
      const float s2 = h16(s2w[k >> 1], k);
      const float qt = (float)(128 * hi[1 + k][j] + lo[1 + k][j]) *
                       (sq[j] * vdiv) * vs;
      quad += s2 * qt * qt;
    }
    const float qmu = (float)(128 * hi[0][j] + lo[0][j]) * sq[j];
    S[j] = qmu * mus * a.scale + quad * a.coef;
  }
  const int p = it.p0 + m + 8 * half;
  const bool pv = half ? it.vb : it.va;
  const int cq = c & 1;
  if constexpr (WRITE_H) {
    float* base = a.score_h + ((int64_t)it.r * a.n_kv + it.h) * a.G * a.SHS;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int g = 2 * cq + j;
      if (g < a.G && pv) {
        base[(int64_t)g * a.SHS + p] = S[j];
        rmx[j] = fmaxf(rmx[j], S[j]);
      }
    }
  } else {
    float mx = (2 * cq < a.G) ? S[0] : -INFINITY;
    if (2 * cq + 1 < a.G) mx = fmaxf(mx, S[1]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    if (pv && cq == 0)
      a.score[((int64_t)it.r * a.n_kv + it.h) * a.MP + p] = mx;
  }
}

// Folds the lanes' running maxima of score_item_pk into hmax of (r, h) and
// resets them (whole warp).
AMASS_DEV void flush_hmax(const QuadArgs& a, int r, int h, int lane,
                          float* rmx) {
  const int cq = lane & 1;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float mx = rmx[j];
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const int g = 2 * cq + j;
    if (lane == cq && g < a.G && mx > -INFINITY)
      atomic_max_float(a.hmax + ((int64_t)r * a.n_kv + h) * a.G + g, mx);
    rmx[j] = -INFINITY;
  }
}

// Warp 0's prologue of the quad scorers: this step's page parameters
// (derived here from seq_lens, CTA 0 writing them for the select and decode
// launches, or read) and the per-request tile offsets prefix[0..n_req].
AMASS_DEV void quad_prologue(const QuadArgs& a, int* prefix, int* nshs,
                             int lane) {
  // this step's page parameters: derived here from seq_lens (CTA 0 writes
  // them for the select and decode launches), or read
  const double bud = a.dv_sl ? a.dv_budget[0] : 0.0;
  int run = 0;
  for (int base = 0; base < a.n_req; base += 32) {
    const int r = base + lane;
    int nsh = 0;
    if (r < a.n_req) {
      if (a.dv_sl) {
        int32_t npg_r, nsh_r, b_r;
        derive_one(a.dv_sl[r], bud, a.page, a.dv_win, a.dv_sink, &npg_r,
                   &nsh_r, &b_r);
        if (blockIdx.x == 0) {
          a.dv_npg[r] = npg_r;
          a.dv_nsh[r] = nsh_r;
          a.dv_b[r] = b_r;
        }
        nsh = max(nsh_r, 0);
      } else {
        nsh = max(a.nsh[r], 0);
      }
    }
    const int t = (nsh + 15) / 16;
    int incl = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    if (r < a.n_req) { prefix[r] = run + incl - t; nshs[r] = nsh; }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) prefix[a.n_req] = run;
}

// two CTAs per SM (<= 128 registers) when a lane's V slice is <= 32 bytes
template <int D, int R, int VB>
constexpr int quad_min_blocks() {
  return (D / 4) * ((VB == 8) ? R : R / 2) <= 32 ? 2 : 1;
}

// QIN: the q limbs are split from the bf16 query by each warp (and the page
// parameters derived in the prologue when asked) -- no limb launch; else
// they come from q_limbs_kernel.
// PK: packed limbs (score_item_pk; G <= 4, V slice in registers)
template <int D, int R, int VB, bool WRITE_H, bool QIN, bool PK = false>
__global__ void __launch_bounds__(kQuadWarps * 32, (quad_min_blocks<D, R, VB>()))
quad_score_kernel(QuadArgs a) {
  grid_dep_wait();     // inputs written by the previous kernel
  grid_dep_launch();
  __shared__ int prefix[kQuadMaxReq + 1];   // per-request tile offsets
  __shared__ int nshs[kQuadMaxReq];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) quad_prologue(a, prefix, nshs, lane);
  __syncthreads();
  // warp gw owns head gw % n_kv and a contiguous range of tiles, so its q
  // operand changes only when the range crosses into the next request; the
  // n_kv heads of a tile run on sibling warps at the same time
  const int T = prefix[a.n_req];
  const int gw = blockIdx.x * kQuadWarps + warp;
  const int NJ = gridDim.x * kQuadWarps / a.n_kv;
  const int j = gw / a.n_kv;
  if (j >= NJ) return;
  const int h = gw - j * a.n_kv;
  const int t_lo = (int)((int64_t)T * j / NJ);
  const int t_hi = (int)((int64_t)T * (j + 1) / NJ);
  if (t_lo >= t_hi) return;
  // three-deep pipeline per warp: block ids two tiles ahead, summary data
  // one tile ahead, compute on the current one
  int rh = 0;
  {
    int lo = 0, hi = a.n_req - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= t_lo) lo = mid; else hi = mid - 1;
    }
    rh = lo;
  }
  Item<D, R, VB> cur, nxt, nn;
  QFrag<D> qf;
  int qr = -1;
  float rmx[2] = {-INFINITY, -INFINITY};   // PK: running per-head maxima
  int t = t_lo;
  load_idx(cur, a, prefix, nshs, t * a.n_kv + h, lane, &rh);
  load_data(cur, a, lane);
  if (t + 1 < t_hi) load_idx(nxt, a, prefix, nshs, (t + 1) * a.n_kv + h, lane, &rh);
  while (true) {
    const bool more = t + 1 < t_hi;
    if (t + 2 < t_hi) load_idx(nn, a, prefix, nshs, (t + 2) * a.n_kv + h, lane, &rh);
    if (more) load_data(nxt, a, lane);
    if (cur.r != qr) {
      if constexpr (PK && WRITE_H)
        if (qr >= 0) flush_hmax(a, qr, h, lane, rmx);
      if constexpr (QIN) qfrag_from_q<D, PK>(qf, a, cur.r, h, lane);
      else load_qfrag<D, PK>(qf, a, cur.r, h, lane);
      qr = cur.r;
    }
    if constexpr (PK) score_item_pk<D, R, VB, WRITE_H>(cur, qf, a, lane, rmx);
    else score_item<D, R, VB, WRITE_H>(cur, qf, a, lane);
    if (!more) break;
    cur = nxt;
    nxt = nn;
    ++t;
  }
  if constexpr (PK && WRITE_H) flush_hmax(a, qr, h, lane, rmx);
}

// ---------------------------------------------------------------------------
// Pipelined quad scorer (8 kv heads, a lane's V slice in registers).
//
// A CTA owns one contiguous range of 16-page tiles and scores all 8 heads of
// each: warp h < 8 is the consumer for kv head h, warp 8 the producer.  The
// producer streams each tile's summaries into a ring of S shared-memory
// stages: per page, the block's mu row and V-code row (all heads, 1 KB each
// at C3 geometry -- contiguous in the reference's (L, NB, n_kv, ...) slabs)
// as two bulk copies (cp.async.bulk, complete_tx on the stage's full
// barrier), and its three scale rows (16 + 32 + 32 B) as 16-byte cp.async
// pieces that arrive on the same barrier.  Block-table entries are read one
// tile ahead.  Consumers wait on the full barrier, move their head's slice
// into registers (rows padded by 16 B, so the 8 lanes of a 16-byte shared
// load phase hit distinct banks), release the stage (empty barrier, one
// arrival per warp) and run the same integer-MMA math and epilogue as
// quad_score_kernel, so the two kernels' scores are bit-identical.  Up to S
// tiles (S x 34.5 KB per CTA, two CTAs per SM) are in flight without holding
// registers, where the register pipeline holds one tile per warp.
//
// Every mbarrier wait is bounded (about a second of %globaltimer): on expiry
// the warp records the fault in g_quad_pipe_fault (1 = consumer, 2 =
// producer) and unwinds; the producer waits (bounded) for its last copies to
// land before it returns.
// ---------------------------------------------------------------------------
constexpr int kPipeHeads = 8;
constexpr int kPipeThreads = (kPipeHeads + 1) * 32;
// two stages per CTA: three measured slower in the step (64 requests 115.1
// vs 114.3 us) -- the larger ring keeps the select's CTAs off the SMs longer
constexpr int kPipeStages = 2;
__device__ int g_quad_pipe_fault;

template <int D, int R, int VB>
struct PipeLayout {
  static constexpr int RB = (VB == 8) ? R : R / 2;
  static constexpr int MU_ROW = kPipeHeads * D;        // bytes per block
  static constexpr int V_ROW = kPipeHeads * D * RB;
  static constexpr int MS_ROW = kPipeHeads * 2;
  static constexpr int VS_ROW = kPipeHeads * R * 2;
  static constexpr int MU_P = MU_ROW + 16;             // padded smem rows
  static constexpr int V_P = V_ROW + 16;
  static constexpr int OFF_V = 16 * MU_P;
  static constexpr int OFF_MS = OFF_V + 16 * V_P;
  static constexpr int OFF_VS = OFF_MS + 16 * MS_ROW;
  static constexpr int OFF_S2 = OFF_VS + 16 * VS_ROW;
  static constexpr int STAGE = OFF_S2 + 16 * VS_ROW;
  static constexpr uint32_t TX = MU_ROW + V_ROW;       // bulk bytes per page
  static_assert(MS_ROW % 16 == 0 && VS_ROW % 16 == 0 && STAGE % 16 == 0,
                "16-byte copy pieces");
};

template <int D, int R, int VB, int S>
constexpr size_t pipe_smem_bytes(int n_req) {
  return (size_t)S * PipeLayout<D, R, VB>::STAGE + 16 * S +
         4 * (2 * (size_t)n_req + 1);
}

// R fp16 values at shared address p into RW words (as load_halves)
template <int R>
AMASS_DEV void lds_halves(uint32_t* w, uint32_t p) {
  if constexpr (R == 1) {
    w[0] = lds16(p);
  } else {
#pragma unroll
    for (int k = 0; k < R / 2; ++k) w[k] = lds32(p + 4 * k);
  }
}

// PK: packed limbs (score_item_pk), else the two-limb form
template <int D, int R, int VB, bool WRITE_H, bool QIN, int S, bool PK>
__global__ void __launch_bounds__(kPipeThreads, 2)
quad_score_pipe_kernel(QuadArgs a) {
  using PL = PipeLayout<D, R, VB>;
  using I = Item<D, R, VB>;
  static_assert(I::V_PRE, "the pipelined scorer keeps the V slice in registers");
  extern __shared__ __align__(128) uint8_t pipe_smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(pipe_smem + S * PL::STAGE);
  int* prefix = reinterpret_cast<int*>(bars + 2 * S);
  int* nshs = prefix + a.n_req + 1;
  grid_dep_wait();     // inputs written by the previous kernel
  grid_dep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ring = smem_u32(pipe_smem);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * S;
  if (warp == 0) quad_prologue(a, prefix, nshs, lane);
  if (threadIdx.x == 32) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1 + 32);     // expect_tx arrive + 32 lanes
      mbar_init(empty0 + 8 * s, kPipeHeads);
    }
    mbar_init_fence();
  }
  __syncthreads();
  const int T = prefix[a.n_req];
  const int t_lo = (int)((int64_t)T * blockIdx.x / gridDim.x);
  const int t_hi = (int)((int64_t)T * (blockIdx.x + 1) / gridDim.x);
  if (t_lo >= t_hi) return;
  int rq;
  {
    int lo = 0, hi = a.n_req - 1;     // request of tile t_lo
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= t_lo) lo = mid; else hi = mid - 1;
    }
    rq = lo;
  }

  if (warp == kPipeHeads) {
    // ---- producer ----
    // block ids of the next kIdsAhead tiles stay in flight (slot j = tile
    // t + j), so a tile's copies never wait on its block-table read
    constexpr int kIdsAhead = 4;
    int pr = rq;
    int blk_q[kIdsAhead];
    bool ok_q[kIdsAhead];
    auto fetch = [&](int t, int& blk, bool& ok) {
      ok = false;
      blk = 0;
      if (t >= t_hi) return;
      while (prefix[pr + 1] <= t) ++pr;
      const int p = (t - prefix[pr]) * 16 + (lane & 15);
      ok = lane < 16 && p < nshs[pr];
      if (ok) blk = __ldg(a.bt + (int64_t)pr * a.bt_stride + p);
    };
#pragma unroll
    for (int j = 0; j < kIdsAhead; ++j) fetch(t_lo + j, blk_q[j], ok_q[j]);
    int issued = 0;
    for (int t = t_lo; t < t_hi; ++t) {
      const int i = t - t_lo, s = i % S;
      const int blk = blk_q[0];
      const bool ok = ok_q[0];
#pragma unroll
      for (int j = 0; j + 1 < kIdsAhead; ++j) {
        blk_q[j] = blk_q[j + 1];
        ok_q[j] = ok_q[j + 1];
      }
      fetch(t + kIdsAhead, blk_q[kIdsAhead - 1], ok_q[kIdsAhead - 1]);
      if (i >= S && !mbar_wait(empty0 + 8 * s, ((i / S) - 1) & 1)) {
        atomicCAS(&g_quad_pipe_fault, 0, 2);
        break;
      }
      const uint32_t full = full0 + 8 * s;
      const int nv = __popc(__ballot_sync(0xffffffffu, ok));
      if (lane == 0) mbar_arrive_expect_tx(full, (uint32_t)nv * PL::TX);
      __syncwarp();
      if (ok) {
        const uint32_t st = ring + s * PL::STAGE;
        const int64_t b = blk;
        bulk_g2s(st + lane * PL::MU_P, a.mu + b * PL::MU_ROW, PL::MU_ROW, full);
        bulk_g2s(st + PL::OFF_V + lane * PL::V_P, a.V + b * PL::V_ROW,
                 PL::V_ROW, full);
        const uint8_t* ms = reinterpret_cast<const uint8_t*>(a.mus) + b * PL::MS_ROW;
        const uint8_t* vs = reinterpret_cast<const uint8_t*>(a.Vs) + b * PL::VS_ROW;
        const uint8_t* s2 = reinterpret_cast<const uint8_t*>(a.sig2) + b * PL::VS_ROW;
#pragma unroll
        for (int k = 0; k < PL::MS_ROW; k += 16)
          cp_async16(st + PL::OFF_MS + lane * PL::MS_ROW + k, ms + k, true);
#pragma unroll
        for (int k = 0; k < PL::VS_ROW; k += 16) {
          cp_async16(st + PL::OFF_VS + lane * PL::VS_ROW + k, vs + k, true);
          cp_async16(st + PL::OFF_S2 + lane * PL::VS_ROW + k, s2 + k, true);
        }
      }
      cp_async_mbar_arrive(full);
      issued = i + 1;
    }
    // the last fills (at most S) land before this warp leaves
    for (int j = issued > S ? issued - S : 0; j < issued; ++j)
      if (!mbar_wait(full0 + 8 * (j % S), (j / S) & 1)) {
        atomicCAS(&g_quad_pipe_fault, 0, 2);
        break;
      }
    return;
  }

  // ---- consumers: warp h scores kv head h of every tile ----
  const int h = warp;
  const int m = lane >> 2, c = lane & 3;
  int cr = rq, qr = -1;
  QFrag<D> qf;
  float rmx[2] = {-INFINITY, -INFINITY};   // PK: running per-head maxima
  bool done = true;
  for (int t = t_lo; t < t_hi; ++t) {
    const int i = t - t_lo, s = i % S;
    while (prefix[cr + 1] <= t) ++cr;
    Item<D, R, VB> it;
    it.r = cr;
    it.h = h;
    it.p0 = (t - prefix[cr]) * 16;
    const int nsh = nshs[cr];
    it.va = it.p0 + m < nsh;
    it.vb = it.p0 + m + 8 < nsh;
    it.rowa = it.rowb = 0;
    // warp-uniform verdict: the score epilogue shuffles over all 32 lanes
    if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8 * s, (i / S) & 1))) {
      if (lane == 0) atomicCAS(&g_quad_pipe_fault, 0, 1);
      done = false;
      break;
    }
    const uint32_t st = ring + s * PL::STAGE;
    const uint32_t ma = st + m * PL::MU_P + h * D + c * (D / 4);
    const uint32_t va = st + PL::OFF_V + m * PL::V_P + h * D * PL::RB +
                        c * I::V_BYTES;
#pragma unroll
    for (int k = 0; k < I::MU_U4; ++k) {
      it.mu[0][k] = lds128(ma + 16 * k);
      it.mu[1][k] = lds128(ma + 8 * PL::MU_P + 16 * k);
    }
#pragma unroll
    for (int k = 0; k < I::V_U4; ++k) {
      it.v[0][k] = lds128(va + 16 * k);
      it.v[1][k] = lds128(va + 8 * PL::V_P + 16 * k);
    }
    const uint32_t msa = st + PL::OFF_MS + m * PL::MS_ROW + 2 * h;
    it.mus = __halves2half2(__ushort_as_half(lds16(msa)),
                            __ushort_as_half(lds16(msa + 8 * PL::MS_ROW)));
    const uint32_t vsa = st + PL::OFF_VS + m * PL::VS_ROW + h * R * 2;
    const uint32_t s2a = st + PL::OFF_S2 + m * PL::VS_ROW + h * R * 2;
    lds_halves<R>(it.vs[0], vsa);
    lds_halves<R>(it.vs[1], vsa + 8 * PL::VS_ROW);
    lds_halves<R>(it.s2[0], s2a);
    lds_halves<R>(it.s2[1], s2a + 8 * PL::VS_ROW);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
    if (cr != qr) {
      if constexpr (PK && WRITE_H)
        if (qr >= 0) flush_hmax(a, qr, h, lane, rmx);
      if constexpr (QIN) qfrag_from_q<D, PK>(qf, a, cr, h, lane);
      else load_qfrag<D, PK>(qf, a, cr, h, lane);
      qr = cr;
    }
    if constexpr (PK) score_item_pk<D, R, VB, WRITE_H>(it, qf, a, lane, rmx);
    else score_item<D, R, VB, WRITE_H>(it, qf, a, lane);
  }
  if constexpr (PK && WRITE_H)
    if (done && qr >= 0) flush_hmax(a, qr, h, lane, rmx);
}

// ---------------------------------------------------------------------------
// r8 low-rank scorer (reference selection/score.py:30-120):
//   q~_g   = Vk^T q_g                       (rank R columns, integer MMA as above)
//   tok_gt = s * c_scale_t * (c_code_t . (Vk_scale * q~_g))   t < page, tok < seq_len
//   S_g    = s * mu_scale * (mu_code . q_g) + logsumexp_t tok_gt   (or max_t)
//   score  = max_g S_g
// The item's per-token coordinate codes (16 pages x page x rank) and scales
// are staged in a warp-private shared buffer; lane (m, c) evaluates the page
// tokens of pages m, m+8 for query heads 2c, 2c+1 on the FP32 pipe.
// ---------------------------------------------------------------------------
constexpr int kR8MaxReq = 2048;

template <int R, int CB>
struct R8Tok {
  static constexpr int RC = (CB == 8) ? R : R / 2;   // code bytes per token
};

// Coordinate staging of one tile: 16-byte cp.async pieces into the warp's
// buffer, page-major codes then (token grain) the per-token scales.  Lane
// (m, c) stages the pieces of its own pages m and m+8 (their rows are known
// to it), lanes c = 0..3 interleaved; pages past n_sel_hi are zero-filled.
template <int D, int R, int VB, int CB>
AMASS_DEV void stage_coords(const Item<D, R, VB>& it, const QuadArgs& a,
                            int lane, uint32_t cbase) {
  constexpr int RC = R8Tok<R, CB>::RC;
  constexpr int PG = 16;
  constexpr int kCBytes = 16 * PG * RC;
  constexpr int NPC = PG * RC / 16;                 // code pieces per page
  const int NP = NPC + (a.ctok ? 2 : 0);            // pieces per page
  const int m = lane >> 2, c = lane & 3;
  for (int i = c; i < 2 * NP; i += 4) {
    const int half = i >= NP;
    const int k = i - half * NP;
    const int pl = m + 8 * half;
    const int row = half ? it.rowb : it.rowa;
    const bool ok = half ? it.vb : it.va;
    if (k < NPC) {
      cp_async16(cbase + pl * PG * RC + k * 16,
                 a.c + (int64_t)row * PG * RC + k * 16, ok);
    } else {
      const int k2 = k - NPC;
      cp_async16(cbase + kCBytes + pl * PG * 2 + k2 * 16,
                 reinterpret_cast<const uint8_t*>(a.cs) + (int64_t)row * PG * 2 + k2 * 16,
                 ok);
    }
  }
}

// V-row staging of one tile (rank-8 items): lane (m, c) copies the lane
// slices of its own pages m and m+8, 16-byte cp.async pieces; pages past
// n_sel_hi are zero-filled.
template <int D, int R, int VB>
AMASS_DEV void stage_v(const Item<D, R, VB>& it, const QuadArgs& a, int lane,
                       uint32_t vbase) {
  using VSt = VStage<D, R, VB>;
  const int m = lane >> 2;
  constexpr int NPC = VSt::V_BYTES / 16;            // pieces per lane slice
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = half ? it.rowb : it.rowa;
    const bool ok = half ? it.vb : it.va;
    const int8_t* src = a.V + (int64_t)row * (D * VSt::RB);
    const uint32_t dst = vbase + (m + 8 * half) * VSt::ROW;
    for (int k = lane & 3; k < 4 * NPC; k += 4) {
      const int sl = k / NPC, pc = k - sl * NPC;
      cp_async16(dst + sl * VSt::SLICE + pc * 16,
                 src + sl * VSt::V_BYTES + pc * 16, ok);
    }
  }
}

// byte kk of four words, as one A-fragment word
template <int KK>
AMASS_DEV uint32_t byte_col4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
  const uint32_t x = __byte_perm(w0, w1, KK | ((4 + KK) << 4));
  const uint32_t y = __byte_perm(w2, w3, KK | ((4 + KK) << 4));
  return __byte_perm(x, y, 0x5410);
}

// The r8 scorer's integer dots of one tile: accmu = the two-limb mu dots,
// qtl[half][jj][k] = q~ of rank column k for page (m + 8 * half) and query
// head 2c + jj, in float.  V comes from the warp's shared stage (vsm) or,
// when it fits, from the item's registers.  Int8 rank-8 V runs as two passes
// of four columns: column k reads bytes k % 4 of the odd or even words of a
// d-row, so a pass loads only its 8 words per page and step and holds only
// its four columns' accumulators (the one-pass form needs 255 registers).
template <int D, int R, int VB>
AMASS_DEV void r8_dots(const Item<D, R, VB>& it, const QFrag<D>& qf,
                       const QuadArgs& a, int lane, const uint8_t* vsm,
                       int (*accmu)[4], float (*qtl)[2][R]) {
  using I = Item<D, R, VB>;
  constexpr float vdiv = (VB == 8) ? 1.f : 1.f / 16.f;
  if constexpr (!(VB == 8 && R == 8 && !I::V_PRE)) {
    int acc[1 + R][2][4];
    item_dots(it, qf, a, lane, acc, vsm);
#pragma unroll
    for (int l = 0; l < 2; ++l)
#pragma unroll
      for (int i = 0; i < 4; ++i) accmu[l][i] = acc[0][l][i];
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj)
#pragma unroll
        for (int k = 0; k < R; ++k)
          qtl[half][jj][k] = (float)(128 * acc[1 + k][0][2 * half + jj] +
                                     acc[1 + k][1][2 * half + jj]) *
                             (qf.sq[jj] * vdiv) * it.vsf(half, k);
  } else {
    using VSt = VStage<D, R, VB>;
    constexpr int KS = D / 32;
    const int m = lane >> 2, c = lane & 3;
    const uint32_t* Va = reinterpret_cast<const uint32_t*>(
        vsm + m * VSt::ROW + c * VSt::SLICE);
    const uint32_t* Vb = Va + 8 * VSt::ROW / 4;
    const uint32_t* mwa = reinterpret_cast<const uint32_t*>(it.mu[0]);
    const uint32_t* mwb = reinterpret_cast<const uint32_t*>(it.mu[1]);
#pragma unroll
    for (int l = 0; l < 2; ++l)
      accmu[l][0] = accmu[l][1] = accmu[l][2] = accmu[l][3] = 0;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      int acc[4][2][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int l = 0; l < 2; ++l)
          acc[kk][l][0] = acc[kk][l][1] = acc[kk][l][2] = acc[kk][l][3] = 0;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const uint32_t* bh = qf.bh[s];
        const uint32_t* bl = qf.bl[s];
        if (p == 0) {
          const uint32_t am[4] = {mwa[2 * s], mwb[2 * s], mwa[2 * s + 1], mwb[2 * s + 1]};
          mma_s8(accmu[0], am, bh[0], bh[1]);
          mma_s8(accmu[1], am, bl[0], bl[1]);
        }
        // words 2*dd + p of the step's 16 (d-rows dd = 0..7, 8 rank bytes each)
        uint32_t wa[8], wb[8];
#pragma unroll
        for (int dd = 0; dd < 8; ++dd) {
          wa[dd] = Va[16 * s + 2 * dd + p];
          wb[dd] = Vb[16 * s + 2 * dd + p];
        }
#define AMASS_R8_COL(KK)                                                      \
        {                                                                     \
          const uint32_t av[4] = {                                            \
              byte_col4<KK>(wa[0], wa[1], wa[2], wa[3]),                      \
              byte_col4<KK>(wb[0], wb[1], wb[2], wb[3]),                      \
              byte_col4<KK>(wa[4], wa[5], wa[6], wa[7]),                      \
              byte_col4<KK>(wb[4], wb[5], wb[6], wb[7])};                     \
          mma_s8(acc[KK][0], av, bh[0], bh[1]);                               \
          mma_s8(acc[KK][1], av, bl[0], bl[1]);                               \
        }
        AMASS_R8_COL(0) AMASS_R8_COL(1) AMASS_R8_COL(2) AMASS_R8_COL(3)
#undef AMASS_R8_COL
      }
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int jj = 0; jj < 2; ++jj)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            qtl[half][jj][4 * p + kk] =
                (float)(128 * acc[kk][0][2 * half + jj] + acc[kk][1][2 * half + jj]) *
                (qf.sq[jj] * vdiv) * it.vsf(half, 4 * p + kk);
    }
  }
}

template <int D, int R, int VB, int CB, bool TS = false>
__global__ void __launch_bounds__(kQuadWarps * 32,
                                  (TS && R <= 4) ? 2 : 1)
r8_score_kernel(QuadArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  constexpr int RC = R8Tok<R, CB>::RC;
  constexpr int PG = 16;                                    // tokens per page
  constexpr int kCBytes = 16 * PG * RC;                     // 16 pages of codes
  constexpr int kSBytes = 16 * PG * 2;                      // their scales
  constexpr int kBuf = kCBytes + kSBytes;
  __shared__ int prefix[kR8MaxReq + 1];
  __shared__ int nshs[kR8MaxReq];
  extern __shared__ __align__(16) uint8_t r8dyn[];          // warps x 2 x kBuf
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    int run = 0;
    for (int base = 0; base < a.n_req; base += 32) {
      const int r = base + lane;
      const int nsh = r < a.n_req ? max(a.nsh[r], 0) : 0;
      const int t = (nsh + 15) / 16;
      int incl = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
      }
      if (r < a.n_req) { prefix[r] = run + incl - t; nshs[r] = nsh; }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[a.n_req] = run;
  }
  __syncthreads();
  const int T = prefix[a.n_req];
  const int gw = blockIdx.x * kQuadWarps + warp;
  const int NJ = gridDim.x * kQuadWarps / a.n_kv;
  const int j = gw / a.n_kv;
  if (j >= NJ) return;
  const int h = gw - j * a.n_kv;
  const int t_lo = (int)((int64_t)T * j / NJ);
  const int t_hi = (int)((int64_t)T * (j + 1) / NJ);
  if (t_lo >= t_hi) return;
  int rh = 0;
  {
    int lo = 0, hi = a.n_req - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= t_lo) lo = mid; else hi = mid - 1;
    }
    rh = lo;
  }
  const int m = lane >> 2, c = lane & 3;
  uint8_t* wbuf = r8dyn + warp * 2 * kBuf;
  const uint32_t wbuf_s = smem_u32(wbuf);
  // rank-8 V rows go through one warp-private shared stage: the next
  // tile's rows are copied while this tile's token logits are computed
  constexpr bool VS = !Item<D, R, VB>::V_PRE;
  uint8_t* vbuf = r8dyn + kQuadWarps * 2 * kBuf + warp * VStage<D, R, VB>::BYTES;
  const uint32_t vbuf_s = smem_u32(vbuf);
  QFrag<D> qf;
  int qr = -1;
  // three-deep pipeline as the quad scorer (block ids two tiles ahead,
  // summary registers and the coordinate copies one tile ahead)
  Item<D, R, VB> cur, nxt, nn;
  __half2 csp_cur, csp_nxt;                 // page-grain coordinate scales
  auto page_scales = [&](const Item<D, R, VB>& x) {
    __half2 v;
    v.x = x.va ? a.cs[x.rowa] : __ushort_as_half(0);
    v.y = x.vb ? a.cs[x.rowb] : __ushort_as_half(0);
    return v;
  };
  int t = t_lo;
  load_idx(cur, a, prefix, nshs, t * a.n_kv + h, lane, &rh);
  load_data<D, R, VB, false>(cur, a, lane);
  stage_coords<D, R, VB, CB>(cur, a, lane, wbuf_s);
  cp_async_commit();
  if constexpr (VS) {
    stage_v<D, R, VB>(cur, a, lane, vbuf_s);
    cp_async_commit();
  }
  if (!a.ctok) csp_cur = page_scales(cur);
  if (t + 1 < t_hi) load_idx(nxt, a, prefix, nshs, (t + 1) * a.n_kv + h, lane, &rh);
  constexpr float kL2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
  while (true) {
    const bool more = t + 1 < t_hi;
    if (t + 2 < t_hi) load_idx(nn, a, prefix, nshs, (t + 2) * a.n_kv + h, lane, &rh);
    if (more) {
      load_data<D, R, VB, false>(nxt, a, lane);
      stage_coords<D, R, VB, CB>(nxt, a, lane, wbuf_s + ((t + 1 - t_lo) & 1) * kBuf);
      if (!a.ctok) csp_nxt = page_scales(nxt);
    }
    cp_async_commit();
    if (cur.r != qr) {
      load_qfrag(qf, a, cur.r, h, lane);
      qr = cur.r;
    }
    int accmu[2][4];
    float qtl[2][2][R];                    // q~ [page half][head jj][rank]
    if constexpr (VS) {
      cp_async_wait<1>();                  // this tile's coordinates and V
      __syncwarp();
      r8_dots(cur, qf, a, lane, vbuf, accmu, qtl);
      __syncwarp();                        // every lane is done with vbuf
      if (more) stage_v<D, R, VB>(nxt, a, lane, vbuf_s);
      cp_async_commit();
    } else {
      r8_dots(cur, qf, a, lane, nullptr, accmu, qtl);
      cp_async_wait<1>();                  // this tile's coordinates landed
      __syncwarp();
    }
    const uint8_t* cb = wbuf + ((t - t_lo) & 1) * kBuf;
    const __half* csb = reinterpret_cast<const __half*>(cb + kCBytes);
    const int sl_r = __ldg(a.sl + cur.r);
    float best[2] = {-INFINITY, -INFINITY};
    float Sv[2][2];
    float qsqv[2] = {0.f, 0.f};
    if (a.resid) {
      const int H = a.n_kv * a.G;
      const float* qr_ = a.qsq + (int64_t)cur.r * H + h * a.G;
      qsqv[0] = __ldg(qr_ + min(2 * c, a.G - 1));
      qsqv[1] = __ldg(qr_ + min(2 * c + 1, a.G - 1));
    }
    if constexpr (TS) {
      // token split (G <= 4): lane c evaluates tokens 4c..4c+3
      // of its two pages for all four head slots, so each token's code is
      // decoded once per quad of lanes instead of four times and no logits
      // are spent on head slots >= 4; the per-(page, head) log-sum-exp is
      // then combined across the quad's lanes
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int pl = m + 8 * half;
        const int p = cur.p0 + pl;
        float qa[4][R];
#pragma unroll
        for (int g = 0; g < 4; ++g)
#pragma unroll
          for (int k = 0; k < R; ++k)
            qa[g][k] = __shfl_sync(0xffffffffu, qtl[half][g & 1][k],
                                   (lane & ~3) | (g >> 1));
        constexpr int RCT = R8Tok<R, CB>::RC;
        const uint8_t* rowp = cb + (pl * PG + 4 * c) * RCT;
        uint32_t cw[RCT];
        if constexpr (RCT == 1) {
          cw[0] = *reinterpret_cast<const uint32_t*>(rowp);
        } else if constexpr (RCT == 2) {
          const uint2 x = *reinterpret_cast<const uint2*>(rowp);
          cw[0] = x.x; cw[1] = x.y;
        } else {
#pragma unroll
          for (int w4 = 0; w4 < RCT; w4 += 4) {
            const uint4 x = *reinterpret_cast<const uint4*>(rowp + 4 * w4);
            cw[w4] = x.x; cw[w4 + 1] = x.y; cw[w4 + 2] = x.z; cw[w4 + 3] = x.w;
          }
        }
        float csv[4];
        if (a.ctok) {
          const uint2 sw = *reinterpret_cast<const uint2*>(csb + pl * PG + 4 * c);
          csv[0] = __half2float(__ushort_as_half((uint16_t)(sw.x & 0xffffu)));
          csv[1] = __half2float(__ushort_as_half((uint16_t)(sw.x >> 16)));
          csv[2] = __half2float(__ushort_as_half((uint16_t)(sw.y & 0xffffu)));
          csv[3] = __half2float(__ushort_as_half((uint16_t)(sw.y >> 16)));
        } else {
          const float csp = half ? __high2float(csp_cur) : __low2float(csp_cur);
          csv[0] = csv[1] = csv[2] = csv[3] = csp;
        }
        float lg[4][4];                              // [head slot][token]
#pragma unroll
        for (int tk = 0; tk < 4; ++tk) {
          float code[R];
#pragma unroll
          for (int k = 0; k < (CB == 8 ? R : R / 2); ++k) {
            const int bi = tk * RCT + k;
            const int b = (int)(int8_t)((cw[bi >> 2] >> (8 * (bi & 3))) & 0xffu);
            if constexpr (CB == 8) {
              code[k] = (float)b;
            } else {
              code[2 * k] = (float)((b << 28) >> 28);
              code[2 * k + 1] = (float)(b >> 4);
            }
          }
          const bool tv = p * PG + 4 * c + tk < sl_r;
          const float cs = csv[tk] * a.scale * kL2e;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            float d = 0.f;
#pragma unroll
            for (int k = 0; k < R; ++k) d += code[k] * qa[g][k];
            lg[g][tk] = tv ? d * cs : -INFINITY;
          }
        }
        float agg[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float mx = fmaxf(fmaxf(lg[g][0], lg[g][1]), fmaxf(lg[g][2], lg[g][3]));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          if (a.tokmax) {
            agg[g] = mx * kLn2;
          } else {
            // hardware 2^x / log2 (rel. error ~2^-22); 2^-inf = 0 covers
            // masked tokens, and an all-masked row keeps agg = -inf
            float sm = 0.f;
#pragma unroll
            for (int tk = 0; tk < 4; ++tk) sm += ex2_approx(lg[g][tk] - mx);
            sm += __shfl_xor_sync(0xffffffffu, sm, 1);
            sm += __shfl_xor_sync(0xffffffffu, sm, 2);
            agg[g] = mx == -INFINITY ? -INFINITY : (mx + lg2_approx(sm)) * kLn2;
          }
        }
        const float mus = half ? __high2float(cur.mus) : __low2float(cur.mus);
        const float res = a.resid ? __half2float(a.resid[half ? cur.rowb : cur.rowa]) : 0.f;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int g = 2 * c + jj;
          float ag = -INFINITY;
#pragma unroll
          for (int gg = 0; gg < 4; ++gg) ag = gg == g ? agg[gg] : ag;
          const int idx = 2 * half + jj;
          const float qmu = (float)(128 * accmu[0][idx] + accmu[1][idx]) * qf.sq[jj] *
                            mus * a.scale;
          float S = qmu + ag;
          if (a.resid) {
            float qh = 0.f;
#pragma unroll
            for (int k = 0; k < R; ++k) qh += qtl[half][jj][k] * qtl[half][jj][k];
            S += fmaxf(qsqv[jj] - qh, 0.f) * res * a.iso_coef;
          }
          Sv[half][jj] = S;
          if (g < a.G) best[half] = fmaxf(best[half], S);
        }
      }
    } else {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int pl = m + 8 * half;                 // page within the tile
        const int p = cur.p0 + pl;
        const float mus = half ? __high2float(cur.mus) : __low2float(cur.mus);
        const float (*qt)[R] = qtl[half];
        const float csp = half ? __high2float(csp_cur) : __low2float(csp_cur);
        // token logits in the log2 domain: two passes (max, then sum)
        float tk2[2][PG];
  #pragma unroll
        for (int tk = 0; tk < PG; ++tk) {
          const bool tv = p * PG + tk < sl_r;
          const uint8_t* row = cb + (pl * PG + tk) * RC;
          float code[R];
          if constexpr (CB == 8) {
  #pragma unroll
            for (int k = 0; k < R; ++k) code[k] = (float)(int8_t)row[k];
          } else {
  #pragma unroll
            for (int k = 0; k < R; k += 2) {
              const int b = (int8_t)row[k / 2];
              code[k] = (float)((b << 28) >> 28);
              code[k + 1] = (float)(b >> 4);
            }
          }
          const float cs = (a.ctok ? __half2float(csb[pl * PG + tk]) : csp) * a.scale;
  #pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            float d = 0.f;
  #pragma unroll
            for (int k = 0; k < R; ++k) d += code[k] * qt[jj][k];
            tk2[jj][tk] = tv ? d * cs * kL2e : -INFINITY;
          }
        }
        // CLSE: the out-of-subspace energy (|q|^2 - |q~|^2) * resid * coef
        const float res = a.resid ? __half2float(a.resid[half ? cur.rowb : cur.rowa]) : 0.f;
  #pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          float mx = -INFINITY;
  #pragma unroll
          for (int tk = 0; tk < PG; ++tk) mx = fmaxf(mx, tk2[jj][tk]);
          float agg;
          if (a.tokmax) {
            agg = mx * kLn2;
          } else {
            float sm = 0.f;
  #pragma unroll
            for (int tk = 0; tk < PG; ++tk) sm += ex2_approx(tk2[jj][tk] - mx);
            agg = mx == -INFINITY ? -INFINITY : (mx + lg2_approx(sm)) * kLn2;
          }
          const int idx = 2 * half + jj;
          const float qmu = (float)(128 * accmu[0][idx] + accmu[1][idx]) * qf.sq[jj] *
                            mus * a.scale;
          float S = qmu + agg;
          if (a.resid) {
            float qh = 0.f;
  #pragma unroll
            for (int k = 0; k < R; ++k) qh += qt[jj][k] * qt[jj][k];
            S += fmaxf(qsqv[jj] - qh, 0.f) * res * a.iso_coef;
          }
          Sv[half][jj] = S;
          if (2 * c + jj < a.G) best[half] = fmaxf(best[half], S);
        }
      }
    }
    if (a.write_h) {
      // per-head scores and the per-head page maximum (the nrm fold's hmax)
      float* base = a.score_h + ((int64_t)cur.r * a.n_kv + h) * a.G * a.SHS;
      const int pa = cur.p0 + m, pb = pa + 8;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int g = 2 * c + jj;
        float mxh = -INFINITY;
        if (g < a.G) {
          if (cur.va) { base[(int64_t)g * a.SHS + pa] = Sv[0][jj]; mxh = Sv[0][jj]; }
          if (cur.vb) { base[(int64_t)g * a.SHS + pb] = Sv[1][jj]; mxh = fmaxf(mxh, Sv[1][jj]); }
        }
        mxh = fmaxf(mxh, __shfl_xor_sync(0xffffffffu, mxh, 4));
        mxh = fmaxf(mxh, __shfl_xor_sync(0xffffffffu, mxh, 8));
        mxh = fmaxf(mxh, __shfl_xor_sync(0xffffffffu, mxh, 16));
        if (m == 0 && g < a.G && mxh > -INFINITY)
          atomic_max_float(a.hmax + ((int64_t)cur.r * a.n_kv + h) * a.G + g, mxh);
      }
    } else {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v = best[half];
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
        const bool pv = half ? cur.vb : cur.va;
        if (pv && c == 0)
          a.score[((int64_t)cur.r * a.n_kv + h) * a.MP + cur.p0 + m + 8 * half] = v;
      }
    }
    __syncwarp();                          // buffer reused two tiles later
    if (!more) break;
    cur = nxt;
    nxt = nn;
    csp_cur = csp_nxt;
    ++t;
  }
  cp_async_wait<0>();
}

template <int D, int CB, int VB, int R, bool TS>
int launch_r8_k(const QuadArgs& a, cudaStream_t st);

template <int D, int CB, int VB, int R = 8>
int launch_r8(const QuadArgs& a, cudaStream_t st) {
  if (a.G <= 4) return launch_r8_k<D, CB, VB, R, true>(a, st);
  return launch_r8_k<D, CB, VB, R, false>(a, st);
}

template <int D, int CB, int VB, int R, bool TS>
int launch_r8_k(const QuadArgs& a, cudaStream_t st) {
  auto k = r8_score_kernel<D, R, VB, CB, TS>;
  constexpr int RC = R8Tok<R, CB>::RC;
  constexpr size_t vst = Item<D, R, VB>::V_PRE ? 0 : VStage<D, R, VB>::BYTES;
  const size_t smem = (size_t)kQuadWarps * (2 * (16 * 16 * RC + 16 * 16 * 2) + vst);
  static int ps = 0;
  static unsigned long long attr = 0;
  if (first_on_device(attr))
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (ps == 0) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ps, k, kQuadWarps * 32, smem);
    if (ps < 1) ps = 1;
  }
  const int heads = a.n_req * a.n_kv * a.G;
  if (int rc = launch_pdl(q_limbs_kernel<D>, dim3((heads + 7) / 8), dim3(256), 0, st, a)) return rc;
  int grid = num_sms() * ps;
  const int per = a.n_kv > kQuadWarps ? a.n_kv / kQuadWarps : 1;
  grid = (grid / per) * per;
  if (int rc = launch_pdl(k, dim3(grid), dim3(kQuadWarps * 32), smem, st, a)) return rc;
  return launch_status();
}

// Batches of at least kQuadQinReq requests split q in the scorer (each warp
// changes request rarely, so its limb split is amortised: C3 step 117.2 ->
// 115.9 us on B200); smaller batches keep the limb launch, where a warp's
// one or two tiles would wait on its own split (8 requests: 33.9 -> 35.0 us).
constexpr int kQuadQinReq = 32;

// Which scorer serves a call (amass_quad_pipeline): 1 (default) the
// pipelined scorer from kQuadQinReq requests up where the geometry allows,
// 2 wherever the geometry allows, 0 never.  Measured on B200 (layer-step,
// us, pipelined vs register-pipelined): 64 requests 114.3 vs 114.7, 32
// requests 70.0 vs 70.0, 16 requests 48.7 vs 48.6, 8 requests 33.0 vs 34.2,
// C2 (1 request) 42.7 vs 42.0, C5 (16 requests) 154.7 vs 151.7 -- below 32
// requests the ring's shared memory keeps the next kernels' CTAs off the SMs
// for longer than the scorer gains.
int g_quad_pipe_mode = 1;
long long g_quad_pipe_launches = 0;   // host count of pipelined launches
// amass_quad_pack: the quad scorers' packed-limb form for G <= 4 (1,
// default) or the two-limb form (0); bit-identical scores.
int g_quad_pack = 1;

// The pipelined scorer when the geometry allows it: 8 kv heads, a lane's V
// slice of at most 32 bytes (int4 rank 2 or int8 rank 1 at head_dim 128),
// 16-byte aligned scale slabs, the ring and the request table within the
// shared-memory budget of two CTAs per SM.  Returns -1 when it does not
// apply.
template <int D, int R, int VB>
int launch_quad_pipe(const QuadArgs& a, bool write_h, bool qin,
                     cudaStream_t st) {
  constexpr int S = kPipeStages;
  if constexpr (Item<D, R, VB>::V_BYTES > 32) {
    return -1;        // wider V slices exceed the consumers' register budget
  } else {
    if (g_quad_pipe_mode == 0 || (g_quad_pipe_mode == 1 && !qin) ||
        a.n_kv != kPipeHeads)
      return -1;
    if ((reinterpret_cast<uintptr_t>(a.mus) |
         reinterpret_cast<uintptr_t>(a.Vs) |
         reinterpret_cast<uintptr_t>(a.sig2)) & 15)
      return -1;
    const size_t smem = pipe_smem_bytes<D, R, VB, S>(a.n_req);
    if (smem > 110 * 1024) return -1;
    using K = void (*)(QuadArgs);
    // G <= 4: packed limbs (half the MMAs, half the epilogue per lane)
    const int pk = a.G <= 4 ? g_quad_pack : 0;
    K k;
#define AMASS_PIPE_K(W, Q)                                              \
    (pk ? quad_score_pipe_kernel<D, R, VB, W, Q, S, true>               \
        : quad_score_pipe_kernel<D, R, VB, W, Q, S, false>)
    if (qin) k = write_h ? AMASS_PIPE_K(true, true) : AMASS_PIPE_K(false, true);
    else k = write_h ? AMASS_PIPE_K(true, false) : AMASS_PIPE_K(false, false);
#undef AMASS_PIPE_K
    static unsigned long long attr_set[8] = {};
    if (first_on_device(attr_set[(write_h ? 1 : 0) + (qin ? 2 : 0) + 4 * pk]))
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           110 * 1024);
    QuadArgs b = a;
    if (!qin) {
      const int heads = a.n_req * a.n_kv * a.G;
      if (int rc = launch_pdl(q_limbs_kernel<D>, dim3((heads + 7) / 8),
                              dim3(256), 0, st, a))
        return rc;
      b.dv_sl = nullptr;
    }
    if (int rc = launch_pdl(k, dim3(2 * num_sms()), dim3(kPipeThreads), smem,
                            st, b))
      return rc;
    ++g_quad_pipe_launches;
    return launch_status();
  }
}

template <int D, int R, int VB>
int launch_quad(const QuadArgs& a, bool write_h, cudaStream_t st) {
  const bool qin = a.n_req >= kQuadQinReq;
  {
    const int rc = launch_quad_pipe<D, R, VB>(a, write_h, qin, st);
    if (rc >= 0) return rc;
  }
  using K = void (*)(QuadArgs);
  K k;
  // G <= 4 with the V slice in registers: packed limbs
  constexpr bool kPkOk = Item<D, R, VB>::V_PRE;
  const bool pk = kPkOk && a.G <= 4 && g_quad_pack;
#define AMASS_QUAD_K(W, Q)                                               \
    (pk ? quad_score_kernel<D, R, VB, W, Q, kPkOk>                       \
        : quad_score_kernel<D, R, VB, W, Q, false>)
  if (qin) k = write_h ? AMASS_QUAD_K(true, true) : AMASS_QUAD_K(false, true);
  else k = write_h ? AMASS_QUAD_K(true, false) : AMASS_QUAD_K(false, false);
#undef AMASS_QUAD_K
  static int per_sm[8] = {};
  int& ps = per_sm[(write_h ? 1 : 0) + (qin ? 2 : 0) + (pk ? 4 : 0)];
  if (ps == 0) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ps, k, kQuadWarps * 32, 0);
    if (ps < 1) ps = 1;
  }
  QuadArgs b = a;
  if (!qin) {
    const int heads = a.n_req * a.n_kv * a.G;
    if (int rc = launch_pdl(q_limbs_kernel<D>, dim3((heads + 7) / 8), dim3(256), 0, st, a))
      return rc;
    b.dv_sl = nullptr;          // derived by the limb launch; the scorer reads nsh
  }
  int grid = num_sms() * ps;
  const int per = a.n_kv > kQuadWarps ? a.n_kv / kQuadWarps : 1;
  grid = (grid / per) * per;   // warps per grid a multiple of n_kv
  if (int rc = launch_pdl(k, dim3(grid), dim3(kQuadWarps * 32), 0, st, b)) return rc;
  return launch_status();
}

template <int D>
int dispatch_rank(const QuadArgs& a, int rank, int v_bits, bool write_h,
                  cudaStream_t st) {
  if (v_bits == 8) {
    switch (rank) {
      case 1: return launch_quad<D, 1, 8>(a, write_h, st);
      case 2: return launch_quad<D, 2, 8>(a, write_h, st);
      case 4: return launch_quad<D, 4, 8>(a, write_h, st);
      case 8: return launch_quad<D, 8, 8>(a, write_h, st);
    }
  } else if (v_bits == 4) {
    switch (rank) {
      case 2: return launch_quad<D, 2, 4>(a, write_h, st);
      case 4: return launch_quad<D, 4, 4>(a, write_h, st);
      case 8: return launch_quad<D, 8, 4>(a, write_h, st);
    }
  }
  return AMASS_ERR_UNSUPPORTED;
}

}  // namespace
}  // namespace amass

namespace amass {
namespace {
int quad_score_impl(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                    const int8_t* mu, const void* mu_scale, const int8_t* V,
                    const void* V_scale, const void* sig2,
                    const int32_t* block_table, int64_t bt_stride,
                    const int32_t* n_sel_hi, float* score, float* score_h,
                    int64_t sh_stride, float* hmax, int8_t* q8_ws,
                    float* qs_ws, float scale, int n_req, int n_kv, int G,
                    int head_dim, int page, int rank, int v_bits,
                    int max_pages, int write_h, void* stream,
                    const QuadArgs* derive) {
  if (n_req < 0 || n_kv <= 0 || G <= 0 || max_pages <= 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!q || !mu || !mu_scale || !V || !V_scale || !sig2 || !block_table ||
      !n_sel_hi || !q8_ws || !qs_ws)
    return AMASS_ERR_ARG;
  if (write_h ? (!score_h || !hmax || sh_stride < max_pages) : !score)
    return AMASS_ERR_ARG;
  if (G > 8 || page != 16 || n_req > kQuadMaxReq) return AMASS_ERR_UNSUPPORTED;
  // 16-byte loads of summary rows and of the q limbs
  if ((q_stride_h % 2) || (q_stride_t % 2) ||
      (reinterpret_cast<uintptr_t>(mu) & 15) ||
      (reinterpret_cast<uintptr_t>(V) & 15) ||
      (reinterpret_cast<uintptr_t>(q8_ws) & 15))
    return AMASS_ERR_ARG;
  QuadArgs a{};
  if (derive) {
    a.dv_sl = derive->dv_sl;
    a.dv_budget = derive->dv_budget;
    a.dv_npg = derive->dv_npg;
    a.dv_nsh = derive->dv_nsh;
    a.dv_b = derive->dv_b;
    a.dv_win = derive->dv_win;
    a.dv_sink = derive->dv_sink;
  }
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.mu = mu;
  a.mus = static_cast<const __half*>(mu_scale);
  a.V = V;
  a.Vs = static_cast<const __half*>(V_scale);
  a.sig2 = static_cast<const __half*>(sig2);
  a.bt = block_table;
  a.bt_stride = bt_stride;
  a.nsh = n_sel_hi;
  a.score = score;
  a.score_h = score_h;
  a.SHS = sh_stride;
  a.hmax = hmax;
  a.q8 = q8_ws;
  a.qs = qs_ws;
  a.scale = scale;
  a.coef = scale * scale * (1.0f / (2.0f * page));
  a.n_req = n_req;
  a.n_kv = n_kv;
  a.G = G;
  a.MP = max_pages;
  a.page = page;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) return dispatch_rank<128>(a, rank, v_bits, write_h, st);
  if (head_dim == 64) return dispatch_rank<64>(a, rank, v_bits, write_h, st);
  return AMASS_ERR_UNSUPPORTED;
}
}  // namespace
}  // namespace amass

extern "C" int amass_quad_score(const void* q, int64_t q_stride_t,
                                int64_t q_stride_h, const int8_t* mu,
                                const void* mu_scale, const int8_t* V,
                                const void* V_scale, const void* sig2,
                                const int32_t* block_table, int64_t bt_stride,
                                const int32_t* n_sel_hi, float* score,
                                float* score_h, int64_t sh_stride,
                                float* hmax, int8_t* q8_ws,
                                float* qs_ws, float scale, int n_req,
                                int n_kv, int G, int head_dim, int page,
                                int rank, int v_bits, int max_pages,
                                int write_h, void* stream) {
  return amass::quad_score_impl(q, q_stride_t, q_stride_h, mu, mu_scale, V,
                                V_scale, sig2, block_table, bt_stride,
                                n_sel_hi, score, score_h, sh_stride, hmax,
                                q8_ws, qs_ws, scale, n_req, n_kv, G, head_dim,
                                page, rank, v_bits, max_pages, write_h, stream,
                                nullptr);
}

extern "C" int amass_quad_score_derive(
    const int32_t* seq_lens, const double* budget64, int32_t* n_pages,
    int32_t* n_sel_hi, int32_t* b_fix, int window_pages, int sink_pages,
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const int8_t* mu,
    const void* mu_scale, const int8_t* V, const void* V_scale,
    const void* sig2, const int32_t* block_table, int64_t bt_stride,
    float* score, float* score_h, int64_t sh_stride, float* hmax,
    int8_t* q8_ws, float* qs_ws, float scale, int n_req, int n_kv, int G,
    int head_dim, int page, int rank, int v_bits, int max_pages, int write_h,
    void* stream) {
  using namespace amass;
  if (!seq_lens || !budget64 || !n_pages || !n_sel_hi || !b_fix ||
      window_pages < 0 || sink_pages < 0)
    return AMASS_ERR_ARG;
  QuadArgs d{};
  d.dv_sl = seq_lens;
  d.dv_budget = budget64;
  d.dv_npg = n_pages;
  d.dv_nsh = n_sel_hi;
  d.dv_b = b_fix;
  d.dv_win = window_pages;
  d.dv_sink = sink_pages;
  return quad_score_impl(q, q_stride_t, q_stride_h, mu, mu_scale, V, V_scale,
                         sig2, block_table, bt_stride, n_sel_hi, score,
                         score_h, sh_stride, hmax, q8_ws, qs_ws, scale, n_req,
                         n_kv, G, head_dim, page, rank, v_bits, max_pages,
                         write_h, stream, &d);
}


extern "C" int amass_r8_score(const void* q, int64_t q_stride_t,
                              int64_t q_stride_h, const int8_t* mu,
                              const void* mu_scale, const int8_t* Vk,
                              const void* Vk_scale, const int8_t* c,
                              const void* c_scale, const int32_t* block_table,
                              int64_t bt_stride, const int32_t* seq_lens,
                              const int32_t* n_sel_hi, float* score,
                              int8_t* q8_ws, float* qs_ws, float scale,
                              int n_req, int n_kv, int G, int head_dim,
                              int page, int rank, int vk_bits, int c_bits,
                              int max_pages, int token_agg, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || G <= 0 || max_pages <= 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!q || !mu || !mu_scale || !Vk || !Vk_scale || !c || !c_scale ||
      !block_table || !seq_lens || !n_sel_hi || !score || !q8_ws || !qs_ws)
    return AMASS_ERR_ARG;
  if (G > 8 || page != 16 || rank != 8 || n_req > kR8MaxReq ||
      (vk_bits != 8 && vk_bits != 4) || (c_bits != 8 && c_bits != 4))
    return AMASS_ERR_UNSUPPORTED;
  if ((q_stride_h % 2) || (q_stride_t % 2) ||
      (reinterpret_cast<uintptr_t>(mu) & 15) ||
      (reinterpret_cast<uintptr_t>(Vk) & 15) ||
      (reinterpret_cast<uintptr_t>(c) & 15) ||
      (reinterpret_cast<uintptr_t>(c_scale) & 15) ||
      (reinterpret_cast<uintptr_t>(Vk_scale) & 3) ||
      (reinterpret_cast<uintptr_t>(q8_ws) & 15))
    return AMASS_ERR_ARG;
  QuadArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.mu = mu;
  a.mus = static_cast<const __half*>(mu_scale);
  a.V = Vk;
  a.Vs = static_cast<const __half*>(Vk_scale);
  a.sig2 = static_cast<const __half*>(Vk_scale);   // unused by r8
  a.c = c;
  a.cs = static_cast<const __half*>(c_scale);
  a.sl = seq_lens;
  a.bt = block_table;
  a.bt_stride = bt_stride;
  a.nsh = n_sel_hi;
  a.score = score;
  a.q8 = q8_ws;
  a.qs = qs_ws;
  a.scale = scale;
  a.n_req = n_req;
  a.n_kv = n_kv;
  a.G = G;
  a.MP = max_pages;
  a.page = page;
  a.tokmax = token_agg == AMASS_R8_TOKMAX ? 1 : 0;
  a.ctok = 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto d) -> int {
    constexpr int D = decltype(d)::value;
    if (vk_bits == 8 && c_bits == 8) return launch_r8<D, 8, 8>(a, st);
    if (vk_bits == 8 && c_bits == 4) return launch_r8<D, 4, 8>(a, st);
    if (vk_bits == 4 && c_bits == 8) return launch_r8<D, 8, 4>(a, st);
    return launch_r8<D, 4, 4>(a, st);
  };
  if (head_dim == 128) return go(std::integral_constant<int, 128>{});
  if (head_dim == 64) return go(std::integral_constant<int, 64>{});
  return AMASS_ERR_UNSUPPORTED;
}

extern "C" int amass_clse_score(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const int8_t* mu,
    const void* mu_scale, const int8_t* V, const void* V_scale,
    const int8_t* c, const void* c_scale, int c_token_grain,
    const void* resid, const int32_t* block_table, int64_t bt_stride,
    const int32_t* seq_lens, const int32_t* n_sel_hi, float* score,
    float* score_h, int64_t sh_stride, float* hmax, int8_t* q8_ws,
    float* qs_ws, float* qsq_ws, float scale, int n_req, int n_kv, int G,
    int head_dim, int page, int rank, int v_bits, int c_bits, int max_pages,
    int write_h, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || G <= 0 || max_pages <= 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!q || !mu || !mu_scale || !V || !V_scale || !c || !c_scale || !resid ||
      !block_table || !seq_lens || !n_sel_hi || !q8_ws || !qs_ws || !qsq_ws)
    return AMASS_ERR_ARG;
  if (write_h ? (!score_h || !hmax || sh_stride < max_pages) : !score)
    return AMASS_ERR_ARG;
  if (G > 8 || page != 16 || n_req > kR8MaxReq ||
      (rank != 2 && rank != 4 && rank != 8) || (v_bits != 8 && v_bits != 4) ||
      (c_bits != 8 && c_bits != 4))
    return AMASS_ERR_UNSUPPORTED;
  if ((q_stride_h % 2) || (q_stride_t % 2) ||
      (reinterpret_cast<uintptr_t>(mu) & 15) ||
      (reinterpret_cast<uintptr_t>(V) & 15) ||
      (reinterpret_cast<uintptr_t>(c) & 15) ||
      (c_token_grain && (reinterpret_cast<uintptr_t>(c_scale) & 15)) ||
      (reinterpret_cast<uintptr_t>(V_scale) & 3) ||
      (reinterpret_cast<uintptr_t>(q8_ws) & 15))
    return AMASS_ERR_ARG;
  QuadArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.mu = mu;
  a.mus = static_cast<const __half*>(mu_scale);
  a.V = V;
  a.Vs = static_cast<const __half*>(V_scale);
  a.sig2 = static_cast<const __half*>(V_scale);   // unused here
  a.c = c;
  a.cs = static_cast<const __half*>(c_scale);
  a.sl = seq_lens;
  a.bt = block_table;
  a.bt_stride = bt_stride;
  a.nsh = n_sel_hi;
  a.score = score;
  a.score_h = score_h;
  a.SHS = sh_stride;
  a.hmax = hmax;
  a.q8 = q8_ws;
  a.qs = qs_ws;
  a.qsq = qsq_ws;
  a.resid = static_cast<const __half*>(resid);
  a.scale = scale;
  a.iso_coef = scale * scale / (2.f * page * (float)std::max(head_dim - rank, 1));
  a.ctok = c_token_grain ? 1 : 0;
  a.write_h = write_h ? 1 : 0;
  a.n_req = n_req;
  a.n_kv = n_kv;
  a.G = G;
  a.MP = max_pages;
  a.page = page;
  a.tokmax = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto d, auto r) -> int {
    constexpr int D = decltype(d)::value;
    constexpr int R = decltype(r)::value;
    if (v_bits == 8 && c_bits == 8) return launch_r8<D, 8, 8, R>(a, st);
    if (v_bits == 8 && c_bits == 4) return launch_r8<D, 4, 8, R>(a, st);
    if (v_bits == 4 && c_bits == 8) return launch_r8<D, 8, 4, R>(a, st);
    return launch_r8<D, 4, 4, R>(a, st);
  };
  auto by_rank = [&](auto d) -> int {
    if (rank == 2) return go(d, std::integral_constant<int, 2>{});
    if (rank == 4) return go(d, std::integral_constant<int, 4>{});
    return go(d, std::integral_constant<int, 8>{});
  };
  if (head_dim == 128) return by_rank(std::integral_constant<int, 128>{});
  if (head_dim == 64) return by_rank(std::integral_constant<int, 64>{});
  return AMASS_ERR_UNSUPPORTED;
}

extern "C" int amass_quad_pipeline(int mode) {
  using namespace amass;
  const int prev = g_quad_pipe_mode;
  if (mode >= 0 && mode <= 2) g_quad_pipe_mode = mode;
  return prev;
}

extern "C" int amass_quad_pack(int on) {
  using namespace amass;
  const int prev = g_quad_pack;
  if (on == 0 || on == 1) g_quad_pack = on;
  return prev;
}

extern "C" int amass_quad_pipeline_status(int* fault, long long* launches,
                                          int clear) {
  using namespace amass;
  if (fault) {
    if (cudaMemcpyFromSymbol(fault, g_quad_pipe_fault, sizeof(int)) !=
        cudaSuccess)
      return AMASS_ERR_CUDA;
    if (clear) {
      const int zero = 0;
      if (cudaMemcpyToSymbol(g_quad_pipe_fault, &zero, sizeof(int)) !=
          cudaSuccess)
        return AMASS_ERR_CUDA;
    }
  }
  if (launches) {
    *launches = g_quad_pipe_launches;
    if (clear) g_quad_pipe_launches = 0;
  }
  return AMASS_OK;
}
