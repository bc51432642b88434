// Stage A.1: the quad (Gaussian-MGF) page scorer on sm_100a.
//
// Math (reference selection/quad_score.py:55-107), per (request r, kv-head h,
// page p < n_sel_hi, query head g of the GQA group):
//     qmu_g  = mu_code . q_g            q~_{g,k} = V_code[:,k] . q_g
//     S_g    = s*mu_scale*qmu_g + s^2/(2P) * sum_k sig2_k (V_scale_k q~_{g,k})^2
//
// Layout of the work.  One CTA = 8 warps covers 16*TPC pages of one request
// for every kv-head; a warp owns (16-page tile, kv-head) items, so the 8 heads
// of a block -- whose summaries are contiguous rows -- are read by sibling
// warps at the same time and share their DRAM sectors.  Within a warp the
// three (or 1+rank) dot products per (page, head) run on the tensor cores as
// m16n8k16 MMAs:  A = integer codes (16 pages x 16 d) converted exactly to
// fp16 in registers,  B = q^T (16 d x 8 query heads, fp16),  C = fp32.  The
// d <-> k-slot assignment is a fixed permutation shared by A and B, chosen so
// each lane's loads are contiguous.
#include "common.cuh"

namespace amass {
namespace {

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
  float scale, coef;
  int n_kv, G, MP, tpc;
};

template <int NB>
struct VecLoad;
template <>
struct VecLoad<4> {
  static AMASS_DEV void ld(const int8_t* p, uint32_t* w) {
    w[0] = __ldg(reinterpret_cast<const unsigned int*>(p));
  }
};
template <>
struct VecLoad<8> {
  static AMASS_DEV void ld(const int8_t* p, uint32_t* w) {
    uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  }
};
template <>
struct VecLoad<16> {
  static AMASS_DEV void ld(const int8_t* p, uint32_t* w) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  }
};
template <>
struct VecLoad<32> {
  static AMASS_DEV void ld(const int8_t* p, uint32_t* w) {
    VecLoad<16>::ld(p, w);
    VecLoad<16>::ld(p + 16, w + 4);
  }
};

// Code pair (d0+i, d0+i+1) of column k from a k-step's V bytes (4 d values).
template <int R, int VB, int K, int I>
AMASS_DEV uint32_t v_pair(const uint32_t* w) {
  if constexpr (VB == 8) {
    constexpr int BI = I * R + K, BJ = (I + 1) * R + K;
    return i8pair_to_h2(pick2<BI, BJ>(w[BI / 4], w[BJ / 4]));
  } else {
    constexpr int RB = R / 2;
    constexpr int BI = I * RB + K / 2, BJ = (I + 1) * RB + K / 2;
    uint32_t x = pick2<BI, BJ>(w[BI / 4], w[BJ / 4]);
    if (K & 1) x >>= 4;
    return i4pair_to_h2(x);
  }
}

template <int R, int VB, int K>
struct VCols {
  static AMASS_DEV void run(float (*acc)[4], const uint32_t* wa,
                            const uint32_t* wb, uint32_t b0, uint32_t b1) {
    uint32_t a[4];
    a[0] = v_pair<R, VB, K, 0>(wa);
    a[1] = v_pair<R, VB, K, 0>(wb);
    a[2] = v_pair<R, VB, K, 2>(wa);
    a[3] = v_pair<R, VB, K, 2>(wb);
    mma_f16(acc[1 + K], a, b0, b1);
    if constexpr (K + 1 < R) VCols<R, VB, K + 1>::run(acc, wa, wb, b0, b1);
  }
};

template <int D, int R, int VB, bool WRITE_H>
__global__ void __launch_bounds__(256)
quad_score_kernel(QuadArgs a) {
  constexpr int KS = D / 16;                 // MMA k-steps over head_dim
  constexpr int RB = (VB == 8) ? R : R / 2;  // V code bytes per d
  constexpr int VSTEP = 4 * RB;              // V bytes per k-step per page
  const int r = blockIdx.y;
  const int nsh = a.nsh[r];
  const int pbase = blockIdx.x * 16 * a.tpc;
  if (pbase >= nsh) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = lane >> 2, c = lane & 3;
  const int n_items = a.tpc * a.n_kv;

  for (int item = warp; item < n_items; item += 8) {
    const int t = item / a.n_kv, h = item - t * a.n_kv;
    const int p0 = pbase + 16 * t;
    if (p0 >= nsh) break;
    const int pa = p0 + m, pb = pa + 8;
    const bool va = pa < nsh, vb = pb < nsh;
    const int32_t* btr = a.bt + (int64_t)r * a.bt_stride;
    const int64_t blka = va ? btr[pa] : 0;
    const int64_t blkb = vb ? btr[pb] : 0;
    const int64_t rowa = blka * a.n_kv + h, rowb = blkb * a.n_kv + h;

    // B operand: q^T for query heads g = m of this kv group (zero beyond G)
    uint32_t qb[KS][2];
    {
      const bool gv = m < a.G;
      const __nv_bfloat16* qp =
          a.q + (int64_t)r * a.q_st + (int64_t)(h * a.G + (gv ? m : 0)) * a.q_sh;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        uint2 w = __ldg(reinterpret_cast<const uint2*>(qp + 16 * s + 4 * c));
        qb[s][0] = gv ? pack_h2(bf16_lo(w.x), bf16_hi(w.x)) : 0u;
        qb[s][1] = gv ? pack_h2(bf16_lo(w.y), bf16_hi(w.y)) : 0u;
      }
    }

    float acc[1 + R][4];
#pragma unroll
    for (int i = 0; i <= R; ++i)
      acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    const int8_t* mua = a.mu + rowa * D;
    const int8_t* mub = a.mu + rowb * D;
    const int8_t* Va = a.V + rowa * (D * RB);
    const int8_t* Vb = a.V + rowb * (D * RB);
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int d0 = 16 * s + 4 * c;
      uint32_t wma, wmb;
      VecLoad<4>::ld(mua + d0, &wma);
      VecLoad<4>::ld(mub + d0, &wmb);
      uint32_t wva[VSTEP / 4 > 0 ? VSTEP / 4 : 1], wvb[VSTEP / 4 > 0 ? VSTEP / 4 : 1];
      VecLoad<VSTEP>::ld(Va + d0 * RB, wva);
      VecLoad<VSTEP>::ld(Vb + d0 * RB, wvb);
      uint32_t am[4];
      am[0] = i8pair_to_h2(pick2<0, 1>(wma, wma));
      am[1] = i8pair_to_h2(pick2<0, 1>(wmb, wmb));
      am[2] = i8pair_to_h2(pick2<2, 3>(wma, wma));
      am[3] = i8pair_to_h2(pick2<2, 3>(wmb, wmb));
      mma_f16(acc[0], am, qb[s][0], qb[s][1]);
      VCols<R, VB, 0>::run(acc, wva, wvb, qb[s][0], qb[s][1]);
    }

    // epilogue: rows pa (acc[.][0..1]) and pb (acc[.][2..3]); cols g = 2c, 2c+1
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int p = half ? pb : pa;
      const bool pv = half ? vb : va;
      const int64_t row = half ? rowb : rowa;
      float S[2] = {-INFINITY, -INFINITY};
      if (pv) {
        const float mus = __half2float(a.mus[row]);
        float vs[R], s2[R];
#pragma unroll
        for (int k = 0; k < R; ++k) {
          vs[k] = __half2float(a.Vs[row * R + k]);
          s2[k] = __half2float(a.sig2[row * R + k]);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int idx = 2 * half + j;
          float quad = 0.f;
#pragma unroll
          for (int k = 0; k < R; ++k) {
            const float qt = acc[1 + k][idx] * vs[k];
            quad += s2[k] * qt * qt;
          }
          S[j] = acc[0][idx] * mus * a.scale + quad * a.coef;
        }
      }
      if constexpr (WRITE_H) {
        if (pv) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int g = 2 * c + j;
            if (g < a.G)
              a.score_h[(((int64_t)r * a.n_kv + h) * a.G + g) * a.MP + p] = S[j];
          }
        }
      } else {
        float mx = (2 * c < a.G) ? S[0] : -INFINITY;
        if (2 * c + 1 < a.G) mx = fmaxf(mx, S[1]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (pv && c == 0)
          a.score[((int64_t)r * a.n_kv + h) * a.MP + p] = mx;
      }
    }
  }
}

template <int D, int R, int VB>
int launch_quad(const QuadArgs& a, int n_req, bool write_h, cudaStream_t st) {
  dim3 grid((a.MP + 16 * a.tpc - 1) / (16 * a.tpc), n_req);
  if (write_h)
    quad_score_kernel<D, R, VB, true><<<grid, 256, 0, st>>>(a);
  else
    quad_score_kernel<D, R, VB, false><<<grid, 256, 0, st>>>(a);
  return launch_status();
}

template <int D>
int dispatch_rank(const QuadArgs& a, int n_req, int rank, int v_bits,
                  bool write_h, cudaStream_t st) {
  if (v_bits == 8) {
    switch (rank) {
      case 1: return launch_quad<D, 1, 8>(a, n_req, write_h, st);
      case 2: return launch_quad<D, 2, 8>(a, n_req, write_h, st);
      case 4: return launch_quad<D, 4, 8>(a, n_req, write_h, st);
      case 8: return launch_quad<D, 8, 8>(a, n_req, write_h, st);
    }
  } else if (v_bits == 4) {
    switch (rank) {
      case 2: return launch_quad<D, 2, 4>(a, n_req, write_h, st);
      case 4: return launch_quad<D, 4, 4>(a, n_req, write_h, st);
      case 8: return launch_quad<D, 8, 4>(a, n_req, write_h, st);
    }
  }
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
                                float* score_h, float scale, int n_req,
                                int n_kv, int G, int head_dim, int page,
                                int rank, int v_bits, int max_pages,
                                int write_h, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || G <= 0 || max_pages <= 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!q || !mu || !mu_scale || !V || !V_scale || !sig2 || !block_table ||
      !n_sel_hi)
    return AMASS_ERR_ARG;
  if (write_h ? !score_h : !score) return AMASS_ERR_ARG;
  if (G > 8 || page != 16) return AMASS_ERR_UNSUPPORTED;
  if ((q_stride_h % 4) != 0 || (q_stride_t % 4) != 0 ||
      (reinterpret_cast<uintptr_t>(q) & 7))
    return AMASS_ERR_ARG;
  QuadArgs a;
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
  a.scale = scale;
  a.coef = scale * scale * (1.0f / (2.0f * page));
  a.n_kv = n_kv;
  a.G = G;
  a.MP = max_pages;
  // pages per CTA: 16 * tpc; aim for >= 8 warp items per CTA
  int tpc = (n_kv >= 8) ? 1 : 8 / n_kv;
  if (n_req >= 16) tpc *= 4;
  a.tpc = tpc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) return dispatch_rank<128>(a, n_req, rank, v_bits, write_h, st);
  if (head_dim == 64) return dispatch_rank<64>(a, n_req, rank, v_bits, write_h, st);
  return AMASS_ERR_UNSUPPORTED;
}
