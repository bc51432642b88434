// Page summary build on sm_100a: quad (and r8 / CLSE) summaries of finalized
// KV pages (reference selection/build.py:297-452, quad_build.py:37-84).
//
// Per (layer, block, kv-head) page of 16 keys:
//   mu = mean_t K;  dc = K - mu;  Gm = dc dc^T (16 x 16);  eigh(Gm)
//   S2r = the rank top eigenvalues in ascending order (clamped >= 1e-10),
//   U8 their eigenvectors;  Vk = dc^T U8 / sqrt(S2r)           (d, rank)
//   mu -> int8 (one scale), Vk -> int8/int4 (per column or one scale),
//   sig2 = S2r (fp16), tag = the last key's first tagw values,
//   coordinates c = U8 * sqrt(S2r) (page, rank) -> int8/int4 with per-token
//   or per-page scales, resid = sum K^2 - P |mu|^2 - sum S2r  (CLSE).
//
// One warp per page-head.  Each lane holds d/32 consecutive columns of the
// 16 centred keys in registers; the Gram's 136 distinct entries are lane
// partial dot products reduced through shared memory; the 16 x 16 symmetric
// eigenproblem is solved by cyclic Jacobi in parallel (round-robin) order:
// 8 disjoint rotations per round, 15 rounds per sweep, sweeps until the
// off-diagonal mass is negligible (at most 12).  Eigenvectors are unique up
// to sign, as in the reference.
#include <algorithm>

#include "common.cuh"

namespace amass {
namespace {

constexpr int kSumWarps = 4;
constexpr int kMaxLayers = 128;
constexpr int kPg = 16;

struct SumArgs {
  const __nv_bfloat16* k[kMaxLayers];  // per-layer key caches
  int64_t kb, kt, kh;                  // element strides: block, token, head
  const int32_t* blocks;               // (n_blocks,)
  int n_blocks, n_layers, l0, NB, n_kv;
  int8_t* mu;                          // (Ltot, NB, n_kv, d)
  __half* mus;                         // (Ltot, NB, n_kv)
  int8_t* V;                           // (Ltot, NB, n_kv, d, rv)
  __half* Vs;                          // (Ltot, NB, n_kv, r)
  __half* sig2;                        // (Ltot, NB, n_kv, r) or null
  __nv_bfloat16* tag;                  // (Ltot, NB, n_kv, tagw) or null
  int8_t* c;                           // (Ltot, NB, n_kv, page, rc) or null
  __half* cs;                          // token: (.., page); page: (..) or (.., page)
  __half* resid;                       // (Ltot, NB, n_kv) or null
  int tagw, r, v_bits, v_tensor, c_bits, c_mode;
};

struct SumSmem {
  float part[136][33];     // Gram partials, transposed for the reduction
  float A[kPg][kPg + 1];
  float U[kPg][kPg + 1];
  float rc[8], rs[8];
  int rp[8], rq[8];
  int idx[8];              // eigen-index of rank slot k (ascending)
  float s2[8], s8[8];
  float red[4];
};

AMASS_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
AMASS_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// symmetric quantisation code: round half to even of x / s, clamped
AMASS_DEV int qcode(float x, float s, float lvl) {
  return (int)fminf(fmaxf(rintf(x / s), -lvl), lvl);
}

template <int D>
__global__ void __launch_bounds__(kSumWarps * 32)
summary_kernel(SumArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  constexpr int PER = D / 32;                  // columns per lane
  extern __shared__ __align__(16) uint8_t ssm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  SumSmem& sm = reinterpret_cast<SumSmem*>(ssm)[warp];
  const int per_layer = a.n_blocks * a.n_kv;
  const int total = a.n_layers * per_layer;
  const int r = a.r;
  for (int item = blockIdx.x * kSumWarps + warp; item < total;
       item += gridDim.x * kSumWarps) {
    const int l = item / per_layer;
    const int rem = item - l * per_layer;
    const int bi = rem / a.n_kv, h = rem - bi * a.n_kv;
    const int64_t blk = a.blocks[bi];
    if (blk < 0) continue;                       // not stale (delta rebuild)
    const __nv_bfloat16* kp = a.k[l] + blk * a.kb + h * a.kh + lane * PER;
    // ---- keys -> registers; mean; centred keys; sum of squares -----------
    float x[kPg][PER];
#pragma unroll
    for (int t = 0; t < kPg; ++t) {
      const __nv_bfloat16* kr = kp + t * a.kt;
#pragma unroll
      for (int i = 0; i < PER; i += 2) {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(kr + i);
        x[t][i] = __low2float(v);
        x[t][i + 1] = __high2float(v);
      }
    }
    float mu[PER], ksq = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      float s = 0.f;
#pragma unroll
      for (int t = 0; t < kPg; ++t) s += x[t][i];
      mu[i] = s / (float)kPg;
    }
#pragma unroll
    for (int t = 0; t < kPg; ++t)
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        ksq += x[t][i] * x[t][i];
        x[t][i] -= mu[i];
      }
    // tag: the last key's first tagw raw values
    if (a.tag) {
      const __nv_bfloat16* last = a.k[l] + blk * a.kb + h * a.kh + (kPg - 1) * a.kt;
      const int64_t row = ((int64_t)(a.l0 + l) * a.NB + blk) * a.n_kv + h;
      for (int j = lane; j < a.tagw; j += 32) a.tag[row * a.tagw + j] = last[j];
    }
    // ---- Gram: 136 lane partials, reduced through shared memory ----------
    {
      int e = 0;
#pragma unroll
      for (int i = 0; i < kPg; ++i)
#pragma unroll
        for (int j = i; j < kPg; ++j, ++e) {
          float s = 0.f;
#pragma unroll
          for (int q = 0; q < PER; ++q) s += x[i][q] * x[j][q];
          sm.part[e][lane] = s;
        }
    }
    __syncwarp();
    for (int e = lane; e < 136; e += 32) {
      float s = 0.f;
#pragma unroll 8
      for (int q = 0; q < 32; ++q) s += sm.part[e][q];
      // entry e -> (i, j), i <= j
      int i = 0, base = 0;
      while (e >= base + (kPg - i)) { base += kPg - i; ++i; }
      const int j = i + (e - base);
      sm.A[i][j] = s;
      sm.A[j][i] = s;
    }
    for (int e = lane; e < kPg * kPg; e += 32)
      sm.U[e / kPg][e % kPg] = (e / kPg == e % kPg) ? 1.f : 0.f;
    __syncwarp();
    // ---- cyclic Jacobi, round-robin pairs --------------------------------
    float fro = 0.f;
    for (int e = lane; e < kPg * kPg; e += 32) {
      const float v = sm.A[e / kPg][e % kPg];
      fro += v * v;
    }
    fro = warp_sum(fro);
    for (int sweep = 0; sweep < 12; ++sweep) {
      float off = 0.f;
      for (int e = lane; e < kPg * kPg; e += 32)
        if (e / kPg != e % kPg) {
          const float v = sm.A[e / kPg][e % kPg];
          off += v * v;
        }
      off = warp_sum(off);
      if (off <= 1e-14f * fro) break;
      for (int rnd = 0; rnd < kPg - 1; ++rnd) {
        if (lane < 8) {
          int p, q;
          if (lane == 0) { p = kPg - 1; q = rnd; }
          else { p = (rnd + lane) % (kPg - 1); q = (rnd - lane + kPg - 1) % (kPg - 1); }
          if (p > q) { const int t = p; p = q; q = t; }
          const float apq = sm.A[p][q];
          float c = 1.f, s = 0.f;
          if (fabsf(apq) > 1e-30f) {
            const float tau = (sm.A[q][q] - sm.A[p][p]) / (2.f * apq);
            const float t = (tau >= 0.f ? 1.f : -1.f) /
                            (fabsf(tau) + sqrtf(1.f + tau * tau));
            c = rsqrtf(1.f + t * t);
            s = t * c;
          }
          sm.rp[lane] = p; sm.rq[lane] = q;
          sm.rc[lane] = c; sm.rs[lane] = s;
        }
        __syncwarp();
        // rows: A <- J^T A
        for (int e = lane; e < 8 * kPg; e += 32) {
          const int pi = e / kPg, j = e % kPg;
          const int p = sm.rp[pi], q = sm.rq[pi];
          const float c = sm.rc[pi], s = sm.rs[pi];
          const float ap = sm.A[p][j], aq = sm.A[q][j];
          sm.A[p][j] = c * ap - s * aq;
          sm.A[q][j] = s * ap + c * aq;
        }
        __syncwarp();
        // columns: A <- A J, U <- U J
        for (int e = lane; e < 8 * kPg; e += 32) {
          const int pi = e / kPg, j = e % kPg;
          const int p = sm.rp[pi], q = sm.rq[pi];
          const float c = sm.rc[pi], s = sm.rs[pi];
          const float ap = sm.A[j][p], aq = sm.A[j][q];
          sm.A[j][p] = c * ap - s * aq;
          sm.A[j][q] = s * ap + c * aq;
          const float up = sm.U[j][p], uq = sm.U[j][q];
          sm.U[j][p] = c * up - s * uq;
          sm.U[j][q] = s * up + c * uq;
        }
        __syncwarp();
      }
    }
    // ---- top-r eigenpairs in ascending order (the reference's S2[-r:]) ----
    if (lane < kPg) {
      const float li = sm.A[lane][lane];
      int rank = 0;                              // descending rank
      for (int j = 0; j < kPg; ++j) {
        const float lj = sm.A[j][j];
        rank += (lj > li) || (lj == li && j > lane);
      }
      if (rank < r) {
        const int k = r - 1 - rank;
        sm.idx[k] = lane;
        const float s2 = fmaxf(li, 1e-10f);
        sm.s2[k] = s2;
        sm.s8[k] = sqrtf(s2);
      }
    }
    __syncwarp();
    const int64_t row = ((int64_t)(a.l0 + l) * a.NB + blk) * a.n_kv + h;
    // ---- Vk = dc^T U8 / S8, quantised ------------------------------------
    float vk[PER][8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= r) break;
      const int ei = sm.idx[k];
      const float inv = 1.f / sm.s8[k];
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        float s = 0.f;
#pragma unroll
        for (int t = 0; t < kPg; ++t) s += x[t][i] * sm.U[t][ei];
        vk[i][k] = s * inv;
      }
    }
    const float vlvl = a.v_bits == 4 ? 7.f : 127.f;
    float vsc[8];
    {
      float amax_all = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k >= r) break;
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < PER; ++i) am = fmaxf(am, fabsf(vk[i][k]));
        am = warp_max(am);
        vsc[k] = fmaxf(am / vlvl, 1e-8f);
        amax_all = fmaxf(amax_all, am);
      }
      if (a.v_tensor) {
        const float st = fmaxf(amax_all / vlvl, 1e-8f);
#pragma unroll
        for (int k = 0; k < 8; ++k) vsc[k] = st;
      }
    }
    if (lane < r) {
      float v = vsc[0];
#pragma unroll
      for (int k = 1; k < 8; ++k) if (k == lane) v = vsc[k];
      a.Vs[row * r + lane] = __float2half_rn(v);
      if (a.sig2) a.sig2[row * r + lane] = __float2half_rn(sm.s2[lane]);
    }
    {
      const int rv = a.v_bits == 4 ? r / 2 : r;
      int8_t* vout = a.V + row * (int64_t)D * rv;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane * PER + i;
        if (a.v_bits == 8) {
          for (int k = 0; k < r; ++k)
            vout[d * rv + k] = (int8_t)qcode(vk[i][k], vsc[k], vlvl);
        } else {
          for (int k = 0; k < r; k += 2) {
            const int lo = qcode(vk[i][k], vsc[k], vlvl) & 0xF;
            const int hi = qcode(vk[i][k + 1], vsc[k + 1], vlvl) & 0xF;
            vout[d * rv + k / 2] = (int8_t)(lo | (hi << 4));
          }
        }
      }
    }
    // ---- mu, quantised ----------------------------------------------------
    {
      float am = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) am = fmaxf(am, fabsf(mu[i]));
      am = warp_max(am);
      const float s = fmaxf(am / 127.f, 1e-8f);
#pragma unroll
      for (int i = 0; i < PER; ++i)
        a.mu[row * D + lane * PER + i] = (int8_t)qcode(mu[i], s, 127.f);
      if (lane == 0) a.mus[row] = __float2half_rn(s);
    }
    // ---- coordinates c = U8 * S8 and the residual energy ------------------
    if (a.c) {
      const float clvl = a.c_bits == 4 ? 7.f : 127.f;
      float cv[8];
      float am = 0.f;
      if (lane < kPg) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          cv[k] = (k < r) ? sm.U[lane][sm.idx[k]] * sm.s8[k] : 0.f;
          am = fmaxf(am, fabsf(cv[k]));
        }
      }
      float s;
      if (a.c_mode == 0) {
        s = fmaxf(am / clvl, 1e-8f);                    // per token
      } else {
        s = fmaxf(warp_max(am) / clvl, 1e-8f);          // per page
      }
      if (lane < kPg) {
        const int rcb = a.c_bits == 4 ? r / 2 : r;
        int8_t* co = a.c + (row * kPg + lane) * rcb;
        if (a.c_bits == 8) {
          for (int k = 0; k < r; ++k) co[k] = (int8_t)qcode(cv[k], s, clvl);
        } else {
          for (int k = 0; k < r; k += 2) {
            const int lo = qcode(cv[k], s, clvl) & 0xF;
            const int hi = qcode(cv[k + 1], s, clvl) & 0xF;
            co[k / 2] = (int8_t)(lo | (hi << 4));
          }
        }
        if (a.c_mode == 2) {
          if (lane == 0) a.cs[row] = __float2half_rn(s);
        } else {
          a.cs[row * kPg + lane] = __float2half_rn(s);
        }
      }
    }
    if (a.resid) {
      float musq = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) musq += mu[i] * mu[i];
      const float tr = warp_sum(ksq) - (float)kPg * warp_sum(musq);
      float s2sum = 0.f;
      for (int k = 0; k < r; ++k) s2sum += sm.s2[k];
      if (lane == 0) a.resid[row] = __float2half_rn(fmaxf(tr - s2sum, 0.f));
    }
    __syncwarp();
  }
}

}  // namespace
}  // namespace amass

extern "C" int amass_summarize_pages(
    const void* const* k_layers, int n_layers, int64_t k_sb, int64_t k_st,
    int64_t k_sh, const int32_t* blocks, int n_blocks, int layer0,
    int num_blocks, int n_kv, int head_dim, int page, int rank, int8_t* mu,
    void* mu_scale, int8_t* V, void* V_scale, int v_bits, int v_tensor,
    void* sig2, void* tag, int tagw, int8_t* c, void* c_scale, int c_bits,
    int c_mode, void* resid, void* stream) {
  using namespace amass;
  if (!k_layers || n_layers <= 0 || n_layers > kMaxLayers || n_blocks < 0 ||
      layer0 < 0 || num_blocks <= 0 || n_kv <= 0 || !mu || !mu_scale || !V ||
      !V_scale || rank < 1 || rank > 8)
    return AMASS_ERR_ARG;
  if (n_blocks == 0) return AMASS_OK;
  if (!blocks) return AMASS_ERR_ARG;
  if (page != kPg || (head_dim != 64 && head_dim != 128) ||
      (v_bits != 8 && v_bits != 4) || (v_bits == 4 && rank % 2) ||
      (c && ((c_bits != 8 && c_bits != 4) || (c_bits == 4 && rank % 2) ||
             c_mode < 0 || c_mode > 2 || !c_scale)) ||
      (tag && (tagw <= 0 || tagw > head_dim)))
    return AMASS_ERR_UNSUPPORTED;
  if ((k_st % 2) || (k_sh % 2) || (k_sb % 2)) return AMASS_ERR_ARG;
  SumArgs a{};
  for (int l = 0; l < n_layers; ++l) {
    if (!k_layers[l] || (reinterpret_cast<uintptr_t>(k_layers[l]) & 3))
      return AMASS_ERR_ARG;
    a.k[l] = static_cast<const __nv_bfloat16*>(k_layers[l]);
  }
  a.kb = k_sb; a.kt = k_st; a.kh = k_sh;
  a.blocks = blocks; a.n_blocks = n_blocks; a.n_layers = n_layers;
  a.l0 = layer0; a.NB = num_blocks; a.n_kv = n_kv;
  a.mu = mu; a.mus = static_cast<__half*>(mu_scale);
  a.V = V; a.Vs = static_cast<__half*>(V_scale);
  a.sig2 = static_cast<__half*>(sig2);
  a.tag = static_cast<__nv_bfloat16*>(tag); a.tagw = tagw;
  a.c = c; a.cs = static_cast<__half*>(c_scale);
  a.resid = static_cast<__half*>(resid);
  a.r = rank; a.v_bits = v_bits; a.v_tensor = v_tensor ? 1 : 0;
  a.c_bits = c_bits; a.c_mode = c_mode;
  const size_t smem = sizeof(SumSmem) * kSumWarps;
  const long long items = (long long)n_layers * n_blocks * n_kv;
  const int grid = (int)std::min<long long>((items + kSumWarps - 1) / kSumWarps,
                                            (long long)num_sms() * 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static unsigned long long conf = 0;  // both variants, once per device
  if (first_on_device(conf)) {
    cudaFuncSetAttribute(summary_kernel<128>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(summary_kernel<64>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  auto kern = head_dim == 128 ? summary_kernel<128> : summary_kernel<64>;
  if (int rc = launch_pdl(kern, dim3(grid), dim3(kSumWarps * 32), smem, st, a))
    return rc;
  return launch_status();
}

// ---------------------------------------------------------------------------
// Content-tag staleness of candidate blocks (reference selection/build.py:
// 532-545): a block is stale when, in ANY layer and kv-head, its stored tag
// differs from the leading tagw channels of its page-final key (compared as
// floats: a NaN-initialised tag is always stale).  One warp per candidate.
// ---------------------------------------------------------------------------
namespace amass {
namespace {

struct TagArgs {
  const __nv_bfloat16* k[kMaxLayers];
  int64_t kb, kt, kh;
  const __nv_bfloat16* tag;   // (Ltot, NB, n_kv, tagw)
  const int32_t* in;
  int32_t* out;
  int32_t* count;
  int n, n_layers, l0, NB, n_kv, tagw, page;
};

__global__ void __launch_bounds__(256) tag_stale_kernel(TagArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (i >= a.n) return;
  const int blk = a.in[i];
  bool stale = false;
  if (blk >= 0) {
    const int per = a.n_kv * a.tagw;
    for (int e = lane; e < a.n_layers * per && !stale; e += 32) {
      const int l = e / per, rem = e - l * per;
      const int kv = rem / a.tagw, w = rem - kv * a.tagw;
      const float cur = __bfloat162float(
          a.k[l][(int64_t)blk * a.kb + (int64_t)(a.page - 1) * a.kt + kv * a.kh + w]);
      const float old = __bfloat162float(
          a.tag[(((int64_t)(a.l0 + l) * a.NB + blk) * a.n_kv + kv) * a.tagw + w]);
      stale = cur != old;
    }
  }
  stale = __any_sync(0xffffffffu, stale);
  if (lane == 0) {
    a.out[i] = stale ? blk : -1;
    if (stale) atomicAdd(a.count, 1);
  }
}

}  // namespace
}  // namespace amass

extern "C" int amass_tag_stale(const void* const* k_layers, int n_layers,
                               int64_t k_sb, int64_t k_st, int64_t k_sh,
                               const void* tag, int layer0, int num_blocks,
                               int n_kv, int tagw, int page,
                               const int32_t* blocks_in, int n_blocks,
                               int32_t* blocks_out, int32_t* count,
                               void* stream) {
  using namespace amass;
  if (!k_layers || n_layers <= 0 || n_layers > kMaxLayers || !tag ||
      layer0 < 0 || num_blocks <= 0 || n_kv <= 0 || tagw <= 0 || page <= 0 ||
      n_blocks < 0 || !count)
    return AMASS_ERR_ARG;
  if (n_blocks > 0 && (!blocks_in || !blocks_out)) return AMASS_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(count, 0, sizeof(int32_t), st) != cudaSuccess)
    return AMASS_ERR_CUDA;
  if (n_blocks == 0) return AMASS_OK;
  TagArgs a{};
  for (int l = 0; l < n_layers; ++l) {
    if (!k_layers[l]) return AMASS_ERR_ARG;
    a.k[l] = static_cast<const __nv_bfloat16*>(k_layers[l]);
  }
  a.kb = k_sb; a.kt = k_st; a.kh = k_sh;
  a.tag = static_cast<const __nv_bfloat16*>(tag);
  a.in = blocks_in; a.out = blocks_out; a.count = count;
  a.n = n_blocks; a.n_layers = n_layers; a.l0 = layer0; a.NB = num_blocks;
  a.n_kv = n_kv; a.tagw = tagw; a.page = page;
  if (int rc = launch_pdl(tag_stale_kernel, dim3((n_blocks + 7) / 8), dim3(256),
                          0, st, a))
    return rc;
  return launch_status();
}
