// Stage A.2 on sm_100a: per-step page parameters, the nrm GQA fold and the
// per-(request, kv-head) page selection (fixed top-b or nucleus coverage).
//
// Selection is a threshold rule (reference selection/select.py:60-101): tau is
// the b-th largest score of the selectable region [sink, n_sel_hi); every page
// with score >= tau is kept (ties all kept), plus the sinks, the recent window
// and the partial tail; ids are written ascending and -1 padded.  tau is found
// by an MSD radix select over order-preserving 32-bit keys held in shared
// memory (4 passes x 8-bit digits).  The coverage mode runs the same radix
// walk on per-digit MASS sums instead of counts, which lands on the smallest
// b whose top-b pages hold the required mass.
#include "common.cuh"

namespace amass {
namespace {

constexpr int kSelThreads = 512;
constexpr int kSelWarps = kSelThreads / 32;

// ---------------------------------------------------------------------------
// derive_page_params (reference selection/select.py:30-45)
// ---------------------------------------------------------------------------
__global__ void derive_kernel(const int32_t* __restrict__ sl,
                              const double* __restrict__ budget,
                              int32_t* npg_o, int32_t* nsh_o, int32_t* b_o,
                              int n_req, int page, int win, int sink) {
  const double bud = budget[0];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_req;
       i += gridDim.x * blockDim.x) {
    const int s = sl[i];
    const int npg = (s + page - 1) / page;
    const int nsh = npg - win;
    const int nsel = nsh - sink;
    const double bf = ceil((double)nsel * bud);
    int b = (int)bf;
    b = max(b, 1);
    b = min(b, max(nsel, 1));
    npg_o[i] = npg;
    nsh_o[i] = nsh;
    b_o[i] = b;
  }
}

// block-wide reductions for 512 threads
template <typename T, typename Op>
AMASS_DEV T block_reduce(T v, T* red, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int w = 1; w < kSelWarps; ++w) v = op(v, red[w]);
  return v;
}

struct SelArgs {
  const float* score_h;   // (R, n_kv, G, MP)      NRM input
  float* score;           // (R, n_kv, MP)         MAX input / NRM output
  const int32_t* npg;
  const int32_t* nsh;
  const int32_t* b_fix;
  int32_t* tab;
  int32_t* cnt;
  int32_t* b_unit;
  int n_kv, G, sink, MP;
  float coverage;
};

// nrm fold of one unit into shared sc[0, nsh); also writes score (contract of
// reference quad_score.py:293-315).  hmax_out (R, n_kv, G) optional.
AMASS_DEV void nrm_fold(const SelArgs& a, int unit, int nsh, float* sc,
                        float* red, float* hmax_out) {
  const float* sh = a.score_h + (int64_t)unit * a.G * a.MP;
  float hm[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) hm[g] = -INFINITY;
  for (int p = threadIdx.x; p < nsh; p += kSelThreads) {
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (g < a.G) hm[g] = fmaxf(hm[g], sh[(int64_t)g * a.MP + p]);
  }
  auto mx = [](float x, float y) { return fmaxf(x, y); };
#pragma unroll
  for (int g = 0; g < 8; ++g)
    if (g < a.G) hm[g] = block_reduce(hm[g], red, mx);
  if (hmax_out && threadIdx.x < a.G) {
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (g == (int)threadIdx.x) hmax_out[(int64_t)unit * a.G + g] = hm[g];
  }
  float* so = a.score + (int64_t)unit * a.MP;
  for (int p = threadIdx.x; p < nsh; p += kSelThreads) {
    float s = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (g < a.G) s += expf(sh[(int64_t)g * a.MP + p] - hm[g]);
    sc[p] = s;
    so[p] = s;
  }
}

__global__ void __launch_bounds__(kSelThreads)
nrm_combine_kernel(SelArgs a, float* hmax) {
  extern __shared__ float sc[];
  __shared__ float red[kSelWarps];
  const int unit = blockIdx.x;
  const int r = unit / a.n_kv;
  const int nsh = a.nsh[r];
  if (nsh <= 0) return;
  nrm_fold(a, unit, nsh, sc, red, hmax);
}

// Radix walk: returns the key tau of the selected threshold element.
//   COVERAGE = false: the k-th largest key (1-based) among the selectable.
//   COVERAGE = true : the key at which the descending cumulative mass first
//                     reaches `need` (the lowest key if it never does).
template <bool COVERAGE>
AMASS_DEV uint32_t radix_tau(const float* sc, int lo, int hi, int k,
                             float need, float mass_shift, bool mass_exp,
                             uint32_t* hist, float* hmass, int* bcast,
                             float* fbcast) {
  uint32_t prefix = 0, pmask = 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kSelThreads) {
      hist[i] = 0;
      if (COVERAGE) hmass[i] = 0.f;
    }
    __syncthreads();
    for (int p = lo + threadIdx.x; p < hi; p += kSelThreads) {
      const float v = sc[p];
      const uint32_t key = float_key(v);
      if ((key & pmask) == prefix) {
        const int dg = (key >> shift) & 255;
        atomicAdd(&hist[dg], 1u);
        if (COVERAGE) atomicAdd(&hmass[dg], mass_exp ? expf(v - mass_shift) : v);
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns digits [255-8l .. 248-8l] (descending)
      uint32_t c[8];
      float ms[8];
      uint32_t csum = 0;
      float msum = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = hist[255 - 8 * lane - i];
        csum += c[i];
        if (COVERAGE) {
          ms[i] = hmass[255 - 8 * lane - i];
          msum += ms[i];
        }
      }
      // exclusive scan over lanes (lane 0 = highest digits)
      uint32_t cex = csum;
      float mex = msum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t tc = __shfl_up_sync(0xffffffffu, cex, o);
        float tm = __shfl_up_sync(0xffffffffu, mex, o);
        if (lane >= o) { cex += tc; mex += tm; }
      }
      cex -= csum;
      mex -= msum;
      int found = -1;
      uint32_t above_c = cex;
      float above_m = mex;
      int last_nz = -1;
      uint32_t last_c = 0;
      float last_m = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (c[i] != 0) {
          if (found < 0) {
            bool hit;
            if (COVERAGE) hit = above_m + ms[i] >= need;
            else hit = above_c + c[i] >= (uint32_t)k;
            if (hit) found = i;
          }
          if (found < 0) { last_nz = i; last_c = above_c; last_m = above_m; }
        }
        if (found < 0) {
          above_c += c[i];
          if (COVERAGE) above_m += ms[i];
        }
      }
      const unsigned hitmask = __ballot_sync(0xffffffffu, found >= 0);
      if (hitmask) {
        const int src = __ffs(hitmask) - 1;
        if (lane == src) {
          bcast[0] = 255 - 8 * lane - found;
          bcast[1] = (int)above_c;
          fbcast[0] = above_m;
        }
      } else {
        // mass never reached `need` (rounding): descend into the lowest
        // non-empty digit so that every selectable page ends up kept
        const unsigned nzmask = __ballot_sync(0xffffffffu, last_nz >= 0);
        const int src = nzmask ? 31 - __clz(nzmask) : 0;
        if (lane == src) {
          bcast[0] = last_nz >= 0 ? 255 - 8 * lane - last_nz : 0;
          bcast[1] = (int)last_c;
          fbcast[0] = last_m;
        }
      }
    }
    __syncthreads();
    const uint32_t dg = (uint32_t)bcast[0];
    prefix |= dg << shift;
    pmask |= 0xFFu << shift;
    if (COVERAGE) need -= fbcast[0];
    else k -= bcast[1];
    __syncthreads();
  }
  return prefix;
}

// FOLD: fold score_h (nrm) into score first.  LIN: page mass = score (nrm
// semantics) instead of exp(score - max) (max semantics).
template <bool FOLD, bool LIN, bool COVERAGE>
__global__ void __launch_bounds__(kSelThreads)
select_kernel(SelArgs a) {
  extern __shared__ float sc[];
  __shared__ uint32_t hist[256];
  __shared__ float hmass[COVERAGE ? 256 : 1];
  __shared__ float red[kSelWarps];
  __shared__ int bcast[2];
  __shared__ float fbcast[1];
  __shared__ int wsum[kSelWarps];
  const int unit = blockIdx.x;
  const int r = unit / a.n_kv;
  const int npg = max(a.npg[r], 0);
  const int nsh = a.nsh[r];
  const int sink = a.sink;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  if (nsh > 0) {
    if (FOLD) {
      nrm_fold(a, unit, nsh, sc, red, nullptr);
    } else {
      const float* si = a.score + (int64_t)unit * a.MP;
      for (int p = threadIdx.x; p < nsh; p += kSelThreads) sc[p] = si[p];
    }
  }
  __syncthreads();

  const int nsel = nsh - sink;
  const bool keep_all = nsel <= 1;
  uint32_t tau = 0;
  int b_used = 1;
  if (!keep_all) {
    if (COVERAGE) {
      // page masses over the scored region [0, nsh)
      float shiftv = 0.f;
      const bool mexp = !LIN;
      if (mexp) {
        float mx = -INFINITY;
        for (int p = threadIdx.x; p < nsh; p += kSelThreads) mx = fmaxf(mx, sc[p]);
        mx = block_reduce(mx, red, [](float x, float y) { return fmaxf(x, y); });
        shiftv = mx;
      }
      float tot = 0.f, alw = 0.f;
      for (int p = threadIdx.x; p < nsh; p += kSelThreads) {
        const float m = mexp ? expf(sc[p] - shiftv) : sc[p];
        tot += m;
        if (p < sink) alw += m;
      }
      auto add = [](float x, float y) { return x + y; };
      tot = block_reduce(tot, red, add);
      alw = block_reduce(alw, red, add);
      const float need = fmaxf(a.coverage * tot - alw, 0.f);
      tau = radix_tau<true>(sc, sink, nsh, 0, need, shiftv, mexp, hist, hmass,
                            bcast, fbcast);
      // b_u = (# selectable strictly above tau) + 1
      int above = 0;
      for (int p = sink + threadIdx.x; p < nsh; p += kSelThreads)
        above += float_key(sc[p]) > tau;
      above = block_reduce(above, reinterpret_cast<int*>(red),
                           [](int x, int y) { return x + y; });
      b_used = above + 1;
    } else {
      const int b = a.b_fix[r];
      b_used = b;
      tau = radix_tau<false>(sc, sink, nsh, b, 0.f, 0.f, false, hist, hmass,
                             bcast, fbcast);
    }
  }
  if (a.b_unit && threadIdx.x == 0) a.b_unit[unit] = b_used;

  // ascending compaction of kept pages over [0, npg)
  int32_t* tab = a.tab + (int64_t)unit * a.MP;
  int base_out = 0;
  for (int base = 0; base < npg; base += kSelThreads) {
    const int p = base + threadIdx.x;
    bool keep = false;
    if (p < npg) {
      if (keep_all || p < sink || p >= nsh) keep = true;
      else keep = float_key(sc[p]) >= tau;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    int off = base_out, tot = 0;
#pragma unroll
    for (int w = 0; w < kSelWarps; ++w) {
      const int v = wsum[w];
      if (w < warp) off += v;
      tot += v;
    }
    if (keep) tab[off + __popc(bal & ((1u << lane) - 1u))] = p;
    base_out += tot;
    __syncthreads();
  }
  for (int p = base_out + threadIdx.x; p < a.MP; p += kSelThreads) tab[p] = -1;
  if (threadIdx.x == 0) a.cnt[unit] = base_out;
}

template <bool FOLD, bool LIN, bool COV>
int launch_select(const SelArgs& a, int units, cudaStream_t st) {
  const size_t smem = (size_t)a.MP * sizeof(float);
  auto k = select_kernel<FOLD, LIN, COV>;
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  }
  k<<<units, kSelThreads, smem, st>>>(a);
  return launch_status();
}

}  // namespace
}  // namespace amass

extern "C" int amass_derive_page_params(const int32_t* seq_lens,
                                        const double* budget64,
                                        int32_t* n_pages, int32_t* n_sel_hi,
                                        int32_t* b_fix, int n_req, int page,
                                        int window_pages, int sink_pages,
                                        void* stream) {
  using namespace amass;
  if (n_req < 0 || page <= 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!seq_lens || !budget64 || !n_pages || !n_sel_hi || !b_fix)
    return AMASS_ERR_ARG;
  const int threads = 256;
  const int blocks = (n_req + threads - 1) / threads;
  derive_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      seq_lens, budget64, n_pages, n_sel_hi, b_fix, n_req, page, window_pages,
      sink_pages);
  return launch_status();
}

static int max_pages_ok(int mp) {
  return mp > 0 && (size_t)mp * sizeof(float) <= 200 * 1024;
}

extern "C" int amass_nrm_combine(const float* score_h, const int32_t* n_sel_hi,
                                 float* hmax, float* score, int n_req,
                                 int n_kv, int G, int max_pages, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || G <= 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!score_h || !n_sel_hi || !score) return AMASS_ERR_ARG;
  if (G > 8 || !max_pages_ok(max_pages)) return AMASS_ERR_UNSUPPORTED;
  SelArgs a{};
  a.score_h = score_h;
  a.score = score;
  a.nsh = n_sel_hi;
  a.n_kv = n_kv;
  a.G = G;
  a.MP = max_pages;
  const size_t smem = (size_t)max_pages * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(nrm_combine_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  nrm_combine_kernel<<<n_req * n_kv, kSelThreads, smem,
                       static_cast<cudaStream_t>(stream)>>>(a, hmax);
  return launch_status();
}

extern "C" int amass_select_pages(const float* score_h, float* score,
                                  const int32_t* n_pages,
                                  const int32_t* n_sel_hi,
                                  const int32_t* b_fix, int32_t* page_table,
                                  int32_t* page_cnt, int32_t* b_unit,
                                  int n_req, int n_kv, int G, int sink_pages,
                                  int max_pages, int combine, int mode,
                                  float coverage, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || sink_pages < 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!score || !n_pages || !n_sel_hi || !page_table || !page_cnt)
    return AMASS_ERR_ARG;
  if (score_h && (G <= 0 || combine != AMASS_COMBINE_NRM)) return AMASS_ERR_ARG;
  if (mode == AMASS_SELECT_TOPB && !b_fix) return AMASS_ERR_ARG;
  if (mode == AMASS_SELECT_COVERAGE && !(coverage > 0.f && coverage <= 1.f))
    return AMASS_ERR_ARG;
  if ((score_h && G > 8) || !max_pages_ok(max_pages))
    return AMASS_ERR_UNSUPPORTED;
  SelArgs a{};
  a.score_h = score_h;
  a.score = score;
  a.npg = n_pages;
  a.nsh = n_sel_hi;
  a.b_fix = b_fix;
  a.tab = page_table;
  a.cnt = page_cnt;
  a.b_unit = b_unit;
  a.n_kv = n_kv;
  a.G = G;
  a.sink = sink_pages;
  a.MP = max_pages;
  a.coverage = coverage;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int units = n_req * n_kv;
  const bool fold = score_h != nullptr;
  const bool lin = combine == AMASS_COMBINE_NRM;
  const bool cov = mode == AMASS_SELECT_COVERAGE;
  if (!cov) {
    if (fold) return launch_select<true, true, false>(a, units, st);
    return launch_select<false, false, false>(a, units, st);
  }
  if (fold) return launch_select<true, true, true>(a, units, st);
  if (lin) return launch_select<false, true, true>(a, units, st);
  return launch_select<false, false, true>(a, units, st);
}

extern "C" int amass_topb_select(const float* score, const int32_t* n_pages,
                                 const int32_t* n_sel_hi, const int32_t* b_fix,
                                 int32_t* page_table, int32_t* page_cnt,
                                 int n_req, int n_kv, int sink_pages,
                                 int max_pages, void* stream) {
  return amass_select_pages(nullptr, const_cast<float*>(score), n_pages,
                            n_sel_hi, b_fix, page_table, page_cnt, nullptr,
                            n_req, n_kv, 0, sink_pages, max_pages,
                            AMASS_COMBINE_MAX, AMASS_SELECT_TOPB, 0.f, stream);
}
