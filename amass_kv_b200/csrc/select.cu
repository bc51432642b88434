// Stage A.2 on sm_100a: per-step page parameters, the nrm GQA fold and the
// per-(request, kv-head) page selection (fixed top-b or nucleus coverage);
// the selection algorithm itself is in select_dev.cuh.
#include "select_dev.cuh"

namespace amass {
namespace {

// ---------------------------------------------------------------------------
// derive_page_params (reference selection/select.py:30-45)
// ---------------------------------------------------------------------------
__global__ void derive_kernel(const int32_t* __restrict__ sl,
                              const double* __restrict__ budget,
                              int32_t* npg_o, int32_t* nsh_o, int32_t* b_o,
                              int n_req, int page, int win, int sink) {
  grid_dep_wait();     // inputs written by the previous kernel
  grid_dep_launch();
  const double bud = budget[0];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_req;
       i += gridDim.x * blockDim.x)
    derive_one(sl[i], bud, page, win, sink, npg_o + i, nsh_o + i, b_o + i);
}

__global__ void __launch_bounds__(kSelThreads)
nrm_combine_kernel(SelArgs a) {
  grid_dep_wait();     // inputs written by the previous kernel
  grid_dep_launch();
  extern __shared__ float sc[];
  const int unit = blockIdx.x;
  const int nsh = a.nsh[unit / a.n_kv];
  if (nsh <= 0) {
    if (threadIdx.x < a.G) a.hmax[(int64_t)unit * a.G + threadIdx.x] = -INFINITY;
    return;
  }
  nrm_fold(a, unit, 0, nsh, sc);
}

template <bool FOLD, bool LIN, bool COVERAGE, int GM = 8, bool CLU = false,
          int NT = kSelThreads>
__global__ void __launch_bounds__(NT, 1024 / NT)
select_kernel(SelArgs a) {
  grid_dep_wait();     // inputs written by the previous kernel
  grid_dep_launch();
  extern __shared__ float sc[];                 // this CTA's slice
  __shared__ SelShared sh;
  int nb = 1, rank = 0;
  if constexpr (CLU) {
    cg::cluster_group cl = cg::this_cluster();
    nb = (int)cl.num_blocks();
    rank = (int)cl.block_rank();
  }
  select_unit<FOLD, LIN, COVERAGE, GM, CLU, NT>(a, blockIdx.x / nb, nb, rank,
                                                sc, sh);
}

constexpr int kMaxSmem = 160 * 1024;

// cluster launch (one unit per cluster of `cl` CTAs) with programmatic
// dependent launch
template <typename... KArgs, typename... Args>
int launch_cluster_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                       size_t smem, cudaStream_t st, int cl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = cl;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess
             ? AMASS_OK
             : AMASS_ERR_CUDA;
}

// CTAs per unit for top-b selection: a cluster of up to 8 when the units
// are long (max_pages above 4096) and alone would leave most of the GPU idle
// (units x CTAs kept within about 4 CTAs per SM).  Measured on B200, whole
// step: C5 (128 units of up to 8191 pages) 176.2 us at 1 CTA per unit,
// 158.3 at 2, 152.9 at 4; the C3 batch split 8 ways (64 units of up to 4094
// pages) 36.7 us at 1 CTA per unit against 49.8 with 4-CTA clusters, and
// 56.0 vs 56.5 split 4 ways.  Coverage selection stays at one CTA per unit:
// its mass-weighted walk merges more levels across the cluster and was
// slower (C2, 8 units: 45.4 -> 55.2 us at 2 CTAs).
inline int select_cluster_size(int units, int max_pages) {
  if (max_pages <= 4096) return 1;
  int cl = 1;
  while (cl < 8 && (long long)units * cl * 2 <= (long long)num_sms() * 4) cl *= 2;
  return cl;
}

template <bool FOLD, bool LIN, bool COV>
int launch_select(const SelArgs& a, int units, cudaStream_t st) {
  const bool g4 = FOLD && a.G <= 4;
  const int cl = COV ? 1 : select_cluster_size(units, a.MP);
  static unsigned long long configured[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (cl > 1) {
    auto k = g4 ? select_kernel<FOLD, LIN, COV, 4, true>
                : select_kernel<FOLD, LIN, COV, 8, true>;
    const int chunk = ((a.MP + cl - 1) / cl + 3) & ~3;
    const size_t smem = (size_t)chunk * sizeof(float);
    if (first_on_device(configured[2 + (g4 ? 1 : 0)]))
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kMaxSmem);
    if (int rc = launch_cluster_pdl(k, dim3(units * cl), dim3(kSelThreads),
                                    smem, st, cl, a))
      return rc;
    return launch_status();
  }
  const size_t smem = (size_t)a.MP * sizeof(float);
  // one CTA per unit; with few units (at most one or two per SM) wider CTAs
  // shorten each unit's fold / histogram / compaction latency
  const int nt = units <= num_sms() ? 1024 : units <= 2 * num_sms() ? 512 : 256;
  using K = void (*)(SelArgs);
  K k;
  int ci;
  if (nt == 1024) {
    k = g4 ? select_kernel<FOLD, LIN, COV, 4, false, 1024>
           : select_kernel<FOLD, LIN, COV, 8, false, 1024>;
    ci = 4;
  } else if (nt == 512) {
    k = g4 ? select_kernel<FOLD, LIN, COV, 4, false, 512>
           : select_kernel<FOLD, LIN, COV, 8, false, 512>;
    ci = 6;
  } else {
    k = g4 ? select_kernel<FOLD, LIN, COV, 4> : select_kernel<FOLD, LIN, COV, 8>;
    ci = 0;
  }
  if (first_on_device(configured[ci + (g4 ? 1 : 0)])) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kMaxSmem);
  }
  if (int rc = launch_pdl(k, dim3(units), dim3(nt), smem, st, a)) return rc;
  return launch_status();
}

int max_pages_ok(int mp) {
  // compaction keeps one 64-bit keep mask per thread: MP <= 64 * kSelThreads
  return mp > 0 && mp <= 64 * kSelThreads &&
         (size_t)mp * sizeof(float) <= (size_t)kMaxSmem;
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
  if (int rc = launch_pdl(derive_kernel, dim3(blocks), dim3(threads), 0,
                          static_cast<cudaStream_t>(stream), seq_lens, budget64,
                          n_pages, n_sel_hi, b_fix, n_req, page, window_pages,
                          sink_pages))
    return rc;
  return launch_status();
}

extern "C" int amass_nrm_combine(const float* score_h, int64_t sh_stride,
                                 const int32_t* n_sel_hi, float* hmax,
                                 float* score, int n_req, int n_kv, int G,
                                 int max_pages, void* stream) {
  using namespace amass;
  if (n_req < 0 || n_kv <= 0 || G <= 0) return AMASS_ERR_ARG;
  if (n_req == 0) return AMASS_OK;
  if (!score_h || !n_sel_hi || !score || !hmax) return AMASS_ERR_ARG;
  if (G > 8 || !max_pages_ok(max_pages)) return AMASS_ERR_UNSUPPORTED;
  if (sh_stride < max_pages) return AMASS_ERR_ARG;
  SelArgs a{};
  a.score_h = score_h;
  a.SHS = sh_stride;
  a.hmax = hmax;
  a.score = score;
  a.nsh = n_sel_hi;
  a.n_kv = n_kv;
  a.G = G;
  a.MP = max_pages;
  const size_t smem = (size_t)max_pages * sizeof(float);
  static unsigned long long configured = 0;
  if (first_on_device(configured)) {
    cudaFuncSetAttribute(nrm_combine_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  }
  if (int rc = launch_pdl(nrm_combine_kernel, dim3(n_req * n_kv),
                          dim3(kSelThreads), smem,
                          static_cast<cudaStream_t>(stream), a))
    return rc;
  return launch_status();
}

extern "C" int amass_select_pages(const float* score_h, int64_t sh_stride,
                                  float* hmax, float* score, const int32_t* n_pages,
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
  if (score_h && (G <= 0 || !hmax || combine != AMASS_COMBINE_NRM ||
                  sh_stride < max_pages))
    return AMASS_ERR_ARG;
  if (mode == AMASS_SELECT_TOPB && !b_fix) return AMASS_ERR_ARG;
  if (mode == AMASS_SELECT_COVERAGE && !(coverage > 0.f && coverage <= 1.f))
    return AMASS_ERR_ARG;
  if ((score_h && G > 8) || !max_pages_ok(max_pages))
    return AMASS_ERR_UNSUPPORTED;
  SelArgs a{};
  a.score_h = score_h;
  a.SHS = sh_stride;
  a.hmax = hmax;
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
  return amass_select_pages(nullptr, 0, nullptr, const_cast<float*>(score),
                            n_pages, n_sel_hi, b_fix, page_table, page_cnt,
                            nullptr, n_req, n_kv, 0, sink_pages, max_pages,
                            AMASS_COMBINE_MAX, AMASS_SELECT_TOPB, 0.f, stream);
}
