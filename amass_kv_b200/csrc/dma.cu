// Copy-engine miss fetch of the tier: host-side run coalescing of the planned
// (block, slot) installs and their issue as strided 2-D copies.
//
// The kernel fetch moves pinned pages with SM loads; this mode moves them with
// the copy engines on a side stream, so a prefetch for the next step can
// overlap this step's compute.  A run is a maximal sequence of installs of one
// kv-head whose blocks and hot slots both advance by one and whose pages are
// all flushed (pool_valid): one cudaMemcpy2DAsync of `height` rows of one
// page, source rows n_kv pages apart (pinned layout (L, NB, n_kv, page, d)),
// destination rows one page apart (hot layout (n_kv, S, page, d)).  Staged
// (unflushed) installs are left to the staged-only kernel fetch.
#include "common.cuh"

extern "C" int amass_tier_dma_plan(const int32_t* fetch_list,
                                   const int32_t* fetch_cnt,
                                   const int8_t* pool_valid, int layer,
                                   int num_blocks, int n_kv, int hot_slots,
                                   int page, int head_dim, uint64_t pool_base,
                                   uint64_t hot_base, uint64_t pool_k_base,
                                   uint64_t hot_k_base, AmassDmaRun* runs,
                                   int max_runs, int* n_runs,
                                   int* has_staged) {
  if (!fetch_list || !fetch_cnt || !pool_valid || !runs || !n_runs ||
      !has_staged || layer < 0 || num_blocks <= 0 || n_kv <= 0 ||
      hot_slots <= 0 || page <= 0 || head_dim <= 0 || max_runs < 0 ||
      !pool_base || !hot_base || ((pool_k_base != 0) != (hot_k_base != 0)))
    return AMASS_ERR_ARG;
  const int64_t pbytes = (int64_t)page * head_dim * 2;
  const int64_t layer_off = (int64_t)layer * num_blocks * n_kv * pbytes;
  int n = 0, staged = 0;
  for (int kv = 0; kv < n_kv; ++kv) {
    const int m = fetch_cnt[kv];
    if (m < 0 || m > hot_slots) return AMASS_ERR_ARG;
    const int32_t* fl = fetch_list + (int64_t)kv * hot_slots * 2;
    const int8_t* vld = pool_valid + (int64_t)kv * num_blocks;
    int i = 0;
    while (i < m) {
      const int blk = fl[2 * i], slot = fl[2 * i + 1];
      if (blk < 0 || blk >= num_blocks || slot < 0 || slot >= hot_slots)
        return AMASS_ERR_ARG;
      if (vld[blk] == 0) {
        staged = 1;
        ++i;
        continue;
      }
      int run = 1;
      while (i + run < m && fl[2 * (i + run)] == blk + run &&
             fl[2 * (i + run) + 1] == slot + run && blk + run < num_blocks &&
             slot + run < hot_slots && vld[blk + run] != 0)
        ++run;
      if (n >= max_runs) return AMASS_ERR_CAPACITY;
      AmassDmaRun& r = runs[n++];
      const int64_t src = layer_off + ((int64_t)blk * n_kv + kv) * pbytes;
      const int64_t dst = ((int64_t)kv * hot_slots + slot) * pbytes;
      r.dst = hot_base + dst;
      r.src = pool_base + src;
      r.dst_k = hot_k_base ? hot_k_base + dst : 0;
      r.src_k = pool_k_base ? pool_k_base + src : 0;
      r.dpitch = pbytes;
      r.spitch = (int64_t)n_kv * pbytes;
      r.width = pbytes;
      r.height = run;
      i += run;
    }
  }
  *n_runs = n;
  *has_staged = staged;
  return AMASS_OK;
}

extern "C" int amass_dma_issue(const AmassDmaRun* runs, int n_runs,
                               void* stream) {
  if (n_runs < 0 || (n_runs > 0 && !runs)) return AMASS_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n_runs; ++i) {
    const AmassDmaRun& r = runs[i];
    if (r.width <= 0 || r.height <= 0 || !r.dst || !r.src) return AMASS_ERR_ARG;
    for (int k = 0; k < (r.dst_k ? 2 : 1); ++k) {
      void* dst = reinterpret_cast<void*>(k ? r.dst_k : r.dst);
      const void* src = reinterpret_cast<const void*>(k ? r.src_k : r.src);
      cudaError_t e =
          r.height == 1
              ? cudaMemcpyAsync(dst, src, (size_t)r.width, cudaMemcpyDefault, st)
              : cudaMemcpy2DAsync(dst, (size_t)r.dpitch, src, (size_t)r.spitch,
                                  (size_t)r.width, (size_t)r.height,
                                  cudaMemcpyDefault, st);
      if (e != cudaSuccess) {
        cudaGetLastError();
        return AMASS_ERR_CUDA;
      }
    }
  }
  return AMASS_OK;
}
