/*
 * amass_b200.h -- C ABI of libamass_b200.so, the sm_100a implementation of
 * the AMASS decode-time sparse paged-attention hot path.
 *
 * Every entry point takes raw device pointers (or UVA device pointers of
 * pinned host memory), element strides, sizes and a cudaStream_t passed as
 * void*.  No entry point allocates, frees or synchronises; all launches are
 * fixed-shape for given sizes, so they can be captured in a CUDA graph.
 * Return value: AMASS_OK or one of the error codes below.  Dtypes:
 * bf16/fp16 tensors are passed as void*, fp32 as float*, indices as int32_t*.
 *
 * Citations name the reference interface each entry point replaces, as
 * path:line inside the reference project (Js-Hwang1/amass-kv, src/amass/).
 */
#ifndef AMASS_B200_H
#define AMASS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  AMASS_OK = 0,
  AMASS_ERR_ARG = 1,          /* null pointer / negative size / bad stride   */
  AMASS_ERR_UNSUPPORTED = 2,  /* geometry outside the compiled variants       */
  AMASS_ERR_CAPACITY = 3,     /* a caller buffer is too small for the request */
  AMASS_ERR_CUDA = 4          /* a CUDA launch error (cudaGetLastError)       */
};

/* combine modes for the GQA group (AmassConfig.quad_combine) */
enum { AMASS_COMBINE_MAX = 0, AMASS_COMBINE_NRM = 1 };
/* selection modes */
enum { AMASS_SELECT_TOPB = 0, AMASS_SELECT_COVERAGE = 1 };
/* r8 token aggregation */
enum { AMASS_R8_LSE = 0, AMASS_R8_TOKMAX = 1 };

const char* amass_status_string(int status);
int amass_version(void);

/* One-time per-device setup (kernel attributes).  Call once per device
 * before stream capture; every other entry point calls it lazily too. */
int amass_init(void);

/* derive_page_params -- replaces selection/select.py:48-56 (kernel :30-45).
 * n_pages = ceil(seq_len/page); n_sel_hi = n_pages - window;
 * b_fix = clamp(ceil(fp64(n_sel_hi - sink) * budget64[0]), 1, max(n_sel,1)). */
int amass_derive_page_params(const int32_t* seq_lens, const double* budget64,
                             int32_t* n_pages, int32_t* n_sel_hi,
                             int32_t* b_fix, int n_req, int page,
                             int window_pages, int sink_pages, void* stream);

/* quad_score -- replaces selection/quad_score_cuda.py:1724-1794 (Triton
 * golden selection/quad_score.py:35-139).  Reads one layer's quad slabs:
 *   mu (NB, n_kv, d) int8, mu_scale (NB, n_kv) fp16,
 *   V (NB, n_kv, d, rv) int8 (rv = rank, or rank/2 packed int4),
 *   V_scale (NB, n_kv, rank) fp16, sig2 (NB, n_kv, rank) fp16 (contiguous,
 *   mu and V 16-byte aligned).
 * write_h = 0: score[r, kv, p] = max_g S_g (R, n_kv, MP) fp32.
 * write_h = 1: score_h[r, kv, g, p] = S_g (R, n_kv, G, sh_stride) fp32, rows
 *              of sh_stride >= MP elements (a multiple of 4 enables 16-byte
 *              loads in the fold) (the nrm
 *              path) and hmax[r, kv, g] = max(hmax, max_p S_g) (R, n_kv, G)
 *              fp32; hmax must hold -inf before the call -- the fold
 *              (amass_nrm_combine / amass_select_pages) consumes it and
 *              resets it to -inf.
 * q8_ws (n_req, H, 2, d) int8 (16-byte aligned) and qs_ws (n_req, H) fp32
 * are caller scratch for the exact two-limb int8 form of q the integer MMAs
 * use (|dq| <= max|q_head| / 32512); from 32 requests up the scorer splits
 * q itself (same limbs) and leaves the scratch untouched.
 * Pages p < n_sel_hi[r] are written; others are left untouched.
 * Compiled variants: head_dim in {64, 128}, rank in {1, 2, 4, 8},
 * v_bits in {4, 8} (int4 needs an even rank), G <= 8, page = 16,
 * n_req <= 4096. */
int amass_quad_score(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                     const int8_t* mu, const void* mu_scale, const int8_t* V,
                     const void* V_scale, const void* sig2,
                     const int32_t* block_table, int64_t bt_stride,
                     const int32_t* n_sel_hi, float* score, float* score_h,
                     int64_t sh_stride, float* hmax, int8_t* q8_ws,
                     float* qs_ws, float scale,
                     int n_req, int n_kv, int G, int head_dim, int page,
                     int rank, int v_bits, int max_pages, int write_h,
                     void* stream);

/* quad_score_derive -- derive_page_params (selection/select.py:30-54) and
 * quad_score_cuda (selection/quad_score_cuda.py:1724-1794), the first two
 * calls of the reference's _quad_select_adapter (backend/_runtime.py:
 * 183-263), in the launches of amass_quad_score alone: n_pages / n_sel_hi /
 * b_fix are written from seq_lens and budget64 (as amass_derive_page_params)
 * by the q-limb launch, or from 32 requests up by the scorer's own prologue
 * (one launch).  Other arguments as amass_quad_score. */
int amass_quad_score_derive(
    const int32_t* seq_lens, const double* budget64, int32_t* n_pages,
    int32_t* n_sel_hi, int32_t* b_fix, int window_pages, int sink_pages,
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const int8_t* mu,
    const void* mu_scale, const int8_t* V, const void* V_scale,
    const void* sig2, const int32_t* block_table, int64_t bt_stride,
    float* score, float* score_h, int64_t sh_stride, float* hmax,
    int8_t* q8_ws, float* qs_ws, float scale, int n_req, int n_kv, int G,
    int head_dim, int page, int rank, int v_bits, int max_pages, int write_h,
    void* stream);

/* quad_pipeline -- no counterpart in the reference (a choice between two
 * kernels of this library for amass_quad_score / amass_quad_score_derive).
 * The pipelined scorer (a producer warp streams each 16-page tile's summary
 * rows into a shared-memory ring with bulk copies; eight consumer warps
 * score them) serves calls with 8 kv heads, a V-code slice of at most 32
 * bytes per lane (int4 rank 2 or int8 rank 1 at head_dim 128), 16-byte
 * aligned scale slabs (any batch up to the scorer's 4096 requests: the
 * request table fits beside the ring).
 * mode 1 (default): those calls from 32 requests up; mode 2: all of them;
 * mode 0: none -- the register-pipelined scorer serves every call.  Both
 * give bit-identical scores.  Other values only query.  Returns the
 * previous mode.  Process-wide; not synchronised with calls in flight. */
int amass_quad_pipeline(int mode);

/* quad_pack -- no counterpart in the reference (a choice between two forms
 * of the quad scorers).  on = 1 (default): when a kv head has at most 4
 * query heads and a lane's V-code slice fits its registers (at head_dim
 * 128: int4 V up to rank 4, int8 V up to rank 2), the two int8 limbs of q
 * share one integer MMA's 8 columns
 * (hi limbs in columns 0-3, lo limbs in 4-7), half the MMAs and half the
 * per-lane epilogue of the two-limb form; on = 0: the two-limb form.  Both
 * give bit-identical scores.  Other values only query.  Returns the
 * previous setting.  Process-wide; not synchronised with calls in flight. */
int amass_quad_pack(int on);

/* quad_pipeline_status -- no counterpart in the reference.  fault (may be
 * null) receives the pipelined scorer's device fault word: 0, or 1 / 2 when a
 * consumer / the producer warp gave up a bounded barrier wait (its scores
 * are then incomplete); launches (may be null) the number of pipelined
 * launches this process issued.  clear = 1 resets both.  Synchronous copy
 * from the current device. */
int amass_quad_pipeline_status(int* fault, long long* launches, int clear);

/* nrm combine -- replaces the two passes of selection/quad_score.py:276-315
 * (CUDA twin quad_score_cuda.py:1446-1547): with hmax[r,kv,g] = the per-head
 * page max that amass_quad_score accumulated, score[r,kv,p] =
 * sum_g exp(score_h[r,kv,g,p] - hmax[r,kv,g]) for p < n_sel_hi; hmax is then
 * reset to -inf for the next call. */
int amass_nrm_combine(const float* score_h, int64_t sh_stride,
                      const int32_t* n_sel_hi, float* hmax, float* score,
                      int n_req, int n_kv, int G, int max_pages, void* stream);

/* topb_select -- replaces selection/select_cuda.py:370-391 (Triton golden
 * selection/select.py:60-116): tau = b_fix[r]-th largest score over the
 * selectable region [sink, n_sel_hi); keep score >= tau, sinks, window and
 * tail; ascending page ids, -1 padded to max_pages; page_cnt per unit. */
int amass_topb_select(const float* score, const int32_t* n_pages,
                      const int32_t* n_sel_hi, const int32_t* b_fix,
                      int32_t* page_table, int32_t* page_cnt, int n_req,
                      int n_kv, int sink_pages, int max_pages, void* stream);

/* select_pages -- fused Stage-A.2: (optional nrm fold of score_h into score)
 * then per-(request, kv-head) selection.  mode TOPB uses b_fix (as
 * amass_topb_select); mode COVERAGE computes each unit's nucleus budget b_u
 * (smallest b whose top-b selectable pages hold `coverage` of the scored page
 * mass minus the sink share; the per-unit form of the reference's
 * backend/_selection_bridge.py:117-133) and applies the same threshold rule.
 * With score_h (and hmax) given, the nrm fold runs first (as
 * amass_nrm_combine) and writes score.  combine MAX: page mass =
 * exp(score - max); NRM: page mass = score.  b_unit (R, n_kv) receives the b used per unit
 * (may be NULL).  Has no single reference counterpart: it replaces the pair
 * nrm_combine + topb_select_cuda on the graph-safe path
 * (backend/_runtime.py:183-263) and adds the per-head coverage the
 * reference only has in its eager bridge. */
int amass_select_pages(const float* score_h, int64_t sh_stride, float* hmax,
                       float* score,
                       const int32_t* n_pages, const int32_t* n_sel_hi,
                       const int32_t* b_fix, int32_t* page_table,
                       int32_t* page_cnt, int32_t* b_unit, int n_req, int n_kv,
                       int G, int sink_pages, int max_pages, int combine,
                       int mode, float coverage, void* stream);

/* r8_score -- replaces selection/score_cuda.py:888-913 (Triton golden
 * selection/score.py:30-148).  One layer's R8State slabs: mu (NB,n_kv,d) int8
 * + mu_scale (NB,n_kv) fp16, Vk (NB,n_kv,d,rv) int8 (rv = 8, or 4 packed
 * int4) + Vk_scale (NB,n_kv,8) fp16, c (NB,n_kv,page,rc) int8 (rc = 8 or 4)
 * + c_scale (NB,n_kv,page) fp16.  score[r,kv,p] = max_g (s*mu.q_g +
 * agg_t(s*c_t.(Vk^T q_g))), agg = log-sum-exp over tokens < seq_len
 * (token_agg AMASS_R8_LSE, the reference form) or max (AMASS_R8_TOKMAX).
 * q8_ws/qs_ws: scratch as for amass_quad_score.  rank 8, page 16, G <= 8,
 * head_dim in {64, 128}. */
int amass_r8_score(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                   const int8_t* mu, const void* mu_scale, const int8_t* Vk,
                   const void* Vk_scale, const int8_t* c, const void* c_scale,
                   const int32_t* block_table, int64_t bt_stride,
                   const int32_t* seq_lens, const int32_t* n_sel_hi,
                   float* score, int8_t* q8_ws, float* qs_ws, float scale,
                   int n_req, int n_kv, int G, int head_dim, int page,
                   int rank, int vk_bits, int c_bits, int max_pages,
                   int token_agg, void* stream);

/* clse_score -- replaces selection/quad_score_cuda.py:1797 (Triton golden
 * selection/quad_score.py:156-374).  The quad geometry plus rank-r' per-key
 * coordinates c (NB, n_kv, page, rc) int8 (rc = rank, or rank/2 packed int4)
 * with fp16 scales per token (c_token_grain = 1: (NB, n_kv, page)) or per
 * page (0: (NB, n_kv)), and resid (NB, n_kv) fp16 = trace - sum sig2:
 *   S_g = s*mu.q_g + logsumexp_{t < seq_len} (s * c_t . V^T q_g)
 *         + max(|q_g|^2 - |V^T q_g|^2, 0) * resid * s^2 / (2P(d - rank)).
 * write_h = 0: score = max_g S_g; write_h = 1: score_h / hmax as in
 * amass_quad_score (the nrm fold follows).  qsq_ws (n_req, H) fp32 scratch
 * receives |q_g|^2.  rank in {2, 4, 8}, v_bits / c_bits in {4, 8},
 * head_dim in {64, 128}, G <= 8, page = 16, n_req <= 2048. */
int amass_clse_score(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                     const int8_t* mu, const void* mu_scale, const int8_t* V,
                     const void* V_scale, const int8_t* c, const void* c_scale,
                     int c_token_grain, const void* resid,
                     const int32_t* block_table, int64_t bt_stride,
                     const int32_t* seq_lens, const int32_t* n_sel_hi,
                     float* score, float* score_h, int64_t sh_stride,
                     float* hmax, int8_t* q8_ws, float* qs_ws, float* qsq_ws,
                     float scale, int n_req, int n_kv, int G, int head_dim,
                     int page, int rank, int v_bits, int c_bits, int max_pages,
                     int write_h, void* stream);

/* Page summary build -- replaces the page-finalize summarizers
 * selection/build.py:396-452 (_page_eigh, _r8_write) and
 * selection/quad_build.py:37-84 (_quad_write): for every layer l of
 * k_layers[0..n_layers) (each a key cache addressed as
 * base + block*k_sb + token*k_st + head*k_sh, bf16) and every block in
 * blocks[0..n_blocks), per kv-head: page mean, the top `rank` eigenpairs of
 * the 16 x 16 Gram of the centred keys (ascending order, eigenvalues clamped
 * >= 1e-10), Vk = dc^T U / sqrt(lambda), quantised and written at slab layer
 * layer0 + l:  mu (NB, n_kv, d) int8 + mu_scale fp16; V (NB, n_kv, d, rv)
 * int8 or packed int4 + V_scale (NB, n_kv, rank) per column (v_tensor = 0)
 * or one scale (1); sig2 (NB, n_kv, rank) fp16 or NULL; tag (NB, n_kv,
 * tagw) bf16 or NULL.  With c != NULL also the coordinates c = U sqrt(lambda)
 * (NB, n_kv, 16, rc) and c_scale: c_mode 0 = per token (.., 16), 1 = one
 * scale per page repeated over (.., 16), 2 = one per page (..); resid
 * (NB, n_kv) fp16 = sum K^2 - 16 |mu|^2 - sum lambda, or NULL.  Slabs are the
 * whole layer-major arrays (first layer at index 0).  Eigenvectors are
 * unique up to sign.  head_dim in {64, 128}, page = 16, rank <= 8,
 * n_layers <= 128.  Negative entries of `blocks` are skipped. */
int amass_summarize_pages(const void* const* k_layers, int n_layers,
                          int64_t k_sb, int64_t k_st, int64_t k_sh,
                          const int32_t* blocks, int n_blocks, int layer0,
                          int num_blocks, int n_kv, int head_dim, int page,
                          int rank, int8_t* mu, void* mu_scale, int8_t* V,
                          void* V_scale, int v_bits, int v_tensor, void* sig2,
                          void* tag, int tagw, int8_t* c, void* c_scale,
                          int c_bits, int c_mode, void* resid, void* stream);

/* Content-tag staleness for the delta rebuild -- replaces the tag pass of
 * quad_build_delta / r8_build_delta (selection/build.py:532-545,
 * quad_build.py:110-121): blocks_out[i] = blocks_in[i] when, in any of the
 * n_layers layers (slab layer layer0 + l) and any kv-head, the stored tag
 * (Ltot, NB, n_kv, tagw) bf16 differs (as floats; NaN always differs) from
 * the first tagw channels of the block's last-token key, else -1 (also for
 * negative inputs); *count = number of stale entries.  Feed blocks_out to
 * amass_summarize_pages, which skips the -1 entries. */
int amass_tag_stale(const void* const* k_layers, int n_layers, int64_t k_sb,
                    int64_t k_st, int64_t k_sh, const void* tag, int layer0,
                    int num_blocks, int n_kv, int tagw, int page,
                    const int32_t* blocks_in, int n_blocks, int32_t* blocks_out,
                    int32_t* count, void* stream);

/* sparse_paged_decode -- replaces attention/decode_cuda.py:1376-1465
 * (Triton golden attention/decode.py:247-304 + merge.py:21-50).
 * K/V tiles are addressed as base + blk*s_b + tok*s_t + kv*s_h (elements,
 * bf16), which covers vLLM's (nb, 2, page, n_kv, d) and (2, nb, ...) caches.
 * The selected pages of all units form one flat list cut into equal runs
 * (at least pps_min pages, one per warp of the persistent grid, and long
 * enough that no unit needs more than `split` of them); each run writes one
 * partial per unit it touches to m_part/l_part (R, n_kv, split, G) and
 * acc_part (R, n_kv, split, G, d) fp32; a merge writes out (T, H, d) bf16
 * rows [0, n_req) in place (0 for empty units).  split >= 2, head_dim in
 * {64, 128}, G <= 8, page = 16. */
int amass_sparse_decode(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                        const void* k, int64_t k_sb, int64_t k_st,
                        int64_t k_sh, const void* v, int64_t v_sb,
                        int64_t v_st, int64_t v_sh,
                        const int32_t* block_table, int64_t bt_stride,
                        const int32_t* page_table, const int32_t* page_cnt,
                        const int32_t* seq_lens, float* m_part, float* l_part,
                        float* acc_part, int split, int pps_min, void* out,
                        int64_t o_stride_t, int64_t o_stride_h, float scale,
                        int n_req, int n_kv, int G, int head_dim, int page,
                        int max_pages, void* stream);

/* sparse_paged_decode_noalloc -- no counterpart in the reference.  For
 * callers that cannot allocate device memory (a plugin running inside another
 * runtime's memory pool, a serving loop that must not touch the allocator, a
 * binding with no tensor library): the same decode as amass_sparse_decode,
 * but the split-K partials live in a fixed file-scope device array of
 * amass_sparse_decode_noalloc_capacity() floats (16 MiB) that every GPU
 * loading this library holds until exit.  Requires
 * n_req*n_kv*split*G*(head_dim+2) <= capacity, else AMASS_ERR_CAPACITY (use a
 * smaller split).  Allocates and frees nothing.  The first call on a device
 * resolves the array's device address (cudaGetSymbolAddress), so make that
 * first call before any stream capture.  All calls share the one array:
 * calls that overlap on the GPU (other streams, other threads) race and must
 * be serialised by the caller.  No part of the array needs to start zeroed. */
size_t amass_sparse_decode_noalloc_capacity(void);
int amass_sparse_decode_noalloc(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v, int64_t v_sb,
    int64_t v_st, int64_t v_sh, const int32_t* block_table, int64_t bt_stride,
    const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, int split, int pps_min, void* out,
    int64_t o_stride_t, int64_t o_stride_h, float scale, int n_req, int n_kv,
    int G, int head_dim, int page, int max_pages, void* stream);

/* KV-head-sharded decode with the all-gather fused into the merge.  As
 * amass_sparse_decode over this rank's kv heads (q, k, v, page_table,
 * page_cnt and the partials hold n_kv local heads), but every merged output
 * row is stored into each of the n_peers buffers out_peers[0..n_peers)
 * (this GPU's and the peers' output tensors, mapped into this GPU's address
 * space, all (T, H, d) with strides o_stride_t / o_stride_h) at global head
 * head_offset + local head.  n_peers <= 8.  The stores are plain peer
 * stores over NVLink; the caller orders them before any reader with a
 * cross-GPU barrier after the call.  Replaces the reference's decode
 * (attention/decode_cuda.py:1376-1465) followed by the all-gather of a
 * head-sharded attention output. */
int amass_sparse_decode_gather(
    const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
    int64_t k_sb, int64_t k_st, int64_t k_sh, const void* v, int64_t v_sb,
    int64_t v_st, int64_t v_sh, const int32_t* block_table, int64_t bt_stride,
    const int32_t* page_table, const int32_t* page_cnt,
    const int32_t* seq_lens, float* m_part, float* l_part, float* acc_part,
    int split, int pps_min, void* const* out_peers, int n_peers,
    int head_offset, int64_t o_stride_t, int64_t o_stride_h, float scale,
    int n_req, int n_kv, int G, int head_dim, int page, int max_pages,
    void* stream);

/* Cross-GPU barrier for amass_sparse_decode_gather: peer_flags[i] is rank
 * i's int32[n_ranks] flag array mapped into this GPU (zeroed once before the
 * first call); epoch is this rank's int32 call counter (device, zeroed
 * once).  Makes the stream's earlier peer stores visible, signals every
 * rank, and waits (bounded, about a second) until every rank has signalled
 * this call; on timeout err[0] becomes 1 + the missing rank and the kernel
 * returns.  One launch; CUDA-graph capturable.  n_ranks <= 8. */
int amass_peer_barrier(int32_t* const* peer_flags, int n_ranks, int rank,
                       int32_t* epoch, int32_t* err, void* stream);

/* ------------------------------------------------------------------------
 * mem-v / mem-kv DRAM tier (reference tier/pool.py, tier/residency.py,
 * tier/decode_mem.py).  Per layer the tier keeps a VRAM hot buffer of S page
 * slots per kv-head; V (and K under mem-kv) of every page lives in a pinned,
 * device-mapped host pool (L, NB, n_kv, page, d) bf16, and pages not yet
 * flushed there sit in a VRAM staging pool addressed through vbo.
 * ------------------------------------------------------------------------ */

/* Device address of pinned, mapped host memory -- replaces
 * tier/pool.py:65-80 (host_device_pointer). */
int amass_host_device_pointer(void* host, void** dev);

/* Largest number of misses per kv-head one amass_tier_plan call lists
 * (beyond it the misses stay non-resident and overflow is set); 0 when
 * hot_slots is outside (0, 8192]. */
int amass_tier_plan_capacity(int hot_slots);

/* Residency plan of one layer -- replaces Residency.gather_plan
 * tier/residency.py:385-407 (kernels :45-139).  Exact LRU:
 *   clock[0] advances by one (clock is int32[2]; clock[1] is a CTA ticket
 *   that must be 0 before the first call and is left 0);
 *   hits (selected, complete, page2slot >= 0) set lru = clock;
 *   misses, per kv-head in (request, page-table) order and deduplicated,
 *   take the slot of smallest (lru, index) among slots with lru < clock,
 *   evict its page and are written to fetch_list (n_kv, hot_slots, 2) as
 *   (block, slot) with fetch_cnt[kv] entries (fetch_cnt is int32[n_kv]).
 * A miss without an eligible slot (or beyond amass_tier_plan_capacity)
 * stays non-resident and sets overflow[0] = 1.
 * page2slot (n_kv, NB), slot2page / lru_clock (n_kv, hot_slots) are this
 * layer's rows.  miss_pages (n_req, n_kv, max_pages) int32 receives the
 * classified entries: the block of a miss (>= 0), -(slot + 2) for a hit, -1
 * for a page that is not complete.  Two launches: the
 * classification over the whole GPU, then one CTA per kv-head.
 * hot_slots <= 8192, n_req <= 4096. */
int amass_tier_plan(const int32_t* page_table, const int32_t* page_cnt,
                    const int32_t* block_table, int64_t bt_stride,
                    const int32_t* seq_lens, int32_t* page2slot,
                    int32_t* slot2page, int32_t* lru_clock, int32_t* clock,
                    int32_t* overflow, int32_t* fetch_list, int32_t* fetch_cnt,
                    int32_t* miss_pages, int n_req, int n_kv, int max_pages,
                    int page, int num_blocks, int hot_slots, void* stream);

/* Miss fetch -- replaces Residency.gather_fetch tier/residency.py:409-436
 * (kernel :196-248).  For each planned (block, slot): hot[kv, slot] <- pinned
 * pool page when pool_valid[kv, block]; else, when vbo[block] >= 0, the
 * staging page v_pool + vbo*svb + kv*svh (token stride svt), written through
 * to the pinned pool with pool_valid = 1; else the pinned pool page.  Bit
 * copies of 16-bit elements.  hot (n_kv, S, page, d) of this layer; pool_dev
 * is the device view of the whole (L, NB, n_kv, page, d) pool; pool_valid
 * (n_kv, NB) of this layer.  hot_k / pool_k_dev / k_pool: the K tier under
 * mem-kv (all three null under mem-v).  page = 16, head_dim in {64, 128}. */
int amass_tier_fetch(const int32_t* fetch_list, const int32_t* fetch_cnt,
                     void* hot, void* pool_dev, int8_t* pool_valid,
                     const int32_t* vbo, const void* v_pool, int64_t svb,
                     int64_t svt, int64_t svh, void* hot_k, void* pool_k_dev,
                     const void* k_pool, int layer, int num_blocks, int n_kv,
                     int hot_slots, int page, int head_dim, void* stream);

/* As amass_tier_fetch, but only the installs whose page is not flushed
 * (pool_valid 0: staged, or neither staged nor flushed), exactly the ones
 * amass_tier_dma_plan leaves out: the device half of the copy-engine fetch --
 * Residency._gather_staged_only tier/residency.py:527-548. */
int amass_tier_fetch_staged(
    const int32_t* fetch_list, const int32_t* fetch_cnt, void* hot,
    void* pool_dev, int8_t* pool_valid, const int32_t* vbo, const void* v_pool,
    int64_t svb, int64_t svt, int64_t svh, void* hot_k, void* pool_k_dev,
    const void* k_pool, int layer, int num_blocks, int n_kv, int hot_slots,
    int page, int head_dim, void* stream);

/* One copy-engine copy: `height` rows of `width` bytes, rows dpitch / spitch
 * bytes apart (height 1: a plain copy); dst_k / src_k the same rows of the K
 * tier under mem-kv (0 otherwise).  Addresses are device / UVA pointers. */
typedef struct AmassDmaRun {
  uint64_t dst, src, dst_k, src_k;
  int64_t dpitch, spitch, width, height;
} AmassDmaRun;

/* HOST function (reads host copies of fetch_list (n_kv, S, 2), fetch_cnt
 * (n_kv,) and this layer's pool_valid (n_kv, NB)) -- replaces
 * Residency.build_dma_plan tier/residency.py:438-492.  Coalesces each
 * kv-head's flushed installs into runs whose blocks and slots both advance
 * by one; staged installs are skipped and reported in *has_staged.
 * pool_base / hot_base: the pinned pool (L, NB, n_kv, page, d) and this
 * layer's hot buffer (n_kv, S, page, d); the _k bases under mem-kv, else 0.
 * AMASS_ERR_CAPACITY when more than max_runs runs are needed. */
int amass_tier_dma_plan(const int32_t* fetch_list, const int32_t* fetch_cnt,
                        const int8_t* pool_valid, int layer, int num_blocks,
                        int n_kv, int hot_slots, int page, int head_dim,
                        uint64_t pool_base, uint64_t hot_base,
                        uint64_t pool_k_base, uint64_t hot_k_base,
                        AmassDmaRun* runs, int max_runs, int* n_runs,
                        int* has_staged);

/* Issue a plan's runs on `stream` with the copy engines (cudaMemcpyAsync /
 * cudaMemcpy2DAsync, one call per run and tier) -- replaces
 * Residency.issue_dma_plan tier/residency.py:494-509 and CopyEngine
 * tier/dma.py:77-140. */
int amass_dma_issue(const AmassDmaRun* runs, int n_runs, void* stream);

/* Drop residency and pool validity of the pages (re)written this step in all
 * layers -- replaces Residency.invalidate_written tier/residency.py:352-367
 * (kernel :251-282).  query_start_loc (n_req+1,); page2slot (L, n_kv, NB),
 * slot2page (L, n_kv, S), pool_valid (L, n_kv, NB). */
int amass_tier_invalidate(const int32_t* block_table, int64_t bt_stride,
                          const int32_t* seq_lens,
                          const int32_t* query_start_loc, int32_t* page2slot,
                          int32_t* slot2page, int8_t* pool_valid, int n_req,
                          int num_layers, int n_kv, int num_blocks,
                          int hot_slots, int page, void* stream);

/* Staging lifecycle of one step (write side of the tier) -- replaces
 * Staging.begin_step tier/staging.py:312-346 (kernels :51-232).  In order:
 * v_slot_mapping[:n_tokens] = -1; clear the flushed latch of the pages
 * written this step; collect the complete pages written by earlier steps
 * that hold a staging block (requests in order): the first claim of the
 * latch enters flush_list (blk, vb) (at most max_flush entries, flush_cnt),
 * and the staging block is freed onto free_stack (free_top); copy every
 * flushed page v_pool[l, vb] -> the pinned pool [l, blk] for all layers and
 * kv-heads (and k_pool -> pool_k under mem-kv) and set pool_valid; allocate
 * a staging block (pop) for every page written this step without one
 * (underflow sets overflow[0]); fill v_slot_mapping (int64) for this step's
 * tokens (vb * page + pos % page, or -1).  v_pool (L, NV, page, n_kv, d) at
 * element strides svl/svb/svt/svh; pool_valid (L, n_kv, NB).  Requests with
 * seq_len <= 0 or no new tokens are skipped.  cand (1 + cand_cap int32,
 * cand_cap <= 4096) is scratch for a whole-GPU pre-pass that lists the
 * staged complete pages, so the ordered part only visits those; cand_cap 0,
 * or more staged complete pages than cand_cap, walks every complete page in
 * one CTA instead (same result). */
int amass_staging_begin_step(
    const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
    const int32_t* query_start_loc, int n_req, int n_tokens, int max_query_len,
    int64_t* v_slot_mapping, int32_t* vbo, int32_t* v_flushed,
    int32_t* free_stack, int32_t* free_top, int32_t* flush_list,
    int32_t* flush_cnt, int32_t* overflow, int max_flush, const void* v_pool,
    const void* k_pool, int64_t svl, int64_t svb, int64_t svt, int64_t svh,
    void* pool_dev, void* pool_k_dev, int8_t* pool_valid, int num_layers,
    int num_blocks, int n_kv, int head_dim, int page, int32_t* cand,
    int cand_cap, void* stream);

/* Write path: scatter this step's V (and K under mem-kv) (n_tokens, n_kv, d)
 * 16-bit into one layer's staging pool(s) (NV, page, n_kv, d) at
 * v_slot_mapping (-1 skips) -- replaces Staging.scatter_kv
 * tier/staging.py:348-367 (kernel :51-77).  Bit copies. */
int amass_staging_scatter(const void* value, int64_t v_st, int64_t v_sh,
                          const void* key, int64_t k_st, int64_t k_sh,
                          const int64_t* v_slot_mapping, void* v_pool_layer,
                          void* k_pool_layer, int64_t pb, int64_t pt,
                          int64_t ph, int n_tokens, int n_kv, int head_dim,
                          int page, void* stream);

/* Tiered split-K decode (ptr-select) -- replaces mem_decode_ptrsel
 * tier/decode_mem.py:169-222 (kernel :78-166).  As amass_sparse_decode,
 * but per selected page the V tile (and the K tile when hot_k != NULL,
 * mem-kv) is read from hot (complete page with page2slot >= 0), else the
 * staging pool (vbo >= 0; stg_* at svb/svt/svh), else the pinned pool
 * (pool_* device views).  Under mem-v (hot_k == NULL) K comes from the
 * resident cache k at k_sb/k_st/k_sh.  entry_slots: NULL, or the
 * miss_pages of the amass_tier_plan call made for this same page_table on
 * this layer (entries that were hits carry their hot slot there, which
 * saves the page2slot lookup); with any other array the result is
 * undefined.  Output is bitwise equal to amass_sparse_decode on the same
 * bytes. */
int amass_tier_decode(
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
    int max_pages, void* stream);

/* tier_decode_install -- amass_tier_decode that also does the plan's miss
 * fetch (replaces Residency.gather_fetch, tier/residency.py:196-248,
 * 409-436, which the reference runs between the plan and the decode,
 * tier/decode_mem.py:225-274).  entry_slots (the plan's classified entries)
 * is required: a page whose entry is a miss that the plan gave a hot slot
 * (page2slot >= 0, complete page) is read from staging (vbo >= 0) or the
 * pinned pool -- not from the slot, which is not filled yet -- and its V
 * tile (and K tile under mem-kv) is then written into that slot; when it
 * came from staging and pool_valid (n_kv, NB) is 0 it is also written
 * through to the pinned pool and pool_valid set to 1, as the fetch does.
 * Each miss thus crosses the host link once.  Output, hot slots, pinned
 * pool and pool_valid end equal to plan + amass_tier_fetch +
 * amass_tier_decode. */
int amass_tier_decode_install(
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
    int max_pages, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AMASS_B200_H */
