// Shared device helpers for the AMASS sm_100a kernels.
//
// Tensor-core fragments use the warp-level m16n8k16 MMA (fp16/bf16 inputs,
// fp32 accumulate).  The hot path is HBM-bound (~2-6 flop per byte read), so
// the MMA only has to keep the integer->half conversions and the q.K / P.V
// products off the fp32 pipe; operand staging is cp.async into XOR-swizzled
// shared memory.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/amass_b200.h"

#define AMASS_DEV __device__ __forceinline__

namespace amass {

constexpr float kLog2e = 1.4426950408889634f;

// --------------------------------------------------------------------------
// launch helpers
// --------------------------------------------------------------------------
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AMASS_OK : AMASS_ERR_CUDA;
}

// Launch with programmatic dependent launch enabled: the grid may be
// scheduled while the previous kernel on the stream is still finishing; every
// kernel here calls grid_dep_wait() before touching memory that kernel wrote,
// and grid_dep_launch() early so its own successor can be scheduled.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                      size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess
             ? AMASS_OK
             : AMASS_ERR_CUDA;
}

// Kernel attributes are per device: true the first time this is called for
// the current device with this mask (one bit per device id).
inline bool first_on_device(unsigned long long& mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (mask & bit) return false;
  mask |= bit;
  return true;
}

inline int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

// --------------------------------------------------------------------------
// derive_page_params of one request (reference selection/select.py:30-45):
// npg = ceil(s / page), n_sel_hi = npg - window, b = clamp(ceil(fp64
// (n_sel_hi - sink) * budget), 1, max(n_sel_hi - sink, 1))
// --------------------------------------------------------------------------
AMASS_DEV void derive_one(int s, double bud, int page, int win, int sink,
                          int32_t* npg_o, int32_t* nsh_o, int32_t* b_o) {
  const int npg = (s + page - 1) / page;
  const int nsh = npg - win;
  const int nsel = nsh - sink;
  const double bf = ceil((double)nsel * bud);
  int b = (int)bf;
  b = max(b, 1);
  b = min(b, max(nsel, 1));
  *npg_o = npg;
  *nsh_o = nsh;
  *b_o = b;
}

// --------------------------------------------------------------------------
// order-preserving float <-> uint32 keys (larger float -> larger key)
// --------------------------------------------------------------------------
AMASS_DEV uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
AMASS_DEV float key_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// --------------------------------------------------------------------------
// exact small-integer -> fp16 conversion (magic-bias method: an 8-bit
// unsigned u placed in the low mantissa of 1024.0h reads as 1024+u, so a
// signed code v is recovered by (0x6400 | (v + bias)) - (1024 + bias)).  Each
// helper converts the two bytes at positions 0 and 2 of x into one half2.
// Reference for the method: Kim et al., "Who Says Elephants Can't Run:
// Bringing Large Scale MoE Models into Cloud Scale Production" (2022).
// --------------------------------------------------------------------------
AMASS_DEV uint32_t lop3_sel(uint32_t a, uint32_t b, uint32_t c) {
  // f = b ? (a ^ c) : c   (immLut 0x6A)
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// signed int8 bytes (positions 0,2) -> half2 (exact)
AMASS_DEV uint32_t i8pair_to_h2(uint32_t x) {
  uint32_t h = lop3_sel(x, 0x00FF00FFu, 0x64806480u);  // 1024 + (v + 128)
  const uint32_t bias = 0x64806480u;                   // 1152.0h x2
  uint32_t r;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(bias));
  return r;
}
// signed int4 nibbles (low nibble of bytes 0,2) -> half2 (exact)
AMASS_DEV uint32_t i4pair_to_h2(uint32_t x) {
  uint32_t h = lop3_sel(x, 0x000F000Fu, 0x64086408u);  // 1024 + (v + 8)
  const uint32_t bias = 0x64086408u;                   // 1032.0h x2
  uint32_t r;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(bias));
  return r;
}
// place byte BI of word a at position 0 and byte BJ of word b at position 2
template <int BI, int BJ>
AMASS_DEV uint32_t pick2(uint32_t a, uint32_t b) {
  return __byte_perm(a, b, (BI & 3) | ((4 + (BJ & 3)) << 8));
}

AMASS_DEV uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
AMASS_DEV uint32_t pack_bf2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
AMASS_DEV float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
AMASS_DEV float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// --------------------------------------------------------------------------
// warp MMA m16n8k16, fp32 accumulate
// --------------------------------------------------------------------------
AMASS_DEV void mma_f16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
AMASS_DEV void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

AMASS_DEV void ldsm_x4(uint32_t* r, uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}
// transpose of the 8x8 b16 matrix held as one fragment register per lane
AMASS_DEV uint32_t movmatrix_t(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
AMASS_DEV void ldsm_x4_t(uint32_t* r, uint32_t saddr) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(saddr));
}

// L2 eviction-priority policies: evict_first for data read once (streamed
// summaries and K/V pages), evict_last for data re-read soon (per-head
// scores between the scorer and the select)
AMASS_DEV uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// --------------------------------------------------------------------------
// cp.async (16 B, L2-only caching; src_bytes = 0 zero-fills the destination)
// --------------------------------------------------------------------------
AMASS_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
AMASS_DEV void cp_async16(uint32_t dst, const void* src, bool valid) {
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
               :: "r"(dst), "l"(src), "r"(n));
}
AMASS_DEV void cp_async16_pol(uint32_t dst, const void* src, bool valid,
                              uint64_t pol) {
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;"
               :: "r"(dst), "l"(src), "r"(n), "l"(pol));
}
AMASS_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
AMASS_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" :: "n"(N));
}

// --------------------------------------------------------------------------
// mbarrier + bulk-copy (cp.async.bulk, no multicast) helpers
// --------------------------------------------------------------------------
AMASS_DEV void mbar_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count));
}
// make the initialised barriers visible to the async proxy (bulk copies)
AMASS_DEV void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
AMASS_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
AMASS_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(bar), "r"(bytes) : "memory");
}
// this thread's earlier cp.async copies arrive on bar when they land (the
// arrival counts against the barrier's expected count)
AMASS_DEV void cp_async_mbar_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];"
               :: "r"(bar) : "memory");
}
// one poll: suspends the thread for at most ~1 us (suspend-time hint) while
// the phase is incomplete
AMASS_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
AMASS_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// bounded wait for the phase of parity `parity` to complete: false when
// about a second passed (the caller records the fault and unwinds)
constexpr uint64_t kMbarWaitNs = 1000000000ull;
AMASS_DEV bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kMbarWaitNs) return false;
  }
}
// one contiguous global -> shared bulk copy completing on bar (16-byte
// aligned addresses, size a multiple of 16)
AMASS_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                        uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];"
      :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
AMASS_DEV uint4 lds128(uint32_t a) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
  return r;
}
AMASS_DEV uint32_t lds32(uint32_t a) {
  uint32_t r;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(a));
  return r;
}
AMASS_DEV uint16_t lds16(uint32_t a) {
  uint16_t r;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(r) : "r"(a));
  return r;
}

// read-only global loads that do not allocate in L1 (streamed summaries)
AMASS_DEV uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// the same with an L2 eviction-priority policy (createpolicy)
AMASS_DEV uint4 ldg_nc_v4_pol(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(pol));
  return r;
}
AMASS_DEV uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
AMASS_DEV void stg_f32_pol(float* p, float v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.f32 [%0], %1, %2;"
               :: "l"(p), "f"(v), "l"(pol) : "memory");
}
AMASS_DEV float4 ldcg_f4_pol(const float4* p, uint64_t pol) {
  float4 r;
  asm volatile("ld.global.cg.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p), "l"(pol));
  return r;
}
AMASS_DEV uint2 ldg_nc_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
AMASS_DEV uint32_t ldg_nc_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];"
               : "=r"(r) : "l"(p));
  return r;
}

// Programmatic dependent launch: wait for the producing grid's memory.
// PTX ex2.approx / lg2.approx (relative error about 2^-22; 2^-inf = 0)
AMASS_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
AMASS_DEV float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

AMASS_DEV void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
AMASS_DEV void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;");
}

}  // namespace amass
