// Cross-GPU barrier over peer-mapped flags, for the kv-head-sharded decode
// whose merge kernel stores its output rows into every rank's output buffer.
//
// Every rank owns a flag array of n ints (index = source rank) in memory
// that all ranks map.  A call advances this rank's epoch counter e, makes
// the preceding kernels' peer stores visible (fence.sys), writes e into slot
// `rank` of every rank's flags with a release store, then waits until every
// slot of its own flags holds >= e (acquire loads).  The wait is bounded:
// after kSpinLimit polls the kernel records the waiting slot in err and
// returns, leaving the context usable; the host reads err.
#include "common.cuh"

namespace amass {
namespace {

constexpr int kMaxRanks = 8;
constexpr long long kSpinLimit = 1LL << 20;   // about a second with the back-off

struct BarrierArgs {
  int32_t* flags[kMaxRanks];   // every rank's flag array, mapped here
  int32_t* epoch;              // this rank's call counter (device)
  int32_t* err;                // 0, or 1 + slot that timed out
  int n, rank;
};

AMASS_DEV void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
AMASS_DEV int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(BarrierArgs a) {
  __shared__ int32_t e_s;
  const int t = threadIdx.x;
  if (t == 0) {
    const int32_t e = *a.epoch + 1;
    *a.epoch = e;
    e_s = e;
  }
  __syncthreads();
  const int32_t e = e_s;
  __threadfence_system();
  if (t < a.n) st_release_sys(a.flags[t] + a.rank, e);
  if (t < a.n) {
    const int32_t* mine = a.flags[a.rank] + t;
    long long it = 0;
    while (ld_acquire_sys(mine) - e < 0) {
      if (++it > kSpinLimit) {
        atomicCAS(a.err, 0, 1 + t);
        break;
      }
      __nanosleep(128);
    }
  }
  __threadfence_system();
}

}  // namespace
}  // namespace amass

extern "C" int amass_peer_barrier(int32_t* const* peer_flags, int n_ranks,
                                  int rank, int32_t* epoch, int32_t* err,
                                  void* stream) {
  using namespace amass;
  if (!peer_flags || !epoch || !err || n_ranks < 1 || n_ranks > kMaxRanks ||
      rank < 0 || rank >= n_ranks)
    return AMASS_ERR_ARG;
  BarrierArgs a{};
  for (int i = 0; i < kMaxRanks; ++i)
    a.flags[i] = i < n_ranks ? peer_flags[i] : nullptr;
  for (int i = 0; i < n_ranks; ++i)
    if (!a.flags[i]) return AMASS_ERR_ARG;
  a.epoch = epoch; a.err = err; a.n = n_ranks; a.rank = rank;
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}
