// Device side of the Stage A.2 page selection (the per-unit selection body
// the select kernels in select.cu run).
//
// Selection is a threshold rule (reference selection/select.py:60-101): tau is
// the b-th largest score of the selectable region [sink, n_sel_hi); every page
// with score >= tau is kept (ties all kept), plus the sinks, the recent window
// and the partial tail; ids are written ascending and -1 padded.
//
// tau is found by an adaptive-range histogram select over order-preserving
// 32-bit keys held in shared memory: each level histograms the keys of the
// current range [lo, hi] into at most 1024 power-of-two-wide bins
// (bin = (key - lo) >> shift), one warp scans the bins from the top to the
// one holding the target rank -- or, in coverage mode, the target cumulative
// MASS -- and the range shrinks to that bin.  A bin of at most 64 keys is
// resolved exactly by ranking its members.  Typical units finish in one
// level: one pass over global memory, one histogram pass, one compaction.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace amass {
namespace {

// threads of a selection CTA: 256 (four CTAs per SM) by default; 512 or
// 1024 when there are few units, so one unit's latency chain is spread over
// more threads (NT template parameter below)
constexpr int kSelThreads = 256;
constexpr int kSelMaxWarps = 32;
constexpr int kBins = 1024;
constexpr int kCand = 64;


template <int NT, typename T, typename Op>
AMASS_DEV T block_reduce(T v, T* red, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) v = op(v, red[w]);
  return v;
}

struct SelArgs {
  const float* score_h;   // (R, n_kv, G, MP)   per-head scores (fold input)
  float* hmax;            // (R, n_kv, G)       per-head page max (fold input)
  float* score;           // (R, n_kv, MP)      combined score (in or out)
  const int32_t* npg;
  const int32_t* nsh;
  const int32_t* b_fix;
  int32_t* tab;
  int32_t* cnt;
  int32_t* b_unit;
  int n_kv, G, sink, MP;
  int64_t SHS;            // score_h row stride (elements; >= MP)
  float coverage;
};

// nrm fold of one unit (reference quad_score.py:293-315; 2^x in hardware,
// relative error ~2^-22): sc[p - p_lo] =
// sum_g exp(S_g[p] - hmax_g) for p in [p_lo, p_hi) (p_lo a multiple of 4);
// writes score; resets hmax to -inf when `reset` (after the barrier).
// GM: the largest G this instantiation serves (registers hold GM x KQ
// 16-byte loads per thread, all issued before any use).
template <int GM = 8, int KQ = 1, int NT = kSelThreads>
AMASS_DEV void nrm_fold(const SelArgs& a, int unit, int p_lo, int p_hi,
                        float* sc, bool reset = true,
                        const float* hm_in = nullptr) {
  const int nsh = p_hi;
  const float* sh = a.score_h + (int64_t)unit * a.G * a.SHS;
  float* hm_g = a.hmax + (int64_t)unit * a.G;
  float hm[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g)
    hm[g] = hm_in ? hm_in[g] : (g < a.G ? __ldcg(hm_g + g) : 0.f);
  float* so = a.score + (int64_t)unit * a.MP;
  // batches of pages per thread: every load of a batch issues before any
  // use, so a long unit costs a few memory round trips, not one per page
  if ((a.SHS & 3) == 0 && (reinterpret_cast<uintptr_t>(a.score_h) & 15) == 0) {
    // 16-byte loads: thread owns page quads tid, tid + NT, ...
    constexpr int kQ = KQ;
    const int nq = (nsh + 3) >> 2;
    for (int q0 = (p_lo >> 2) + threadIdx.x; q0 < nq; q0 += kQ * NT) {
      float4 v[kQ][GM];
#pragma unroll
      for (int i = 0; i < kQ; ++i) {
        const int q = q0 + i * NT;
#pragma unroll
        for (int g = 0; g < GM; ++g)
          v[i][g] = (g < a.G && q < nq)
                        ? __ldcg(reinterpret_cast<const float4*>(sh + (int64_t)g * a.SHS) + q)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < kQ; ++i) {
        const int q = q0 + i * NT;
        if (q < nq) {
          float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            if (g < a.G) {
              s4[0] += ex2_approx((v[i][g].x - hm[g]) * kLog2e);
              s4[1] += ex2_approx((v[i][g].y - hm[g]) * kLog2e);
              s4[2] += ex2_approx((v[i][g].z - hm[g]) * kLog2e);
              s4[3] += ex2_approx((v[i][g].w - hm[g]) * kLog2e);
            }
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int p = 4 * q + e;
            if (p < nsh) { sc[p - p_lo] = s4[e]; so[p] = s4[e]; }
          }
        }
      }
    }
  } else {
    constexpr int kB = 8;
    for (int p0 = p_lo + threadIdx.x; p0 < nsh; p0 += kB * NT) {
      float v[kB][GM];
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int p = p0 + i * NT;
#pragma unroll
        for (int g = 0; g < GM; ++g)
          v[i][g] = (g < a.G && p < nsh) ? __ldcg(sh + (int64_t)g * a.SHS + p) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int p = p0 + i * NT;
        if (p < nsh) {
          float s1 = 0.f;
#pragma unroll
          for (int g = 0; g < GM; ++g)
            if (g < a.G) s1 += ex2_approx((v[i][g] - hm[g]) * kLog2e);
          sc[p - p_lo] = s1;
          so[p] = s1;
        }
      }
    }
  }
  __syncthreads();
  if (reset && threadIdx.x < a.G) hm_g[threadIdx.x] = -INFINITY;
}

struct SelShared {
  uint32_t hist[kBins];
  float hmass[kBins];
  uint32_t cand[kCand];
  float cmass[kCand];
  float red[kSelMaxWarps];
  int wsum[kSelMaxWarps];
  uint32_t wc[kSelMaxWarps];
  float wm[kSelMaxWarps];
  int hit;
  int maxd;
  int ncand;
  int bin;
  uint32_t above_c;
  float above_m;
  uint32_t tau;
  uint32_t lowest;
  uint32_t kmin, kmax;
  // cluster form: the merged histogram / candidates and exchange slots
  // that the other CTAs of the unit read through distributed shared memory
  uint32_t mhist[kBins];
  float mmass[kBins];
  uint32_t acand[kCand];
  float amass[kCand];
  int nall;
  uint32_t x_kmin, x_kmax;
  float x_vmax, x_tot, x_alw;
  int x_above, x_cnt;
};

namespace cg = cooperative_groups;

// all-reduce of a per-CTA value over the cluster: every CTA publishes its
// value in `slot` (its own shared memory), then reads all ranks' slots in
// rank order (identical result in every CTA).  One cluster barrier.
template <typename T, typename Op>
AMASS_DEV T cl_allreduce(T* slot, T v, Op op) {
  cg::cluster_group cl = cg::this_cluster();
  if (threadIdx.x == 0) *slot = v;
  cl.sync();
  T r = *cl.map_shared_rank(slot, 0);
  for (unsigned k = 1; k < cl.num_blocks(); ++k)
    r = op(r, *cl.map_shared_rank(slot, k));
  return r;
}

// tau over the keys of sc[lo_p, hi_p).  COV: mass walk to `need`; else the
// k-th largest key.  mass(v) = LIN ? v : exp(v - shift).
// CLU: the unit's pages are spread over the CTAs of a cluster (sc / lo_p /
// hi_p are this CTA's slice); histograms and candidates are merged across
// the cluster, so every CTA walks the same merged bins to the same tau.
template <bool COV, bool LIN, bool CLU = false, int NT = kSelThreads>
AMASS_DEV uint32_t find_tau(const float* sc, int lo_p, int hi_p, int k,
                            float need, float shift_v, uint32_t kmin,
                            uint32_t kmax, SelShared& sh) {
  uint32_t* H = CLU ? sh.mhist : sh.hist;
  float* HM = CLU ? sh.mmass : sh.hmass;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t lo = kmin, hi = kmax;
  if (COV && !(need > 0.f)) return kmax;      // b = 1: the top page only
  for (int level = 0; level < 6; ++level) {
    const uint64_t width = (uint64_t)(hi - lo) + 1;
    int shift = 0;
    while (((width - 1) >> shift) >= (uint64_t)kBins) ++shift;
    for (int i = threadIdx.x; i < kBins; i += NT) {
      sh.hist[i] = 0;
      if (COV) sh.hmass[i] = 0.f;
    }
    if (threadIdx.x == 0) sh.ncand = 0;
    __syncthreads();
    for (int p = lo_p + threadIdx.x; p < hi_p; p += NT) {
      const float v = sc[p];
      const uint32_t key = float_key(v);
      if (key >= lo && key <= hi) {
        const int b = (int)((key - lo) >> shift);
        atomicAdd(&sh.hist[b], 1u);
        if (COV) atomicAdd(&sh.hmass[b], LIN ? v : expf(v - shift_v));
      }
    }
    if constexpr (CLU) {
      cg::cluster_group cl = cg::this_cluster();
      cl.sync();                       // every slice's histogram is built
      for (int i = threadIdx.x; i < kBins; i += NT) {
        uint32_t c = 0;
        float mm = 0.f;
        for (unsigned q = 0; q < cl.num_blocks(); ++q) {
          c += cl.map_shared_rank(sh.hist, q)[i];
          if (COV) mm += cl.map_shared_rank(sh.hmass, q)[i];
        }
        sh.mhist[i] = c;
        if (COV) sh.mmass[i] = mm;
      }
      cl.sync();                       // remote reads done before reuse
    } else {
      __syncthreads();
    }
    // bin scan by the whole block: warp w owns the w-th 1/(NT / 32) of the
    // bins counted from the top, each lane kPL consecutive bins
    {
      constexpr int kPW = kBins / (NT / 32), kPL = kPW / 32;
      const int d0 = warp * kPW + lane * kPL;          // descending index
      uint32_t cl = 0;
      float ml = 0.f;
#pragma unroll
      for (int i = 0; i < kPL; ++i) {
        cl += H[kBins - 1 - (d0 + i)];
        if (COV) ml += HM[kBins - 1 - (d0 + i)];
      }
      uint32_t ci = cl;
      float mi = ml;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t tc = __shfl_up_sync(0xffffffffu, ci, o);
        const float tm = __shfl_up_sync(0xffffffffu, mi, o);
        if (lane >= o) { ci += tc; mi += tm; }
      }
      if (lane == 31) { sh.wc[warp] = ci; sh.wm[warp] = mi; }
      if (threadIdx.x == 0) { sh.hit = 0; sh.maxd = -1; }
      __syncthreads();
      uint32_t cex = ci - cl;
      float mex = mi - ml;
      for (int w = 0; w < warp; ++w) { cex += sh.wc[w]; if (COV) mex += sh.wm[w]; }
      bool mine;
      if (COV) mine = cl > 0 && (mex + ml >= need) && (mex < need);
      else mine = cl > 0 && (cex < (uint32_t)k) && (cex + cl >= (uint32_t)k);
      if (mine) {
        uint32_t ac = cex;
        float am = mex;
        for (int i = 0; i < kPL; ++i) {
          const int b = kBins - 1 - (d0 + i);
          const uint32_t cb = H[b];
          if (cb == 0) continue;
          const float mm = COV ? HM[b] : 0.f;
          if (COV ? (am + mm >= need) : (ac + cb >= (uint32_t)k)) {
            sh.bin = b; sh.above_c = ac; sh.above_m = am; sh.hit = 1;
            break;
          }
          ac += cb;
          am += mm;
        }
      }
      if (cl > 0) atomicMax(&sh.maxd, d0 + kPL - 1);
      __syncthreads();
      if (!sh.hit) {
        // coverage never reached (fp rounding): the lowest non-empty bin
        const int md = sh.maxd;
        if (md >= d0 && md < d0 + kPL) {
          uint32_t ac = cex;
          float am = mex;
          int last = -1;
          uint32_t lc = 0;
          float lm = 0.f;
          for (int i = 0; i < kPL; ++i) {
            const int b = kBins - 1 - (d0 + i);
            const uint32_t cb = H[b];
            if (cb == 0) continue;
            last = b; lc = ac; lm = am;
            ac += cb;
            am += COV ? HM[b] : 0.f;
          }
          sh.bin = last < 0 ? 0 : last;
          sh.above_c = lc;
          sh.above_m = lm;
        }
      }
    }
    __syncthreads();
    const int bin = sh.bin;
    const uint32_t cnt_bin = H[bin];
    k -= (int)sh.above_c;
    need -= sh.above_m;
    const uint32_t blo = lo + ((uint32_t)bin << shift);
    const uint64_t bend = (uint64_t)blo + ((1ull << shift) - 1);
    const uint32_t bhi = bend < (uint64_t)hi ? (uint32_t)bend : hi;
    if (blo == bhi) return blo;
    if (cnt_bin <= (uint32_t)kCand) {
      for (int p = lo_p + threadIdx.x; p < hi_p; p += NT) {
        const float v = sc[p];
        const uint32_t key = float_key(v);
        if (key >= blo && key <= bhi) {
          const int j = atomicAdd(&sh.ncand, 1);
          sh.cand[j] = key;
          if (COV) sh.cmass[j] = LIN ? v : expf(v - shift_v);
        }
      }
      if (threadIdx.x == 0) { sh.tau = 0xffffffffu; sh.lowest = 0xffffffffu; }
      uint32_t* CK = sh.cand;
      float* CM = sh.cmass;
      if constexpr (CLU) {
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();                     // every slice's candidates listed
        if (threadIdx.x == 0) {
          int off = 0;
          for (unsigned q = 0; q < cl.num_blocks(); ++q) {
            const int nq = *cl.map_shared_rank(&sh.ncand, q);
            const uint32_t* ck = cl.map_shared_rank(sh.cand, q);
            const float* cm = cl.map_shared_rank(sh.cmass, q);
            for (int j = 0; j < nq && off < kCand; ++j, ++off) {
              sh.acand[off] = ck[j];
              if (COV) sh.amass[off] = cm[j];
            }
          }
          sh.nall = off;
        }
        CK = sh.acand;
        CM = sh.amass;
      }
      __syncthreads();
      {
        // rank the members in parallel: 4 threads per candidate, each
        // comparing against a quarter of the members
        const int n = CLU ? sh.nall : sh.ncand;
        const int j = threadIdx.x >> 2, part = threadIdx.x & 3;
        const uint32_t key = j < n ? CK[j] : 0u;
        uint32_t ab = 0, eq = 0;
        float mab = 0.f, meq = 0.f;
        if (j < n) {
          for (int t = part; t < n; t += 4) {
            const uint32_t o = CK[t];
            if (o > key) { ab++; if (COV) mab += CM[t]; }
            else if (o == key) { eq++; if (COV) meq += CM[t]; }
          }
        }
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
          ab += __shfl_xor_sync(0xffffffffu, ab, o);
          eq += __shfl_xor_sync(0xffffffffu, eq, o);
          if (COV) {
            mab += __shfl_xor_sync(0xffffffffu, mab, o);
            meq += __shfl_xor_sync(0xffffffffu, meq, o);
          }
        }
        if (j < n && part == 0) {
          atomicMin(&sh.lowest, key);
          bool ok;
          if (COV) ok = (mab < need) && (mab + meq >= need);
          else ok = (ab < (uint32_t)k) && (ab + eq >= (uint32_t)k);
          if (ok) atomicMin(&sh.tau, key);
        }
      }
      __syncthreads();
      if (threadIdx.x == 0 && sh.tau == 0xffffffffu) sh.tau = sh.lowest;
      __syncthreads();
      return sh.tau;
    }
    lo = blo;
    hi = bhi;
    __syncthreads();
  }
  return lo;
}

// FOLD: fold score_h (nrm) into score first.  LIN: page mass = score (nrm
// semantics) instead of exp(score - max) (max semantics).  CLU: one unit per
// thread-block cluster -- CTA `rank` owns the slice [s0, s1) of the scored
// pages (fold, statistics and histograms of its slice, merged over the
// cluster through distributed shared memory) and compacts that slice (the
// last rank also the unscored tail) at an offset taken from the lower
// ranks' counts; used when there are few units, so a long unit's latency is
// spread over several SMs.
// Selection of one (request, kv-head) unit by the calling CTA (all
// NT threads): the nrm fold (FOLD), the threshold search and the
// ascending compaction.  CLU: the unit is spread over the nb CTAs of a
// thread-block cluster and this CTA is `rank`.  `sc` holds at least this
// CTA's slice of the scored pages; the caller separates consecutive calls
// with a barrier.
template <bool FOLD, bool LIN, bool COVERAGE, int GM = 8, bool CLU = false,
          int NT = kSelThreads>
AMASS_DEV void select_unit(const SelArgs& a, const int unit, const int nb,
                           const int rank, float* sc, SelShared& sh) {
  const int r = unit / a.n_kv;
  // every per-unit scalar the selection needs, loaded together
  const int npg_raw = a.npg[r];
  const int nsh = a.nsh[r];
  const int bfix = COVERAGE ? 0 : a.b_fix[r];
  float hm_pre[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g)
    hm_pre[g] = (FOLD && g < a.G) ? __ldcg(a.hmax + (int64_t)unit * a.G + g) : 0.f;
  const int npg = max(npg_raw, 0);
  const int sink = a.sink;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nsc = max(nsh, 0);
  const int chunk = ((nsc + nb - 1) / nb + 3) & ~3;
  const int s0 = min(rank * chunk, nsc), s1 = min(s0 + chunk, nsc);
  if (threadIdx.x == 0) { sh.kmin = 0xffffffffu; sh.kmax = 0u; }
  if (nsh > 0) {
    if (FOLD) {
      nrm_fold<GM, (GM <= 4 && NT <= 256 ? 2 : 1), NT>(a, unit, s0, s1, sc, !CLU, hm_pre);
    } else {
      const float* si = a.score + (int64_t)unit * a.MP;
      constexpr int kB = 8;
      for (int p0 = s0 + threadIdx.x; p0 < s1; p0 += kB * NT) {
        float v[kB];
#pragma unroll
        for (int i = 0; i < kB; ++i) {
          const int p = p0 + i * NT;
          v[i] = p < s1 ? __ldcg(si + p) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kB; ++i) {
          const int p = p0 + i * NT;
          if (p < s1) sc[p - s0] = v[i];
        }
      }
    }
  } else if (FOLD && !CLU && threadIdx.x < a.G) {
    a.hmax[(int64_t)unit * a.G + threadIdx.x] = -INFINITY;
  }
  if constexpr (CLU) {
    cg::this_cluster().sync();               // every slice has read hmax
    if (FOLD && rank == 0 && threadIdx.x < a.G)
      a.hmax[(int64_t)unit * a.G + threadIdx.x] = -INFINITY;
  }
  __syncthreads();
  const int nsel = nsh - sink;
  const bool keep_all = nsel <= 1;
  const int lo_sel = max(sink, s0);            // selectable part of the slice
  uint32_t tau = 0;
  int b_used = 1;
  if (!keep_all) {
    uint32_t kmin = 0xffffffffu, kmax = 0;
    for (int p = lo_sel + threadIdx.x; p < s1; p += NT) {
      const uint32_t key = float_key(sc[p - s0]);
      kmin = min(kmin, key);
      kmax = max(kmax, key);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
      kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    }
    if (lane == 0) {
      atomicMin(&sh.kmin, kmin);
      atomicMax(&sh.kmax, kmax);
    }
    __syncthreads();
    kmin = sh.kmin;
    kmax = sh.kmax;
    if constexpr (CLU) {
      kmin = cl_allreduce(&sh.x_kmin, kmin,
                          [](uint32_t x, uint32_t y) { return min(x, y); });
      kmax = cl_allreduce(&sh.x_kmax, kmax,
                          [](uint32_t x, uint32_t y) { return max(x, y); });
    }
    if (COVERAGE) {
      float shiftv = 0.f;
      if (!LIN) {
        float vmax = -INFINITY;
        for (int p = s0 + threadIdx.x; p < s1; p += NT)
          vmax = fmaxf(vmax, sc[p - s0]);
        shiftv = block_reduce<NT>(vmax, sh.red,
                              [](float x, float y) { return fmaxf(x, y); });
        if constexpr (CLU)
          shiftv = cl_allreduce(&sh.x_vmax, shiftv,
                                [](float x, float y) { return fmaxf(x, y); });
      }
      float tot = 0.f, alw = 0.f;
      for (int p = s0 + threadIdx.x; p < s1; p += NT) {
        const float m = LIN ? sc[p - s0] : expf(sc[p - s0] - shiftv);
        tot += m;
        if (p < sink) alw += m;
      }
      auto add = [](float x, float y) { return x + y; };
      tot = block_reduce<NT>(tot, sh.red, add);
      alw = block_reduce<NT>(alw, sh.red, add);
      if constexpr (CLU) {
        tot = cl_allreduce(&sh.x_tot, tot, add);
        alw = cl_allreduce(&sh.x_alw, alw, add);
      }
      const float need = fmaxf(a.coverage * tot - alw, 0.f);
      tau = find_tau<true, LIN, CLU, NT>(sc, lo_sel - s0, s1 - s0, 0, need, shiftv,
                                     kmin, kmax, sh);
      int above = 0;
      for (int p = lo_sel + threadIdx.x; p < s1; p += NT)
        above += float_key(sc[p - s0]) > tau;
      auto iadd = [](int x, int y) { return x + y; };
      above = block_reduce<NT>(above, reinterpret_cast<int*>(sh.red), iadd);
      if constexpr (CLU) above = cl_allreduce(&sh.x_above, above, iadd);
      b_used = above + 1;
    } else {
      const int b = bfix;
      b_used = b;
      tau = find_tau<false, true, CLU, NT>(sc, lo_sel - s0, s1 - s0, b, 0.f, 0.f,
                                       kmin, kmax, sh);
    }
  }
  if (a.b_unit && threadIdx.x == 0 && rank == 0) a.b_unit[unit] = b_used;

  // ascending compaction of this CTA's range [c0, c1) (the whole [0, npg)
  // without a cluster): each thread owns a contiguous run of pages; one
  // block-wide exclusive scan of the per-thread counts
  int32_t* tab = a.tab + (int64_t)unit * a.MP;
  const int c0 = s0, c1 = (rank == nb - 1) ? max(npg, s1) : s1;
  const int per = (c1 - c0 + NT - 1) / NT;
  const int p_lo = c0 + threadIdx.x * per, p_hi = min(p_lo + per, c1);
  auto keep_page = [&](int p) {
    return keep_all || p < sink || p >= nsh || float_key(sc[p - s0]) >= tau;
  };
  // keep bits of this thread's run (at most 64 pages per thread: MP <= 16K)
  uint64_t bits = 0;
  for (int p = p_lo; p < p_hi; ++p)
    if (keep_page(p)) bits |= 1ull << (p - p_lo);
  const int mine = __popcll(bits);
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sh.wsum[warp] = incl;
  __syncthreads();
  int off = 0, total = 0;
#pragma unroll
  for (int w = 0; w < (NT / 32); ++w) {
    const int v = sh.wsum[w];
    if (w < warp) off += v;
    total += v;
  }
  int base = 0, all = total;
  if constexpr (CLU) {
    cg::cluster_group cl = cg::this_cluster();
    if (threadIdx.x == 0) sh.x_cnt = total;
    cl.sync();
    all = 0;
    for (int q = 0; q < nb; ++q) {
      const int cq = *cl.map_shared_rank(&sh.x_cnt, q);
      if (q < rank) base += cq;
      all += cq;
    }
  }
  off += base + incl - mine;
  while (bits) {
    const int i = __ffsll(bits) - 1;
    bits &= bits - 1;
    tab[off++] = p_lo + i;
  }
  if (nb == 1 && (a.MP & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(a.tab) & 15) == 0) {
    // -1 padding in 16-byte stores past the first multiple of 4
    const int p4 = min((all + 3) & ~3, a.MP);
    if (all + (int)threadIdx.x < p4) tab[all + threadIdx.x] = -1;
    int4* t4 = reinterpret_cast<int4*>(tab);
    for (int q4 = p4 / 4 + threadIdx.x; q4 < a.MP / 4; q4 += NT)
      t4[q4] = make_int4(-1, -1, -1, -1);
  } else {
    for (int p = all + rank * NT + threadIdx.x; p < a.MP;
         p += nb * NT)
      tab[p] = -1;
  }
  if (threadIdx.x == 0 && rank == 0) a.cnt[unit] = all;
  if constexpr (CLU) cg::this_cluster().sync();   // peers' reads of sh done
}


}  // namespace
}  // namespace amass
