// lss_sampler.cu — batched token sampler for B200 (sm_100a).
//
// What it computes, per row (LocalStrm src/engine/sampling.py:118-163):
//   greedy (T <= 0): argmax of the raw row, NaN largest, lowest index on ties      (:132-133)
//   z = repetition / frequency / presence penalties over the row's history         (:38-68)
//   y = z / T   (IEEE f32 division)                                                 (:146)
//   top-k keeps y >= k-th largest (ties kept); min-p keeps exp(y - max) >= min_p;
//   top-p keeps the sorted prefix whose cumulative mass before each token <= top_p (:71-115)
//   NaN / +inf / all -inf rows: argmax of y (the reference's NaN guard)             (:159-160)
//   draw: inverse CDF in vocabulary order from a supplied uniform                   (:162)
//
// How (one thread-block cluster of CL CTAs per row; no tensor cores — this is a
// memory-bound select, not a contraction):
//   K0 lss_hist_dedup   per row: (id, count) pairs of the history (torch.unique, :52)
//   K1 lss_rows_kernel  each CTA stages a contiguous 1/CL slice of the row in shared
//                       memory with bulk async copies (one HBM read), applies the
//                       penalties, divides by T and reduces the row max across the
//                       cluster through distributed shared memory.  A value-space
//                       histogram (counts, merged by DSMEM atomics) bounds the top-k
//                       window; min-p is an exact key threshold.  The survivors are
//                       compacted, pushed into CTA 0's shared memory and resolved
//                       there (sort, top-k / top-p cut, renormalise, draw).  When the
//                       survivors do not fit, a cluster-wide radix select over the
//                       order-preserving u32 keys of y (counts for top-k, 2^-40 fixed
//                       point mass for top-p) finds the exact cut, and the CTA whose
//                       slice holds the uniform's CDF position finds the token.
//   lss_argmax_kernel   the all-greedy seam (llm_engine.py:1139-1141).
//
// Error handling: every bounded wait that gives up sets a flag in the workspace
// header; host entry points return int statuses and never abort.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cooperative_groups.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "lsampler.h"

namespace cg = cooperative_groups;

namespace lss {

constexpr int NT = 512;                 // threads per CTA
constexpr int NWARP = NT / 32;
constexpr int MAXCL = 8;                // CTAs per cluster (portable limit)
constexpr int NBIN = 256;               // histogram bins per pass (+1 "far" bucket)
constexpr int CAP = 4096;               // survivors one CTA can resolve
constexpr float BIN_PER_NAT = 16.0f;    // value-space bins: 1/16 nat wide, 16 nats deep
constexpr uint32_t KEY_FINITE_MIN = 0x00800000u;  // key of -FLT_MAX
constexpr double FIX_ONE = 1099511627776.0;       // 2^40: fixed-point unit of mass
constexpr int RES_BYTES = CAP * 8 + CAP * 4;      // resolve buffers in CTA 0
constexpr long long WAIT_CYCLES = 4000000000LL;   // ~2 s at 1.9 GHz

// ---------------------------------------------------------------------------
// Order-preserving keys and small numeric helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(__fadd_rn(f, 0.0f));   // -0 -> +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// torch.argmax order: NaN above everything.
__device__ __forceinline__ uint32_t gkey(float f) { return (f != f) ? 0xffffffffu : f2key(f); }
__device__ __forceinline__ uint64_t argmax_code(float f, int idx) {
  return ((uint64_t)gkey(f) << 32) | (uint32_t)(~(uint32_t)idx);
}
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t efix(float e) {
  return __float2ull_rn(__fmul_rn(e, 1099511627776.0f));
}
// Value-space bin: 0 for the max, NBIN ("far") for >= 16 nats below or -inf.
__device__ __forceinline__ int vbin(float y, float m) {
  float d = __fmul_rn(__fsub_rn(m, y), BIN_PER_NAT);
  return d < (float)NBIN ? (int)d : NBIN;
}

// ---------------------------------------------------------------------------
// PTX wrappers: mbarrier + bulk async copy (global -> own shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t saddr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          saddr(dst)),
      "l"(src), "r"(bytes), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, "
      "p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after WAIT_CYCLES and reports false.
__device__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > WAIT_CYCLES) return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Block-wide reductions and scans (NT threads)
// ---------------------------------------------------------------------------
template <class T, class Op>
__device__ __forceinline__ T warp_allreduce(T v, Op op) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <class T, class Op>
__device__ T block_allreduce(T v, Op op, T* scr) {
  v = warp_allreduce(v, op);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) scr[threadIdx.x >> 5] = v;
  __syncthreads();
  T r = scr[0];
#pragma unroll
  for (int i = 1; i < NWARP; ++i) r = op(r, scr[i]);
  return r;
}
// Exclusive scan of one value per thread in thread order; `total` gets the sum.
template <class T>
__device__ T block_excl_scan(T v, T* scr, T& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) scr[warp] = x;
  __syncthreads();
  T pre = T(0), tot = T(0);
#pragma unroll
  for (int i = 0; i < NWARP; ++i) {
    T s = scr[i];
    if (i < warp) pre += s;
    tot += s;
  }
  total = tot;
  return pre + x - v;
}
struct MaxF { __device__ float operator()(float a, float b) const { return fmax_nan(a, b); } };
struct MaxU64 { __device__ uint64_t operator()(uint64_t a, uint64_t b) const { return a > b ? a : b; } };
struct SumU64 { __device__ uint64_t operator()(uint64_t a, uint64_t b) const { return a + b; } };
struct SumU32 { __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a + b; } };
struct SumD { __device__ double operator()(double a, double b) const { return a + b; } };
struct MinI { __device__ int operator()(int a, int b) const { return a < b ? a : b; } };

// Bitonic sort of a[0, np) (np a power of two) in shared memory.
__device__ void bitonic_sort(uint64_t* a, int np, bool descending) {
  for (int k = 2; k <= np; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < np; i += NT) {
        int p = i ^ j;
        if (p > i) {
          uint64_t x = a[i], y = a[p];
          bool asc = ((i & k) == 0) != descending;
          if (asc ? (x > y) : (x < y)) {
            a[i] = y;
            a[p] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

__host__ __device__ __forceinline__ int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

// ---------------------------------------------------------------------------
// K0: history -> unique (id, count) pairs per row  (torch.unique, sampling.py:52)
// ---------------------------------------------------------------------------
constexpr int DEDUP_SMEM_SLOTS = 4096;  // histories up to 2,048 ids hash in shared memory
constexpr uint32_t EMPTY = 0xffffffffu;

__global__ void __launch_bounds__(256) lss_hist_dedup(const int32_t* __restrict__ hist_off,
                                                      const int32_t* __restrict__ hist_ids, int V,
                                                      const float* __restrict__ temperature,
                                                      const float* __restrict__ rep,
                                                      const float* __restrict__ freq,
                                                      const float* __restrict__ pres,
                                                      int32_t* __restrict__ uniq_ids,
                                                      int32_t* __restrict__ uniq_cnt,
                                                      int32_t* __restrict__ n_uniq,
                                                      uint32_t* __restrict__ gkeys,
                                                      uint32_t* __restrict__ gcnts,
                                                      uint32_t* __restrict__ err) {
  __shared__ uint32_t skeys[DEDUP_SMEM_SLOTS];
  __shared__ uint32_t scnts[DEDUP_SMEM_SLOTS];
  __shared__ uint32_t nout;
  const int row = blockIdx.x;
  const int b = hist_off[row], e = hist_off[row + 1];
  const int H = e - b;
  const bool active = !(temperature[row] <= 0.0f) && H > 0 &&
                      (rep[row] != 1.0f || freq[row] != 0.0f || pres[row] != 0.0f);
  if (!active) {
    if (threadIdx.x == 0) n_uniq[row] = 0;
    return;
  }
  uint32_t *keys, *cnts;
  uint32_t cap;
  bool pow2;
  if (2 * H <= DEDUP_SMEM_SLOTS) {
    cap = (uint32_t)next_pow2(2 * H);
    keys = skeys;
    cnts = scnts;
    pow2 = true;
  } else {
    cap = (uint32_t)(2 * H);
    keys = gkeys + 2 * (int64_t)b;
    cnts = gcnts + 2 * (int64_t)b;
    pow2 = false;
  }
  for (uint32_t s = threadIdx.x; s < cap; s += blockDim.x) {
    keys[s] = EMPTY;
    cnts[s] = 0;
  }
  if (threadIdx.x == 0) nout = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < H; j += blockDim.x) {
    int id = hist_ids[b + j];
    if (id < 0 || id >= V) {
      atomicOr(err, LSS_FLAG_BAD_HISTORY);
      continue;
    }
    uint32_t h = (uint32_t)id * 2654435761u;
    h = pow2 ? (h & (cap - 1)) : (h % cap);
    for (uint32_t probe = 0; probe < cap; ++probe) {
      uint32_t old = atomicCAS(&keys[h], EMPTY, (uint32_t)id);
      if (old == EMPTY || old == (uint32_t)id) {
        atomicAdd(&cnts[h], 1u);
        break;
      }
      h = (h + 1 == cap) ? 0 : h + 1;
    }
  }
  __syncthreads();
  for (uint32_t s = threadIdx.x; s < cap; s += blockDim.x) {
    uint32_t k = keys[s];
    if (k != EMPTY) {
      uint32_t pos = atomicAdd(&nout, 1u);
      uniq_ids[b + pos] = (int32_t)k;
      uniq_cnt[b + pos] = (int32_t)cnts[s];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) n_uniq[row] = (int32_t)nout;
}

// ---------------------------------------------------------------------------
// K1: one cluster per row
// ---------------------------------------------------------------------------
struct RowArgs {
  const void* logits;
  int64_t row_stride;  // elements
  int B, V, TE;        // TE: tile elements per CTA (multiple of 16)
  int tile_bytes;      // bytes reserved for the tile / resolve area
  int use_hist;
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* min_p;
  const float* rep;
  const float* freq;
  const float* pres;
  const int32_t* hist_off;
  const int32_t* uniq_ids;
  const int32_t* uniq_cnt;
  const int32_t* n_uniq;
  const float* uniforms;
  int32_t* tokens;
  uint8_t* kept_out;
  float* probs_out;
  uint32_t* err;
  int32_t* row_path;
};

struct __align__(16) Ctl {
  uint64_t mbar;
  uint64_t xs[2][MAXCL][4];   // scalar exchange slots, written by peers (double-buffered)
  uint64_t r64[NWARP];
  double rd[NWARP];
  float rf[NWARP];
  uint32_t r32[NWARP];
  int ri[NWARP];
  uint32_t lcount;            // local survivor count
  uint32_t pad[3];
};

template <int CL>
struct Smem {
  static constexpr int LCAP = CAP / CL;
  // layout after the tile area: Ctl | lh_cnt[NBIN+1] | lh_mass[NBIN+1] |
  //                             mh_cnt[2][NBIN+1] | mh_mass[2][NBIN+1] | lcand[LCAP]
  static constexpr int CTL = (int)((sizeof(Ctl) + 15) & ~15);
  static constexpr int LHC = ((NBIN + 1) * 4 + 15) & ~15;
  static constexpr int LHM = (NBIN + 1) * 8;
  static constexpr int MHC = 2 * LHC;
  static constexpr int MHM = 2 * LHM;
  static constexpr int LC = LCAP * 8;
  static constexpr int EXTRA = CTL + LHC + LHM + MHC + MHM + LC;
};

template <int CL>
struct Row {
  cg::cluster_group cl;
  int me, row, lo, n, n4;
  float* tile;
  Ctl* ctl;
  uint32_t* lh_cnt;
  uint64_t* lh_mass;
  uint32_t* mh_cnt;   // [2][NBIN+1]
  uint64_t* mh_mass;  // [2][NBIN+1]
  uint64_t* lcand;
  uint32_t* err;
  int xpar, hpar;

  __device__ Row() : cl(cg::this_cluster()) {}

  // Every CTA publishes four u64 values; afterwards xs[p][r][*] holds rank r's values.
  __device__ int exchange(uint64_t v0, uint64_t v1, uint64_t v2, uint64_t v3) {
    const int p = xpar;
    xpar ^= 1;
    const int t = threadIdx.x;
    if (t < CL * 4) {
      const int r = t >> 2, j = t & 3;
      uint64_t v = j == 0 ? v0 : j == 1 ? v1 : j == 2 ? v2 : v3;
      uint64_t* dst = cl.map_shared_rank(&ctl->xs[p][me][j], r);
      *dst = v;
    }
    cl.sync();
    return p;
  }
  // Adds this CTA's local histogram into every CTA's merged buffer; returns its parity.
  template <bool MASS>
  __device__ int merge_hist() {
    const int p = hpar;
    hpar ^= 1;
    __syncthreads();
    for (int i = threadIdx.x; i < CL * (NBIN + 1); i += NT) {
      const int r = i / (NBIN + 1), b = i - r * (NBIN + 1);
      uint32_t c = lh_cnt[b];
      if (c) {
        atomicAdd(cl.map_shared_rank(&mh_cnt[p * (NBIN + 1) + b], r), c);
        if (MASS) {
          unsigned long long m = lh_mass[b];
          if (m) atomicAdd((unsigned long long*)cl.map_shared_rank(&mh_mass[p * (NBIN + 1) + b], r), m);
        }
      }
    }
    cl.sync();
    return p;
  }
  __device__ void zero_merged(int p) {
    for (int i = threadIdx.x; i < NBIN + 1; i += NT) {
      mh_cnt[p * (NBIN + 1) + i] = 0;
      mh_mass[p * (NBIN + 1) + i] = 0;
    }
  }
  __device__ void zero_local() {
    for (int i = threadIdx.x; i < NBIN + 1; i += NT) {
      lh_cnt[i] = 0;
      lh_mass[i] = 0;
    }
    __syncthreads();
  }
};

// Smallest key K with exp(key2f(K) - m) >= mp (min-p keeps y with key >= K).
__device__ uint32_t minp_key(float m, float mp) {
  const uint32_t hiK = f2key(m);
  auto pred = [&](uint32_t k) { return expf(__fsub_rn(key2f(k), m)) >= mp; };
  float y0 = __fadd_rn(m, logf(mp));
  uint32_t k = f2key(y0);
  if (k < KEY_FINITE_MIN) k = KEY_FINITE_MIN;
  if (k > hiK) k = hiK;
  uint32_t lo, hi;  // binary-search bracket [lo, hi], pred(hi) true
  if (pred(k)) {
    int s = 0;
    while (s < 64 && k > KEY_FINITE_MIN && pred(k - 1)) { --k; ++s; }
    if (s < 64) return k;
    lo = KEY_FINITE_MIN;
    hi = k;
  } else {
    int s = 0;
    while (s < 64 && !pred(k)) { ++k; ++s; }
    if (s < 64) return k;
    lo = k;
    hi = hiK;
  }
  while (lo < hi) {
    uint32_t mid = lo + ((hi - lo) >> 1);
    if (pred(mid)) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// Result of a cluster-wide radix select.
struct Sel {
  bool found;     // false when the whole measure is <= target (nothing to cut)
  uint32_t K;     // key of the group that crosses the target
  uint64_t A;     // measure of all elements with key > K
  uint32_t neq;   // elements with key == K
  uint64_t eeq;   // fixed-point mass of one element at K (MASS only)
  uint64_t total; // measure of all candidate elements (key >= floorK)
};

// Finds the key group at which the descending cumulative measure (count, or fixed-point
// mass exp(y - m) * 2^40) of the elements with key >= floorK first exceeds `target`.
// For MASS the target is floor(top_p * total), computed after the first pass.
template <int CL, bool MASS>
__device__ Sel radix_select(Row<CL>& R, uint32_t floorK, float m, uint64_t target_count,
                            float tp) {
  Sel s{};
  const float4* t4 = reinterpret_cast<const float4*>(R.tile);
  // Level 0: value-space bins relative to the max.
  R.zero_local();
  {
    uint32_t far_c = 0;
    uint64_t far_m = 0;
    for (int q = threadIdx.x; q < R.n4; q += NT) {
      float4 v = t4[q];
      float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float y = ys[j];
        uint32_t k = f2key(y);
        if (k < floorK) continue;
        int b = vbin(y, m);
        uint64_t e = MASS ? efix(expf(__fsub_rn(y, m))) : 0;
        if (b < NBIN) {
          atomicAdd(&R.lh_cnt[b], 1u);
          if (MASS && e) atomicAdd((unsigned long long*)&R.lh_mass[b], (unsigned long long)e);
        } else {
          far_c++;
          far_m += e;
        }
      }
    }
    far_c = block_allreduce(far_c, SumU32(), R.ctl->r32);
    if (MASS) far_m = block_allreduce(far_m, SumU64(), R.ctl->r64);
    if (threadIdx.x == 0) {
      R.lh_cnt[NBIN] = far_c;
      R.lh_mass[NBIN] = far_m;
    }
  }
  int p = R.template merge_hist<MASS>();
  const uint32_t* hc = R.mh_cnt + p * (NBIN + 1);
  const uint64_t* hm = R.mh_mass + p * (NBIN + 1);
  uint64_t total = 0;
  for (int b = 0; b <= NBIN; ++b) total += MASS ? hm[b] : (uint64_t)hc[b];
  s.total = total;
  uint64_t target = MASS ? (uint64_t)floor((double)total * (double)tp) : target_count;
  if (total <= target) {
    s.found = false;
    __syncthreads();
    R.zero_merged(p);
    return s;
  }
  uint64_t acc = 0;
  int b0 = NBIN;
  for (int b = 0; b <= NBIN; ++b) {
    uint64_t mb = MASS ? hm[b] : (uint64_t)hc[b];
    if (acc + mb > target) { b0 = b; break; }
    acc += mb;
  }
  __syncthreads();
  R.zero_merged(p);
  // Key range that holds bin b0 (widened; the vbin predicate keeps it exact).
  const float span = fmaxf(fabsf(m), 16.0f) * 9.5367431640625e-07f;  // 2^-20 relative slack
  uint32_t lo, hi;
  if (b0 < NBIN) {
    float yhi = __fadd_rn(__fsub_rn(m, (float)b0 / BIN_PER_NAT), span);
    float ylo = __fsub_rn(__fsub_rn(m, (float)(b0 + 1) / BIN_PER_NAT), span);
    hi = min(f2key(yhi), f2key(m));
    lo = max(f2key(ylo), floorK);
  } else {
    float yhi = __fadd_rn(__fsub_rn(m, (float)NBIN / BIN_PER_NAT), span);
    hi = min(f2key(yhi), f2key(m));
    lo = floorK;
  }
  if (lo > hi) lo = hi;
  uint64_t A = acc;
  // Key-space levels.
  for (int level = 0; level < 8; ++level) {
    const uint32_t range = hi - lo;
    const int sh = range < NBIN ? 0 : (32 - __clz(range) - 8);
    R.zero_local();
    for (int q = threadIdx.x; q < R.n4; q += NT) {
      float4 v = t4[q];
      float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float y = ys[j];
        uint32_t k = f2key(y);
        if (k < lo || k > hi || k < floorK) continue;
        if (vbin(y, m) != b0) continue;
        int bb = (int)((k - lo) >> sh);
        atomicAdd(&R.lh_cnt[bb], 1u);
        if (MASS) {
          uint64_t e = efix(expf(__fsub_rn(y, m)));
          if (e) atomicAdd((unsigned long long*)&R.lh_mass[bb], (unsigned long long)e);
        }
      }
    }
    p = R.template merge_hist<MASS>();
    hc = R.mh_cnt + p * (NBIN + 1);
    hm = R.mh_mass + p * (NBIN + 1);
    const int nb = (int)(range >> sh);  // highest bin index in use
    int c = -1;
    uint64_t a2 = A;
    for (int bb = nb; bb >= 0; --bb) {
      uint64_t mb = MASS ? hm[bb] : (uint64_t)hc[bb];
      if (a2 + mb > target) { c = bb; break; }
      a2 += mb;
    }
    uint32_t cnt_c = c >= 0 ? hc[c] : 0;
    uint64_t mass_c = c >= 0 ? hm[c] : 0;
    __syncthreads();
    R.zero_merged(p);
    if (c < 0) {  // cannot happen with exact arithmetic; report and stop
      if (threadIdx.x == 0) atomicOr(R.err, LSS_FLAG_INTERNAL);
      s.found = false;
      return s;
    }
    A = a2;
    const uint32_t nlo = lo + ((uint32_t)c << sh);
    const uint32_t nhi = min(hi, nlo + ((1u << sh) - 1u));
    if (sh == 0) {
      s.found = true;
      s.K = nlo;
      s.A = A;
      s.neq = cnt_c;
      s.eeq = (MASS && cnt_c) ? mass_c / cnt_c : 0;
      return s;
    }
    lo = nlo;
    hi = nhi;
  }
  s.found = false;
  return s;
}

template <int CL, int DT>
__global__ void __launch_bounds__(NT, 2) lss_rows_kernel(const RowArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  using SM = Smem<CL>;
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  Row<CL> R;
  R.me = (int)R.cl.block_rank();
  R.row = blockIdx.x / CL;
  R.xpar = 0;
  R.hpar = 0;
  R.err = a.err;
  const int tid = threadIdx.x;
  const int row = R.row;
  const int V = a.V;
  R.lo = R.me * a.TE;
  R.n = max(0, min(V, R.lo + a.TE) - R.lo);
  R.n4 = (R.n + 3) >> 2;
  R.tile = reinterpret_cast<float*>(smem);
  unsigned char* ex = smem + a.tile_bytes;
  R.ctl = reinterpret_cast<Ctl*>(ex);
  R.lh_cnt = reinterpret_cast<uint32_t*>(ex + SM::CTL);
  R.lh_mass = reinterpret_cast<uint64_t*>(ex + SM::CTL + SM::LHC);
  R.mh_cnt = reinterpret_cast<uint32_t*>(ex + SM::CTL + SM::LHC + SM::LHM);
  R.mh_mass = reinterpret_cast<uint64_t*>(ex + SM::CTL + SM::LHC + SM::LHM + SM::MHC);
  R.lcand = reinterpret_cast<uint64_t*>(ex + SM::CTL + SM::LHC + SM::LHM + SM::MHC + SM::MHM);
  float* tile = R.tile;
  Ctl* ctl = R.ctl;
  const int lo = R.lo, n = R.n, n4 = R.n4;

  // ---- zero the merged histograms (peers add into them after the first cluster barrier)
  for (int i = tid; i < 2 * (NBIN + 1); i += NT) {
    R.mh_cnt[i] = 0;
    R.mh_mass[i] = 0;
  }

  // ---- stage this CTA's slice of the row in shared memory
  const char* g0 = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
  const bool bulk = n > 0 && ((reinterpret_cast<uintptr_t>(g0) & 15) == 0);
  const int nbytes = bulk ? ((n * ES) & ~15) : 0;
  const int nbulk = nbytes / ES;
  if (tid == 0) {
    mbar_init(&ctl->mbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0 && nbytes > 0) {
    mbar_expect_tx(&ctl->mbar, (uint32_t)nbytes);
    constexpr int CH = 32768;
    for (int off = 0; off < nbytes; off += CH)
      bulk_g2s(reinterpret_cast<unsigned char*>(tile) + off, g0 + off, (uint32_t)min(CH, nbytes - off),
               &ctl->mbar);
  }
  // Every CTA of the cluster must be running before any distributed-shared-memory access.
  R.cl.sync();
  // Elements the bulk copy does not cover (ragged tail / unaligned rows): plain loads.
  auto load_elem = [&](int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(g0)[i];
    if (DT == LSS_DTYPE_BF16)
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g0)[i]);
    return __half2float(reinterpret_cast<const __half*>(g0)[i]);
  };
  float tailv[1];
  const int ntail = n - nbulk;  // < 8 when bulk, else n
  if (DT == LSS_DTYPE_F32 || !bulk) {
    for (int i = nbulk + tid; i < n; i += NT) tile[i] = load_elem(i);
  } else {
    tailv[0] = (tid < ntail) ? load_elem(nbulk + tid) : 0.0f;
  }
  if (nbytes > 0) {
    if (!mbar_wait_bounded(&ctl->mbar, 0) && tid == 0) atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
  }
  if (DT != LSS_DTYPE_F32 && nbulk > 0) {
    // Widen 16-bit values in place, back to front: chunk c's f32 writes only
    // overwrite 16-bit data of chunks >= 2c, which earlier iterations consumed.
    const uint16_t* h = reinterpret_cast<const uint16_t*>(tile);
    constexpr int W = NT * 8;
    const int nch = (nbulk + W - 1) / W;
    for (int c = nch - 1; c >= 0; --c) {
      const int i0 = c * W + tid * 8;
      float v[8];
      const bool act = i0 < nbulk;  // nbulk is a multiple of 8
      if (act) {
        uint4 raw = *reinterpret_cast<const uint4*>(h + i0);
        uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint16_t l16 = (uint16_t)(w[j] & 0xffffu), h16 = (uint16_t)(w[j] >> 16);
          if (DT == LSS_DTYPE_BF16) {
            v[2 * j] = __uint_as_float((uint32_t)l16 << 16);
            v[2 * j + 1] = __uint_as_float((uint32_t)h16 << 16);
          } else {
            v[2 * j] = __half2float(__ushort_as_half(l16));
            v[2 * j + 1] = __half2float(__ushort_as_half(h16));
          }
        }
      }
      __syncthreads();
      if (act) {
        float4* d = reinterpret_cast<float4*>(tile + i0);
        d[0] = make_float4(v[0], v[1], v[2], v[3]);
        d[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
    __syncthreads();
    if (tid < ntail) tile[nbulk + tid] = tailv[0];
  }
  // Pad to a whole float4 with -inf (never a survivor, never the argmax of a real row).
  if (tid < n4 * 4 - n) tile[n + tid] = -INFINITY;
  __syncthreads();

  const float T = a.temperature[row];
  const bool greedy = T <= 0.0f;
  float4* t4 = reinterpret_cast<float4*>(tile);

  if (greedy) {
    uint64_t best = 0;
    for (int q = tid; q < n4; q += NT) {
      float4 v = t4[q];
      const int i = lo + 4 * q;
      best = max(best, argmax_code(v.x, i));
      best = max(best, argmax_code(v.y, i + 1));
      best = max(best, argmax_code(v.z, i + 2));
      best = max(best, argmax_code(v.w, i + 3));
    }
    best = block_allreduce(best, MaxU64(), ctl->r64);
    const int p = R.exchange(best, 0, 0, 0);
    if (R.me == 0 && tid == 0) {
      uint64_t b = 0;
      for (int r = 0; r < CL; ++r) b = max(b, ctl->xs[p][r][0]);
      a.tokens[row] = (int32_t)(~(uint32_t)b);
      a.row_path[row] = LSS_PATH_GREEDY;
    }
    return;
  }

  // ---- penalties (sampling.py:55-66), then y = z / T (sampling.py:146) and the row max
  if (a.use_hist) {
    const int nu = a.n_uniq[row];
    if (nu > 0) {
      const int base = a.hist_off[row];
      const float rp = a.rep[row], fq = a.freq[row], pr = a.pres[row];
      const bool do_rep = rp != 1.0f, do_add = (fq != 0.0f || pr != 0.0f);
      for (int j = tid; j < nu; j += NT) {
        const int id = a.uniq_ids[base + j];
        if (id >= lo && id < lo + n) {
          float v = tile[id - lo];
          if (do_rep) v = v > 0.0f ? __fdiv_rn(v, rp) : __fmul_rn(v, rp);
          if (do_add) v = __fsub_rn(v, __fadd_rn(__fmul_rn(fq, (float)a.uniq_cnt[base + j]), pr));
          tile[id - lo] = v;
        }
      }
      __syncthreads();
    }
  }
  float lmax = -INFINITY;
  for (int q = tid; q < n4; q += NT) {
    float4 v = t4[q];
    const int i = 4 * q;
    v.x = __fdiv_rn(v.x, T);
    v.y = __fdiv_rn(v.y, T);
    v.z = __fdiv_rn(v.z, T);
    v.w = __fdiv_rn(v.w, T);
    if (i + 3 >= n) {  // keep the -inf padding
      if (i + 1 >= n) v.y = -INFINITY;
      if (i + 2 >= n) v.z = -INFINITY;
      if (i + 3 >= n) v.w = -INFINITY;
    }
    lmax = fmax_nan(lmax, fmax_nan(fmax_nan(v.x, v.y), fmax_nan(v.z, v.w)));
    t4[q] = v;
  }
  lmax = block_allreduce(lmax, MaxF(), ctl->rf);
  int p = R.exchange((uint64_t)__float_as_uint(lmax), 0, 0, 0);
  float m = -INFINITY;
  for (int r = 0; r < CL; ++r) m = fmax_nan(m, __uint_as_float((uint32_t)ctl->xs[p][r][0]));

  if (!(m == m) || m == INFINITY || m == -INFINITY) {
    // NaN guard (sampling.py:159-160): argmax of y with NaN largest, lowest index.
    uint64_t best = 0;
    for (int q = tid; q < n4; q += NT) {
      float4 v = t4[q];
      const int i = lo + 4 * q;
      best = max(best, argmax_code(v.x, i));
      best = max(best, argmax_code(v.y, i + 1));
      best = max(best, argmax_code(v.z, i + 2));
      best = max(best, argmax_code(v.w, i + 3));
    }
    best = block_allreduce(best, MaxU64(), ctl->r64);
    p = R.exchange(best, 0, 0, 0);
    if (R.me == 0 && tid == 0) {
      uint64_t b = 0;
      for (int r = 0; r < CL; ++r) b = max(b, ctl->xs[p][r][0]);
      a.tokens[row] = (int32_t)(~(uint32_t)b);
      a.row_path[row] = LSS_PATH_SPECIAL;
    }
    return;
  }

  // ---- per-row filter parameters
  const int k = a.top_k[row];
  const float mp = a.min_p[row], tp = a.top_p[row];
  const bool tk_on = k > 0 && k < V;
  const bool mp_on = mp > 0.0f && mp < 1.0f;
  const bool tp_on = tp > 0.0f && tp < 1.0f;
  const float u = a.uniforms[row];
  const uint32_t Kmp = mp_on ? minp_key(m, mp) : KEY_FINITE_MIN;

  // ---- top-k window from a value-space count histogram (elements with key >= Kmp)
  bool tk_bind = false;  // top-k cuts inside the min-p survivors
  int bk = NBIN;         // window: vbin <= bk
  bool need_dense = false;
  if (tk_on) {
    R.zero_local();
    uint32_t far_c = 0;
    for (int q = tid; q < n4; q += NT) {
      float4 v = t4[q];
      float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (f2key(ys[j]) < Kmp) continue;
        int b = vbin(ys[j], m);
        if (b < NBIN) atomicAdd(&R.lh_cnt[b], 1u); else far_c++;
      }
    }
    far_c = block_allreduce(far_c, SumU32(), ctl->r32);
    if (tid == 0) R.lh_cnt[NBIN] = far_c;
    const int hp = R.template merge_hist<false>();
    const uint32_t* hc = R.mh_cnt + hp * (NBIN + 1);
    uint32_t acc = 0;
    int b = 0;
    for (; b < NBIN; ++b) {
      acc += hc[b];
      if (acc >= (uint32_t)k) break;
    }
    uint32_t total = acc;
    if (b == NBIN) total += hc[NBIN];
    if (b < NBIN) {
      tk_bind = true;
      bk = b;
    } else if (total > (uint32_t)k) {
      need_dense = true;  // the k-th largest is more than 16 nats below the max
    }
    __syncthreads();
    R.zero_merged(hp);
  }

  // ---- compaction of the window into a local list
  if (!need_dense) {
    if (tid == 0) ctl->lcount = 0;
    __syncthreads();
    const int lane = tid & 31;
    for (int q = tid; q - lane < n4; q += NT) {  // warp-uniform trip count
      float4 v = q < n4 ? t4[q] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t key = f2key(ys[j]);
        bool keep = key >= Kmp && ys[j] > -INFINITY && (!tk_bind || vbin(ys[j], m) <= bk);
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (bal) {
          uint32_t base = 0;
          const int leader = __ffs(bal) - 1;
          if (lane == leader) base = atomicAdd(&ctl->lcount, (uint32_t)__popc(bal));
          base = __shfl_sync(0xffffffffu, base, leader);
          if (keep) {
            const uint32_t pos = base + __popc(bal & ((1u << lane) - 1u));
            if (pos < (uint32_t)SM::LCAP)
              R.lcand[pos] = ((uint64_t)key << 32) | (uint32_t)(~(uint32_t)(lo + 4 * q + j));
          }
        }
      }
    }
    __syncthreads();
  }
  const uint32_t lcount = need_dense ? 0xffffffffu : ctl->lcount;
  p = R.exchange(lcount, 0, 0, 0);
  uint32_t total = 0, before = 0;
  bool overflow = need_dense;
  for (int r = 0; r < CL; ++r) {
    const uint32_t c = (uint32_t)ctl->xs[p][r][0];
    if (c > (uint32_t)SM::LCAP) overflow = true;
    if (r < R.me) before += c;
    total += c;
  }

  if (!overflow) {
    // ---- gather: push the local lists into CTA 0's tile area, then CTA 0 resolves.
    uint64_t* G = reinterpret_cast<uint64_t*>(tile);
    uint64_t* Gdst = R.cl.map_shared_rank(G, 0);
    for (uint32_t i = tid; i < lcount; i += NT) Gdst[before + i] = R.lcand[i];
    R.cl.sync();
    if (R.me != 0) return;

    const int nc = (int)total;
    const int np = next_pow2(max(nc, 1));
    for (int i = nc + tid; i < np; i += NT) G[i] = 0ull;
    __syncthreads();
    bitonic_sort(G, np, true);  // key desc, index asc
    float* E = reinterpret_cast<float*>(tile) + 2 * CAP;  // after G[CAP]
    // top-k cut (ties kept, sampling.py:85)
    int n1 = nc;
    if (tk_bind && k <= nc) {
      const uint32_t Kk = (uint32_t)(G[k - 1] >> 32);
      uint32_t c = 0;
      for (int i = tid; i < nc; i += NT) c += ((uint32_t)(G[i] >> 32) >= Kk) ? 1u : 0u;
      n1 = (int)block_allreduce(c, SumU32(), ctl->r32);
    }
    // e_j = exp(y_j - m); S in f64 (thread-ordered, deterministic)
    constexpr int PER = CAP / NT;  // 8 items per thread, contiguous
    double part = 0.0;
    for (int j = 0; j < PER; ++j) {
      const int i = tid * PER + j;
      float e = 0.0f;
      if (i < n1) e = expf(__fsub_rn(key2f((uint32_t)(G[i] >> 32)), m));
      E[i] = e;
      part += (double)e;
    }
    double S = block_allreduce(part, SumD(), ctl->rd);
    int n2 = n1;
    if (tp_on && n1 > 1) {
      // top-p (sampling.py:98-108): p = e / S (f32), c = cumsum in f64 rounded to f32,
      // token j kept iff j == 0 or c_{j-1} <= top_p.
      const float S32 = (float)S;
      double loc[PER];
      double run = 0.0;
      for (int j = 0; j < PER; ++j) {
        const int i = tid * PER + j;
        const double pj = i < n1 ? (double)__fdiv_rn(E[i], S32) : 0.0;
        run += pj;
        loc[j] = run;
      }
      double tot;
      const double pre = block_excl_scan(run, ctl->rd, tot);
      uint32_t c = 0;
      for (int j = 0; j < PER; ++j) {
        const int i = tid * PER + j;
        if (i < n1 - 1 && (float)(pre + loc[j]) <= tp) c++;
      }
      n2 = 1 + (int)block_allreduce(c, SumU32(), ctl->r32);
      if (n2 > n1) n2 = n1;
      double part2 = 0.0;
      for (int j = 0; j < PER; ++j) {
        const int i = tid * PER + j;
        if (i < n2) part2 += (double)E[i];
      }
      S = block_allreduce(part2, SumD(), ctl->rd);
    }
    // final probabilities (sampling.py:157) and the draw in vocabulary order
    const float Sf = (float)S;
    __syncthreads();
    for (int i = tid; i < CAP; i += NT) {
      if (i < n2) {
        const uint32_t idx = ~(uint32_t)G[i];
        const float pr = __fdiv_rn(E[i], Sf);
        G[i] = ((uint64_t)idx << 32) | __float_as_uint(pr);
        if (a.kept_out) a.kept_out[(int64_t)row * V + idx] = 1;
        if (a.probs_out) a.probs_out[(int64_t)row * V + idx] = pr;
      }
    }
    const int np2 = next_pow2(max(n2, 1));
    for (int i = n2 + tid; i < np2; i += NT) G[i] = ~0ull;
    __syncthreads();
    bitonic_sort(G, np2, false);  // index asc
    double loc[PER];
    double run = 0.0;
    for (int j = 0; j < PER; ++j) {
      const int i = tid * PER + j;
      run += i < n2 ? (double)__uint_as_float((uint32_t)G[i]) : 0.0;
      loc[j] = run;
    }
    double tot;
    const double pre = block_excl_scan(run, ctl->rd, tot);
    const double target = (double)u * tot;
    int first = 0x7fffffff;
    for (int j = 0; j < PER; ++j) {
      const int i = tid * PER + j;
      if (i < n2 && pre + loc[j] > target) { first = i; break; }
    }
    first = block_allreduce(first, MinI(), ctl->ri);
    if (tid == 0) {
      if (first >= n2) first = n2 - 1;
      a.tokens[row] = (int32_t)(G[first] >> 32);
      a.row_path[row] = LSS_PATH_GATHER;
    }
    return;
  }

  // ---- dense path: exact cuts by cluster-wide radix select over the whole row
  uint32_t Klo = Kmp;
  if (tk_on) {
    Sel sk = radix_select<CL, false>(R, Kmp, m, (uint64_t)(k - 1), 0.0f);
    if (sk.found && sk.K > Klo) Klo = sk.K;
  }
  bool cut = false;
  uint32_t Kp = 0;
  uint64_t eeq = 0;
  uint32_t rmax = 0;
  if (tp_on) {
    Sel sp = radix_select<CL, true>(R, Klo, m, 0, tp);
    if (sp.found) {
      cut = true;
      Kp = sp.K;
      eeq = sp.eeq;
      const uint64_t target = (uint64_t)floor((double)sp.total * (double)tp);
      uint64_t r = (eeq > 0) ? (target - sp.A) / eeq + 1 : (uint64_t)sp.neq;
      rmax = (uint32_t)(r < (uint64_t)sp.neq ? r : (uint64_t)sp.neq);
    }
  }
  // Per-CTA kept mass (excluding the tie group at the cut) and tie counts.
  uint64_t Mc = 0;
  uint32_t tc = 0;
  for (int q = tid; q < n4; q += NT) {
    float4 v = t4[q];
    float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t key = f2key(ys[j]);
      if (key < Klo || !(ys[j] > -INFINITY)) continue;
      if (cut && key < Kp) continue;
      if (cut && key == Kp) { tc++; continue; }
      Mc += efix(expf(__fsub_rn(ys[j], m)));
    }
  }
  Mc = block_allreduce(Mc, SumU64(), ctl->r64);
  tc = block_allreduce(tc, SumU32(), ctl->r32);
  p = R.exchange(Mc, tc, 0, 0);
  uint64_t Mall[MAXCL];
  uint32_t allow_me = 0;
  uint64_t Sfix = 0, Pme = 0;
  {
    uint32_t tprev = 0;
    for (int r = 0; r < CL; ++r) {
      const uint64_t mr = ctl->xs[p][r][0];
      const uint32_t tr = (uint32_t)ctl->xs[p][r][1];
      uint32_t al = 0;
      if (cut) al = rmax > tprev ? min(rmax - tprev, tr) : 0u;
      tprev += tr;
      Mall[r] = mr + (uint64_t)al * eeq;
      if (r == R.me) allow_me = al;
      if (r < R.me) Pme += Mall[r];
      Sfix += Mall[r];
    }
  }
  uint64_t target = (uint64_t)floor((double)u * (double)Sfix);
  if (target >= Sfix) target = Sfix ? Sfix - 1 : 0;
  // The CTA whose slice holds the target scans it in vocabulary order.
  int owner = CL - 1;
  {
    uint64_t acc = 0;
    for (int r = 0; r < CL; ++r) {
      if (Mall[r] > 0 && target < acc + Mall[r]) { owner = r; break; }
      acc += Mall[r];
    }
    if (Sfix == 0) owner = 0;
  }
  const bool scan_me = (R.me == owner) || a.kept_out || a.probs_out;
  if (scan_me) {
    const float Sf = (float)((double)Sfix / FIX_ONE);
    uint64_t run_base = Pme;
    uint32_t tie_base = 0;
    int found = 0x7fffffff;
    for (int c0 = 0; c0 < n4 * 4; c0 += NT * 4) {
      const int i0 = c0 + tid * 4;
      float ys[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (i0 < n4 * 4) {
        float4 v = t4[i0 >> 2];
        ys[0] = v.x; ys[1] = v.y; ys[2] = v.z; ys[3] = v.w;
      }
      uint32_t keyv[4];
      uint32_t ties = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        keyv[j] = f2key(ys[j]);
        if (cut && keyv[j] == Kp && keyv[j] >= Klo && ys[j] > -INFINITY) ties++;
      }
      uint32_t ttot;
      const uint32_t tpre = block_excl_scan(ties, ctl->r32, ttot) + tie_base;
      uint64_t mloc[4];
      uint64_t msum = 0;
      uint32_t tseen = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bool kept = keyv[j] >= Klo && ys[j] > -INFINITY;
        if (kept && cut) {
          if (keyv[j] < Kp) kept = false;
          else if (keyv[j] == Kp) { kept = (tpre + tseen) < allow_me; tseen++; }
        }
        mloc[j] = kept ? efix(expf(__fsub_rn(ys[j], m))) : 0;
        msum += mloc[j];
        if (kept && (a.kept_out || a.probs_out)) {
          const int64_t o = (int64_t)row * V + lo + i0 + j;
          if (a.kept_out) a.kept_out[o] = 1;
          if (a.probs_out) a.probs_out[o] = __fdiv_rn(expf(__fsub_rn(ys[j], m)), Sf);
        }
      }
      uint64_t mtot;
      const uint64_t mpre = block_excl_scan(msum, ctl->r64, mtot) + run_base;
      if (R.me == owner && found == 0x7fffffff) {
        int f = 0x7fffffff;
        uint64_t run = mpre;
        for (int j = 0; j < 4; ++j) {
          run += mloc[j];
          if (mloc[j] > 0 && run > target) { f = lo + i0 + j; break; }
        }
        f = block_allreduce(f, MinI(), ctl->ri);
        found = f;
      }
      run_base += mtot;
      tie_base += ttot;
    }
    if (R.me == owner && tid == 0) {
      a.tokens[row] = found == 0x7fffffff ? (int32_t)(lo + n - 1) : found;
      a.row_path[row] = LSS_PATH_DENSE;
    }
  }
}

// ---------------------------------------------------------------------------
// Batched greedy argmax: CL CTAs per row stream the row with 16-byte loads.
// ---------------------------------------------------------------------------
template <int CL, int DT>
__global__ void __launch_bounds__(NT) lss_argmax_kernel(const void* logits, int64_t row_stride, int V,
                                                        int TE, int32_t* tokens) {
  __shared__ uint64_t scr[NWARP];
  __shared__ uint64_t slots[MAXCL];
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  cg::cluster_group cl = cg::this_cluster();
  const int me = (int)cl.block_rank();
  const int row = blockIdx.x / CL;
  const int lo = me * TE;
  const int n = max(0, min(V, lo + TE) - lo);
  const char* g0 = reinterpret_cast<const char*>(logits) + ((int64_t)row * row_stride + lo) * ES;
  cl.sync();  // all CTAs of the cluster are running before slots[] is written remotely
  uint64_t best = 0;
  auto val = [&](int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(g0)[i];
    if (DT == LSS_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g0)[i]);
    return __half2float(reinterpret_cast<const __half*>(g0)[i]);
  };
  constexpr int VE = 16 / ES;  // elements per 16-byte vector
  int head = 0;
  if ((reinterpret_cast<uintptr_t>(g0) & 15) != 0) head = n;  // unaligned rows: scalar path
  const int nvec = (n - head) / VE;
  for (int i = threadIdx.x; i < head; i += NT) best = max(best, argmax_code(val(i), lo + i));
  for (int q = threadIdx.x; q < nvec; q += NT) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(g0) + q);
    const int i = lo + q * VE;
    uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    if (DT == LSS_DTYPE_F32) {
#pragma unroll
      for (int j = 0; j < 4; ++j) best = max(best, argmax_code(__uint_as_float(w[j]), i + j));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a0, a1;
        if (DT == LSS_DTYPE_BF16) {
          a0 = __uint_as_float(w[j] << 16);
          a1 = __uint_as_float(w[j] & 0xffff0000u);
        } else {
          a0 = __half2float(__ushort_as_half((uint16_t)(w[j] & 0xffffu)));
          a1 = __half2float(__ushort_as_half((uint16_t)(w[j] >> 16)));
        }
        best = max(best, argmax_code(a0, i + 2 * j));
        best = max(best, argmax_code(a1, i + 2 * j + 1));
      }
    }
  }
  for (int i = head + nvec * VE + threadIdx.x; i < n; i += NT) best = max(best, argmax_code(val(i), lo + i));
  best = block_allreduce(best, MaxU64(), scr);
  if (threadIdx.x < CL) *cl.map_shared_rank(&slots[me], (int)threadIdx.x) = best;
  cl.sync();
  if (me == 0 && threadIdx.x == 0) {
    uint64_t b = 0;
    for (int r = 0; r < CL; ++r) b = max(b, slots[r]);
    tokens[row] = (int32_t)(~(uint32_t)b);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
constexpr int TILE_TARGET_BYTES = 80 * 1024;   // two CTAs per SM
constexpr int TILE_MAX_BYTES = 160 * 1024;     // one CTA per SM
constexpr int MAX_VOCAB = MAXCL * (TILE_MAX_BYTES / 4);

struct Plan {
  int CL, TE, tile_bytes, smem;
};

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

static Plan make_plan(int V) {
  Plan pl{};
  int CL = 1;
  while (CL < MAXCL && round_up((V + CL - 1) / CL, 16) * 4 > TILE_TARGET_BYTES) CL <<= 1;
  const int TE = round_up((V + CL - 1) / CL, 16);
  pl.CL = CL;
  pl.TE = TE;
  pl.tile_bytes = round_up(std::max(TE * 4, RES_BYTES), 1024);
  int extra = 0;
  switch (CL) {
    case 1: extra = Smem<1>::EXTRA; break;
    case 2: extra = Smem<2>::EXTRA; break;
    case 4: extra = Smem<4>::EXTRA; break;
    default: extra = Smem<8>::EXTRA; break;
  }
  pl.smem = pl.tile_bytes + extra;
  return pl;
}

struct WsLayout {
  size_t header, row_path, n_uniq, uniq_ids, uniq_cnt, gkeys, gcnts, total;
};
static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }
static WsLayout ws_layout(int B, int64_t H) {
  WsLayout L{};
  size_t o = 0;
  L.header = o; o += 256;
  L.row_path = o; o = align256(o + sizeof(int32_t) * (size_t)std::max(B, 1));
  L.n_uniq = o; o = align256(o + sizeof(int32_t) * (size_t)std::max(B, 1));
  L.uniq_ids = o; o = align256(o + sizeof(int32_t) * (size_t)std::max<int64_t>(H, 1));
  L.uniq_cnt = o; o = align256(o + sizeof(int32_t) * (size_t)std::max<int64_t>(H, 1));
  L.gkeys = o; o = align256(o + sizeof(uint32_t) * 2 * (size_t)std::max<int64_t>(H, 1));
  L.gcnts = o; o = align256(o + sizeof(uint32_t) * 2 * (size_t)std::max<int64_t>(H, 1));
  L.total = o;
  return L;
}

template <int CL, int DT>
static cudaError_t launch_rows(const RowArgs& a, const Plan& pl, int B, cudaStream_t st) {
  auto kern = lss_rows_kernel<CL, DT>;
  static int configured_smem[64] = {0};   // per template instance and device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (configured_smem[dev] < pl.smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
    if (e != cudaSuccess) return e;
    configured_smem[dev] = pl.smem;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(B * CL), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = (size_t)pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int DT>
static cudaError_t launch_rows_dt(const RowArgs& a, const Plan& pl, int B, cudaStream_t st) {
  switch (pl.CL) {
    case 1: return launch_rows<1, DT>(a, pl, B, st);
    case 2: return launch_rows<2, DT>(a, pl, B, st);
    case 4: return launch_rows<4, DT>(a, pl, B, st);
    default: return launch_rows<8, DT>(a, pl, B, st);
  }
}

template <int CL, int DT>
static cudaError_t launch_argmax(const void* logits, int64_t stride, int B, int V, int TE, int32_t* tok,
                                 cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(B * CL), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lss_argmax_kernel<CL, DT>, logits, stride, V, TE, tok);
}

template <int DT>
static cudaError_t launch_argmax_dt(const void* logits, int64_t stride, int B, int V, int32_t* tok,
                                    cudaStream_t st) {
  // Enough CTAs to cover the machine: split rows until B * CL >= 2 * 148 or slices get small.
  int CL = 1;
  while (CL < MAXCL && B * CL < 296 && (V + CL - 1) / CL > 4096) CL <<= 1;
  const int TE = round_up((V + CL - 1) / CL, 16);
  switch (CL) {
    case 1: return launch_argmax<1, DT>(logits, stride, B, V, TE, tok, st);
    case 2: return launch_argmax<2, DT>(logits, stride, B, V, TE, tok, st);
    case 4: return launch_argmax<4, DT>(logits, stride, B, V, TE, tok, st);
    default: return launch_argmax<8, DT>(logits, stride, B, V, TE, tok, st);
  }
}

}  // namespace lss

using namespace lss;

extern "C" {

int lss_version(void) { return (0 << 16) | (1 << 8) | 0; }

const char* lss_status_string(int s) {
  switch (s) {
    case LSS_OK: return "ok";
    case LSS_ERR_INVALID_ARG: return "invalid argument";
    case LSS_ERR_WORKSPACE: return "workspace missing or too small";
    case LSS_ERR_CUDA: return "CUDA runtime error";
    case LSS_ERR_UNSUPPORTED: return "unsupported size or device";
    case LSS_ERR_DEVICE: return "device reported an error flag";
    case LSS_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch of lss_sample_noalloc";
    default: return "unknown status";
  }
}

int lss_max_vocab(void) { return MAX_VOCAB; }

size_t lss_workspace_bytes(int B, int V, int64_t hist_total) {
  (void)V;
  if (B < 0 || hist_total < 0) return 0;
  return ws_layout(B, hist_total).total;
}

static int check_common(int B, int V, int64_t hist_total, const int32_t* hist_offsets,
                        const void* workspace, size_t workspace_bytes) {
  if (B < 0 || V < 1 || hist_total < 0 || hist_total > 0x3fffffff) return LSS_ERR_INVALID_ARG;
  if (V > MAX_VOCAB) return LSS_ERR_UNSUPPORTED;
  if (B == 0) return LSS_OK;
  if (hist_total > 0 && !hist_offsets) return LSS_ERR_INVALID_ARG;
  const WsLayout L = ws_layout(B, hist_total);
  if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return LSS_ERR_WORKSPACE;
  return LSS_OK;
}

int lss_history_prepare(int B, int V, const int32_t* hist_offsets, const int32_t* hist_ids,
                        int64_t hist_total, const float* temperature, const float* repetition_penalty,
                        const float* frequency_penalty, const float* presence_penalty, void* workspace,
                        size_t workspace_bytes, void* stream) {
  int rc = check_common(B, V, hist_total, hist_offsets, workspace, workspace_bytes);
  if (rc != LSS_OK || B == 0) return rc;
  if (hist_total > 0 && (!hist_ids || !temperature || !repetition_penalty || !frequency_penalty ||
                         !presence_penalty))
    return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  const WsLayout L = ws_layout(B, hist_total);
  if (cudaMemsetAsync(ws + L.header, 0, 256, st) != cudaSuccess) return LSS_ERR_CUDA;
  if (hist_total > 0) {
    lss_hist_dedup<<<B, 256, 0, st>>>(hist_offsets, hist_ids, V, temperature, repetition_penalty,
                                      frequency_penalty, presence_penalty,
                                      reinterpret_cast<int32_t*>(ws + L.uniq_ids),
                                      reinterpret_cast<int32_t*>(ws + L.uniq_cnt),
                                      reinterpret_cast<int32_t*>(ws + L.n_uniq),
                                      reinterpret_cast<uint32_t*>(ws + L.gkeys),
                                      reinterpret_cast<uint32_t*>(ws + L.gcnts),
                                      reinterpret_cast<uint32_t*>(ws + L.header));
    if (cudaGetLastError() != cudaSuccess) return LSS_ERR_CUDA;
  }
  return LSS_OK;
}

int lss_sample_rows(const void* logits, int dtype, int B, int V, int64_t row_stride,
                    const float* temperature, const int32_t* top_k, const float* top_p,
                    const float* min_p, const float* repetition_penalty, const float* frequency_penalty,
                    const float* presence_penalty, const int32_t* hist_offsets, int64_t hist_total,
                    const float* uniforms, int32_t* tokens_out, uint8_t* kept_out, float* probs_out,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (row_stride < V) return LSS_ERR_INVALID_ARG;
  if (dtype != LSS_DTYPE_F32 && dtype != LSS_DTYPE_BF16 && dtype != LSS_DTYPE_F16) return LSS_ERR_INVALID_ARG;
  int rc = check_common(B, V, hist_total, hist_offsets, workspace, workspace_bytes);
  if (rc != LSS_OK || B == 0) return rc;
  if (!logits || !temperature || !top_k || !top_p || !min_p || !repetition_penalty || !frequency_penalty ||
      !presence_penalty || !uniforms || !tokens_out)
    return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  const WsLayout L = ws_layout(B, hist_total);
  const Plan pl = make_plan(V);
  if (kept_out && cudaMemsetAsync(kept_out, 0, (size_t)B * V, st) != cudaSuccess) return LSS_ERR_CUDA;
  if (probs_out && cudaMemsetAsync(probs_out, 0, (size_t)B * V * sizeof(float), st) != cudaSuccess)
    return LSS_ERR_CUDA;
  RowArgs a{};
  a.logits = logits;
  a.row_stride = row_stride;
  a.B = B;
  a.V = V;
  a.TE = pl.TE;
  a.tile_bytes = pl.tile_bytes;
  a.use_hist = hist_total > 0 ? 1 : 0;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.min_p = min_p;
  a.rep = repetition_penalty;
  a.freq = frequency_penalty;
  a.pres = presence_penalty;
  a.hist_off = hist_offsets;
  a.uniq_ids = reinterpret_cast<int32_t*>(ws + L.uniq_ids);
  a.uniq_cnt = reinterpret_cast<int32_t*>(ws + L.uniq_cnt);
  a.n_uniq = reinterpret_cast<int32_t*>(ws + L.n_uniq);
  a.uniforms = uniforms;
  a.tokens = tokens_out;
  a.kept_out = kept_out;
  a.probs_out = probs_out;
  a.err = reinterpret_cast<uint32_t*>(ws + L.header);
  a.row_path = reinterpret_cast<int32_t*>(ws + L.row_path);
  cudaError_t e;
  switch (dtype) {
    case LSS_DTYPE_F32: e = launch_rows_dt<LSS_DTYPE_F32>(a, pl, B, st); break;
    case LSS_DTYPE_BF16: e = launch_rows_dt<LSS_DTYPE_BF16>(a, pl, B, st); break;
    default: e = launch_rows_dt<LSS_DTYPE_F16>(a, pl, B, st); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return LSS_ERR_CUDA;
  }
  return LSS_OK;
}

int lss_sample(const void* logits, int dtype, int B, int V, int64_t row_stride, const float* temperature,
               const int32_t* top_k, const float* top_p, const float* min_p,
               const float* repetition_penalty, const float* frequency_penalty,
               const float* presence_penalty, const int32_t* hist_offsets, const int32_t* hist_ids,
               int64_t hist_total, const float* uniforms, int32_t* tokens_out, uint8_t* kept_out,
               float* probs_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (row_stride < V) return LSS_ERR_INVALID_ARG;
  if (dtype != LSS_DTYPE_F32 && dtype != LSS_DTYPE_BF16 && dtype != LSS_DTYPE_F16) return LSS_ERR_INVALID_ARG;
  int rc = check_common(B, V, hist_total, hist_offsets, workspace, workspace_bytes);
  if (rc != LSS_OK || B == 0) return rc;
  if (!logits || !temperature || !top_k || !top_p || !min_p || !repetition_penalty || !frequency_penalty ||
      !presence_penalty || !uniforms || !tokens_out)
    return LSS_ERR_INVALID_ARG;
  if (hist_total > 0 && !hist_ids) return LSS_ERR_INVALID_ARG;
  rc = lss_history_prepare(B, V, hist_offsets, hist_ids, hist_total, temperature, repetition_penalty,
                           frequency_penalty, presence_penalty, workspace, workspace_bytes, stream);
  if (rc != LSS_OK) return rc;
  return lss_sample_rows(logits, dtype, B, V, row_stride, temperature, top_k, top_p, min_p,
                         repetition_penalty, frequency_penalty, presence_penalty, hist_offsets, hist_total,
                         uniforms, tokens_out, kept_out, probs_out, workspace, workspace_bytes, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant: the workspace is a fixed file-scope device array.
// ---------------------------------------------------------------------------
namespace lss {
static __device__ __align__(256) unsigned char g_noalloc_scratch[LSS_NOALLOC_SCRATCH_BYTES];
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch on the current device, looked up once per device.
static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LSS_ERR_CUDA;
  if (dev < 0 || dev >= 64) return LSS_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return LSS_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return LSS_OK;
}
}  // namespace lss

extern "C" {

int lss_sample_noalloc(const void* logits, int dtype, int B, int V, int64_t row_stride,
                       const float* temperature, const int32_t* top_k, const float* top_p,
                       const float* min_p, const float* repetition_penalty,
                       const float* frequency_penalty, const float* presence_penalty,
                       const int32_t* hist_offsets, const int32_t* hist_ids, int64_t hist_total,
                       const float* uniforms, int32_t* tokens_out, uint8_t* kept_out, float* probs_out,
                       void* stream) {
  if (B < 0 || V < 1 || hist_total < 0) return LSS_ERR_INVALID_ARG;
  if (B == 0) return LSS_OK;
  const size_t need = lss_workspace_bytes(B, V, hist_total);
  if (need == 0) return LSS_ERR_INVALID_ARG;
  if (need > (size_t)LSS_NOALLOC_SCRATCH_BYTES) return LSS_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  int rc = lss::noalloc_scratch(&ws);
  if (rc != LSS_OK) return rc;
  return lss_sample(logits, dtype, B, V, row_stride, temperature, top_k, top_p, min_p, repetition_penalty,
                    frequency_penalty, presence_penalty, hist_offsets, hist_ids, hist_total, uniforms,
                    tokens_out, kept_out, probs_out, ws, (size_t)LSS_NOALLOC_SCRATCH_BYTES, stream);
}

int lss_argmax(const void* logits, int dtype, int B, int V, int64_t row_stride, int32_t* tokens_out,
               void* stream) {
  if (B < 0 || V < 1 || row_stride < V) return LSS_ERR_INVALID_ARG;
  if (dtype != LSS_DTYPE_F32 && dtype != LSS_DTYPE_BF16 && dtype != LSS_DTYPE_F16) return LSS_ERR_INVALID_ARG;
  if (B == 0) return LSS_OK;
  if (!logits || !tokens_out) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (dtype) {
    case LSS_DTYPE_F32: e = launch_argmax_dt<LSS_DTYPE_F32>(logits, row_stride, B, V, tokens_out, st); break;
    case LSS_DTYPE_BF16: e = launch_argmax_dt<LSS_DTYPE_BF16>(logits, row_stride, B, V, tokens_out, st); break;
    default: e = launch_argmax_dt<LSS_DTYPE_F16>(logits, row_stride, B, V, tokens_out, st); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return LSS_ERR_CUDA;
  }
  return LSS_OK;
}

int lss_read_status(const void* workspace, uint32_t* flags_out, void* stream) {
  if (!workspace || !flags_out) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return LSS_ERR_CUDA;
  uint32_t f = 0;
  if (cudaMemcpy(&f, workspace, sizeof(f), cudaMemcpyDeviceToHost) != cudaSuccess) return LSS_ERR_CUDA;
  *flags_out = f;
  return f ? LSS_ERR_DEVICE : LSS_OK;
}

int lss_read_row_paths(const void* workspace, int B, int32_t* paths_out, void* stream) {
  if (!workspace || !paths_out || B < 0) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return LSS_ERR_CUDA;
  const WsLayout L = ws_layout(B, 0);
  if (B == 0) return LSS_OK;
  if (cudaMemcpy(paths_out, reinterpret_cast<const unsigned char*>(workspace) + L.row_path,
                 sizeof(int32_t) * (size_t)B, cudaMemcpyDeviceToHost) != cudaSuccess)
    return LSS_ERR_CUDA;
  return LSS_OK;
}

}  // extern "C"
