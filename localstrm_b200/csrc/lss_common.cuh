// lss_common.cuh — constants, order-preserving keys, PTX wrappers (mbarrier, bulk copy,
// cluster barrier), block reductions and the argument block shared by the sampler kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cooperative_groups.h>
#include <float.h>
#include <stdint.h>

#include "lsampler.h"

namespace cg = cooperative_groups;

namespace lss {

constexpr int NT = 512;                 // threads per CTA
constexpr int NWARP = NT / 32;
constexpr int MAXCL = 8;                // CTAs per cluster (portable limit)
constexpr int NBIN = 256;               // histogram bins per pass (+1 "far" bucket)
constexpr float BIN_PER_NAT = 16.0f;    // value-space bins: 1/16 nat wide, 16 nats deep
constexpr uint32_t KEY_FINITE_MIN = 0x00800000u;  // key of -FLT_MAX
constexpr double FIX_ONE = 1099511627776.0;       // 2^40: fixed-point unit of mass
constexpr long long WAIT_CYCLES = 4000000000LL;   // ~2 s at 1.9 GHz

// Survivors of one row that the resolve kernel sorts in shared memory; rows whose
// vocabulary has at most FAST_CAP / 2 entries are resolved there even without a filter.
constexpr int FAST_CAP = 2048;
// Second kernel (rows the resolve kernel defers): survivors one CTA can resolve.
constexpr int SLOW_CAP = 4096;

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
__host__ __device__ __forceinline__ int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}
// Penalties of sampling.py:55-66 on one value: sign-dependent multiplicative repetition
// penalty, then the additive frequency / presence penalty, each an f32 op.
__device__ __forceinline__ float penalise(float v, float rp, float fq, float pr, int cnt) {
  if (rp != 1.0f) v = v > 0.0f ? __fdiv_rn(v, rp) : __fmul_rn(v, rp);
  if (fq != 0.0f || pr != 0.0f) v = __fsub_rn(v, __fadd_rn(__fmul_rn(fq, (float)cnt), pr));
  return v;
}

// ---------------------------------------------------------------------------
// PTX wrappers: mbarrier, bulk async copy (global -> own shared memory), cluster barrier
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
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > WAIT_CYCLES) return false;
  }
  return true;
}
// Bounded wait of a whole warp (all 32 lanes call it together): every lane tests the phase
// (so that each lane acquires the data the phase publishes) and the loop exits for all lanes at
// once, so that no lane spins on its own while the others wait at a warp-synchronous
// instruction.  Returns false (for every lane) after WAIT_CYCLES of lane 0's clock.
__device__ __forceinline__ bool warp_mbar_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  for (;;) {
    const bool ok = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, ok)) return true;
    const int late = (threadIdx.x & 31) == 0 && clock64() - t0 > WAIT_CYCLES;
    if (__shfl_sync(0xffffffffu, late, 0)) return false;
  }
}
// Bounded wait that lets the thread sleep until the phase completes (suspend-time hint), for
// waits that are not on the critical path of the waiting warp.
__device__ __forceinline__ bool mbar_wait_bounded_sleep(uint64_t* bar, uint32_t parity) {
  long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, "
        "p;\n}\n"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > WAIT_CYCLES) return false;
  }
}
// Generic-proxy shared-memory writes made before this call are ordered before later
// bulk-copy (async-proxy) writes into the same memory.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Distributed shared memory: the shared::cluster address of `local` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_u32(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr(local)), "r"(rank));
  return r;
}
// Arrive (release, cluster scope) on an mbarrier in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* local_bar, uint32_t rank) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mapa_u32(local_bar, rank))
               : "memory");
}
// Wait (acquire, cluster scope) for the phase of `parity` of a local mbarrier that other CTAs
// arrive on; gives up after WAIT_CYCLES and reports false.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n "
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > WAIT_CYCLES) return false;
  }
}
__device__ __forceinline__ void fence_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
// 4-byte asynchronous global -> shared copy (completed by cp_async_wait_all).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(saddr(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Waits until at most N of this thread's most recent cp.async groups are still pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Programmatic dependent launch: let the next kernel of the stream start launching, and wait
// until the previous one has completed with its memory visible (both no-ops without it).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Plain arrival (release, CTA scope) on a local mbarrier.
__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

// Cluster barrier halves.  A warp that wrote into another CTA's shared memory arrives
// with release semantics; the others arrive relaxed.  The wait acquires.
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync_warp_release(bool warp_wrote) {
  if (warp_wrote) cluster_arrive_release(); else cluster_arrive_relaxed();
  cluster_wait();
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
struct MaxU32 { __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a > b ? a : b; } };
struct MaxU64 { __device__ uint64_t operator()(uint64_t a, uint64_t b) const { return a > b ? a : b; } };
struct SumU64 { __device__ uint64_t operator()(uint64_t a, uint64_t b) const { return a + b; } };
struct SumU32 { __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a + b; } };
struct OrU32 { __device__ uint32_t operator()(uint32_t a, uint32_t b) const { return a | b; } };
struct SumD { __device__ double operator()(double a, double b) const { return a + b; } };
struct MinI { __device__ int operator()(int a, int b) const { return a < b ? a : b; } };

// Bitonic sort of a[0, np) (np a power of two) in shared memory, whole CTA.
// Steps whose partner distance j is below 32 pair elements inside aligned runs of 32: each
// warp takes such runs, one element per lane, and does those steps with shuffles, so only
// the steps with j >= 32 go through shared memory with a block barrier each (28 barriers
// instead of 66 for np = 2048).
__device__ __forceinline__ void bitonic_sort(uint64_t* a, int np, bool descending) {
  const int lane = threadIdx.x & 31;
  // Levels k_first .. k_last on every run of 32, the last one from step jmax_last down
  // (lanes past np hold placeholders and pair only with each other, np being a power of two).
  auto runs = [&](int k_first, int k_last, int jmax_last) {
    for (int base = (threadIdx.x >> 5) * 32; base < np; base += NT) {
      const int i = base + lane;
      uint64_t v = i < np ? a[i] : 0ull;
      for (int k = k_first; k <= k_last; k <<= 1) {
        for (int j = k == k_last ? jmax_last : k >> 1; j > 0; j >>= 1) {
          const uint64_t o = __shfl_xor_sync(0xffffffffu, v, j);
          const bool asc = ((i & k) == 0) != descending;
          const bool keep_small = ((i & j) == 0) == asc;
          v = keep_small ? (o < v ? o : v) : (o > v ? o : v);
        }
      }
      if (i < np) a[i] = v;
    }
    __syncthreads();
  };
  if (np < 2) return;
  const int k0 = np < 32 ? np : 32;
  runs(2, k0, k0 >> 1);  // levels 2 .. 32 entirely inside the runs
  for (int k = 64; k <= np; k <<= 1) {
    for (int j = k >> 1; j >= 32; j >>= 1) {
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
    runs(k, k, 16);
  }
}
// Bitonic sort of one u64 per lane across a warp (descending when `descending`).
__device__ __forceinline__ uint64_t warp_sort(uint64_t v, bool descending) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      uint64_t o = __shfl_xor_sync(0xffffffffu, v, j);
      const bool lower = (lane & j) == 0;
      const bool asc = ((lane & k) == 0) != descending;
      // lower lane keeps the smaller value in an ascending segment
      const bool keep_small = (lower == asc);
      v = keep_small ? (o < v ? o : v) : (o > v ? o : v);
    }
  }
  return v;
}

// k-th largest of the u32 keys key(0 .. n-1) (1 <= k <= n): radix select, eight bits per pass,
// down to bit `low` (0 for the exact key; 16 gives the largest multiple of 2^16 that at least k
// keys reach, in two passes).  Whole CTA (NT threads); `bins` holds 258 words.
template <class KeyAt>
__device__ uint32_t block_kth_largest(KeyAt key_at, int n, int k, uint32_t* bins, int low = 0) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t prefix = 0u, mask = 0u;
  for (int shift = 24; shift >= low; shift -= 8) {
    for (int b = tid; b < 256; b += NT) bins[b] = 0u;
    __syncthreads();
    for (int i = tid; i < n; i += NT) {
      const uint32_t key = key_at(i);
      if ((key & mask) == prefix) atomicAdd(&bins[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid < 32) {
      // Lane l holds bins 255 - 8l .. 248 - 8l (largest digits first).
      uint32_t c8[8], loc = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        c8[q] = bins[255 - (8 * lane + q)];
        loc += c8[q];
      }
      uint32_t incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, incl >= (uint32_t)k);
      const int L = hit ? __ffs(hit) - 1 : 31;
      if (lane == L) {
        uint32_t acc = incl - loc;
        int d = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (acc + c8[q] >= (uint32_t)k) {
            d = 255 - (8 * lane + q);
            break;
          }
          acc += c8[q];
        }
        bins[256] = (uint32_t)d;
        bins[257] = acc;  // keys with a larger digit
      }
    }
    __syncthreads();
    prefix |= bins[256] << shift;
    mask |= 255u << shift;
    k -= (int)bins[257];
    __syncthreads();
  }
  return prefix;
}

// Smallest key K with exp(key2f(K) - m) >= mp (min-p keeps y with key >= K).
__device__ __forceinline__ uint32_t minp_key(float m, float mp) {
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

// A value of y at or below the exact min-p threshold of a row whose max is m (the threshold
// is the smallest y with exp(y - m) >= mp; expf / logf err by a few ulps, the slack here is
// 2^-13 relative).
__device__ __forceinline__ float minp_floor_y(float m, float mp) {
  const float l = logf(mp);
  const float y = __fadd_rn(m, l);
  return __fsub_rn(y, (fabsf(m) + fabsf(l) + 1.0f) * 1.220703125e-04f);
}

// A pre-temperature value below which z / T cannot reach y_thr (conservative: the true
// boundary lies above it by at least 2^-20 relative).  Used to choose candidates without
// dividing every element; candidates are then divided exactly and filtered on y.
__device__ __forceinline__ float z_floor_for(float y_thr, float T) {
  const double z = (double)y_thr * (double)T;
  const double slack = fabs(z) * 9.5367431640625e-07 + 1e-37;
  return __double2float_rd(z - slack);
}

// History range [b, e) of a row from the caller's CSR offsets.  Offsets outside [0, H] or
// decreasing ones give an empty range and false (the caller raises LSS_FLAG_BAD_HISTORY), so
// that no kernel reads or writes outside the id arrays and the workspace regions sized by H.
__device__ __forceinline__ bool hist_range(const int32_t* off, int row, int H, int& b, int& e) {
  const int b0 = off[row], e0 = off[row + 1];
  const bool ok = 0 <= b0 && b0 <= e0 && e0 <= H;
  b = ok ? b0 : 0;
  e = ok ? e0 : 0;
  return ok;
}

// ---------------------------------------------------------------------------
// Arguments of the per-row kernels
// ---------------------------------------------------------------------------
struct RowArgs {
  const void* logits;
  int64_t row_stride;  // elements
  int B, V, TE;        // TE: tile elements per CTA (multiple of 16)
  int tile_bytes;      // bytes reserved for the tile
  int use_hist;
  int H;                     // total history ids (hist_total)
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* min_p;
  const float* rep;
  const float* freq;
  const float* pres;
  const int32_t* hist_off;   // CSR offsets of the histories
  const int32_t* hist_ids;   // CSR ids of the histories
  int32_t* uniq_ids;         // per row: unique ids grouped by CTA slice
  int32_t* uniq_cnt;         //          their counts
  int32_t* seg_off;          // [B][CL+1] slice segment offsets (relative to hist_off[row])
  uint32_t* gkeys;           // hash tables of histories too long for shared memory (2 slots per id)
  uint32_t* gcnts;
  int CL;                    // CTAs per cluster of the second kernel
  const float* uniforms;
  int32_t* tokens;
  uint8_t* kept_out;
  float* probs_out;
  uint32_t* err;             // workspace header word 0: device error flags
  uint32_t* counters;        // header word [2]: deferred rows
  int32_t* defer_rows;       // [B]
  int32_t* row_path;         // [B]
};

// Applies the penalties of one row to this CTA's slice [lo, lo+n) of `tile` from the prep
// kernel's per-slice (id, count) segment, entries [first, last).
__device__ __forceinline__ void apply_patches_global(const RowArgs& a, int row, int me, int lo, int n,
                                                     float* tile, int first) {
  int base = 0, hend = 0;
  hist_range(a.hist_off, row, a.H, base, hend);
  const int* so = a.seg_off + (int64_t)row * (MAXCL + 1);
  const int s0 = so[me], s1 = so[me + 1];
  const float rp = a.rep[row], fq = a.freq[row], pr = a.pres[row];
  for (int j = s0 + first + (int)threadIdx.x; j < s1; j += NT) {
    const int id = a.uniq_ids[base + j];
    if (id >= lo && id < lo + n) tile[id - lo] = penalise(tile[id - lo], rp, fq, pr, a.uniq_cnt[base + j]);
  }
}

}  // namespace lss
