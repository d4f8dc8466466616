// lss_shard.cuh — vocabulary-sharded sampling: each GPU holds the slice [voff, voff + Vs) of
// every row's vocabulary.
//
// K_S (lss_shard_kernel): one CTA per row of the shard: y = z / T (sampling.py:146), the
// shard's max of y, the sum of exp(y - max) (for callers that normalise over shards), and
// the shard's K largest y as codes (key(y) << 32 | ~global index), value descending, index
// ascending.  Three passes over the shard row: max; a 1/16-nat count histogram of the values
// below the max that locates the K-th largest (and the sum); the values at or above a floor
// two bins below it, compacted, sorted, cut to K.
// K_M (lss_merge_kernel): one CTA per row after the records of every shard are gathered: the
// global max, the union of the shards' candidates, then the reference's top-k with k = K
// (ties kept), top-p, renormalisation and inverse-CDF draw (sampling.py:82-113,157-162).
// The union holds the row's K largest because every one of them is among its shard's K
// largest (exact ties across the K-th value are the one exception and are documented).
// Rows with NaN / +inf or only -inf after scaling take the NaN guard (sampling.py:159-160):
// the argmax of y, NaN first.
#pragma once

#include "lss_common.cuh"
#include "lss_resolve.cuh"

namespace lss {

constexpr int SHARD_CAND = 2048;   // candidates one shard CTA sorts
constexpr int SH_U = 12;           // loads in flight per thread in the shard passes
constexpr int MERGE_CAP = 2048;    // shards x K codes the merge CTA holds
constexpr uint32_t SHARD_OVER = 1u;     // more values at the floor than SHARD_CAND
constexpr uint32_t SHARD_SPECIAL = 2u;  // NaN / +inf in the shard

// Record of one row of one shard: K codes, then {max y, sum exp(y - max), flags, count}.
__host__ __device__ constexpr size_t shard_record_bytes(int K) { return (size_t)K * 8 + 16; }

template <int DT>
__global__ void __launch_bounds__(NT) lss_shard_kernel(const void* logits, int64_t row_stride, int Vs, int64_t voff,
                                                       const float* temperature, int K, unsigned char* rec) {
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  __shared__ uint64_t C[SHARD_CAND];
  __shared__ uint32_t HLw[NWARP][NBIN + 1];
  __shared__ float rf[NWARP];
  __shared__ double rd[NWARP];
  __shared__ uint64_t r64[NWARP];
  __shared__ uint32_t s_n;
  __shared__ int s_bk;
  __shared__ float s_thr;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const char* g0 = reinterpret_cast<const char*>(logits) + (int64_t)row * row_stride * ES;
  auto z_at = [&](int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(g0)[i];
    if (DT == LSS_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g0)[i]);
    return __half2float(reinterpret_cast<const __half*>(g0)[i]);
  };
  const float T = temperature[row];
  const bool greedy = T <= 0.0f;  // codes of the raw values (their order is all a greedy row needs)
  auto y_of = [&](float z) -> float { return greedy ? z : __fdiv_rn(z, T); };
  // Each pass loads SH_U values per thread (elements i0 + u * NT) before it works on them, so
  // that SH_U loads per thread are in flight; a thread sees its elements in the same order as
  // with one load per step.
  auto load_batch = [&](int i0, float (&zb)[SH_U]) {
#pragma unroll
    for (int u = 0; u < SH_U; ++u) {
      const int i = i0 + u * NT;
      zb[u] = i < Vs ? z_at(i) : -INFINITY;
    }
  };
  // ---- pass 1: the shard max of y (y is monotone in z for T > 0) and its argmax, NaN first
  float zm = -INFINITY;
  uint64_t best = 0;
  for (int i0 = tid; i0 < Vs; i0 += SH_U * NT) {
    float zb[SH_U];
    load_batch(i0, zb);
#pragma unroll
    for (int u = 0; u < SH_U; ++u) {
      const int i = i0 + u * NT;
      if (i < Vs) {
        zm = fmax_nan(zm, zb[u]);
        const uint64_t c = argmax_code(zb[u], i);
        best = c > best ? c : best;
      }
    }
  }
  zm = block_allreduce(zm, MaxF(), rf);
  best = block_allreduce(best, MaxU64(), r64);
  const float my = y_of(zm);
  // NaN / +inf, or nothing finite: the shard contributes its argmax only (the NaN guard).
  const bool special = !(my == my) || my == INFINITY || my == -INFINITY;
  unsigned char* r = rec + (size_t)row * shard_record_bytes(K);
  uint64_t* codes = reinterpret_cast<uint64_t*>(r);
  uint32_t* tail = reinterpret_cast<uint32_t*>(r + (size_t)K * 8);
  if (special) {
    for (int i = tid; i < K; i += NT) {
      uint64_t c = 0ull;
      if (i == 0) {
        const int bi = (int)(~(uint32_t)best);
        c = ((uint64_t)gkey(y_of(z_at(bi))) << 32) | (uint32_t)(~(uint32_t)(voff + bi));
      }
      codes[i] = c;
    }
    if (tid == 0) {
      tail[0] = __float_as_uint(my);
      tail[1] = __float_as_uint(my == -INFINITY ? 0.0f : __int_as_float(0x7fc00000));
      tail[2] = (my == -INFINITY) ? 0u : SHARD_SPECIAL;
      tail[3] = 1u;
    }
    return;
  }
  // ---- pass 2: count histogram of (my - y), bins of 1/16 nat (then 1 and 16 nats when the
  //      K-th largest lies deeper), and the sum of exp(y - my)
  double se = 0.0;
  int bk = NBIN;
  float bw = 1.0f / BIN_PER_NAT;  // nats per bin
  for (int scale = 0; scale < 3 && bk == NBIN; ++scale, bw *= 16.0f) {
    for (int i = tid; i < NWARP * (NBIN + 1); i += NT) (&HLw[0][0])[i] = 0u;
    __syncthreads();
    const float bs = __fdiv_rn(1.0f, bw);
    double sl = 0.0;
    for (int i0 = tid; i0 < Vs; i0 += SH_U * NT) {
      float zb[SH_U];
      load_batch(i0, zb);
#pragma unroll
      for (int u = 0; u < SH_U; ++u) {
        if (i0 + u * NT >= Vs) continue;
        const float y = y_of(zb[u]);
        if (y == -INFINITY) continue;
        if (scale == 0) sl += (double)expf(__fsub_rn(y, my));
        const float d = __fmul_rn(__fsub_rn(my, y), bs);
        atomicAdd(&HLw[warp][d < (float)NBIN ? (int)d : NBIN], 1u);
      }
    }
    if (scale == 0) se = block_allreduce(sl, SumD(), rd);
    __syncthreads();
    // Warp 0 merges the per-warp histograms and finds the bin of the K-th largest.
    if (warp == 0) {
      uint32_t c8[8];
      uint32_t loc = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t c = 0;
        for (int w = 0; w < NWARP; ++w) c += HLw[w][8 * lane + q];
        c8[q] = c;
        loc += c;
      }
      uint32_t incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      uint32_t far = 0;
      for (int w = 0; w < NWARP; ++w) far += HLw[w][NBIN];
      const uint32_t total = __shfl_sync(0xffffffffu, incl, 31) + far;
      const unsigned hit = __ballot_sync(0xffffffffu, incl >= (uint32_t)K);
      int b2 = NBIN;
      if (hit) {
        const int L = __ffs(hit) - 1;
        int b = 0;
        uint32_t acc = incl - loc;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          acc += c8[q];
          if (acc < (uint32_t)K) b = q + 1;
        }
        b2 = __shfl_sync(0xffffffffu, 8 * lane + b, L);
      } else if (total <= (uint32_t)K) {
        b2 = -1;  // K or fewer finite values: every one is a candidate
      }
      if (lane == 0) s_bk = b2;
    }
    __syncthreads();
    bk = s_bk;
    if (bk >= 0 && bk < NBIN) {
      // The K-th largest lies in bin bk: (my - y_K) / bw < bk + 1; two bins of slack.
      if (tid == 0) s_thr = __fsub_rn(my, __fmul_rn((float)(bk + 2), bw));
      __syncthreads();
    }
  }
  // ---- pass 3: the values at or above the floor, compacted
  float ythr = -INFINITY;  // candidates: finite y >= ythr
  if (bk >= 0 && bk < NBIN) {
    ythr = s_thr;
    ythr = __fsub_rn(ythr, fabsf(ythr) * 2.384185791015625e-07f + 1e-37f);
  }
  if (tid == 0) s_n = 0u;
  __syncthreads();
  for (int j0 = 0; j0 < Vs; j0 += SH_U * NT) {  // uniform trip count
    float zb[SH_U];
    load_batch(j0 + tid, zb);
#pragma unroll
    for (int u = 0; u < SH_U; ++u) {
      const int i = j0 + u * NT + tid;
      bool keep = false;
      uint64_t code = 0;
      if (i < Vs) {
        const float y = y_of(zb[u]);
        keep = y > -INFINITY && y >= ythr;
        code = ((uint64_t)f2key(y) << 32) | (uint32_t)(~(uint32_t)(voff + i));
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, keep);
      if (bal) {
        const int leader = __ffs(bal) - 1;
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(&s_n, (uint32_t)__popc(bal));
        base = __shfl_sync(0xffffffffu, base, leader);
        const uint32_t pos = base + __popc(bal & ((1u << lane) - 1u));
        if (keep && pos < (uint32_t)SHARD_CAND) C[pos] = code;
      }
    }
  }
  __syncthreads();
  const uint32_t n_all = s_n;
  const int nc = (int)min(n_all, (uint32_t)SHARD_CAND);
  const int np = next_pow2(nc > 1 ? nc : 1);
  for (int i = nc + tid; i < np; i += NT) C[i] = 0ull;
  __syncthreads();
  bitonic_sort(C, np, true);
  // ---- record
  for (int i = tid; i < K; i += NT) codes[i] = i < nc ? C[i] : 0ull;
  if (tid == 0) {
    tail[0] = __float_as_uint(my);
    tail[1] = __float_as_uint((float)se);
    tail[2] = n_all > (uint32_t)SHARD_CAND ? SHARD_OVER : 0u;
    tail[3] = (uint32_t)min(nc, K);
  }
}

// ---------------------------------------------------------------------------------------
// K_SC (lss_shard_cluster_kernel): the same record in one pass over HBM.  A cluster of P CTAs
// takes one row of the shard; CTA r stages the part [r PS, (r + 1) PS) of the row in its
// shared memory with one bulk copy and reads it from there:
//   1. the part's max of z and whether it holds NaN / +inf, and the max of every group of L
//      lanes' values (the "group maxima");
//   2. cluster barrier; every CTA reads the CTAs' maxima and all group maxima through
//      distributed shared memory and takes F, the K-th largest group max: K groups reach F,
//      so K values do, and every value among the row's K largest is at least F;
//   3. each CTA adds exp(y - max) over its finite values and sends the values with
//      y >= y(F) as codes to rank 0's candidate buffer (one remote atomic per warp);
//   4. cluster barrier; rank 0 sorts the ~K candidates and writes the record.
// With about 4K group maxima the candidates number little more than K.  A row with NaN / +inf
// (or nothing finite) after scaling sends its argmax code (NaN first, lowest index) instead.
// ---------------------------------------------------------------------------------------
constexpr int SC_NT = NT;                 // threads per CTA (bitonic_sort works on NT threads)
constexpr int SC_MAXCL = 16;              // CTAs per row at most
constexpr int SC_CAP = SHARD_CAND;        // candidates rank 0 collects
constexpr int SC_GKMAX = 2048;            // group maxima of a row at most
constexpr int SC_PART_MAX = 64 * 1024;    // bytes of a part at most (64 values per thread)
constexpr uint32_t SHARD_TIMEOUT = 4u;    // a bulk copy did not land in time

struct ScCtl {
  uint64_t bar;
  uint32_t n;                   // rank 0: candidates sent
  uint32_t zkey;                // this CTA's max key of z
  uint32_t spec;                // this CTA saw NaN / +inf
  uint32_t pad;
  double psum[SC_MAXCL];        // rank 0: partial sums of exp(y - max), by rank
  uint64_t best[SC_MAXCL];      // rank 0: argmax codes of a special row, by rank
  uint32_t flags[SC_MAXCL];     // rank 0: flags, by rank
  uint32_t bins[260];
  uint32_t gk[SC_NT];           // this CTA's group maxima
  uint32_t allk[SC_GKMAX];      // every group max of the row
  uint64_t cand[SC_CAP];        // rank 0: candidates
};

// 2^x (PTX ex2.approx: relative error about 2^-22; -inf gives +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__host__ __device__ constexpr size_t sc_part_bytes(int PS, int es) { return ((size_t)PS * es + 15) & ~(size_t)15; }

template <int DT>
__global__ void __launch_bounds__(SC_NT) lss_shard_cluster_kernel(const void* logits, int64_t row_stride, int Vs,
                                                                  int64_t voff, const float* temperature, int K,
                                                                  int PS, int L, unsigned char* rec) {
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  constexpr int VE = 16 / ES;             // values per 16-byte vector
  constexpr int MAXV = SC_PART_MAX / 16 / SC_NT;  // vectors per thread at most (8)
  extern __shared__ __align__(128) unsigned char scm[];
  cg::cluster_group cl = cg::this_cluster();
  const int P = (int)cl.num_blocks();
  const int me = (int)cl.block_rank();
  const int row = blockIdx.x / P;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned char* part = scm;
  ScCtl& c = *reinterpret_cast<ScCtl*>(scm + sc_part_bytes(PS, ES));
  __shared__ uint32_t r32[NWARP];
  __shared__ uint64_t r64[NWARP];
  __shared__ double rd[NWARP];
  const int lo = me * PS;
  const int n = max(0, min(Vs, lo + PS) - lo);
  const char* src = reinterpret_cast<const char*>(logits) + ((int64_t)row * row_stride + lo) * ES;
  const float T = temperature[row];
  const bool greedy = T <= 0.0f;  // codes of the raw values (their order is all a greedy row needs)
  auto y_of = [&](float z) -> float { return greedy ? z : __fdiv_rn(z, T); };
  // ---- the part into shared memory: one bulk copy of its 16-byte aligned body, plain loads
  // for the rest (a misaligned row, a ragged tail)
  const uint32_t nb = (reinterpret_cast<uintptr_t>(src) & 15) == 0 ? (uint32_t)((n * ES) & ~15) : 0u;
  if (tid == 0) {
    c.n = 0u;
    c.pad = 0u;
    mbar_init(&c.bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_expect_tx(&c.bar, nb);
    if (nb > 0) bulk_g2s(part, src, nb, &c.bar);
  }
  for (int i = (int)nb / ES + tid; i < n; i += SC_NT) {
    if (ES == 4) reinterpret_cast<float*>(part)[i] = reinterpret_cast<const float*>(src)[i];
    else reinterpret_cast<uint16_t*>(part)[i] = reinterpret_cast<const uint16_t*>(src)[i];
  }
  uint32_t myflags = 0u;
  if (!mbar_wait_bounded(&c.bar, 0)) myflags |= SHARD_TIMEOUT;
  __syncthreads();
  // Values of vector q of the part (elements q VE .. q VE + VE - 1), widened.
  auto vec = [&](int q, float* x) {
    const uint4 r = reinterpret_cast<const uint4*>(part)[q];
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (DT == LSS_DTYPE_F32) {
        x[j] = __uint_as_float(w[j]);
      } else if (DT == LSS_DTYPE_BF16) {
        x[2 * j] = __uint_as_float(w[j] << 16);
        x[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      } else {
        x[2 * j] = __half2float(__ushort_as_half((uint16_t)(w[j] & 0xffffu)));
        x[2 * j + 1] = __half2float(__ushort_as_half((uint16_t)(w[j] >> 16)));
      }
    }
  };
  const int nvec = (n + VE - 1) / VE;
  const int nfull = n / VE;  // vectors whose values all belong to the part
  // ---- 1. maxima: this thread's vectors are q = tid + v NT.  fmaxf passes over NaN, which
  // the flag records (+inf shows up as the max).
  float tmax = -INFINITY;
  bool spec = false;
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int q = tid + v * SC_NT;
    if (q < nvec) {
      float x[VE];
      vec(q, x);
      const int lim = q < nfull ? VE : n - q * VE;
#pragma unroll
      for (int j = 0; j < VE; ++j) {
        if (j < lim) {
          tmax = fmaxf(tmax, x[j]);
          spec |= x[j] != x[j];
        }
      }
    }
  }
  const uint32_t tkey = f2key(tmax);
  uint32_t gkey = tkey;
  for (int o = 1; o < L; o <<= 1) gkey = max(gkey, __shfl_xor_sync(0xffffffffu, gkey, o));
  const int G1 = SC_NT / L;  // groups per CTA
  if ((lane & (L - 1)) == 0) c.gk[warp * (32 / L) + lane / L] = gkey;
  // The part's max key and NaN / +inf flag in one reduction (flag above the key).
  const uint64_t cm = block_allreduce(((uint64_t)(spec ? 1u : 0u) << 32) | tkey, MaxU64(), r64);
  if (tid == 0) {
    c.zkey = (uint32_t)cm;
    c.spec = (uint32_t)(cm >> 32);
  }
  cl.sync();  // 2. every CTA's maxima are visible cluster-wide
  uint64_t rm = 0ull;
  if (tid < P) {
    const ScCtl* rc = cl.map_shared_rank(&c, tid);
    rm = ((uint64_t)rc->spec << 32) | rc->zkey;
  }
  rm = block_allreduce(rm, MaxU64(), r64);
  const uint32_t zk = (uint32_t)rm, sp = (uint32_t)(rm >> 32);
  const int GK = P * G1;
  for (int t = tid; t < GK; t += SC_NT) c.allk[t] = cl.map_shared_rank(&c, t / G1)->gk[t % G1];
  // Max of y: NaN when the row holds a NaN; +inf when it holds +inf (or the division
  // overflows); -inf when nothing is finite (zk then is the key of -inf or 0).
  float my;
  if (sp) {
    my = INFINITY;  // refined below: NaN if any NaN
  } else {
    my = zk >= KEY_FINITE_MIN ? y_of(key2f(zk)) : -INFINITY;
  }
  const bool special = sp || !(my > -INFINITY && my < INFINITY);
  ScCtl* c0 = cl.map_shared_rank(&c, 0);
  unsigned char* r = rec + (size_t)row * shard_record_bytes(K);
  uint64_t* codes = reinterpret_cast<uint64_t*>(r);
  uint32_t* tail = reinterpret_cast<uint32_t*>(r + (size_t)K * 8);
  if (special) {
    // The NaN guard's argmax over the row's y (NaN first, lowest index), and whether a NaN is
    // in the row (then the max is NaN).
    uint64_t best = 0;
    bool nan = false;
    for (int i = tid; i < n; i += SC_NT) {
      const float z = DT == LSS_DTYPE_F32 ? reinterpret_cast<const float*>(part)[i]
                      : DT == LSS_DTYPE_BF16
                          ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(part)[i] << 16)
                          : __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(part)[i]));
      const float y = y_of(z);
      nan |= !(y == y);
      best = max(best, argmax_code(y, (int)(voff + lo + i)));
    }
    best = block_allreduce(best, MaxU64(), r64);
    const uint32_t anynan = block_allreduce(nan ? 1u : 0u, OrU32(), r32);
    if (tid == 0) {
      c0->best[me] = best;
      c0->flags[me] = myflags | (anynan ? 0x80000000u : 0u);
    }
    cl.sync();  // 4. rank 0 has every part's argmax
    if ((myflags & SHARD_TIMEOUT) && tid == 0) mbar_wait_bounded(&c.bar, 0);
    if (me == 0) {
      uint64_t b = 0;
      uint32_t fl = 0;
      for (int q = 0; q < P; ++q) {
        b = max(b, c.best[q]);
        fl |= c.flags[q];
      }
      const float m = (fl & 0x80000000u) ? __int_as_float(0x7fc00000) : my;
      for (int i = tid; i < K; i += SC_NT) codes[i] = i == 0 ? b : 0ull;
      if (tid == 0) {
        tail[0] = __float_as_uint(m);
        tail[1] = __float_as_uint(m == -INFINITY ? 0.0f : __int_as_float(0x7fc00000));
        tail[2] = (m == -INFINITY ? 0u : SHARD_SPECIAL) | (fl & SHARD_TIMEOUT);
        tail[3] = 1u;
      }
    }
    return;
  }
  __syncthreads();  // allk complete
  // F: a key at most the K-th largest group max, to within 2^-7 of its value (the top 16 bits
  // of the key: sign, exponent, seven mantissa bits); at least K groups reach it.  No bound
  // when fewer than K groups hold a finite value.
  const uint32_t F = block_kth_largest([&](int i) { return c.allk[i]; }, GK, K, c.bins, 16);
  const float yF = F >= KEY_FINITE_MIN ? y_of(key2f(F)) : -INFINITY;
  // Values below zlow cannot reach y(F); only the others are divided exactly.
  const float zlow = (yF == -INFINITY) ? -INFINITY : (greedy ? yF : z_floor_for(yF, T));
  const float zmax = key2f(zk);
  const float invT = greedy ? 1.0f : __frcp_rn(T);
  // ---- 3. sum of exp(y - max) over the finite values, as 2^((z - zmax) log2(e) / T) (within a
  // few ulp of the exact terms; per vector in f32, then in f64), and the candidates y >= y(F)
  const float c2 = __fmul_rn(invT, 1.4426950408889634f);
  using Mask = unsigned long long;
  Mask m = 0;
  double sl = 0.0;
  int cnt = 0;
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int q = tid + v * SC_NT;
    if (q < nvec) {
      float x[VE];
      vec(q, x);
      const int lim = q < nfull ? VE : n - q * VE;
      float e[VE];
#pragma unroll
      for (int j = 0; j < VE; ++j) {
        e[j] = 0.0f;
        if (j < lim) {
          e[j] = ex2_approx(__fmul_rn(__fsub_rn(x[j], zmax), c2));
          if (x[j] >= zlow && x[j] > -INFINITY) {
            const float y = y_of(x[j]);
            if (y >= yF && y > -INFINITY) {
              m |= (Mask)1 << (v * VE + j);
              ++cnt;
            }
          }
        }
      }
#pragma unroll
      for (int w2 = VE / 2; w2 >= 1; w2 /= 2)
#pragma unroll
        for (int j = 0; j < w2; ++j) e[j] += e[j + w2];
      sl += (double)e[0];
    }
  }
  uint32_t incl = (uint32_t)cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  uint32_t base = 0;
  if (lane == 31 && incl) base = atomicAdd(&c0->n, incl);
  base = __shfl_sync(0xffffffffu, base, 31) + incl - (uint32_t)cnt;
  while (m) {
    const int b = __ffsll((long long)m) - 1;
    m &= m - 1;
    const int v = b / VE, j = b % VE;
    const int i = (tid + v * SC_NT) * VE + j;
    float x[VE];
    vec(tid + v * SC_NT, x);
    if (base < (uint32_t)SC_CAP)
      c0->cand[base] = ((uint64_t)f2key(y_of(x[j])) << 32) | (uint32_t)(~(uint32_t)(voff + lo + i));
    ++base;
  }
  const double se = block_allreduce(sl, SumD(), rd);
  if (tid == 0) {
    c0->psum[me] = se;
    c0->flags[me] = myflags;
  }
  cl.sync();  // 4. rank 0 holds every candidate and partial sum
  // After a bulk copy gave up, wait (bounded) once more for it before the memory is released.
  if ((myflags & SHARD_TIMEOUT) && tid == 0) mbar_wait_bounded(&c.bar, 0);
  if (me != 0) return;
  const uint32_t n_all = c.n;
  const int nc = (int)min(n_all, (uint32_t)SC_CAP);
  const int np = next_pow2(nc > 1 ? nc : 1);
  for (int i = nc + tid; i < np; i += SC_NT) c.cand[i] = 0ull;
  __syncthreads();
  bitonic_sort(c.cand, np, true);
  __syncthreads();
  for (int i = tid; i < K; i += SC_NT) codes[i] = i < nc ? c.cand[i] : 0ull;
  if (tid == 0) {
    double S = 0.0;
    uint32_t fl = 0;
    for (int q = 0; q < P; ++q) {
      S += c.psum[q];
      fl |= c.flags[q];
    }
    tail[0] = __float_as_uint(my);
    tail[1] = __float_as_uint((float)S);
    tail[2] = (n_all > (uint32_t)SC_CAP ? SHARD_OVER : 0u) | (fl & SHARD_TIMEOUT);
    tail[3] = (uint32_t)min(nc, K);
  }
}

// The records are gathered shard-major: shard s, row b at (s * B + b) * shard_record_bytes(K).
__global__ void __launch_bounds__(NT) lss_merge_kernel(const unsigned char* recs, int nshards, int B, int K,
                                                       const RowArgs a) {
  __shared__ uint64_t G[MERGE_CAP];
  __shared__ float E[MERGE_CAP];
  __shared__ uint64_t r64[NWARP];
  __shared__ double rd[NWARP];
  __shared__ uint32_t r32[NWARP];
  __shared__ int ri[NWARP];
  __shared__ uint32_t s_n, s_flags;
  __shared__ float s_my;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const size_t rb = shard_record_bytes(K);
  if (tid == 0) {
    float m = -INFINITY;
    uint32_t fl = 0;
    for (int s = 0; s < nshards; ++s) {
      const uint32_t* tail = reinterpret_cast<const uint32_t*>(recs + ((size_t)s * B + row) * rb + (size_t)K * 8);
      m = fmax_nan(m, __uint_as_float(tail[0]));
      fl |= tail[2];
    }
    s_my = m;
    s_flags = fl;
    s_n = 0u;
  }
  __syncthreads();
  const int tot = nshards * K;
  const float gm = s_my;
  const bool finite_row = gm == gm && gm > -INFINITY && gm < INFINITY && !(s_flags & SHARD_SPECIAL);
  for (int i = tid; i < tot; i += NT) {
    const int s = i / K, j = i - s * K;
    const uint64_t c = reinterpret_cast<const uint64_t*>(recs + ((size_t)s * B + row) * rb)[j];
    // An all -inf shard's argmax code only matters when the whole row is -inf.
    if (c != 0ull && (!finite_row || key2f((uint32_t)(c >> 32)) > -INFINITY)) {
      const uint32_t pos = atomicAdd(&s_n, 1u);
      if (pos < (uint32_t)MERGE_CAP) G[pos] = c;
    }
  }
  __syncthreads();
  const int nc = (int)min(s_n, (uint32_t)MERGE_CAP);
  const float my = s_my;
  const bool special = !(my == my) || my == INFINITY || my == -INFINITY || (s_flags & SHARD_SPECIAL);
  const float T = a.temperature[row];
  if (T <= 0.0f || special || nc == 0) {
    // Greedy rows and the NaN guard: the largest code (NaN first, then lowest index).
    uint64_t best = 0;
    for (int i = tid; i < nc; i += NT) best = G[i] > best ? G[i] : best;
    best = block_allreduce(best, MaxU64(), r64);
    if (tid == 0) {
      a.tokens[row] = (int32_t)(~(uint32_t)best);
      a.row_path[row] = T <= 0.0f ? LSS_PATH_GREEDY : LSS_PATH_SPECIAL;
      if (s_flags & SHARD_OVER) atomicOr(a.err, LSS_FLAG_INTERNAL);
      if (s_flags & SHARD_TIMEOUT) atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
    }
    return;
  }
  if (tid == 0 && (s_flags & SHARD_OVER)) atomicOr(a.err, LSS_FLAG_INTERNAL);
  if (tid == 0 && (s_flags & SHARD_TIMEOUT)) atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
  const float tp = a.top_p[row];
  const ResolveIn in{my, true, K, tp > 0.0f && tp < 1.0f, tp, a.uniforms[row], row, a.V};
  const RedScratch rs{r64, rd, r32, ri};
  resolve_block<MERGE_CAP>(G, E, nc, in, a, rs, LSS_PATH_GATHER);
}

}  // namespace lss
