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
  __shared__ uint32_t r32[NWARP];
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
    }
    return;
  }
  if (tid == 0 && (s_flags & SHARD_OVER)) atomicOr(a.err, LSS_FLAG_INTERNAL);
  const float tp = a.top_p[row];
  const ResolveIn in{my, true, K, tp > 0.0f && tp < 1.0f, tp, a.uniforms[row], row, a.V};
  const RedScratch rs{r64, rd, r32, ri};
  resolve_block<MERGE_CAP>(G, E, nc, in, a, rs, LSS_PATH_GATHER);
}

}  // namespace lss
