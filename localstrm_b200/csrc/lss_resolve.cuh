// lss_resolve.cuh — final stage of a row once its survivors sit in one CTA's shared memory:
// sort (value desc, index asc), top-k cut (ties kept), exp(y - max), top-p cut, renormalise
// and draw by inverse CDF in vocabulary order (sampling.py:82-113,157-162); and K2, the
// resolve kernel, which gathers each row's candidates from the streaming kernel's slice segments
// and its history values.
//
// Candidates are u64 codes (key(y) << 32) | ~index, where key() is the order-preserving u32
// key of the scaled logit y; sorting the codes in descending order gives value descending
// then index ascending, the tie rule of the oracle.
#pragma once

#include "lss_common.cuh"

namespace lss {

struct ResolveIn {
  float m;       // row max of y
  bool tk;       // top-k active (k < V)
  int k;
  bool tp_on;    // 0 < top_p < 1
  float tp;
  float u;       // uniform of the row
  int row;
  int V;
};

// Scratch for block-level reductions (lives in each kernel's control block).
struct RedScratch {
  uint64_t* r64;
  double* rd;
  uint32_t* r32;
  int* ri;
};

// Whole-CTA resolve of G[0, nc) (nc <= cap, cap a power of two >= NT * per-thread items).
// E must hold `cap` floats.  Writes the token and, when requested, kept/probs.
template <int CAPN>
__device__ void resolve_block(uint64_t* G, float* E, int nc, const ResolveIn& in, const RowArgs& a,
                              const RedScratch& rs, int path) {
  constexpr int PER = CAPN / NT;  // items per thread, contiguous
  const int tid = threadIdx.x;
  const int np = next_pow2(nc > 1 ? nc : 1);
  for (int i = nc + tid; i < np; i += NT) G[i] = 0ull;
  __syncthreads();
  bitonic_sort(G, np, true);  // key desc, index asc
  int n1 = nc;
  if (in.tk && in.k <= nc) {  // top-k keeps every value >= the k-th largest (sampling.py:85)
    const uint32_t Kk = (uint32_t)(G[in.k - 1] >> 32);
    uint32_t c = 0;
    for (int i = tid; i < nc; i += NT) c += ((uint32_t)(G[i] >> 32) >= Kk) ? 1u : 0u;
    n1 = (int)block_allreduce(c, SumU32(), rs.r32);
  }
  double part = 0.0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = tid * PER + j;
    float e = 0.0f;
    if (i < n1) e = expf(__fsub_rn(key2f((uint32_t)(G[i] >> 32)), in.m));
    E[i] = e;
    part += (double)e;
  }
  double S = block_allreduce(part, SumD(), rs.rd);
  int n2 = n1;
  if (in.tp_on && n1 > 1) {
    // p = e / S in f32; c = cumsum in f64 rounded to f32; keep j iff j == 0 or c_{j-1} <= top_p.
    const float S32 = (float)S;
    double loc[PER];
    double run = 0.0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid * PER + j;
      run += i < n1 ? (double)__fdiv_rn(E[i], S32) : 0.0;
      loc[j] = run;
    }
    double tot;
    const double pre = block_excl_scan(run, rs.rd, tot);
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid * PER + j;
      if (i < n1 - 1 && (float)(pre + loc[j]) <= in.tp) c++;
    }
    n2 = 1 + (int)block_allreduce(c, SumU32(), rs.r32);
    if (n2 > n1) n2 = n1;
    double part2 = 0.0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid * PER + j;
      if (i < n2) part2 += (double)E[i];
    }
    S = block_allreduce(part2, SumD(), rs.rd);
  }
  const float Sf = (float)S;
  __syncthreads();
  for (int i = tid; i < n2; i += NT) {
    const uint32_t idx = ~(uint32_t)G[i];
    const float pr = __fdiv_rn(E[i], Sf);
    G[i] = ((uint64_t)idx << 32) | __float_as_uint(pr);
    if (a.kept_out) a.kept_out[(int64_t)in.row * in.V + idx] = 1;
    if (a.probs_out) a.probs_out[(int64_t)in.row * in.V + idx] = pr;
  }
  const int np2 = next_pow2(n2 > 1 ? n2 : 1);
  for (int i = n2 + tid; i < np2; i += NT) G[i] = ~0ull;
  __syncthreads();
  bitonic_sort(G, np2, false);  // index asc
  double loc[PER];
  double run = 0.0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = tid * PER + j;
    run += i < n2 ? (double)__uint_as_float((uint32_t)G[i]) : 0.0;
    loc[j] = run;
  }
  double tot;
  const double pre = block_excl_scan(run, rs.rd, tot);
  const double target = (double)in.u * tot;
  int first = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = tid * PER + j;
    if (first == 0x7fffffff && i < n2 && pre + loc[j] > target) first = i;
  }
  first = block_allreduce(first, MinI(), rs.ri);
  if (tid == 0) {
    if (first >= n2) first = n2 - 1;
    a.tokens[in.row] = (int32_t)(G[first] >> 32);
    a.row_path[in.row] = path;
  }
}

// One-warp resolve of up to 32 candidates: lane i holds code v (0 for "no candidate").
// Same arithmetic as resolve_block; nc is the number of non-zero codes.
__device__ void resolve_warp(uint64_t v, int nc, const ResolveIn& in, const RowArgs& a, int path) {
  const int lane = threadIdx.x & 31;
  const unsigned FULL = 0xffffffffu;
  v = warp_sort(v, true);  // key desc, index asc; zeros last
  int n1 = nc;
  if (in.tk && in.k <= nc) {
    const uint64_t vk = __shfl_sync(FULL, v, in.k - 1);
    const uint32_t Kk = (uint32_t)(vk >> 32);
    n1 = __popc(__ballot_sync(FULL, lane < nc && (uint32_t)(v >> 32) >= Kk));
  }
  float e = 0.0f;
  if (lane < n1) e = expf(__fsub_rn(key2f((uint32_t)(v >> 32)), in.m));
  double S = warp_allreduce((double)e, SumD());
  int n2 = n1;
  if (in.tp_on && n1 > 1) {
    const float S32 = (float)S;
    double c = lane < n1 ? (double)__fdiv_rn(e, S32) : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      double y = __shfl_up_sync(FULL, c, o);
      if (lane >= o) c += y;
    }
    n2 = 1 + __popc(__ballot_sync(FULL, lane < n1 - 1 && (float)c <= in.tp));
    if (n2 > n1) n2 = n1;
    S = warp_allreduce(lane < n2 ? (double)e : 0.0, SumD());
  }
  const float Sf = (float)S;
  const uint32_t idx = ~(uint32_t)v;
  float pr = 0.0f;
  if (lane < n2) {
    pr = __fdiv_rn(e, Sf);
    if (a.kept_out) a.kept_out[(int64_t)in.row * in.V + idx] = 1;
    if (a.probs_out) a.probs_out[(int64_t)in.row * in.V + idx] = pr;
  }
  uint64_t w = lane < n2 ? (((uint64_t)idx << 32) | __float_as_uint(pr)) : ~0ull;
  w = warp_sort(w, false);  // index asc
  double c = lane < n2 ? (double)__uint_as_float((uint32_t)w) : 0.0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    double y = __shfl_up_sync(FULL, c, o);
    if (lane >= o) c += y;
  }
  const double tot = __shfl_sync(FULL, c, 31);
  const double target = (double)in.u * tot;
  const unsigned hit = __ballot_sync(FULL, lane < n2 && c > target);
  int first = hit ? (__ffs(hit) - 1) : (n2 - 1);
  const uint64_t wf = __shfl_sync(FULL, w, first);
  if (lane == 0) {
    a.tokens[in.row] = (int32_t)(wf >> 32);
    a.row_path[in.row] = path;
  }
}

// =========================================================================================
// K2: resolve kernel — one CTA per row.
//
// Greedy rows: the largest argmax code of the row's slices.  Sampled rows: the exact row max
// of z over the slices' maxima of the non-history values and over the history values, whose
// penalties are applied here from the raw logits the streaming kernel set aside
// (sampling.py:52-66: x > 0 ? x / rep : x * rep, then x - (freq * count + pres)); y = z / T
// (sampling.py:146); every candidate and every history value divided exactly and kept when y
// is finite and at or above the exact min-p key (sampling.py:89-94), then the sort / top-k /
// top-p / draw of resolve_warp or resolve_block.  Rows that need the whole vocabulary (top-p
// only or no filter on a large vocabulary), rows with NaN / +inf / only -inf after scaling
// (the NaN guard, sampling.py:159-160), and rows whose candidates overflow the fixed buffers go
// to the deferred list for the second kernel.
// =========================================================================================
struct GatherArgs {
  const uint4* summ;        // [B][MAXSL]
  const uint64_t* cand;     // [B][MAXSL][SEGCAP]
  int MAXSL, SEGCAP, C, G;  // slice stride, segment capacity, chunks per row, streaming grid
  int64_t N;                // chunks in all
  int nseg;                 // history segments per row
  const int32_t* seg2;      // [B][nseg + 1] absolute pair offsets (K0)
  const float* hraw;        // raw logit at each pair's id (streaming kernel)
  const uint32_t* rowflag;  // [B] history flags of K0
};

// Largest CTA index whose chunk range [c N / G, (c + 1) N / G) starts at or before chunk x.
__device__ __forceinline__ int resolve_cta_of_chunk(int64_t x, int64_t N, int G) {
  const int64_t c = ((x + 1) * (int64_t)G - 1) / N;
  return (int)(c < G - 1 ? c : G - 1);
}

__global__ void __launch_bounds__(NT, 2) lss_resolve_kernel(const RowArgs a, const GatherArgs g) {
  constexpr int HPT = 4;  // history values kept in registers per thread
  __shared__ uint64_t G[FAST_CAP];
  __shared__ float E[FAST_CAP];
  __shared__ uint64_t r64[NWARP];
  __shared__ double rd[NWARP];
  __shared__ uint32_t r32[NWARP];
  __shared__ int ri[NWARP];
  __shared__ float rf[NWARP];
  __shared__ uint32_t s_pre[NT + 1];
  __shared__ uint32_t s_cnt[NT];
  __shared__ uint32_t s_n, s_kmp;
  __shared__ int s_defer;
  __shared__ float s_my;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int V = a.V;
  const float T = a.temperature[row];
  const int k = a.top_k[row];
  const float mp = a.min_p[row], tp = a.top_p[row], u = a.uniforms[row];
  const float rp = a.rep[row], fq = a.freq[row], pr = a.pres[row];
  const bool greedy = T <= 0.0f;
  const bool tk_on = k > 0 && k < V;
  const bool mp_on = mp > 0.0f && mp < 1.0f;
  const bool bounded = greedy || tk_on || mp_on || V <= FAST_CAP / 2;
  const int cf = resolve_cta_of_chunk((int64_t)row * g.C, g.N, g.G);
  const int cl = resolve_cta_of_chunk((int64_t)(row + 1) * g.C - 1, g.N, g.G);
  const int nsl = cl - cf + 1;  // slices of this row (<= MAXSL)
  const RedScratch rs{r64, rd, r32, ri};
  pdl_trigger();
  pdl_wait();  // the streaming kernel's summaries, candidates and raw history values are visible
  if (tid == 0 && g.rowflag[row]) atomicOr(a.err, g.rowflag[row]);
  const uint4* sm_row = g.summ + (int64_t)row * g.MAXSL;
  if (greedy) {
    uint64_t b = 0;
    for (int s = tid; s < nsl; s += NT) {
      const uint4 sm = sm_row[s];
      const uint64_t c = ((uint64_t)sm.y << 32) | sm.x;
      b = c > b ? c : b;
    }
    b = block_allreduce(b, MaxU64(), r64);
    if (tid == 0) {
      a.tokens[row] = (int32_t)(~(uint32_t)b);
      a.row_path[row] = LSS_PATH_GREEDY;
    }
    return;
  }
  if (!bounded) {
    if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
    return;
  }
  // One round trip for the common case: the summaries, the first SPEC slots of every slice's
  // segment and the row's history values are requested together.
  const int SPEC = max(1, min(256, NT / max(nsl, 1)));
  const int ss = tid / SPEC, si = tid - ss * SPEC;
  uint64_t cspec = 0;
  if (ss < nsl) cspec = g.cand[((int64_t)row * g.MAXSL + ss) * g.SEGCAP + si];
  uint4 sm = make_uint4(0u, 0u, 0u, 0u);
  if (tid < nsl) sm = sm_row[tid];
  const int32_t* so = g.seg2 + (int64_t)row * (g.nseg + 1);
  const int hb = so[0], he = so[g.nseg];
  float hz[HPT];
  int hid[HPT];
  float hmax = -INFINITY;
#pragma unroll
  for (int q = 0; q < HPT; ++q) {
    const int e = hb + tid + q * NT;
    hid[q] = -1;
    hz[q] = -INFINITY;
    if (e < he) {
      hid[q] = a.uniq_ids[e];
      hz[q] = penalise(g.hraw[e], rp, fq, pr, a.uniq_cnt[e]);
      hmax = fmax_nan(hmax, hz[q]);
    }
  }
  for (int e = hb + tid + HPT * NT; e < he; e += NT)
    hmax = fmax_nan(hmax, penalise(g.hraw[e], rp, fq, pr, a.uniq_cnt[e]));
  // Slice summaries: max key of the non-history values (all ones: NaN / +inf), flags, counts.
  const uint32_t mkey = block_allreduce(tid < nsl ? sm.x : 0u, MaxU32(), r32);
  const uint32_t fl = block_allreduce(tid < nsl ? sm.w : 0u, OrU32(), r32);
  const uint32_t over = block_allreduce(tid < nsl && sm.z > (uint32_t)g.SEGCAP ? 1u : 0u, OrU32(), r32);
  hmax = block_allreduce(hmax, MaxF(), rf);
  // Prefix of the counts beyond the speculated slots.
  uint32_t tot;
  const uint32_t rest = (tid < nsl && sm.z > (uint32_t)SPEC) ? min(sm.z, (uint32_t)g.SEGCAP) - (uint32_t)SPEC : 0u;
  const uint32_t pre = block_excl_scan(rest, r32, tot);
  if (tid < nsl) {
    s_pre[tid] = pre;
    s_cnt[tid] = sm.z;
  }
  __syncthreads();
  if (tid == 0) {
    s_pre[nsl] = tot;
    const float mz = mkey == 0xffffffffu ? NAN : key2f(mkey);
    const float M = fmax_nan(mz, hmax);
    const float my = __fdiv_rn(M, T);
    const bool special = !(my == my) || my == INFINITY || my == -INFINITY;
    s_defer = (fl != 0u || over != 0u || special) ? 1 : 0;
    s_my = my;
    s_kmp = (!special && mp_on) ? minp_key(my, mp) : KEY_FINITE_MIN;
    s_n = 0u;
  }
  __syncthreads();
  if (s_defer) {
    if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
    return;
  }
  const float my = s_my;
  const uint32_t Kmp = s_kmp;
  auto push = [&](float y, uint32_t low) {
    const uint32_t yk = f2key(y);
    if (y > -INFINITY && yk >= Kmp) {
      const uint32_t pos = atomicAdd(&s_n, 1u);
      if (pos < (uint32_t)FAST_CAP) G[pos] = ((uint64_t)yk << 32) | low;
    }
  };
  // Streaming kernel's candidates (history positions are not among them).
  if (ss < nsl && (uint32_t)si < s_cnt[ss] && si < g.SEGCAP)
    push(__fdiv_rn(key2f((uint32_t)(cspec >> 32)), T), (uint32_t)cspec);
  const uint32_t total = s_pre[nsl];
  for (uint32_t i = tid; i < total; i += NT) {
    int lo_s = 0, hi_s = nsl - 1;  // last slice whose prefix is <= i
    while (lo_s < hi_s) {
      const int mid = (lo_s + hi_s + 1) >> 1;
      if (s_pre[mid] <= i) lo_s = mid; else hi_s = mid - 1;
    }
    const uint64_t c = g.cand[((int64_t)row * g.MAXSL + lo_s) * g.SEGCAP + SPEC + (i - s_pre[lo_s])];
    push(__fdiv_rn(key2f((uint32_t)(c >> 32)), T), (uint32_t)c);
  }
  // History values (penalised above).
#pragma unroll
  for (int q = 0; q < HPT; ++q)
    if (hid[q] >= 0) push(__fdiv_rn(hz[q], T), ~(uint32_t)hid[q]);
  for (int e = hb + tid + HPT * NT; e < he; e += NT)
    push(__fdiv_rn(penalise(g.hraw[e], rp, fq, pr, a.uniq_cnt[e]), T), ~(uint32_t)a.uniq_ids[e]);
  __syncthreads();
  const uint32_t nk = s_n;
  if (nk == 0u || nk > (uint32_t)FAST_CAP) {
    if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
    return;
  }
  const ResolveIn in{my, tk_on, k, tp > 0.0f && tp < 1.0f, tp, u, row, V};
  if (nk <= 32u) {
    if (tid < 32) resolve_warp(tid < (int)nk ? G[tid] : 0ull, (int)nk, in, a, LSS_PATH_GATHER);
  } else {
    resolve_block<FAST_CAP>(G, E, (int)nk, in, a, rs, LSS_PATH_GATHER);
  }
}

}  // namespace lss
