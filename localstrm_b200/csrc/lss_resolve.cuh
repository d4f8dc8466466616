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
// `presorted`: G[0, nc) is already in that order.
template <int CAPN>
__device__ void resolve_block(uint64_t* G, float* E, int nc, const ResolveIn& in, const RowArgs& a,
                              const RedScratch& rs, int path, bool presorted = false) {
  constexpr int PER = CAPN / NT;  // items per thread, contiguous
  const int tid = threadIdx.x;
  if (!presorted) {
    const int np = next_pow2(nc > 1 ? nc : 1);
    for (int i = nc + tid; i < np; i += NT) G[i] = 0ull;
    __syncthreads();
    bitonic_sort(G, np, true);  // key desc, index asc
  }
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
// Greedy rows: the largest argmax code of the row's slices.  Sampled rows:
//   * before it waits for the streaming kernel (inputs only): the history as unique (id, count)
//     pairs in a shared hash table (torch.unique(..., return_counts=True), sampling.py:52), the
//     raw logit at each id read from the logits, and the penalties applied (sampling.py:55-66:
//     x > 0 ? x / rep : x * rep, then x - (freq * count + pres));
//   * the exact row max of z over the candidates that are not history ids and over the
//     penalised history values; y = z / T (sampling.py:146); every such value kept when y is
//     finite and at or above the exact min-p key (sampling.py:89-94);
//   * the check that makes the candidates exact: every value of a slice that is not a
//     candidate lies below the slice's largest threshold U (streaming kernel), so once the
//     cut (min-p key, and the k-th largest kept value for top-k rows) lies above every U / T,
//     nothing outside the candidates can survive.  A slice whose U / T reaches the cut (a
//     history value counted there with its raw value raised its threshold) is re-read from the
//     logits for every value at or above the cut, and the cut is taken again;
//   * then the sort / top-k / top-p / draw of resolve_warp or resolve_block.
// Rows that need the whole vocabulary (top-p only or no filter on a large vocabulary), rows with
// NaN / +inf / only -inf after scaling (the NaN guard, sampling.py:159-160), rows with more
// than RH_CAP history ids, and rows whose candidates overflow the fixed buffers go to the
// deferred list for the second kernel.
// =========================================================================================
constexpr int RH_CAP = 2048;          // history ids of a row this kernel takes
constexpr int RH_SLOTS = 2 * RH_CAP;  // its shared hash table (load <= 1/2)

struct GatherArgs {
  const uint4* summ;        // [B][MAXSL]: {max key | argmax lo, threshold key | argmax hi, count, flags}
  const uint64_t* cand;     // [B][MAXSL][SEGCAP]
  int MAXSL, SEGCAP, C, G;  // slice stride, segment capacity, chunks per row, streaming grid
  int64_t N;                // chunks in all
  int CE;                   // logits per chunk
  int dtype;                // LSS_DTYPE_* of the logits
  const uint32_t* cmax;     // [B * C]: key of each sampled chunk's max (streaming kernel)
};

// Dynamic shared memory of K2: hash keys and counts, the penalised value and the slot of each
// listed pair.
__host__ __device__ constexpr int resolve_smem_bytes() { return RH_SLOTS * 8 + RH_CAP * 4 + RH_CAP * 2; }

// Largest CTA index whose chunk range [c N / G, (c + 1) N / G) starts at or before chunk x.
__device__ __forceinline__ int resolve_cta_of_chunk(int64_t x, int64_t N, int G) {
  const int64_t c = ((x + 1) * (int64_t)G - 1) / N;
  return (int)(c < G - 1 ? c : G - 1);
}

__device__ __forceinline__ float load_logit(const void* base, int dtype, int64_t i) {
  if (dtype == LSS_DTYPE_F32) return reinterpret_cast<const float*>(base)[i];
  const uint16_t h = reinterpret_cast<const uint16_t*>(base)[i];
  if (dtype == LSS_DTYPE_BF16) return __uint_as_float((uint32_t)h << 16);
  return __half2float(__ushort_as_half(h));
}

__global__ void __launch_bounds__(NT, 2) lss_resolve_kernel(const RowArgs a, const GatherArgs g) {
  constexpr int HPT = RH_CAP / NT;  // history ids per thread
  constexpr int PER = FAST_CAP / NT;
  extern __shared__ __align__(16) uint32_t rsm[];
  uint32_t* hkeys = rsm;
  uint32_t* hcnts = rsm + RH_SLOTS;
  float* hz = reinterpret_cast<float*>(rsm + 2 * RH_SLOTS);
  uint16_t* hslot = reinterpret_cast<uint16_t*>(hz + RH_CAP);
  __shared__ uint64_t G[FAST_CAP];
  __shared__ float E[FAST_CAP];
  __shared__ uint64_t r64[NWARP];
  __shared__ double rd[NWARP];
  __shared__ uint32_t r32[NWARP];
  __shared__ int ri[NWARP];
  __shared__ float rf[NWARP];
  __shared__ uint32_t s_pre[NT + 1];
  __shared__ uint32_t s_cnt[NT];
  __shared__ uint32_t s_uy[NT];
  __shared__ uint32_t s_rbm[NT / 32];
  __shared__ uint32_t s_n, s_kmp, s_nh, s_hflags;
  __shared__ int s_defer;
  __shared__ float s_my;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
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
  const int nsl = cl - cf + 1;  // slices of this row (<= MAXSL <= NT)
  const RedScratch rs{r64, rd, r32, ri};
  const char* zrow = reinterpret_cast<const char*>(a.logits) +
                     (int64_t)row * a.row_stride * (g.dtype == LSS_DTYPE_F32 ? 4 : 2);

  // ---- history (inputs only: runs while the streaming kernel may still be busy elsewhere)
  const bool hist_on = a.use_hist && !greedy && bounded && (rp != 1.0f || fq != 0.0f || pr != 0.0f);
  int hb = 0, he = 0;
  const bool bad_range = hist_on && !hist_range(a.hist_off, row, a.H, hb, he);
  const int H = he - hb;
  const bool hist_long = H > RH_CAP;
  const uint32_t cap = (H > 0 && !hist_long) ? (uint32_t)next_pow2(max(2 * H, 64)) : 0u;
  if (tid == 0) {
    s_nh = 0u;
    s_hflags = bad_range ? LSS_FLAG_BAD_HISTORY : 0u;
  }
  float hmax = -INFINITY;
  bool hspecial = false;
  if (cap) {
    int idv[HPT];
#pragma unroll
    for (int t = 0; t < HPT; ++t) {
      const int j = t * NT + tid;
      idv[t] = j < H ? a.hist_ids[hb + j] : INT32_MIN;
    }
    for (uint32_t s = tid; s < cap; s += NT) {
      hkeys[s] = EMPTY;
      hcnts[s] = 0u;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < HPT; ++t) {
      const int id = idv[t];
      bool fresh = false;
      uint32_t slot = 0;
      if (id != INT32_MIN) {
        if (id < 0 || id >= V) {
          atomicOr(&s_hflags, LSS_FLAG_BAD_HISTORY);
        } else {
          uint32_t h = ((uint32_t)id * 2654435761u) & (cap - 1u);
          for (uint32_t probe = 0; probe < cap; ++probe) {
            const uint32_t old = atomicCAS(&hkeys[h], EMPTY, (uint32_t)id);
            if (old == EMPTY || old == (uint32_t)id) {
              atomicAdd(&hcnts[h], 1u);
              fresh = old == EMPTY;
              slot = h;
              break;
            }
            h = (h + 1u) & (cap - 1u);
          }
        }
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, fresh);
      if (bal) {
        const int leader = __ffs(bal) - 1;
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(&s_nh, (uint32_t)__popc(bal));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (fresh) hslot[base + __popc(bal & ((1u << lane) - 1u))] = (uint16_t)slot;
      }
    }
    __syncthreads();
    const int nh = (int)s_nh;
    // The raw logit at every listed id (all requested at once), then the penalties.
    int ids[HPT];
    float raw[HPT];
#pragma unroll
    for (int t = 0; t < HPT; ++t) {
      const int i = t * NT + tid;
      ids[t] = i < nh ? (int)hkeys[hslot[i]] : -1;
      raw[t] = ids[t] >= 0 ? load_logit(zrow, g.dtype, ids[t]) : 0.0f;
    }
#pragma unroll
    for (int t = 0; t < HPT; ++t) {
      const int i = t * NT + tid;
      if (ids[t] >= 0) {
        const float v = penalise(raw[t], rp, fq, pr, (int)hcnts[hslot[i]]);
        hz[i] = v;
        hmax = fmax_nan(hmax, v);
        hspecial |= !(v == v) || v == INFINITY;
      }
    }
  }
  // Is id one of the row's history ids?
  auto in_hist = [&](uint32_t id) -> bool {
    if (!cap) return false;
    uint32_t h = (id * 2654435761u) & (cap - 1u);
    for (uint32_t probe = 0; probe < cap; ++probe) {
      const uint32_t key = hkeys[h];
      if (key == id) return true;
      if (key == EMPTY) return false;
      h = (h + 1u) & (cap - 1u);
    }
    return false;
  };

  // No early trigger for the deferred-row kernel: its clusters would then wait on SMs where
  // the last rows of this kernel still run (the call measured 0.7-6.5 us slower with one).
  pdl_wait();  // the streaming kernel's summaries and candidates are complete and visible
  if (tid == 0 && s_hflags) atomicOr(a.err, s_hflags);
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
  if (!bounded || (hist_on && hist_long)) {
    if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
    return;
  }
  // One round trip for the common case: the summaries and the first SPEC slots of every
  // slice's segment are requested together.
  const int SPEC = max(1, min(256, NT / max(nsl, 1)));
  const int ss = tid / SPEC, si = tid - ss * SPEC;
  uint64_t cspec = 0;
  if (ss < nsl) cspec = g.cand[((int64_t)row * g.MAXSL + ss) * g.SEGCAP + si];
  uint4 sm = make_uint4(0u, 0u, 0u, 0u);
  if (tid < nsl) sm = sm_row[tid];
  // Per slice: count, and U / T as a key (0: every finite value of the slice is a candidate).
  uint32_t uy = 0u;
  if (tid < nsl && sm.y > KEY_FINITE_MIN) uy = f2key(__fdiv_rn(key2f(sm.y), T));
  const uint32_t fl = block_allreduce((tid < nsl ? sm.w : 0u) | (hspecial ? 1u : 0u) |
                                          (tid < nsl && sm.z > (uint32_t)g.SEGCAP ? 2u : 0u),
                                      OrU32(), r32);
  const uint32_t rest = (tid < nsl && sm.z > (uint32_t)SPEC) ? min(sm.z, (uint32_t)g.SEGCAP) - (uint32_t)SPEC : 0u;
  uint32_t tot;
  const uint32_t pre = block_excl_scan(rest, r32, tot);
  if (tid < nsl) {
    s_pre[tid] = pre;
    s_cnt[tid] = sm.z;
    s_uy[tid] = uy;
  }
  if (tid == 0) s_pre[nsl] = tot;
  __syncthreads();
  if (fl != 0u) {  // NaN / +inf (raw or penalised), or a segment overflowed
    if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
    return;
  }
  // The candidate of flat position i beyond the speculated slots.
  auto cand_at = [&](uint32_t i) -> uint64_t {
    int lo_s = 0, hi_s = nsl - 1;  // last slice whose prefix is <= i
    while (lo_s < hi_s) {
      const int mid = (lo_s + hi_s + 1) >> 1;
      if (s_pre[mid] <= i) lo_s = mid; else hi_s = mid - 1;
    }
    return g.cand[((int64_t)row * g.MAXSL + lo_s) * g.SEGCAP + SPEC + (i - s_pre[lo_s])];
  };
  const bool spec_ok = ss < nsl && (uint32_t)si < s_cnt[ss] && si < g.SEGCAP;
  const bool spec_nh = spec_ok && !in_hist(~(uint32_t)cspec);
  const uint32_t total = s_pre[nsl];
  // Row max of z: the candidates that are not history ids, and the penalised history values.
  float zmax = spec_nh ? key2f((uint32_t)(cspec >> 32)) : -INFINITY;
  for (uint32_t i = tid; i < total; i += NT) {
    const uint64_t c = cand_at(i);
    if (!in_hist(~(uint32_t)c)) zmax = fmaxf(zmax, key2f((uint32_t)(c >> 32)));
  }
  zmax = block_allreduce(fmax_nan(zmax, hmax), MaxF(), rf);
  if (tid == 0) {
    const float my = __fdiv_rn(zmax, T);
    const bool special = !(my == my) || my == INFINITY || my == -INFINITY;
    s_defer = special ? 1 : 0;
    s_my = my;
    s_kmp = (!special && mp_on) ? minp_key(my, mp) : KEY_FINITE_MIN;
    s_n = 0u;
  }
  __syncthreads();
  if (s_defer) {
    if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
    return;
  }
  float my = s_my;
  const uint32_t Kmp = s_kmp;
  auto push_key = [&](uint32_t yk, uint32_t low) {
    const uint32_t pos = atomicAdd(&s_n, 1u);
    if (pos < (uint32_t)FAST_CAP) G[pos] = ((uint64_t)yk << 32) | low;
  };
  auto push = [&](float y, uint32_t low) {
    const uint32_t yk = f2key(y);
    if (y > -INFINITY && yk >= Kmp) push_key(yk, low);
  };
  if (spec_nh) push(__fdiv_rn(key2f((uint32_t)(cspec >> 32)), T), (uint32_t)cspec);
  for (uint32_t i = tid; i < total; i += NT) {
    const uint64_t c = cand_at(i);
    if (!in_hist(~(uint32_t)c)) push(__fdiv_rn(key2f((uint32_t)(c >> 32)), T), (uint32_t)c);
  }
  for (int i = tid; i < (int)s_nh; i += NT) push(__fdiv_rn(hz[i], T), ~hkeys[hslot[i]]);
  __syncthreads();
  int nk = (int)s_n;
  if (nk == 0 || nk > FAST_CAP) {
    if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
    return;
  }
  // Block helpers over G[0, n): the k-th largest key (radix select, eight bits per pass, the
  // bins in s_pre), and an in-place compaction of the entries a predicate keeps.
  auto kth_largest = [&](int n, int kk) -> uint32_t {
    uint32_t prefix = 0u, mask = 0u;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += NT) s_pre[b] = 0u;
      __syncthreads();
      for (int i = tid; i < n; i += NT) {
        const uint32_t key = (uint32_t)(G[i] >> 32);
        if ((key & mask) == prefix) atomicAdd(&s_pre[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid < 32) {
        // Lane l holds bins 255 - 8l .. 248 - 8l (largest digits first).
        uint32_t c8[8], loc = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          c8[q] = s_pre[255 - (8 * lane + q)];
          loc += c8[q];
        }
        uint32_t incl = loc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, incl >= (uint32_t)kk);
        const int L = hit ? __ffs(hit) - 1 : 31;
        if (lane == L) {
          uint32_t acc = incl - loc;
          int d = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (acc + c8[q] >= (uint32_t)kk) {
              d = 255 - (8 * lane + q);
              break;
            }
            acc += c8[q];
          }
          s_pre[256] = (uint32_t)d;
          s_pre[257] = acc;  // entries with a larger digit
        }
      }
      __syncthreads();
      prefix |= s_pre[256] << shift;
      mask |= 255u << shift;
      kk -= (int)s_pre[257];
      __syncthreads();
    }
    return prefix;
  };
  auto compact = [&](int n, auto keep_fn) -> int {
    uint64_t v[PER];
    uint32_t keep = 0;
#pragma unroll
    for (int j2 = 0; j2 < PER; ++j2) {
      const int i = tid * PER + j2;
      v[j2] = i < n ? G[i] : 0ull;
      if (i < n && keep_fn(v[j2])) keep |= 1u << j2;
    }
    uint32_t all;
    const uint32_t at = block_excl_scan((uint32_t)__popc(keep), r32, all);
    __syncthreads();
    uint32_t o = at;
#pragma unroll
    for (int j2 = 0; j2 < PER; ++j2)
      if (keep & (1u << j2)) G[o++] = v[j2];
    __syncthreads();
    return (int)all;
  };
  // The cut: the min-p key, and for top-k rows the k-th largest kept value.
  uint32_t cut = Kmp;
  if (tk_on && k <= nk) cut = max(cut, kth_largest(nk, k));
  const uint32_t umax = block_allreduce(tid < nsl ? s_uy[tid] : 0u, MaxU32(), r32);
  if (umax >= cut) {
    // ---- re-read the slices whose threshold reaches the cut: in such a slice, the chunks whose
    // max reaches it (the streaming kernel recorded every chunk's max).  Their candidates leave
    // G, and every value of theirs at or above the cut that is not a history id comes back.  A
    // row has at most C <= NT chunks: the chunk list fits s_cnt and its bitmap s_rbm.
    const int ES = g.dtype == LSS_DTYPE_F32 ? 4 : 2;
    const int VPC = g.CE * ES / 16;  // 16-byte vectors per chunk
    // Most values lie below zc, under which z / T cannot reach the cut: they cost one compare.
    const float zc = z_floor_for(key2f(cut), T);
    const uint32_t zck = f2key(zc);
    const int64_t r0 = (int64_t)row * g.C;
    for (int w2 = tid; w2 < NT / 32; w2 += NT) s_rbm[w2] = 0u;
    if (tid == 0) s_kmp = 0u;  // chunk-list length
    __syncthreads();
    for (int ch = tid; ch < g.C; ch += NT) {
      const int sl = resolve_cta_of_chunk(r0 + ch, g.N, g.G) - cf;
      if (s_uy[sl] >= cut && g.cmax[r0 + ch] >= zck) {
        s_cnt[atomicAdd(&s_kmp, 1u)] = (uint32_t)ch;
        atomicOr(&s_rbm[ch >> 5], 1u << (ch & 31));
      }
    }
    __syncthreads();
    const int nrc = (int)s_kmp;
    nk = compact(nk, [&](uint64_t c) {
      const uint32_t idx = ~(uint32_t)c;
      const int ch = (int)(idx / (uint32_t)g.CE);
      return !((s_rbm[ch >> 5] >> (ch & 31)) & 1u) || in_hist(idx);
    });
    if (tid == 0) s_n = (uint32_t)nk;
    __syncthreads();
    auto take = [&](float z, int idx) {
      if (!(z >= zc) || idx >= V) return;
      const float y = __fdiv_rn(z, T);
      const uint32_t yk = f2key(y);
      if (y > -INFINITY && yk >= cut && !in_hist((uint32_t)idx)) push_key(yk, ~(uint32_t)idx);
    };
    if ((reinterpret_cast<uintptr_t>(zrow) & 15u) == 0) {
      // Four 16-byte vectors per thread requested at once.
      for (int q0 = 0; q0 < nrc * VPC; q0 += 4 * NT) {
        uint4 w[4];
        int i0[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int q = q0 + t * NT + tid;
          i0[t] = -1;
          w[t] = make_uint4(0u, 0u, 0u, 0u);
          if (q < nrc * VPC) {
            i0[t] = (int)s_cnt[q / VPC] * g.CE + (q % VPC) * (16 / ES);
            if (i0[t] + 16 / ES <= V) w[t] = reinterpret_cast<const uint4*>(zrow + (int64_t)i0[t] * ES)[0];
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (i0[t] < 0 || i0[t] >= V) continue;
          if (i0[t] + 16 / ES > V) {  // the row ends inside this vector: its last values one by one
            for (int i = i0[t]; i < V; ++i) take(load_logit(zrow, g.dtype, i), i);
            continue;
          }
          const uint32_t x[4] = {w[t].x, w[t].y, w[t].z, w[t].w};
#pragma unroll
          for (int j2 = 0; j2 < 4; ++j2) {
            if (ES == 4) {
              take(__uint_as_float(x[j2]), i0[t] + j2);
            } else if (g.dtype == LSS_DTYPE_BF16) {
              take(__uint_as_float(x[j2] << 16), i0[t] + 2 * j2);
              take(__uint_as_float(x[j2] & 0xffff0000u), i0[t] + 2 * j2 + 1);
            } else {
              take(__half2float(__ushort_as_half((uint16_t)(x[j2] & 0xffffu))), i0[t] + 2 * j2);
              take(__half2float(__ushort_as_half((uint16_t)(x[j2] >> 16))), i0[t] + 2 * j2 + 1);
            }
          }
        }
      }
    } else {
      for (int q = tid; q < nrc * g.CE; q += NT) {
        const int i = (int)s_cnt[q / g.CE] * g.CE + q % g.CE;
        if (i < V) take(load_logit(zrow, g.dtype, i), i);
      }
    }
    __syncthreads();
    nk = (int)s_n;
    if (nk > FAST_CAP) {
      if (tid == 0) a.defer_rows[atomicAdd(&a.counters[2], 1u)] = row;
      return;
    }
    // Every value at or above the old cut is now present once, and the exact cut is at least
    // the old one: the max, the min-p key and the k-th largest again.
    uint32_t mk = 0u;
    for (int i = tid; i < nk; i += NT) mk = max(mk, (uint32_t)(G[i] >> 32));
    mk = block_allreduce(mk, MaxU32(), r32);
    my = key2f(mk);
    const uint32_t Kmp2 = mp_on ? minp_key(my, mp) : KEY_FINITE_MIN;
    cut = Kmp2;
    nk = compact(nk, [&](uint64_t c) { return (uint32_t)(c >> 32) >= Kmp2; });
    if (tk_on && k <= nk) cut = max(cut, kth_largest(nk, k));
  }
  // The survivors of the cut, sorted (value desc, index asc) unless one warp takes them.
  if (cut > Kmp) nk = compact(nk, [&](uint64_t c) { return (uint32_t)(c >> 32) >= cut; });
  const ResolveIn in{my, tk_on, k, tp > 0.0f && tp < 1.0f, tp, u, row, V};
  if (nk <= 32) {
    if (tid < 32) resolve_warp(tid < nk ? G[tid] : 0ull, nk, in, a, LSS_PATH_GATHER);
  } else {
    resolve_block<FAST_CAP>(G, E, nk, in, a, rs, LSS_PATH_GATHER);
  }
}

}  // namespace lss
