// lss_stream.cuh — K1: the streaming pass over the logits (the hot path).
//
// The logits of a call are cut into chunks of ST_CB bytes (1,024 f32 or 2,048 16-bit logits; a
// row's last chunk may be short), B * C chunks in row order.  The grid is persistent (one CTA
// per SM) and CTA b owns the contiguous chunk range [b N / G, (b + 1) N / G): every CTA streams
// the same number of bytes to within one chunk.  The part of a row that falls into one CTA's
// range is a slice of that row; a row has one to a few slices.
//
// Inside a CTA every warp works alone: warp w takes chunks w, w + 16, w + 32, ... of the range,
// each through its own ring of ST_R shared-memory stages filled by bulk async copies that its
// lane 0 issues (and bounded mbarrier waits), so that a warp never waits for another warp and
// the CTA keeps 16 x (ST_R - 1) chunks in flight.  The pass reads nothing but the logits and
// the row parameters, so it is the first kernel of a call and starts streaming at once; the
// history (sampling.py:52-66) is left to the resolve kernel.  Per chunk the warp
//   * takes the chunk max of the raw values and folds it into the slice's running max (a
//     shared atomic max in the slice's slot);
//   * for top-k rows, counts its values above the current threshold into the slice's shared
//     count histogram (bins of 1/16 nat of y below a fixed reference) and raises the slice's
//     top-k threshold from it;
//   * writes the values at or above the candidate threshold into the slice's segment, raises
//     the slice's record of the largest threshold used (a shared atomic max), and records the
//     chunk's max (so that a slice the resolve kernel must re-read costs it only the chunks
//     that can hold a survivor).
// The last warp to finish a slice writes the slice summary (running max or argmax code, the
// largest candidate threshold, candidate count, flags) and hands the slot to a later slice.
//
// What the resolve kernel can rely on: every value of the slice that is not a candidate lies
// below the slice's largest threshold U (or is -inf).  Without penalties every threshold is a
// lower bound of the exact one (the min-p floor is taken from a running max over a subset of
// the row, the top-k threshold lies below a value that k values of the slice reach), so the
// candidates hold every survivor.  With penalties a history value counts here with its raw
// value, which can raise a threshold above the exact one; the resolve kernel, which knows the
// penalised values, checks its exact cut against U and re-reads a slice whose U lies at or
// above it.  Thresholds are taken on z (y = z / T is monotone) with margins that cover every
// rounding of the exact filter, which the resolve kernel applies.
#pragma once

#include <type_traits>

#include "lss_common.cuh"

namespace lss {

constexpr int ST_NW = 16;                     // warps per CTA
constexpr int ST_NT = ST_NW * 32;
constexpr int ST_CB = 4096;                   // bytes per chunk
// Ring stages per warp.  Two stream faster than three on B200 (the headline pass 32.5 vs 35.6
// us, 16-bit rows with top-k unchanged) and one is slower (36.2 us): with 32 rather than 48 4 KB
// copies outstanding per SM the HBM stream runs closer to the copy peak.
constexpr int ST_R = 2;
constexpr int ST_NSLOT = 8;                   // slice slots per CTA
constexpr int ST_SEGCAP = 1024;               // candidate slots per slice
constexpr int ST_ROWTAB = 64;                 // rows whose parameters a CTA keeps in shared memory
constexpr int ST_GCAP = 160;                  // largest grid the workspace layout allows for
constexpr int ST_SB = ST_CB;                  // bytes of a stage: one chunk
constexpr int ST_STAGE_BYTES = ST_NW * ST_R * ST_SB;

constexpr int ITEM_SKIP = 1, ITEM_GREEDY = 2, ITEM_SAMPLE = 3;
// Summary flags: NaN / +inf among the slice's values.
constexpr uint32_t SUM_SPECIAL = 1u;

struct __align__(16) SliceSlot {
  uint32_t tag;         // local slice (row - first row of the CTA) that owns the slot
  uint32_t done;        // chunks of the slice finished
  uint32_t maxkey;      // running max key of z (0xffffffff: NaN or +inf seen)
  uint32_t count;       // candidate slots reserved
  uint32_t flags;
  uint32_t r0key;       // top-k: key of the histogram's reference value (0: not set yet)
  uint32_t taukey;      // top-k: key of the current threshold (0: none)
  uint32_t above;       // top-k: counted values above the reference
  unsigned long long best;  // greedy: argmax code
  uint32_t ukey;        // key of the largest candidate threshold any chunk used (0: none yet)
  uint32_t pad;
  uint32_t hist[NBIN];  // top-k: counted values by depth below the reference, 1/16 nat of y per bin
};

struct __align__(16) RowPrm {
  int mode;             // ITEM_*
  int k;                // top-k when active (0 < k < V), else 0
  float T;
  float tl;             // min-p active: T * ln(min_p), the floor's offset in z; else 0
  float sb;             // 16 / T: bins of the top-k histogram per unit of z
  float binw;           // T / 16
  int jsl;              // index of this CTA's slice among the row's slices
  int nch;              // chunks of the row in this CTA's range
};

struct StreamArgs {
  const void* logits;
  int64_t row_stride;   // elements
  int B, V, C;          // C: chunks per row
  int64_t N;            // B * C
  int MAXSL;            // slices per row reserved in the workspace (summary and segment stride)
  const float* temperature;
  const int32_t* top_k;
  const float* min_p;
  uint4* summ;          // [B][MAXSL]: {max key | argmax code lo, threshold key | argmax code hi, count, flags}
  uint64_t* cand;       // [B][MAXSL][ST_SEGCAP]: (key(z) << 32) | ~index
  uint32_t* cmax;       // [B * C]: key of each sampled chunk's max (all ones: NaN / +inf)
  uint32_t* header;     // workspace status words (word 0: error flags; word 2: deferred rows), cleared here
};

__host__ __device__ constexpr int stream_smem_bytes() {
  return ST_STAGE_BYTES + ST_NSLOT * (int)sizeof(SliceSlot) + ST_NW * ST_R * 8 + ST_ROWTAB * (int)sizeof(RowPrm) + 16;
}

// Largest CTA index whose range starts at or before chunk x (ranges [c N / G, (c + 1) N / G)).
__host__ __device__ __forceinline__ int cta_of_chunk(int64_t x, int64_t N, int G) {
  const int64_t c = ((x + 1) * (int64_t)G - 1) / N;
  return (int)(c < G - 1 ? c : G - 1);
}

// Parameters of `row` as the CTA whose range is [g0, g1) of N chunks (G CTAs) sees it.
__device__ __forceinline__ RowPrm make_row_prm(const StreamArgs& a, int row, int64_t g0, int64_t g1) {
  RowPrm p{};
  const int64_t rs = (int64_t)row * a.C;
  p.jsl = (int)blockIdx.x - cta_of_chunk(rs, a.N, (int)gridDim.x);
  p.nch = (int)(min(g1, rs + a.C) - max(g0, rs));
  const float T = a.temperature[row];
  const int k = a.top_k[row];
  const float mp = a.min_p[row];
  const bool greedy = T <= 0.0f;
  const bool tk = k > 0 && k < a.V;
  const bool mpon = mp > 0.0f && mp < 1.0f;
  // Rows whose survivors are not bounded (top-p only or no filter on a large vocabulary) go
  // to the second kernel whole; their chunks are not read here.
  const bool bounded = greedy || tk || mpon || a.V <= FAST_CAP / 2;
  p.mode = !bounded ? ITEM_SKIP : greedy ? ITEM_GREEDY : ITEM_SAMPLE;
  p.k = tk ? k : 0;
  p.T = T;
  p.tl = (!greedy && mpon) ? __fmul_rn(T, logf(mp)) : 0.0f;
  p.sb = greedy ? 0.0f : __fdiv_rn(BIN_PER_NAT, T);
  p.binw = greedy ? 0.0f : __fdiv_rn(T, BIN_PER_NAT);
  return p;
}

template <class T, class Op>
__device__ __forceinline__ T wred(T v, Op op) { return warp_allreduce(v, op); }

// Two 16-bit logits of a word (the lower address in the low half), compared and reduced as a
// pair: one instruction does the work of two widened f32 operations.
template <int DT>
__device__ __forceinline__ uint32_t pk_max(uint32_t a, uint32_t b) {  // NaN-propagating
  uint32_t r;
  if constexpr (DT == LSS_DTYPE_BF16) {
    const __nv_bfloat162 m = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                         *reinterpret_cast<const __nv_bfloat162*>(&b));
    r = *reinterpret_cast<const uint32_t*>(&m);
  } else {
    const __half2 m = __hmax2_nan(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    r = *reinterpret_cast<const uint32_t*>(&m);
  }
  return r;
}
template <int DT>
__device__ __forceinline__ uint32_t pk_ge(uint32_t a, uint32_t lev2) {  // 0xffff per half >= lev
  if constexpr (DT == LSS_DTYPE_BF16)
    return __hge2_mask(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&lev2));
  else
    return __hge2_mask(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&lev2));
}
// The level, in both halves, at or above which a 16-bit value x satisfies the f32 test
// `x >= lev && x > -inf`: the smallest 16-bit value >= max(lev, -FLT_MAX) (rounding toward
// +inf is exact here, since x itself is a 16-bit value).  A NaN level matches nothing.
template <int DT>
__device__ __forceinline__ uint32_t pk_level(float lev) {
  uint32_t h;
  if constexpr (DT == LSS_DTYPE_BF16)
    h = lev != lev ? 0x7fc0u : (uint32_t)__bfloat16_as_ushort(__float2bfloat16_ru(fmaxf(lev, -FLT_MAX)));
  else
    h = lev != lev ? 0x7e00u : (uint32_t)__half_as_ushort(__float2half_ru(fmaxf(lev, -FLT_MAX)));
  return h | (h << 16);
}
template <int DT>
__device__ __forceinline__ float pk_lo(uint32_t w) {
  if constexpr (DT == LSS_DTYPE_BF16) return __uint_as_float(w << 16);
  else return __half2float(__ushort_as_half((uint16_t)(w & 0xffffu)));
}
template <int DT>
__device__ __forceinline__ float pk_hi(uint32_t w) {
  if constexpr (DT == LSS_DTYPE_BF16) return __uint_as_float(w & 0xffff0000u);
  else return __half2float(__ushort_as_half((uint16_t)(w >> 16)));
}

template <int DT>
__global__ void __launch_bounds__(ST_NT, 1) lss_stream_kernel(const StreamArgs a) {
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  constexpr int CE = ST_CB / ES;            // logits per chunk
  constexpr int VPV = 16 / ES;              // logits per 16-byte vector
  constexpr int NV = ST_CB / 16 / 32;       // 16-byte vectors per lane (8)
  extern __shared__ __align__(1024) unsigned char smem[];
  SliceSlot* slots = reinterpret_cast<SliceSlot*>(smem + ST_STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST_STAGE_BYTES + ST_NSLOT * sizeof(SliceSlot));
  RowPrm* rtab = reinterpret_cast<RowPrm*>(bars + ST_NW * ST_R);
  // Set when a bounded wait gives up: every warp of the CTA then stops, waits (bounded) for its
  // own copies in flight and returns, with the error flag raised.
  volatile uint32_t* abort_w = reinterpret_cast<volatile uint32_t*>(rtab + ST_ROWTAB);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  const int64_t N = a.N;
  const int64_t g0 = (int64_t)blockIdx.x * N / G, g1 = (int64_t)(blockIdx.x + 1) * N / G;
  const int C = a.C, V = a.V;
  const int row0 = (int)(g0 / C);

  // ---- set-up: slots (slot q starts out owned by local slice q), barriers, row parameters
  {
    constexpr int W = (int)(sizeof(SliceSlot) / 4);
    uint32_t* sw = reinterpret_cast<uint32_t*>(slots);
    for (int i = tid; i < ST_NSLOT * W; i += ST_NT) sw[i] = (i % W == 0) ? (uint32_t)(i / W) : 0u;
    if (tid < ST_NW * ST_R) mbar_init(&bars[tid], 1);
    for (int i = tid; i < ST_ROWTAB; i += ST_NT)
      if (row0 + i < a.B) rtab[i] = make_row_prm(a, row0 + i, g0, g1);
    if (tid < ST_NW * ST_R) fence_barrier_init();
    if (tid == 0) *abort_w = 0u;
    // This call's status: the error flags and the deferred-row count start at zero.  (The
    // resolve kernel counts deferred rows only after it has waited for this grid; the flags
    // other CTAs may raise come from waits of seconds.)
    if (blockIdx.x == 0 && tid < 64) a.header[tid] = 0u;
  }
  __syncthreads();
  pdl_trigger();  // the resolve kernel may launch; it waits for this grid before reading

  auto prm_of = [&](int row) -> RowPrm {
    return row - row0 < ST_ROWTAB ? rtab[row - row0] : make_row_prm(a, row, g0, g1);
  };
  uint64_t* wbar = bars + warp * ST_R;
  unsigned char* wst = smem + (size_t)warp * ST_R * ST_SB;
  const int64_t gw = g0 + warp;
  // Positions (row, chunk of the row) are carried forward by adding chunks, so that the loop
  // divides only when it crosses into another row.
  struct Pos {
    int row, c;
  };
  auto adv = [&](Pos p, int k) -> Pos {
    p.c += k;
    if (p.c >= C) {
      const int q = p.c / C;
      p.row += q;
      p.c -= q * C;
    }
    return p;
  };
  const Pos pw{(int)(gw / C), (int)(gw - (gw / C) * C)};

  // Lane 0: start the copy of chunk g (at position p) into stage s (an arrival without bytes for
  // a skipped row or a misaligned chunk, whose logits the warp loads itself).
  auto issue = [&](Pos p, int s) {
    const int row = p.row;
    const int lo = p.c * CE;
    const int n = min(CE, V - lo);
    const char* src = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
    const int mode = prm_of(row).mode;
    const int nb = (mode != ITEM_SKIP && (reinterpret_cast<uintptr_t>(src) & 15) == 0) ? ((n * ES) & ~15) : 0;
    mbar_expect_tx(&wbar[s], (uint32_t)nb);
    if (nb > 0) bulk_g2s(wst + s * ST_SB, src, (uint32_t)nb, &wbar[s]);
  };
  if (lane == 0)
    for (int i = 0; i < ST_R; ++i)
      if (gw + (int64_t)i * ST_NW < g1) issue(adv(pw, i * ST_NW), i);
  __syncwarp();

  auto elem = [&](const unsigned char* st, int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(st)[i];
    if (DT == LSS_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(st)[i]);
    return __half2float(reinterpret_cast<const __half*>(st)[i]);
  };
  auto set_neg_inf = [&](unsigned char* st, int i) {
    if (DT == LSS_DTYPE_F32) reinterpret_cast<float*>(st)[i] = -INFINITY;
    else if (DT == LSS_DTYPE_BF16) reinterpret_cast<uint16_t*>(st)[i] = 0xff80u;
    else reinterpret_cast<uint16_t*>(st)[i] = 0xfc00u;
  };
  auto copy_elem = [&](unsigned char* st, int i, const char* src) {
    if (DT == LSS_DTYPE_F32) reinterpret_cast<float*>(st)[i] = reinterpret_cast<const float*>(src)[i];
    else reinterpret_cast<uint16_t*>(st)[i] = reinterpret_cast<const uint16_t*>(src)[i];
  };
  using MaskT = typename std::conditional<(NV * VPV > 32), unsigned long long, uint32_t>::type;
  // The logits of 16-byte vector q of a stage, widened to f32.
  auto widen = [&](const uint4 r, float* x) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
    if (DT == LSS_DTYPE_F32) {
#pragma unroll
      for (int q = 0; q < 4; ++q) x[q] = __uint_as_float(w[q]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (DT == LSS_DTYPE_BF16) {
          x[2 * q] = __uint_as_float(w[q] << 16);
          x[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
        } else {
          x[2 * q] = __half2float(__ushort_as_half((uint16_t)(w[q] & 0xffffu)));
          x[2 * q + 1] = __half2float(__ushort_as_half((uint16_t)(w[q] >> 16)));
        }
      }
    }
  };

  // Stage s of chunk g is no longer read: generic writes to it precede the next bulk copy into it.
  auto release = [&](int64_t g, Pos pi, int s, bool wrote) {
    if (wrote) fence_proxy_async();
    __syncwarp();
    if (lane == 0 && g + (int64_t)ST_R * ST_NW < g1) issue(pi, s);
  };

  const int nwch = gw < g1 ? (int)((g1 - gw + ST_NW - 1) / ST_NW) : 0;  // this warp's chunks
  Pos pc = pw;                       // this chunk
  Pos pr = adv(pw, ST_R * ST_NW);     // ST_R chunks on (the copy started when this one is released)
  int i = 0;
  int s = 0;
  uint32_t par = 0;
  int crow = -1;        // row of the slice this warp is in (its parameters and slot below)
  int mine = 0;         // chunks of that slice this warp has finished
  RowPrm P{};
  SliceSlot* sl = slots;
  for (;; ++i) {
    const int64_t g = gw + (int64_t)i * ST_NW;
    if (g >= g1 || __shfl_sync(0xffffffffu, lane == 0 ? *abort_w : 0u, 0)) break;
    const int row = pc.row;
    const int lo = pc.c * CE;
    const int n = min(CE, V - lo);
    const int ls = row - row0;
    if (!warp_mbar_wait(&wbar[s], par)) {
      if (lane == 0) {
        atomicOr(a.header, LSS_FLAG_TMA_TIMEOUT);
        *abort_w = 1u;
      }
      __syncwarp();
      break;
    }
    // Entering a slice: its parameters, and its slot, free once the slice ST_NSLOT before it has
    // been summarised.  The whole warp waits in one uniform loop (lane 0 reads and decides, the
    // lanes follow).  The slot stays the slice's until this warp has reported its chunks.
    if (row != crow) {
    crow = row;
    P = prm_of(row);
    sl = &slots[ls % ST_NSLOT];
    volatile uint32_t* vtag = &sl->tag;
    if (__shfl_sync(0xffffffffu, lane == 0 ? *vtag : 0u, 0) != (uint32_t)ls) {
      const long long t0 = clock64();
      uint32_t st2 = 0;  // 1: the slot is ours; 2: gave up
      do {
        __nanosleep(64);
        if (lane == 0)
          st2 = *vtag == (uint32_t)ls ? 1u : ((*abort_w || clock64() - t0 > WAIT_CYCLES) ? 2u : 0u);
        st2 = __shfl_sync(0xffffffffu, st2, 0);
      } while (st2 == 0u);
      __threadfence_block();
      if (st2 == 2u) {
        if (lane == 0) {
          atomicOr(a.header, LSS_FLAG_INTERNAL);
          *abort_w = 1u;
        }
        __syncwarp();
        ++i;  // this chunk's copy has landed: nothing of it is in flight any more
        break;
      }
    }
    }
    unsigned char* st = wst + s * ST_SB;
    if (P.mode == ITEM_SKIP) {
      release(g, pr, s, false);
    } else {
      bool wrote = false;
      const char* src = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
      const int nb = (reinterpret_cast<uintptr_t>(src) & 15) == 0 ? ((n * ES) & ~15) : 0;
      // What the bulk copy skipped (a misaligned chunk, a ragged tail) and -inf padding: the only
      // generic writes into a stage (a row's last chunk, or a row that starts misaligned).
      if (nb < ST_CB) {
        for (int e = nb / ES + lane; e < n; e += 32) {
          copy_elem(st, e, src);
          wrote = true;
        }
        for (int e = n + lane; e < CE; e += 32) {
          set_neg_inf(st, e);
          wrote = true;
        }
        __syncwarp();
      }
      const uint4* s16 = reinterpret_cast<const uint4*>(st);
      uint4 rv[NV];
#pragma unroll
      for (int j = 0; j < NV; ++j) rv[j] = s16[j * 32 + lane];
      if (P.mode == ITEM_GREEDY) {
        // Greedy row (sampling.py:132-133): argmax of the raw chunk, NaN first, lowest index.
        uint64_t best = 0;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          float x[VPV];
          widen(rv[j], x);
          const int ix = lo + (j * 32 + lane) * VPV;
#pragma unroll
          for (int q = 0; q < VPV; ++q)
            if (ix + q < lo + n) best = max(best, argmax_code(x[q], ix + q));
        }
        best = wred(best, MaxU64());
        release(g, pr, s, wrote);  // every value has been read (the reduction consumed them)
        if (lane == 0) atomicMax(&sl->best, (unsigned long long)best);
      } else {
        // Max as a tree (short dependency chains): per vector, then across the vectors; the
        // per-vector maxima are kept to skip vectors without candidates below.
        float vmx[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          if constexpr (DT == LSS_DTYPE_F32) {
            float x[VPV];
            widen(rv[j], x);
#pragma unroll
            for (int w2 = VPV / 2; w2 >= 1; w2 /= 2)
#pragma unroll
              for (int q = 0; q < w2; ++q) x[q] = fmax_nan(x[q], x[q + w2]);
            vmx[j] = x[0];
          } else {  // pairs first, f32 only for the last two values
            const uint32_t m2 = pk_max<DT>(pk_max<DT>(rv[j].x, rv[j].y), pk_max<DT>(rv[j].z, rv[j].w));
            vmx[j] = fmax_nan(pk_lo<DT>(m2), pk_hi<DT>(m2));
          }
        }
        float lm = vmx[0];
#pragma unroll
        for (int j = 1; j < NV; ++j) lm = fmax_nan(lm, vmx[j]);
        const float cmax = wred(lm, MaxF());
        const uint32_t ck = (!(cmax == cmax) || cmax == INFINITY) ? 0xffffffffu : f2key(cmax);
        if (lane == 0) a.cmax[g] = ck;
        uint32_t mk = 0;
        if (lane == 0) {
          // The running max as far as this warp can see it: its own chunk's and what the slot
          // holds (a value read before other warps' updates land is only smaller, which keeps
          // every threshold taken from it a lower bound).
          atomicMax(&sl->maxkey, ck);
          const uint32_t cur = *reinterpret_cast<volatile uint32_t*>(&sl->maxkey);
          mk = cur > ck ? cur : ck;
          if (ck == 0xffffffffu) atomicOr(&sl->flags, SUM_SPECIAL);
        }
        mk = __shfl_sync(0xffffffffu, mk, 0);
        const float M = key2f(mk);
        if (mk != 0xffffffffu && M > -INFINITY) {
          const float T = P.T, tl = P.tl;
          // Min-p floor in z: exp(y - max) >= p  <=>  z >= max_z + T ln p, less a margin of
          // 2^-11 relative that covers every rounding of the exact filter.
          const float zmp = tl != 0.0f ? __fsub_rn(__fadd_rn(M, tl), (fabsf(M) + fabsf(tl) + T) * 4.8828125e-04f)
                                       : -INFINITY;
          float thr = (tl != 0.0f || P.k) ? zmp : -FLT_MAX;  // small vocabulary: every finite value
          if (P.k) {
            const int k = P.k;
            const uint32_t tk0 = *reinterpret_cast<volatile uint32_t*>(&sl->taukey);
            float lowc = fmaxf(zmp, tk0 ? key2f(tk0) : -INFINITY);
            auto count_ge = [&](float lev) -> uint32_t {
              uint32_t cnt = 0;
              if constexpr (DT == LSS_DTYPE_F32) {
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                  float x[VPV];
                  widen(rv[j], x);
#pragma unroll
                  for (int q = 0; q < VPV; ++q) cnt += (x[q] >= lev && x[q] > -INFINITY) ? 1u : 0u;
                }
              } else {
                const uint32_t l2 = pk_level<DT>(lev);
#pragma unroll
                for (int j = 0; j < NV; ++j)
                  cnt += __popc(pk_ge<DT>(rv[j].x, l2)) + __popc(pk_ge<DT>(rv[j].y, l2)) +
                         __popc(pk_ge<DT>(rv[j].z, l2)) + __popc(pk_ge<DT>(rv[j].w, l2));
                cnt >>= 4;  // 16 mask bits per value
              }
              return wred(cnt, SumU32());
            };
            // A chunk with many values above the slice's threshold (the slice's first chunks)
            // first bounds it with its own values: at least k of them reach `lev`, so the
            // slice's k-th largest does too.
            const uint32_t nlow = count_ge(lowc);
            if (nlow > 2u * (uint32_t)k && cmax > -INFINITY) {
#pragma unroll 1
              for (float D = 1.0f; D <= 8.0f; D *= 2.0f) {
                float lev = __fsub_rn(cmax, __fmul_rn(D, T));
                lev = __fsub_rn(lev, (fabsf(lev) + fabsf(cmax)) * 2.384185791015625e-07f + 1e-37f);
                if (lev > lowc && count_ge(lev) >= (uint32_t)k) {
                  lowc = lev;
                  break;
                }
              }
            }
            // A chunk without a value at or above lowc adds nothing to the histogram: it keeps
            // tau = lowc (the slice's threshold as last published, or the min-p floor) and leaves
            // refreshing the threshold from the bins to the warps that add counts.
            float tau = lowc;
            if (nlow != 0u) {
              // The histogram's reference: the first running max any warp reports for the slice.
              uint32_t r0 = *reinterpret_cast<volatile uint32_t*>(&sl->r0key);
              if (r0 == 0u) {
                if (lane == 0) {
                  const uint32_t old = atomicCAS(&sl->r0key, 0u, mk);
                  r0 = old ? old : mk;
                }
                r0 = __shfl_sync(0xffffffffu, r0, 0);
              }
              const float R0 = key2f(r0);
              const float sb = P.sb;
              uint32_t ab = 0;
              auto bin = [&](float z) {
                if (z > R0) {
                  ab++;
                } else {
                  const float dd = __fmul_rn(__fsub_rn(R0, z), sb);
                  if (dd < (float)NBIN) atomicAdd(&sl->hist[(int)dd], 1u);
                }
              };
              if constexpr (DT == LSS_DTYPE_F32) {
  #pragma unroll
                for (int j = 0; j < NV; ++j) {
                  float x[VPV];
                  widen(rv[j], x);
  #pragma unroll
                  for (int q = 0; q < VPV; ++q) {
                    const float z = x[q];
                    if (!(z >= lowc) || z == -INFINITY) continue;
                    bin(z);
                  }
                }
              } else {  // a pair test first; most pairs have no value at or above lowc
                const uint32_t l2 = pk_level<DT>(lowc);
  #pragma unroll
                for (int j = 0; j < NV; ++j) {
                  const uint32_t w4[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
  #pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const uint32_t m = pk_ge<DT>(w4[q], l2);
                    if (m & 0xffffu) bin(pk_lo<DT>(w4[q]));
                    if (m >> 16) bin(pk_hi<DT>(w4[q]));
                  }
                }
              }
              ab = wred(ab, SumU32());
              if (lane == 0 && ab) atomicAdd(&sl->above, ab);
              __syncwarp();
              // Bins as counted so far by every warp (lane l reads bins 8l .. 8l+7).  A partial
              // view only counts fewer values, so the threshold stays a lower bound.
              const volatile uint32_t* vh = sl->hist;
              uint32_t c8[8];
              uint32_t loc = 0;
  #pragma unroll
              for (int q = 0; q < 8; ++q) {
                c8[q] = vh[8 * lane + q];
                loc += c8[q];
              }
              uint32_t incl = loc;
  #pragma unroll
              for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
              }
              const uint32_t abv = *reinterpret_cast<volatile uint32_t*>(&sl->above);
              if (abv >= (uint32_t)k) {
                tau = fmaxf(tau, R0);
              } else {
                const unsigned hit = __ballot_sync(0xffffffffu, abv + incl >= (uint32_t)k);
                if (hit) {
                  const int L = __ffs(hit) - 1;
                  int b = 0;
                  uint32_t acc = abv + incl - loc;
  #pragma unroll
                  for (int q = 0; q < 8; ++q) {
                    acc += c8[q];
                    if (acc < (uint32_t)k) b = q + 1;
                  }
                  const int bk = __shfl_sync(0xffffffffu, 8 * lane + b, L);
                  // The k-th largest counted value lies in bin bk: (R0 - z) * sb < bk + 1.  One
                  // more bin of slack covers the rounding of the bins.
                  float zw = __fsub_rn(R0, __fmul_rn((float)(bk + 2), P.binw));
                  zw = __fsub_rn(zw, fabsf(zw) * 2.384185791015625e-07f + 1e-37f);
                  tau = fmaxf(tau, zw);
                }
              }
              if (lane == 0 && tau > -INFINITY) atomicMax(&sl->taukey, f2key(tau));
            }
            thr = fmaxf(thr, tau);
          }
          // ---- candidates: finite z >= thr, into the slice's segment.  Each lane marks its
          // values at or above the threshold in a bit mask, and writes only those, reading the
          // value back from the stage.
          thr = fmaxf(thr, -FLT_MAX);
          if (lane == 0) atomicMax(&sl->ukey, f2key(thr));
          const bool mine = lm >= thr;
          if (__ballot_sync(0xffffffffu, mine)) {
            MaskT m = 0;
            if (mine) {
#pragma unroll
              for (int j = 0; j < NV; ++j) {
                if (vmx[j] >= thr) {
                  float x[VPV];
                  widen(rv[j], x);
#pragma unroll
                  for (int q = 0; q < VPV; ++q)
                    if (x[q] >= thr) m |= (MaskT)1 << (j * VPV + q);
                }
              }
            }
            const uint32_t cnt = (uint32_t)(sizeof(MaskT) == 8 ? __popcll((unsigned long long)m) : __popc((uint32_t)m));
            uint32_t incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
              if (lane >= o) incl += y;
            }
            const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
            uint32_t base = 0;
            if (lane == 0) base = atomicAdd(&sl->count, total);
            base = __shfl_sync(0xffffffffu, base, 0);
            uint64_t* out = a.cand + ((int64_t)row * a.MAXSL + P.jsl) * ST_SEGCAP;
            uint32_t pos = base + incl - cnt;
            while (m) {
              const int b = sizeof(MaskT) == 8 ? __ffsll((long long)m) - 1 : __ffs((int)m) - 1;
              m &= m - 1;
              const int idx = ((b / VPV) * 32 + lane) * VPV + (b % VPV);
              if (pos < (uint32_t)ST_SEGCAP)
                out[pos] = ((uint64_t)f2key(elem(st, idx)) << 32) | (uint32_t)(~(uint32_t)(lo + idx));
              ++pos;
            }
          }
        }
        release(g, pr, s, wrote);  // the stage has been read for the last time
      }
    }
    // ---- chunk done.  A warp leaving a slice reports its chunks of it at once; the report
    // that completes the slice writes the summary and frees the slot.
    ++mine;
    const Pos pnext = adv(pc, ST_NW);
    uint32_t last = 0;
    if (g + ST_NW >= g1 || pnext.row != row) {
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&sl->done, (uint32_t)mine) + (uint32_t)mine == (uint32_t)P.nch ? 1u : 0u;
      }
      mine = 0;
      last = __shfl_sync(0xffffffffu, last, 0);
    }
    if (last) {
      __threadfence_block();
      if (lane == 0) {
        const int jsl = P.jsl;
        const volatile SliceSlot* vs = sl;
        uint4 sm;
        if (P.mode == ITEM_GREEDY) {
          const unsigned long long b = vs->best;
          sm = make_uint4((uint32_t)b, (uint32_t)(b >> 32), 0u, 0u);
        } else {
          sm = make_uint4(vs->maxkey, vs->ukey, vs->count, vs->flags);
        }
        a.summ[(int64_t)row * a.MAXSL + jsl] = sm;
      }
      uint32_t* sw = reinterpret_cast<uint32_t*>(sl);
      constexpr int W = (int)(sizeof(SliceSlot) / 4);
      for (int q = 1 + lane; q < W; q += 32) sw[q] = 0u;
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        *reinterpret_cast<volatile uint32_t*>(&sl->tag) = (uint32_t)(ls + ST_NSLOT);
      }
    }

    pc = pnext;

    pr = adv(pr, ST_NW);
    s = s + 1 == ST_R ? 0 : s + 1;
    par ^= s == 0 ? 1u : 0u;
  }
  // After an early stop: chunks i .. min(nwch, i + ST_R) - 1 were issued and not consumed; wait
  // (bounded) for their copies before the CTA's shared memory is released.  After a normal end
  // nothing is outstanding.
  for (int j = i; j < min(nwch, i + ST_R); ++j) warp_mbar_wait(&wbar[j % ST_R], (uint32_t)((j / ST_R) & 1));
  __syncwarp();
}

}  // namespace lss
