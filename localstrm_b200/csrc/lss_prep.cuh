// lss_prep.cuh — history preparation: the history of a row as unique (id, count) pairs
// (torch.unique of the history, sampling.py:52), grouped by vocabulary slice.
//
// prep_row does one row with the whole CTA: histories of up to PREP_SMEM_SLOTS / 2 ids hash
// in the shared memory handed in, longer ones in a global table of 2H slots.  The pairs of
// slice c ([c*TE, (c+1)*TE)) land in uniq_ids / uniq_cnt[hist_off[row] + so[c] ..
// hist_off[row] + so[c+1]).  K0, lss_hist_kernel, runs it for every row with the scan
// kernel's slices; the second kernel runs it again for the rows it takes, with its own
// slices.
#pragma once

#include "lss_common.cuh"

namespace lss {

constexpr int PREP_SMEM_SLOTS = 4096;   // histories up to 2,048 ids hash in shared memory
constexpr int PREP_MAXSEG = 32;         // slices per row
constexpr uint32_t EMPTY = 0xffffffffu;

struct PrepOut {
  int32_t* so;         // this row's segment offsets, nseg + 1 entries
  uint32_t* bad;       // OR'ed with LSS_FLAG_BAD_HISTORY for an id outside [0, V)
};

// Whole CTA (NTH threads, `sync` its barrier).  `skeys` / `scnts`: PREP_SMEM_SLOTS words each;
// `bcnt`: PREP_MAXSEG + 1 words, `bfill`: PREP_MAXSEG words.  `active`: the row's penalties
// apply (otherwise only empty segments are written).
template <int NTH, class Sync>
__device__ void prep_row(const RowArgs& a, int row, bool active, int TE, int nseg, const PrepOut& o,
                         uint32_t* skeys, uint32_t* scnts, uint32_t* bcnt, uint32_t* bfill, Sync sync) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (!active) {
    if (tid <= nseg) o.so[tid] = 0;
    return;
  }
  const int b = a.hist_off[row], e = a.hist_off[row + 1];
  const int H = e - b;
  if (H <= 0) {
    if (tid <= nseg) o.so[tid] = 0;
    return;
  }
  uint32_t *keys, *cnts;
  uint32_t cap;
  bool pow2;
  if (2 * H <= PREP_SMEM_SLOTS) {
    cap = (uint32_t)next_pow2(2 * H);
    keys = skeys;
    cnts = scnts;
    pow2 = true;
  } else {
    cap = (uint32_t)(2 * H);
    keys = a.gkeys + 2 * (int64_t)b;
    cnts = a.gcnts + 2 * (int64_t)b;
    pow2 = false;
  }
  for (uint32_t s = tid; s < cap; s += NTH) {
    keys[s] = EMPTY;
    cnts[s] = 0;
  }
  if (tid <= PREP_MAXSEG) bcnt[tid] = 0;
  if (tid < PREP_MAXSEG) bfill[tid] = 0;
  sync();
  // Insert: lanes holding the same id are merged first (one atomic per distinct id per warp).
  // U ids per thread are loaded before any is inserted, so their latencies overlap.
  constexpr int U = 8;
  for (int j0 = 0; j0 < H; j0 += NTH * U) {
    int idv[U];
#pragma unroll
    for (int t = 0; t < U; ++t) {
      const int j = j0 + t * NTH + tid;
      idv[t] = j < H ? a.hist_ids[b + j] : INT32_MIN;  // INT32_MIN: no entry
    }
#pragma unroll
    for (int t = 0; t < U; ++t) {
      int id = idv[t] == INT32_MIN ? -1 : idv[t];
      if (idv[t] != INT32_MIN && (id < 0 || id >= a.V)) {
        atomicOr(o.bad, LSS_FLAG_BAD_HISTORY);
        id = -1;
      }
      const unsigned same = __match_any_sync(0xffffffffu, id);
      if (id >= 0 && lane == __ffs(same) - 1) {
        uint32_t h = (uint32_t)id * 2654435761u;
        h = pow2 ? (h & (cap - 1)) : (h % cap);
        for (uint32_t probe = 0; probe < cap; ++probe) {
          const uint32_t old = atomicCAS(&keys[h], EMPTY, (uint32_t)id);
          if (old == EMPTY || old == (uint32_t)id) {
            atomicAdd(&cnts[h], (uint32_t)__popc(same));
            break;
          }
          h = (h + 1 == cap) ? 0 : h + 1;
        }
      }
    }
  }
  sync();
  // Group by slice: count, exclusive scan, scatter (one atomic per slice per warp).
  for (uint32_t s0 = 0; s0 < cap; s0 += NTH) {
    const uint32_t s = s0 + tid;
    const uint32_t k = s < cap ? keys[s] : EMPTY;
    const int c = k != EMPTY ? (int)(k / (uint32_t)TE) : -1;
    const unsigned same = __match_any_sync(0xffffffffu, c);
    if (c >= 0 && lane == __ffs(same) - 1) atomicAdd(&bcnt[c], (uint32_t)__popc(same));
  }
  sync();
  if (tid == 0) {
    uint32_t run = 0;
    for (int c = 0; c <= PREP_MAXSEG; ++c) {
      const uint32_t v = c < nseg ? bcnt[c] : 0u;
      bcnt[c] = run;
      run += v;
    }
  }
  sync();
  for (uint32_t s0 = 0; s0 < cap; s0 += NTH) {
    const uint32_t s = s0 + tid;
    const uint32_t k = s < cap ? keys[s] : EMPTY;
    const int c = k != EMPTY ? (int)(k / (uint32_t)TE) : -1;
    const unsigned same = __match_any_sync(0xffffffffu, c);
    const int leader = __ffs(same) - 1;
    uint32_t base = 0;
    if (c >= 0 && lane == leader) base = atomicAdd(&bfill[c], (uint32_t)__popc(same));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (c >= 0) {
      const uint32_t pos = bcnt[c] + base + (uint32_t)__popc(same & ((1u << lane) - 1u));
      a.uniq_ids[b + pos] = (int32_t)k;
      a.uniq_cnt[b + pos] = (int32_t)cnts[s];
    }
  }
  if (tid <= nseg) o.so[tid] = (int32_t)bcnt[tid];
}

struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

// =========================================================================================
// K0: history kernel — one CTA per row: the (id, count) pairs of the rows whose penalties
// the scan kernel applies, grouped by its slices (seg2[row][0 .. S]); a per-row flag for ids
// outside [0, V).  Block 0 clears the workspace status first (no other block writes it).
// =========================================================================================
constexpr int HIST_NT = 512;

struct HistArgs {
  RowArgs r;
  int S, TS;
  int32_t* seg2;        // [B][S + 1]
  uint32_t* rowflag;    // [B]
  uint32_t* header;     // 64 words
};

__global__ void __launch_bounds__(HIST_NT) lss_hist_kernel(const HistArgs h) {
  __shared__ uint32_t skeys[PREP_SMEM_SLOTS];
  __shared__ uint32_t scnts[PREP_SMEM_SLOTS];
  __shared__ uint32_t bcnt[PREP_MAXSEG + 1];
  __shared__ uint32_t bfill[PREP_MAXSEG];
  const RowArgs& a = h.r;
  const int row = blockIdx.x;
  if (row == 0 && threadIdx.x < 64) h.header[threadIdx.x] = 0u;
  if (threadIdx.x == 0) h.rowflag[row] = 0u;
  const float T = a.temperature[row];
  const int k = a.top_k[row];
  const float mp = a.min_p[row];
  const bool bounded = (k > 0 && k < a.V) || (mp > 0.0f && mp < 1.0f) || a.V <= FAST_CAP / 2;
  const bool active = a.use_hist && T > 0.0f && bounded &&
                      (a.rep[row] != 1.0f || a.freq[row] != 0.0f || a.pres[row] != 0.0f);
  __syncthreads();
  const PrepOut o{h.seg2 + (int64_t)row * (h.S + 1), h.rowflag + row};
  prep_row<HIST_NT>(a, row, active, h.TS, h.S, o, skeys, scnts, bcnt, bfill, BlockSync());
}

}  // namespace lss
