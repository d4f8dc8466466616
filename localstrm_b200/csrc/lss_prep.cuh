// lss_prep.cuh — history preparation of one row for the second kernel.
//
// The history of a non-greedy row with an active penalty becomes unique (id, count) pairs
// (torch.unique, sampling.py:52), grouped by the CTA slice [c*TE, (c+1)*TE) that holds the id,
// so that each CTA of the row's cluster applies only its own segment.  One CTA does the whole
// row: histories of up to PREP_SMEM_SLOTS / 2 ids hash in the shared memory handed in, longer
// ones in a global table of 2H slots.
#pragma once

#include "lss_common.cuh"

namespace lss {

constexpr int PREP_SMEM_SLOTS = 4096;   // histories up to 2,048 ids hash in shared memory
constexpr uint32_t EMPTY = 0xffffffffu;

// `skeys` / `scnts`: PREP_SMEM_SLOTS words each; `bcnt` MAXCL + 1 words, `bfill` MAXCL words.
// Writes uniq_ids / uniq_cnt at hist_off[row] + ... and seg_off[row][0 .. MAXCL].
__device__ void prep_row(const RowArgs& a, int row, int TE, int CL, uint32_t* skeys, uint32_t* scnts,
                         uint32_t* bcnt, uint32_t* bfill) {
  const int tid = threadIdx.x, lane = tid & 31;
  int32_t* so = a.seg_off + (int64_t)row * (MAXCL + 1);
  const float T = a.temperature[row];
  const int b = a.hist_off[row], e = a.hist_off[row + 1];
  const int H = e - b;
  const bool active = T > 0.0f && H > 0 && (a.rep[row] != 1.0f || a.freq[row] != 0.0f || a.pres[row] != 0.0f);
  if (!active) {
    if (tid <= MAXCL) so[tid] = 0;
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
  for (uint32_t s = tid; s < cap; s += NT) {
    keys[s] = EMPTY;
    cnts[s] = 0;
  }
  if (tid <= MAXCL) bcnt[tid] = 0;
  if (tid < MAXCL) bfill[tid] = 0;
  __syncthreads();
  // Insert: lanes holding the same id are merged first (one atomic per distinct id per warp).
  // Eight ids per thread are loaded before any is inserted, so their latencies overlap.
  constexpr int U = 8;
  for (int j0 = 0; j0 < H; j0 += NT * U) {
    int idv[U];
#pragma unroll
    for (int t = 0; t < U; ++t) {
      const int j = j0 + t * NT + tid;
      idv[t] = j < H ? a.hist_ids[b + j] : INT32_MIN;  // INT32_MIN: no entry
    }
#pragma unroll
    for (int t = 0; t < U; ++t) {
      int id = idv[t] == INT32_MIN ? -1 : idv[t];
      if (idv[t] != INT32_MIN && (id < 0 || id >= a.V)) {
        atomicOr(a.err, LSS_FLAG_BAD_HISTORY);
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
  __syncthreads();
  // Group by CTA slice: count, exclusive scan, scatter (one atomic per slice per warp).
  for (uint32_t s0 = 0; s0 < cap; s0 += NT) {
    const uint32_t s = s0 + tid;
    const uint32_t k = s < cap ? keys[s] : EMPTY;
    const int c = k != EMPTY ? (int)(k / (uint32_t)TE) : -1;
    const unsigned same = __match_any_sync(0xffffffffu, c);
    if (c >= 0 && lane == __ffs(same) - 1) atomicAdd(&bcnt[c], (uint32_t)__popc(same));
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t run = 0;
    for (int c = 0; c <= MAXCL; ++c) {
      const uint32_t v = c < CL ? bcnt[c] : 0u;
      bcnt[c] = run;
      run += v;
    }
  }
  __syncthreads();
  for (uint32_t s0 = 0; s0 < cap; s0 += NT) {
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
  if (tid <= MAXCL) so[tid] = (int32_t)bcnt[tid <= CL ? tid : CL];
}

}  // namespace lss
