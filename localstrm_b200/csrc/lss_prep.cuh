// lss_prep.cuh — history preparation: the history of a row as unique (id, count) pairs
// (torch.unique of the history, sampling.py:52), grouped by vocabulary slice.
//
// prep_row does one row with the whole CTA: histories of up to PREP_SMEM_SLOTS / 2 ids hash
// in the shared memory handed in (and the slots they occupy are listed, so that grouping
// walks only those), longer ones in a global table of 2H slots.  The pairs of
// slice c ([c*TE, (c+1)*TE)) land in uniq_ids / uniq_cnt[hist_off[row] + so[c] ..
// hist_off[row] + so[c+1]).  The second kernel runs it for the rows it takes, with its own
// slices (the resolve kernel keeps the pairs of the other rows in its own shared memory).
#pragma once

#include "lss_common.cuh"

namespace lss {

constexpr int PREP_SMEM_SLOTS = 4096;   // histories up to 2,048 ids hash in shared memory
constexpr int PREP_MAXSEG = 320;        // slices (segments) per row: a row of 327,680 logits in 1,024-logit segments
constexpr uint32_t EMPTY = 0xffffffffu;

struct PrepOut {
  int32_t* so;         // this row's segment offsets, nseg + 1 entries
  uint32_t* bad;       // OR'ed with LSS_FLAG_BAD_HISTORY for an id outside [0, V)
};

// Whole CTA (NTH threads, `sync` its barrier).  Scratch `sw` in shared memory: PREP_SCRATCH_WORDS
// words (hash keys and counts, the list of occupied slots, slice counters).  `active`: the
// row's penalties apply (otherwise only empty segments are written).
constexpr int PREP_SCRATCH_WORDS = 2 * PREP_SMEM_SLOTS + PREP_SMEM_SLOTS / 4 + 2 * (PREP_MAXSEG + 1) + 1;

// The segment offsets written are relative to the row's first pair, plus `so_base`.
template <int NTH, class Sync>
__device__ void prep_row(const RowArgs& a, int row, bool active, int TE, int nseg, const PrepOut& o, uint32_t* sw,
                         Sync sync, int so_base = 0) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (!active) {
    for (int t = tid; t <= nseg; t += NTH) o.so[t] = so_base;
    return;
  }
  int b = 0, e = 0;
  if (!hist_range(a.hist_off, row, a.H, b, e)) atomicOr(o.bad, LSS_FLAG_BAD_HISTORY);
  const int H = e - b;
  if (H <= 0) {
    for (int t = tid; t <= nseg; t += NTH) o.so[t] = so_base;
    return;
  }
  uint32_t* skeys = sw;
  uint32_t* scnts = sw + PREP_SMEM_SLOTS;
  uint16_t* slist = reinterpret_cast<uint16_t*>(sw + 2 * PREP_SMEM_SLOTS);  // PREP_SMEM_SLOTS / 2 entries
  uint32_t* bcnt = sw + 2 * PREP_SMEM_SLOTS + PREP_SMEM_SLOTS / 4;
  uint32_t* bfill = bcnt + PREP_MAXSEG + 1;
  uint32_t* nlist = bfill + PREP_MAXSEG + 1;
  uint32_t *keys, *cnts;
  uint32_t cap;
  const bool small = 2 * H <= PREP_SMEM_SLOTS;  // shared hash, occupied slots listed
  if (small) {
    cap = (uint32_t)next_pow2(2 * H);
    keys = skeys;
    cnts = scnts;
  } else {
    cap = (uint32_t)(2 * H);
    keys = a.gkeys + 2 * (int64_t)b;
    cnts = a.gcnts + 2 * (int64_t)b;
  }
  for (uint32_t s = tid; s < cap; s += NTH) {
    keys[s] = EMPTY;
    cnts[s] = 0;
  }
  for (int t = tid; t <= PREP_MAXSEG; t += NTH) {
    bcnt[t] = 0;
    bfill[t] = 0;
  }
  if (tid == 0) *nlist = 0;
  sync();
  // Insert: lanes holding the same id are merged first (one atomic per distinct id per warp).
  // U ids per thread are loaded before any is inserted, so their latencies overlap.  In the
  // shared table a new key's slot is listed (one list reservation per warp).
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
      if (j0 + t * NTH >= H) break;  // warp-uniform: no entry in this or later rounds
      int id = idv[t] == INT32_MIN ? -1 : idv[t];
      if (idv[t] != INT32_MIN && (id < 0 || id >= a.V)) {
        atomicOr(o.bad, LSS_FLAG_BAD_HISTORY);
        id = -1;
      }
      const unsigned same = __match_any_sync(0xffffffffu, id);
      bool fresh = false;
      uint32_t slot = 0;
      if (id >= 0 && lane == __ffs(same) - 1) {
        uint32_t h = (uint32_t)id * 2654435761u;
        h = small ? (h & (cap - 1)) : (h % cap);
        for (uint32_t probe = 0; probe < cap; ++probe) {
          const uint32_t old = atomicCAS(&keys[h], EMPTY, (uint32_t)id);
          if (old == EMPTY || old == (uint32_t)id) {
            atomicAdd(&cnts[h], (uint32_t)__popc(same));
            fresh = old == EMPTY;
            slot = h;
            break;
          }
          h = (h + 1 == cap) ? 0 : h + 1;
        }
      }
      if (small) {
        const uint32_t bal = __ballot_sync(0xffffffffu, fresh);
        if (bal) {
          const int leader = __ffs(bal) - 1;
          uint32_t base = 0;
          if (lane == leader) base = atomicAdd(nlist, (uint32_t)__popc(bal));
          base = __shfl_sync(0xffffffffu, base, leader);
          if (fresh) slist[base + __popc(bal & ((1u << lane) - 1u))] = (uint16_t)slot;
        }
      }
    }
  }
  sync();
  // Group by slice: count, exclusive scan, scatter (one atomic per slice per warp).  The
  // shared table is walked through its list of occupied slots, the global one whole.
  const uint32_t nwalk = small ? *nlist : cap;
  for (uint32_t s0 = 0; s0 < nwalk; s0 += NTH) {
    const uint32_t i = s0 + tid;
    const uint32_t s = small ? (i < nwalk ? (uint32_t)slist[i] : 0u) : i;
    const uint32_t k = i < nwalk ? keys[s] : EMPTY;
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
  for (uint32_t s0 = 0; s0 < nwalk; s0 += NTH) {
    const uint32_t i = s0 + tid;
    const uint32_t s = small ? (i < nwalk ? (uint32_t)slist[i] : 0u) : i;
    const uint32_t k = i < nwalk ? keys[s] : EMPTY;
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
  for (int t = tid; t <= nseg; t += NTH) o.so[t] = so_base + (int32_t)bcnt[t];
}

struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

}  // namespace lss
