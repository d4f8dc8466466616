// lss_prep.cuh — history preparation: the history of a row as unique (id, count) pairs
// (torch.unique of the history, sampling.py:52), grouped by vocabulary slice.
//
// prep_row does one row with the whole CTA: histories of up to PREP_SMEM_SLOTS / 2 ids hash
// in the shared memory handed in (and the slots they occupy are listed, so that grouping
// walks only those), longer ones in a global table of 2H slots.  The pairs of
// slice c ([c*TE, (c+1)*TE)) land in uniq_ids / uniq_cnt[hist_off[row] + so[c] ..
// hist_off[row] + so[c+1]).  K0, lss_hist_kernel, runs it for every row with the scan
// kernel's slices; the second kernel runs it again for the rows it takes, with its own
// slices.
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

// =========================================================================================
// K0: history kernel — one CTA per row: the (id, count) pairs of the rows whose penalties
// apply (torch.unique(history, return_counts=True), sampling.py:52), sorted by id and grouped
// by segments of TS logits: seg2[row][0 .. S] hold the absolute offsets of each segment's pairs
// in the pair arrays, so that the streaming kernel finds a chunk's pairs directly.  A per-row
// flag records ids outside [0, V) or a bad offset range.  Block 0 clears the workspace status
// first (no other block writes it).
//
// Histories of up to HIST_FAST ids take the bitmap path, which needs no hashing: every id sets
// its bit in a shared bitmap of the vocabulary; one warp per segment counts the set bits of its
// 32 words (the rank of each word's first bit within the segment) and a scan over the segments
// gives every id its rank among the unique ids; the counts are atomic additions on the ranks,
// and every set bit writes its pair at its rank, which sorts the pairs by id.  Longer histories
// go through prep_row's global hash table.
// =========================================================================================
constexpr int HIST_NT = 1024;
constexpr int HIST_FAST = 4096;    // history ids of the bitmap path
constexpr int HIST_IPT = HIST_FAST / HIST_NT;

struct HistArgs {
  RowArgs r;
  int S, TS;            // segments per row (TS == 1024 logits each)
  int32_t* seg2;        // [B][S + 1]: absolute pair offsets per segment
  int32_t* pblk;        // [B][S][8]: per segment {first pair, pairs, first six ids}
  uint32_t* rowflag;    // [B]
  uint32_t* header;     // 64 words
};

// The pair blocks of a row whose pairs are in place (seg2 row `so`, pair ids in uniq_ids): one
// 8-word block per segment with the index of its first pair, its number of pairs and the ids
// of its first six pairs, so that the streaming kernel finds a chunk's history positions in
// the bytes it copies with the chunk.  Whole CTA; the pairs and so[] are visible to it.
__device__ __forceinline__ void write_pair_blocks(const HistArgs& h, int row, const int32_t* so, bool empty) {
  const RowArgs& a = h.r;
  int32_t* blk = h.pblk + (int64_t)row * h.S * 8;
  for (int t = threadIdx.x; t < h.S * 8; t += blockDim.x) {
    const int sg = t >> 3, f = t & 7;
    int v = 0;
    if (!empty) {
      const int b0 = so[sg], cnt = so[sg + 1] - so[sg];
      v = f == 0 ? b0 : f == 1 ? cnt : (f - 2 < cnt ? a.uniq_ids[b0 + f - 2] : 0);
    }
    blk[t] = v;
  }
}

// Dynamic shared memory of K0 for a vocabulary of V: the bitmap path's arrays, or prep_row's
// scratch, whichever is larger.
__host__ __device__ constexpr int hist_bm_words(int V) { return (V + 31) / 32; }
__host__ __device__ constexpr int hist_smem_bytes(int V) {
  return ((hist_bm_words(V) * 4 + hist_bm_words(V) * 2 + 15) & ~15) + ((PREP_MAXSEG + 1) * 4) + HIST_FAST * 4 >
                 PREP_SCRATCH_WORDS * 4
             ? ((hist_bm_words(V) * 4 + hist_bm_words(V) * 2 + 15) & ~15) + ((PREP_MAXSEG + 1) * 4) + HIST_FAST * 4
             : PREP_SCRATCH_WORDS * 4;
}

__global__ void __launch_bounds__(HIST_NT, 1) lss_hist_kernel(const HistArgs h) {
  extern __shared__ __align__(16) uint32_t sw[];
  const RowArgs& a = h.r;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_trigger();  // the streaming kernel may launch and start its own set-up
  if (row == 0 && tid < 64) h.header[tid] = 0u;
  if (tid == 0) h.rowflag[row] = 0u;
  // Every per-row input is requested at once (one round trip), the history offsets included.
  const float T = a.temperature[row];
  const int k = a.top_k[row];
  const float mp = a.min_p[row];
  const float rp = a.rep[row], fq = a.freq[row], pr = a.pres[row];
  int b = 0, e = 0;
  bool bad_range = false;
  if (a.use_hist) bad_range = !hist_range(a.hist_off, row, a.H, b, e);
  const bool bounded = (k > 0 && k < a.V) || (mp > 0.0f && mp < 1.0f) || a.V <= FAST_CAP / 2;
  const bool active = a.use_hist && T > 0.0f && bounded && (rp != 1.0f || fq != 0.0f || pr != 0.0f);
  const int nseg = h.S;
  int32_t* so = h.seg2 + (int64_t)row * (nseg + 1);
  const PrepOut o{so, h.rowflag + row};
  const int H = active ? e - b : 0;
  if (bad_range && tid == 0) atomicOr(o.bad, LSS_FLAG_BAD_HISTORY);  // thread 0 cleared it above
  if (!active || H <= 0) {
    if (tid <= nseg) so[tid] = 0;
    if (a.use_hist) write_pair_blocks(h, row, so, true);
    return;
  }
  if (H > HIST_FAST) {
    __syncthreads();  // rowflag cleared before prep_row may raise it
    prep_row<HIST_NT>(a, row, true, h.TS, nseg, o, sw, BlockSync(), b);
    __syncthreads();  // the pairs and so[] of this row are written
    write_pair_blocks(h, row, so, false);
    return;
  }
  // ---- bitmap path
  const int V = a.V;
  const int W = hist_bm_words(V);
  uint32_t* bm = sw;                                                   // [W] one bit per logit
  uint16_t* wpre = reinterpret_cast<uint16_t*>(sw + W);                // [W] rank of the word's first bit in its segment
  uint32_t* segpre = sw + ((W * 4 + W * 2 + 15) & ~15) / 4;            // [nseg + 1] rank of each segment's first id
  uint32_t* cnt = segpre + PREP_MAXSEG + 1;                            // [HIST_FAST] counts by rank
  int idv[HIST_IPT];
#pragma unroll
  for (int t = 0; t < HIST_IPT; ++t) {
    const int j = t * HIST_NT + tid;
    idv[t] = j < H ? a.hist_ids[b + j] : -1;
  }
  for (int w = tid; w < W; w += HIST_NT) bm[w] = 0u;
  for (int j = tid; j < H; j += HIST_NT) cnt[j] = 0u;
  __syncthreads();
#pragma unroll
  for (int t = 0; t < HIST_IPT; ++t) {
    int id = idv[t];
    if (t * HIST_NT + tid < H && (id < 0 || id >= V)) {
      atomicOr(o.bad, LSS_FLAG_BAD_HISTORY);
      id = -1;
    }
    idv[t] = id;
    if (id >= 0) atomicOr(&bm[id >> 5], 1u << (id & 31));
  }
  __syncthreads();
  // One warp per segment of 32 words: each word's rank within the segment, the segment total.
  for (int sgi = warp; sgi < nseg; sgi += HIST_NT / 32) {
    const int w = sgi * 32 + lane;
    const uint32_t c = w < W ? (uint32_t)__popc(bm[w]) : 0u;
    uint32_t incl = c;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    if (w < W) wpre[w] = (uint16_t)(incl - c);
    if (lane == 31) segpre[sgi] = incl;
  }
  __syncthreads();
  {
    // Exclusive scan of the segment totals (thread c holds segment c; nseg <= PREP_MAXSEG <
    // HIST_NT); seg2 gets the absolute offsets, tid == nseg the row's total.
    __shared__ uint32_t wsum[HIST_NT / 32];
    const uint32_t v = tid < nseg ? segpre[tid] : 0u;
    uint32_t incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    uint32_t pre = 0;
    for (int q = 0; q < warp; ++q) pre += wsum[q];
    const uint32_t ex = pre + incl - v;
    __syncthreads();
    if (tid <= nseg) {
      segpre[tid] = ex;
      so[tid] = b + (int32_t)ex;
    }
  }
  __syncthreads();
  // Counts by rank.
#pragma unroll
  for (int t = 0; t < HIST_IPT; ++t) {
    const int id = idv[t];
    if (id >= 0) {
      const int w = id >> 5;
      const uint32_t r = segpre[id >> 10] + wpre[w] + (uint32_t)__popc(bm[w] & ((1u << (id & 31)) - 1u));
      atomicAdd(&cnt[r], 1u);
    }
  }
  __syncthreads();
  // Every set bit writes its pair at its rank (sorted by id), and the first six ids of each
  // segment go to its pair block as well.
  for (int w = tid; w < W; w += HIST_NT) {
    uint32_t bits = bm[w];
    if (!bits) continue;
    const int sg = w >> 5;
    uint32_t r = segpre[sg] + wpre[w];
    int32_t* blk = h.pblk + ((int64_t)row * nseg + sg) * 8;
    while (bits) {
      const int q = __ffs((int)bits) - 1;
      bits &= bits - 1u;
      a.uniq_ids[b + r] = w * 32 + q;
      a.uniq_cnt[b + r] = (int32_t)cnt[r];
      if (r - segpre[sg] < 6u) blk[2 + r - segpre[sg]] = w * 32 + q;
      ++r;
    }
  }
  for (int sg = tid; sg < nseg; sg += HIST_NT) {
    int32_t* blk = h.pblk + ((int64_t)row * nseg + sg) * 8;
    blk[0] = b + (int32_t)segpre[sg];
    blk[1] = (int32_t)(segpre[sg + 1] - segpre[sg]);
  }
}

}  // namespace lss
