// lss_scan.cuh — K1: the streaming pass over the logits (the hot path).
//
// Persistent kernel, one CTA per SM.  The work is the list of items (row, slice), slice s of a
// row being the vocabulary range [s*TS, (s+1)*TS); CTA b takes items b, b + G, b + 2G, ...
// (G = grid size), so the CTAs in flight at any moment cover a band of consecutive rows and
// the history ids of a row are read from HBM once and from L2 by its other slices.
//
//  * 1 producer warp: fetches each item's row parameters with cp.async several items ahead;
//    when a stage of the two-stage ring is free it describes the item in shared memory and
//    starts bulk async copies into the stage — the slice of logits and the slice's history
//    pairs — so the next slice streams in while the current one is processed.
//  * 31 compute warps, per item: the penalties (sampling.py:55-66) from the slice's unique
//    (id, count) history pairs that K0 prepared (torch.unique, sampling.py:52); the slice
//    max of the pre-temperature values z
//    (held in registers, so each logit is read from shared memory once); the candidate
//    threshold; the candidates written to the item's segment in global memory and a 16-byte
//    summary (slice max or argmax code, candidate count, flags).
//
// Items are independent.  The slice max is a lower bound of the row max, so a threshold
// taken from it keeps a superset of the row's survivors: min-p keeps exp(y - max) >= p and a
// smaller max lowers the cut; every value among the k largest of the row that lies in the
// slice is among the slice's k largest.  Thresholds are taken on z (y = z / T is monotone)
// with a conservative margin; the resolve kernel takes the exact row max from the summaries
// and divides and filters the candidates exactly.
#pragma once

#include "lss_common.cuh"

namespace lss {

constexpr int SC_NT = 1024;                   // threads per CTA
constexpr int SC_CW = SC_NT / 32 - 1;         // compute warps
constexpr int SC_CT = SC_CW * 32;             // compute threads
constexpr int SC_PROD = SC_CW;                // index of the producer warp
constexpr int SC_R = 5;                       // float4 of the slice per compute thread
constexpr int SC_TS_MAX = 19200;              // logits per slice (<= SC_CT * SC_R * 4)
static_assert(SC_TS_MAX <= SC_CT * SC_R * 4, "a slice must fit the compute threads' registers");
constexpr int SC_NST = 2;                     // stages of the copy ring
constexpr int SC_HB = 2048;                   // words of history pairs staged per item
constexpr int SC_HP = SC_HB / 2;              // (id, count) pairs staged per item
constexpr int SC_SMEM_MAX = 232448;           // dynamic shared memory of one CTA
constexpr int SC_RING = 8;                    // parameter ring (items)
constexpr int SC_AHEAD = 4;                   // parameters fetched this many items ahead
constexpr int SC_BAR = 3;                     // named barrier of the compute warps
constexpr int SC_SEG_MIN = 256;               // candidate slots per item (at least)

constexpr int ITEM_END = 0, ITEM_SKIP = 1, ITEM_GREEDY = 2, ITEM_SAMPLE = 3;
// Summary flags: NaN / +inf in the slice or y overflow; top-k window deeper than the bins.
constexpr uint32_t SUM_SPECIAL = 1u, SUM_FAR = 2u;

struct __align__(16) ItemDesc {
  int row, slice, mode, nb;     // nb: bytes of the slice the bulk copy stages
  int hcount, hb, hlead, hbn;   // history pairs of the slice, index of the first, staged window
  float T, rep, freq, pres;
  int k, lo, n, pad0;           // k: top-k when active (0 < k < V), else 0; slice [lo, lo + n)
  float tl;                     // min-p: T * ln(min_p) (0: inactive), the floor's offset in z
  float sb, binw, pad1;         // top-k bins: 16 / T per unit of z, and T / 16
};
struct __align__(16) ItemScratch {
  uint32_t cnt, flags, pad0, pad1;  // candidates, summary flags
};
struct __align__(16) ScanCtl {
  uint64_t full[SC_NST];        // stage landed (2 arrivals + bytes)
  uint64_t empty[SC_NST];       // stage released (one arrival per compute warp)
  ItemDesc desc[2 * SC_NST];   // by item (j % 4): a released stage's next item does not overwrite it
  ItemScratch sc[2];            // by item parity
  uint64_t best[2][32];         // greedy items: argmax code per warp
  uint32_t wkey[2][32];         // sampled items: [0] max key of z over the warps (all ones: NaN / +inf)
  uint32_t prm[SC_RING][12];    // T, k, min_p, rep, freq, pres, hist_off[row], segment bounds
};

struct ScanArgs {
  const void* logits;
  int64_t row_stride;
  int B, V, S, TS, SEG;
  int tile_bytes;               // tile part of a stage (multiple of 128 bytes)
  int work_bytes;               // 16-bit logits: the f32 work tile they are widened into (else 0)
  int use_hist;
  const float* temperature;
  const int32_t* top_k;
  const float* min_p;
  const float* rep;
  const float* freq;
  const float* pres;
  const int32_t* hist_off;
  const int32_t* uniq_ids;      // history pairs by slice (K0), with 4 entries of padding
  const int32_t* uniq_cnt;      // either side
  const int32_t* seg2;          // [B][S + 1] slice segments of the pairs
  uint4* summ;                  // [B*S]: {a lo, a hi, count, flags}
  uint64_t* cand;               // [B*S*SEG]: (key(z) << 32) | ~index
  uint32_t* err;
};

__host__ __device__ constexpr int scan_stage_bytes(int tile_bytes) { return tile_bytes + SC_HB * 4; }
__host__ __device__ constexpr int scan_smem_bytes(int tile_bytes, int work_bytes = 0) {
  return SC_NST * scan_stage_bytes(tile_bytes) + work_bytes + (((NBIN + 1) * 4 + 15) & ~15) +
         (int)((sizeof(ScanCtl) + 15) & ~15);
}

__device__ __forceinline__ void sc_sync() { asm volatile("bar.sync %0, %1;" ::"n"(SC_BAR), "n"(SC_CT) : "memory"); }

template <int DT>
__global__ void __launch_bounds__(SC_NT, 1) lss_scan_kernel(const ScanArgs a) {
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr bool W16 = DT != LSS_DTYPE_F32;  // 16-bit logits: widened into a separate f32 tile
  const int stage_bytes = scan_stage_bytes(a.tile_bytes);
  float* WT = reinterpret_cast<float*>(smem + SC_NST * stage_bytes);  // work tile (16-bit logits)
  uint32_t* HL = reinterpret_cast<uint32_t*>(smem + SC_NST * stage_bytes + a.work_bytes);
  ScanCtl* ctl = reinterpret_cast<ScanCtl*>(reinterpret_cast<unsigned char*>(HL) + (((NBIN + 1) * 4 + 15) & ~15));
  const int V = a.V, S = a.S, TS = a.TS;
  const int nitems = a.B * S;
  const int G = gridDim.x;

  if (tid < (int)(2 * sizeof(ItemScratch) / 4)) reinterpret_cast<uint32_t*>(ctl->sc)[tid] = 0u;  // cnt, flags
  if (tid < 2) ctl->wkey[tid][0] = 0u;
  if (tid == 0) {
    for (int q = 0; q < SC_NST; ++q) {
      mbar_init(&ctl->full[q], 2);  // the logits' arrival, then the history pairs'
      mbar_init(&ctl->empty[q], SC_CW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  pdl_trigger();  // the resolve kernel may launch; it waits for this grid before reading
  if (warp == SC_PROD) {
    // =====================================================================================
    // Producer warp
    // =====================================================================================
    auto fetch = [&](int j) {  // parameters of item j into ring slot j % SC_RING (lanes 0..8)
      const int t = blockIdx.x + j * G;
      if (t < nitems && lane < 9) {
        const int row = t / S;
        int slice = t - row * S + row;
        slice -= (slice / S) * S;
        uint32_t* dst = &ctl->prm[j % SC_RING][lane];
        const void* src = nullptr;
        switch (lane) {
          case 0: src = a.temperature + row; break;
          case 1: src = a.top_k + row; break;
          case 2: src = a.min_p + row; break;
          case 3: src = a.rep + row; break;
          case 4: src = a.freq + row; break;
          case 5: src = a.pres + row; break;
          case 6: src = a.use_hist ? static_cast<const void*>(a.hist_off + row) : nullptr; break;
          default: src = a.seg2 + (int64_t)row * (S + 1) + slice + (lane - 7); break;
        }
        if (src) cp_async4(dst, src);
        else *dst = 0u;
      }
      cp_async_commit();
    };
    // The logits of the first SC_NST items stream in while K0 still runs: their copies read
    // nothing K0 writes (the row parameters are inputs).  Their history arrivals follow below.
    if (lane < SC_NST) {  // lane j: item j
      const int j = lane;
      const int t = blockIdx.x + j * G;
      if (t < nitems) {
        const int row = t / S;
        int slice = t - row * S + row;
        slice -= (slice / S) * S;
        const float T = a.temperature[row];
        const int k = a.top_k[row];
        const float mp = a.min_p[row];
        const bool bounded = T <= 0.0f || (k > 0 && k < V) || (mp > 0.0f && mp < 1.0f) || V <= FAST_CAP / 2;
        const int lo = slice * TS;
        const int n = min(V, lo + TS) - lo;
        const char* g0 = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
        const int nb = (bounded && (reinterpret_cast<uintptr_t>(g0) & 15) == 0) ? ((n * ES) & ~15) : 0;
        mbar_expect_tx(&ctl->full[j], (uint32_t)nb);
        unsigned char* dst = smem + j * stage_bytes;
        constexpr int CH = 32768;
        for (int off = 0; off < nb; off += CH)
          bulk_g2s(dst + off, g0 + off, (uint32_t)min(CH, nb - off), &ctl->full[j]);
      }
    }
    __syncwarp();
    pdl_wait();  // K0's pairs and segments are complete and visible
    for (int j = 0; j < SC_AHEAD; ++j) fetch(j);
    for (int j = 0;; ++j) {
      const int s = j % SC_NST;
      const int t = blockIdx.x + j * G;
      cp_async_wait_group<SC_AHEAD - 1>();  // item j's parameters have landed
      __syncwarp();
      fetch(j + SC_AHEAD);
      if (lane == 0) {
        // The item is described before its stage is free, so that only the stores and the
        // copies follow the wait.
        ItemDesc nd{};
        const char* g0 = nullptr;
        uintptr_t w0 = 0;  // first staged pair (index into the pair arrays)
        nd.mode = ITEM_END;
        if (t < nitems) {
          const uint32_t* p = ctl->prm[j % SC_RING];
          // Slices rotate with the row, so that every CTA meets every slice of the vocabulary
          // (the grid size and S share factors; without it a CTA would see two slices only).
          const int row = t / S;
          int slice = t - row * S + row;
          slice -= (slice / S) * S;
          const float T = __uint_as_float(p[0]);
          const int k = (int)p[1];
          const float mp = __uint_as_float(p[2]);
          const float rp = __uint_as_float(p[3]), fq = __uint_as_float(p[4]), pr = __uint_as_float(p[5]);
          const int hoff = (int)p[6], s0 = (int)p[7], s1 = (int)p[8];
          const bool greedy = T <= 0.0f;
          // Rows whose survivors are not bounded (top-p only or no filter on a large
          // vocabulary) go to the second kernel whole; their slices are not read here.
          const bool bounded = greedy || (k > 0 && k < V) || (mp > 0.0f && mp < 1.0f) || V <= FAST_CAP / 2;
          const int mode = !bounded ? ITEM_SKIP : greedy ? ITEM_GREEDY : ITEM_SAMPLE;
          const int lo = slice * TS;
          const int n = min(V, lo + TS) - lo;
          g0 = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
          const int nb = (mode != ITEM_SKIP && (reinterpret_cast<uintptr_t>(g0) & 15) == 0) ? ((n * ES) & ~15) : 0;
          // History pairs of this slice (K0): the 16-byte blocks that cover them, at most SC_HP.
          const int np = mode == ITEM_SAMPLE ? s1 - s0 : 0;
          int hlead = 0, hbn = 0, hb = hoff + s0;
          if (np > 0) {
            const int w0i = hb & ~3;
            hlead = hb - w0i;
            hbn = min(((hb + np + 3) & ~3) - w0i, SC_HP);
            w0 = (uintptr_t)w0i;
          }
          nd.row = row;
          nd.slice = slice;
          nd.mode = mode;
          nd.nb = nb;
          nd.hcount = np;
          nd.hb = hb;
          nd.hlead = hlead;
          nd.hbn = hbn;
          nd.T = T;
          nd.rep = rp;
          nd.freq = fq;
          nd.pres = pr;
          nd.k = (k > 0 && k < V) ? k : 0;
          nd.lo = lo;
          nd.n = n;
          nd.tl = (mp > 0.0f && mp < 1.0f) ? __fmul_rn(T, logf(mp)) : 0.0f;
          nd.sb = __fdiv_rn(BIN_PER_NAT, T);
          nd.binw = __fdiv_rn(T, BIN_PER_NAT);
        }
        if (j >= SC_NST && !mbar_wait_bounded(&ctl->empty[s], (uint32_t)((j / SC_NST - 1) & 1)))
          atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
        ctl->desc[j % (2 * SC_NST)] = nd;
        unsigned char* dst = smem + s * stage_bytes;
        if (j >= SC_NST || t >= nitems) {  // the first SC_NST items' logits are in flight already
          mbar_expect_tx(&ctl->full[s], (uint32_t)nd.nb);
          constexpr int CH = 32768;
          for (int off = 0; off < nd.nb; off += CH)
            bulk_g2s(dst + off, g0 + off, (uint32_t)min(CH, nd.nb - off), &ctl->full[s]);
        }
        mbar_expect_tx(&ctl->full[s], (uint32_t)(nd.hbn * 8));
        if (nd.hbn > 0) {
          bulk_g2s(dst + a.tile_bytes, a.uniq_ids + w0, (uint32_t)(nd.hbn * 4), &ctl->full[s]);
          bulk_g2s(dst + a.tile_bytes + SC_HP * 4, a.uniq_cnt + w0, (uint32_t)(nd.hbn * 4), &ctl->full[s]);
        }
      }
      __syncwarp();
      if (t >= nitems) break;
    }
    cp_async_wait_all();
    return;
  }

  // =======================================================================================
  // Compute warps.  Item j runs in two phases separated by barriers:
  //   M(j): the slice into registers with the history penalties applied, the slice max,
  //         then the release of the stage;
  //   X(j): the threshold, the candidates and the summary.
  // The preparation of item j + 1 (what the bulk copy skipped, 16-bit widening, padding and
  // the history counts) follows X(j) directly, so warps that finish X(j) early overlap it.
  // =======================================================================================
  const int ctid = tid;  // 0 .. SC_CT-1
  auto load_elem = [&](const char* g0, int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(g0)[i];
    if (DT == LSS_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g0)[i]);
    return __half2float(reinterpret_cast<const __half*>(g0)[i]);
  };
  bool wrote = false;     // this thread wrote the stage through the generic proxy
  bool released = false;  // the warp released the current item's stage in the preparation
  // Waits for item jj's stage and prepares it; false at the end of the list (uniform).
  auto prepare = [&](int jj) -> bool {
    const int s = jj % SC_NST;
    if (!mbar_wait_bounded_sleep(&ctl->full[s], (uint32_t)((jj / SC_NST) & 1)) && ctid == 0)
      atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
    const ItemDesc& D = ctl->desc[jj % (2 * SC_NST)];
    const int mode = D.mode;
    wrote = false;
    released = false;
    if (mode == ITEM_END) return false;
    if (mode == ITEM_SKIP) return true;
    const int row = D.row, lo = D.lo, n = D.n;
    const int n4 = (n + 3) >> 2;
    // f32: the values are used in the stage; 16-bit: widened into the work tile, which the
    // bulk copies never write, so the stage is only read and is released below, right after.
    float* tile = W16 ? WT : reinterpret_cast<float*>(smem + s * stage_bytes);
    const char* g0 = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
    const int nbulk = D.nb / ES;
    // ---- widening, what the bulk copy skipped (ragged tail / unaligned rows), padding
    if (W16 && nbulk > 0) {
      const uint16_t* h = reinterpret_cast<const uint16_t*>(smem + s * stage_bytes);
      for (int i0 = ctid * 8; i0 < nbulk; i0 += SC_CT * 8) {  // nbulk is a multiple of 8
        const uint4 raw = *reinterpret_cast<const uint4*>(h + i0);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        float v[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (DT == LSS_DTYPE_BF16) {
            v[2 * q] = __uint_as_float(w[q] << 16);
            v[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
          } else {
            v[2 * q] = __half2float(__ushort_as_half((uint16_t)(w[q] & 0xffffu)));
            v[2 * q + 1] = __half2float(__ushort_as_half((uint16_t)(w[q] >> 16)));
          }
        }
        float4* dd = reinterpret_cast<float4*>(tile + i0);
        dd[0] = make_float4(v[0], v[1], v[2], v[3]);
        dd[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
    for (int i = nbulk + ctid; i < n; i += SC_CT) {
      tile[i] = load_elem(g0, i);
      if (!W16) wrote = true;
    }
    if (ctid < n4 * 4 - n) {
      tile[n + ctid] = -INFINITY;
      if (!W16) wrote = true;
    }
    // ---- history penalties (sampling.py:55-66), once per unique id of the slice
    const int np = D.hcount;
    // Entries written above by other threads (plain loads, widening) are complete first.
    if (np > 0 && (nbulk < n || W16)) sc_sync();
    if (np > 0) {
      const int32_t* ids = reinterpret_cast<const int32_t*>(smem + s * stage_bytes + a.tile_bytes);
      const int32_t* cnt = ids + SC_HP;
      const int hlead = D.hlead, hbn = D.hbn, hb = D.hb;
      const float rp = D.rep, fq = D.freq, pr = D.pres;
      for (int e = ctid; e < np; e += SC_CT) {
        const int w = e + hlead;
        const int id = w < hbn ? ids[w] : a.uniq_ids[hb + e];
        const int c = w < hbn ? cnt[w] : a.uniq_cnt[hb + e];
        tile[id - lo] = penalise(tile[id - lo], rp, fq, pr, c);
        if (!W16) wrote = true;
      }
    }
    if (W16) {  // this warp has read all it needs of the stage (values and pairs)
      __syncwarp();
      if (lane == 0) mbar_arrive_local(&ctl->empty[s]);
      released = true;
    }
    return true;
  };

  // Summary of the previous item, written by warp 0 once the barrier that opens the next item
  // shows every warp done with it.
  int pmode = ITEM_SKIP, prow = 0, pslice = 0, ps = 0;
  uint32_t pkey = 0;
  auto write_summary = [&]() {  // warp 0
    if (pmode == ITEM_SKIP) return;
    uint64_t av = pkey;
    if (pmode == ITEM_GREEDY) {
      uint64_t b = lane < SC_CW ? ctl->best[ps][lane] : 0ull;
      av = warp_allreduce(b, MaxU64());
    }
    if (lane == 0) {
      ctl->wkey[ps][0] = 0u;  // every warp has read it (X of that item); ready for item + 2
      ItemScratch* q = &ctl->sc[ps];
      a.summ[(int64_t)prow * S + pslice] = make_uint4((uint32_t)av, (uint32_t)(av >> 32), q->cnt, q->flags);
      q->cnt = 0u;
      q->flags = 0u;
    }
  };

  pdl_wait();
  if (!prepare(0)) return;
  for (int j = 0;; ++j) {
    const int s = j % SC_NST, ip = j & 1;  // stage, item parity (scratch)
    ItemScratch* sc = &ctl->sc[ip];
    const ItemDesc& D = ctl->desc[j % (2 * SC_NST)];
    sc_sync();  // item j: slice and history counts complete; item j-1 done by every warp
    if (warp == 0) write_summary();
    const int mode = D.mode;
    const int lo = D.lo, n = D.n, n4 = (n + 3) >> 2;
    const float4* t4 = reinterpret_cast<const float4*>(W16 ? reinterpret_cast<unsigned char*>(WT) : smem + s * stage_bytes);
    const int k = D.k;
    float4 v[SC_R];
    float tmax = -INFINITY;  // max of this thread's values

    // ---- M(j)
    if (mode == ITEM_GREEDY) {
      // Greedy row (sampling.py:132-133): argmax of the raw slice, NaN first.
      uint64_t best = 0;
#pragma unroll
      for (int i = 0; i < SC_R; ++i) {
        const int q = i * SC_CT + ctid;
        if (q < n4) {
          const float4 x = t4[q];
          const int ix = lo + 4 * q;
          best = max(best, argmax_code(x.x, ix));
          best = max(best, argmax_code(x.y, ix + 1));
          best = max(best, argmax_code(x.z, ix + 2));
          best = max(best, argmax_code(x.w, ix + 3));
        }
      }
      best = warp_allreduce(best, MaxU64());
      if (lane == 0) ctl->best[ip][warp] = best;
    } else if (mode == ITEM_SAMPLE) {
      // The slice max of z (penalties applied in the preparation).
#pragma unroll
      for (int i = 0; i < SC_R; ++i) {
        const int q = i * SC_CT + ctid;
        v[i] = q < n4 ? t4[q] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        tmax = fmax_nan(tmax, fmax_nan(fmax_nan(v[i].x, v[i].y), fmax_nan(v[i].z, v[i].w)));
      }
      const float wmax = warp_allreduce(tmax, MaxF());
      if (lane == 0) atomicMax(&ctl->wkey[ip][0], (!(wmax == wmax) || wmax == INFINITY) ? 0xffffffffu : f2key(wmax));
      if (k)
        for (int i = ctid; i < NBIN + 1; i += SC_CT) HL[i] = 0u;
    }
    // The values sit in registers: what X needs of the descriptor is copied out and the
    // stage released, so that the next copy into it starts now.
    const int row = D.row, slice = D.slice;
    const float T = D.T, tl = D.tl, sbin = D.sb, binw = D.binw;
    if (!released) {
      if (wrote) fence_proxy_async();  // generic writes to the stage precede the next bulk copy
      __syncwarp();
      if (lane == 0) mbar_arrive_local(&ctl->empty[s]);
    }
    sc_sync();

    // ---- X(j)
    uint32_t mk = 0;
    if (mode == ITEM_SAMPLE) {
      mk = ctl->wkey[ip][0];
      const bool special = mk == 0xffffffffu;
      if (special && ctid == 0) atomicOr(&sc->flags, SUM_SPECIAL);
      const float M = key2f(mk);
      float thr = INFINITY;  // candidates: z >= thr
      if (!special && M > -INFINITY) {
        // Min-p floor in z: exp(y - max) >= p  <=>  z >= max_z + T ln p (y = z / T), less a
        // margin of 2^-11 relative that covers every rounding of the exact filter.
        const float zmp = tl != 0.0f ? __fsub_rn(__fadd_rn(M, tl), (fabsf(M) + fabsf(tl) + T) * 4.8828125e-04f)
                                     : -INFINITY;
        if (k) {
          // Count histogram of z over the slice (bins of 1/16 nat of y below the slice max,
          // values above the min-p floor), then the bin of the slice's k-th largest.
          uint32_t far_c = 0;
#pragma unroll
          for (int i = 0; i < SC_R; ++i) {
            const float zs[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (!(zs[q] >= zmp) || zs[q] == -INFINITY) continue;
              const float dd = __fmul_rn(__fsub_rn(M, zs[q]), sbin);
              if (dd < (float)NBIN) atomicAdd(&HL[(int)dd], 1u); else far_c++;
            }
          }
          far_c = warp_allreduce(far_c, SumU32());
          if (lane == 0 && far_c) atomicAdd(&HL[NBIN], far_c);
          sc_sync();
          // Every warp scans the bins (lane l holds bins 8l .. 8l+7).
          uint32_t c8[8];
          uint32_t loc = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            c8[q] = HL[8 * lane + q];
            loc += c8[q];
          }
          uint32_t incl = loc;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
          }
          const unsigned hit = __ballot_sync(0xffffffffu, incl >= (uint32_t)k);
          int bk = NBIN;
          if (hit) {
            const int L = __ffs(hit) - 1;
            int b = 0;
            uint32_t acc = incl - loc;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              acc += c8[q];
              if (acc < (uint32_t)k) b = q + 1;
            }
            bk = __shfl_sync(0xffffffffu, 8 * lane + b, L);
          }
          const uint32_t total = __shfl_sync(0xffffffffu, incl, 31) + HL[NBIN];
          if (bk < NBIN) {
            // The k-th largest lies in bin bk: (max - z_k) * sb < bk + 1.  One more bin of
            // slack covers the rounding of the bins and values whose y ties with it.
            float zw = __fsub_rn(M, __fmul_rn((float)(bk + 2), binw));
            zw = __fsub_rn(zw, fabsf(zw) * 2.384185791015625e-07f + 1e-37f);
            thr = fmaxf(zw, zmp);
          } else if (total > (uint32_t)k) {
            if (ctid == 0) atomicOr(&sc->flags, SUM_FAR);  // the k-th largest lies > 16 nats down
          } else {
            thr = tl != 0.0f ? zmp : -FLT_MAX;  // fewer than k values: every finite value above the floor
          }
        } else if (tl != 0.0f) {
          thr = zmp;
        } else {
          thr = -FLT_MAX;  // small vocabulary: every finite value is a candidate
        }
      }
      // ---- candidates into the item's segment
      if (__ballot_sync(0xffffffffu, tmax >= thr) != 0u) {
        uint64_t* out = a.cand + ((int64_t)row * S + slice) * a.SEG;
        const uint32_t SEG = (uint32_t)a.SEG;
#pragma unroll
        for (int i = 0; i < SC_R; ++i) {
          const bool any = v[i].x >= thr || v[i].y >= thr || v[i].z >= thr || v[i].w >= thr;
          if (__ballot_sync(0xffffffffu, any) == 0u) continue;
          const int q = i * SC_CT + ctid;
          const float zs[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const bool keep = zs[c] >= thr;
            const uint32_t bal = __ballot_sync(0xffffffffu, keep);
            if (bal) {
              const int leader = __ffs(bal) - 1;
              uint32_t base = 0;
              if (lane == leader) base = atomicAdd(&sc->cnt, (uint32_t)__popc(bal));
              base = __shfl_sync(0xffffffffu, base, leader);
              if (keep) {
                const uint32_t pos = base + __popc(bal & ((1u << lane) - 1u));
                if (pos < SEG) out[pos] = ((uint64_t)f2key(zs[c]) << 32) | (uint32_t)(~(uint32_t)(lo + 4 * q + c));
              }
            }
          }
        }
      }
    }
    pmode = mode;
    prow = row;
    pslice = slice;
    ps = ip;
    pkey = mk;
    if (!prepare(j + 1)) break;
  }
  sc_sync();
  if (warp == 0) write_summary();
}

}  // namespace lss
