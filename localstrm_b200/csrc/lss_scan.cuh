// lss_scan.cuh — K1: the streaming pass over the logits (the hot path).
//
// Persistent kernel, one CTA per SM.  The work is the list of items (row, slice), slice s of a
// row being the vocabulary range [s*TS, (s+1)*TS); CTA b takes items b, b + G, b + 2G, ...
// (G = grid size), so the CTAs in flight at any moment cover a band of consecutive rows and
// the history ids of a row are read from HBM once and from L2 by its other slices.
//
//  * 1 producer warp: fetches each item's row parameters with cp.async several items ahead;
//    when a stage of the two-stage ring is free it describes the item in shared memory and
//    starts two bulk async copies into the stage — the slice of logits and the row's history
//    ids — so the next slice streams in while the current one is processed.
//  * 15 compute warps, per item: the history ids that fall in the slice are counted in a
//    shared hash (torch.unique of the history, sampling.py:52) and the penalties applied
//    once per unique id (sampling.py:55-66); the slice max of the pre-temperature values z
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

constexpr int SC_CW = NWARP - 1;              // compute warps
constexpr int SC_CT = SC_CW * 32;             // compute threads
constexpr int SC_PROD = SC_CW;                // index of the producer warp
constexpr int SC_R = 10;                      // float4 of the slice per compute thread
constexpr int SC_TS_MAX = SC_CT * SC_R * 4;   // logits per slice (19,200)
constexpr int SC_HB = 2048;                   // history ids staged per item
constexpr int SC_HSLOTS = 2048;               // hash slots (unique ids of one slice)
constexpr int SC_HSHIFT = 21;                 // 32 - log2(SC_HSLOTS)
constexpr int SC_RING = 8;                    // parameter ring (items)
constexpr int SC_AHEAD = 4;                   // parameters fetched this many items ahead
constexpr int SC_BAR = 3;                     // named barrier of the compute warps
constexpr int SC_SEG_MIN = 256;               // candidate slots per item (at least)
constexpr uint32_t HASH_EMPTY = 0xffffffffu;

constexpr int ITEM_END = 0, ITEM_SKIP = 1, ITEM_GREEDY = 2, ITEM_SAMPLE = 3;
// Summary flags: NaN / +inf in the slice or y overflow; top-k window deeper than the bins;
// more unique history ids in the slice than the hash holds.
constexpr uint32_t SUM_SPECIAL = 1u, SUM_FAR = 2u, SUM_HASH = 4u;

struct __align__(16) ItemDesc {
  int row, slice, mode, nb;     // nb: bytes of the slice the bulk copy stages
  int hcount, hb, hlead, hbn;   // history: ids (0: no penalties), CSR base, staged window
  float T, mp, rep, freq;
  float pres;
  int k, pad0, pad1;
};
struct __align__(16) ItemScratch {
  unsigned long long best;      // greedy: argmax code of the slice
  uint32_t maxk, flags, cnt, done, nslots, pad;
};
struct __align__(16) ScanCtl {
  uint64_t full[2];             // stage landed (1 arrival + bytes)
  uint64_t empty[2];            // stage released (one arrival per compute warp)
  ItemDesc desc[2];
  ItemScratch sc[2];
  uint32_t prm[SC_RING][8];     // T, k, min_p, rep, freq, pres, hist_off[row], hist_off[row+1]
};

struct ScanArgs {
  const void* logits;
  int64_t row_stride;
  int B, V, S, TS, SEG;
  int tile_bytes;               // tile part of a stage (multiple of 128 bytes)
  int use_hist;
  int64_t hist_total;
  const float* temperature;
  const int32_t* top_k;
  const float* min_p;
  const float* rep;
  const float* freq;
  const float* pres;
  const int32_t* hist_off;
  const int32_t* hist_ids;
  uint4* summ;                  // [B*S]: {a lo, a hi, count, flags}
  uint64_t* cand;               // [B*S*SEG]: (key(z) << 32) | ~index
  uint32_t* err;
};

__host__ __device__ constexpr int scan_stage_bytes(int tile_bytes) { return tile_bytes + SC_HB * 4; }
__host__ __device__ constexpr int scan_smem_bytes(int tile_bytes) {
  return 2 * scan_stage_bytes(tile_bytes) + SC_HSLOTS * 8 + SC_HSLOTS * 2 + (((NBIN + 1) * 4 + 15) & ~15) +
         (int)((sizeof(ScanCtl) + 15) & ~15);
}

__device__ __forceinline__ void sc_sync() { asm volatile("bar.sync %0, %1;" ::"n"(SC_BAR), "n"(SC_CT) : "memory"); }

template <int DT>
__global__ void __launch_bounds__(NT, 1) lss_scan_kernel(const ScanArgs a) {
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int stage_bytes = scan_stage_bytes(a.tile_bytes);
  uint32_t* hkeys = reinterpret_cast<uint32_t*>(smem + 2 * stage_bytes);
  uint32_t* hcnts = hkeys + SC_HSLOTS;
  uint16_t* hlist = reinterpret_cast<uint16_t*>(hcnts + SC_HSLOTS);
  uint32_t* HL = reinterpret_cast<uint32_t*>(hlist + SC_HSLOTS);
  ScanCtl* ctl = reinterpret_cast<ScanCtl*>(reinterpret_cast<unsigned char*>(HL) + (((NBIN + 1) * 4 + 15) & ~15));
  const int V = a.V, S = a.S, TS = a.TS;
  const int nitems = a.B * S;
  const int G = gridDim.x;

  for (int i = tid; i < SC_HSLOTS; i += NT) {
    hkeys[i] = HASH_EMPTY;
    hcnts[i] = 0;
  }
  if (tid < (int)(2 * sizeof(ItemScratch) / 4)) reinterpret_cast<uint32_t*>(ctl->sc)[tid] = 0u;
  if (tid == 0) {
    mbar_init(&ctl->full[0], 1);
    mbar_init(&ctl->full[1], 1);
    mbar_init(&ctl->empty[0], SC_CW);
    mbar_init(&ctl->empty[1], SC_CW);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == SC_PROD) {
    // =====================================================================================
    // Producer warp
    // =====================================================================================
    auto fetch = [&](int j) {  // parameters of item j into ring slot j % SC_RING (lanes 0..7)
      const int t = blockIdx.x + j * G;
      if (t < nitems && lane < 8) {
        const int row = t / S;
        uint32_t* dst = &ctl->prm[j % SC_RING][lane];
        const void* src = nullptr;
        switch (lane) {
          case 0: src = a.temperature + row; break;
          case 1: src = a.top_k + row; break;
          case 2: src = a.min_p + row; break;
          case 3: src = a.rep + row; break;
          case 4: src = a.freq + row; break;
          case 5: src = a.pres + row; break;
          default: src = a.use_hist ? static_cast<const void*>(a.hist_off + row + (lane - 6)) : nullptr; break;
        }
        if (src) cp_async4(dst, src);
        else *dst = 0u;
      }
      cp_async_commit();
    };
    for (int j = 0; j < SC_AHEAD; ++j) fetch(j);
    const uintptr_t hbase = reinterpret_cast<uintptr_t>(a.hist_ids);
    for (int j = 0;; ++j) {
      const int s = j & 1;
      const int t = blockIdx.x + j * G;
      cp_async_wait_group<SC_AHEAD - 1>();  // item j's parameters have landed
      __syncwarp();
      fetch(j + SC_AHEAD);
      if (lane == 0) {
        if (j >= 2 && !mbar_wait_bounded(&ctl->empty[s], (uint32_t)(((j >> 1) - 1) & 1)))
          atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
        ItemDesc& d = ctl->desc[s];
        if (t >= nitems) {
          d.mode = ITEM_END;
          mbar_expect_tx(&ctl->full[s], 0u);
        } else {
          const uint32_t* p = ctl->prm[j % SC_RING];
          const int row = t / S, slice = t - row * S;
          const float T = __uint_as_float(p[0]);
          const int k = (int)p[1];
          const float mp = __uint_as_float(p[2]);
          const float rp = __uint_as_float(p[3]), fq = __uint_as_float(p[4]), pr = __uint_as_float(p[5]);
          const int h0 = (int)p[6], h1 = (int)p[7];
          const bool greedy = T <= 0.0f;
          // Rows whose survivors are not bounded (top-p only or no filter on a large
          // vocabulary) go to the second kernel whole; their slices are not read here.
          const bool bounded = greedy || (k > 0 && k < V) || (mp > 0.0f && mp < 1.0f) || V <= FAST_CAP / 2;
          const int mode = !bounded ? ITEM_SKIP : greedy ? ITEM_GREEDY : ITEM_SAMPLE;
          const int lo = slice * TS;
          const int n = min(V, lo + TS) - lo;
          const char* g0 = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
          const int nb = (mode != ITEM_SKIP && (reinterpret_cast<uintptr_t>(g0) & 15) == 0) ? ((n * ES) & ~15) : 0;
          const int H = h1 - h0;
          const bool pen = mode == ITEM_SAMPLE && a.use_hist && H > 0 && (rp != 1.0f || fq != 0.0f || pr != 0.0f);
          // History window: the 16-byte blocks that cover ids [h0, h1), clipped to the
          // 16-byte blocks inside the id array, at most SC_HB ids.
          int hlead = 0, hbn = 0;
          uintptr_t w0 = 0;
          if (pen) {
            const uintptr_t lo_ok = (hbase + 15) & ~(uintptr_t)15;
            const uintptr_t hi_ok = (hbase + 4 * (uintptr_t)a.hist_total) & ~(uintptr_t)15;
            const uintptr_t b0 = hbase + 4 * (uintptr_t)h0, b1 = hbase + 4 * (uintptr_t)h1;
            w0 = b0 & ~(uintptr_t)15;
            if (w0 < lo_ok) w0 = lo_ok;
            uintptr_t w1 = (b1 + 15) & ~(uintptr_t)15;
            if (w1 > hi_ok) w1 = hi_ok;
            if (w1 > w0) {
              hbn = (int)min((uintptr_t)(SC_HB * 4), w1 - w0) / 4;
              hlead = (int)((intptr_t)b0 - (intptr_t)w0) / 4;
            }
          }
          d.row = row;
          d.slice = slice;
          d.mode = mode;
          d.nb = nb;
          d.hcount = pen ? H : 0;
          d.hb = h0;
          d.hlead = hlead;
          d.hbn = hbn;
          d.T = T;
          d.mp = mp;
          d.rep = rp;
          d.freq = fq;
          d.pres = pr;
          d.k = k;
          mbar_expect_tx(&ctl->full[s], (uint32_t)(nb + hbn * 4));
          unsigned char* dst = smem + s * stage_bytes;
          constexpr int CH = 32768;
          for (int off = 0; off < nb; off += CH)
            bulk_g2s(dst + off, g0 + off, (uint32_t)min(CH, nb - off), &ctl->full[s]);
          if (hbn > 0)
            bulk_g2s(dst + a.tile_bytes, reinterpret_cast<const void*>(w0), (uint32_t)(hbn * 4), &ctl->full[s]);
        }
      }
      __syncwarp();
      if (t >= nitems) break;
    }
    cp_async_wait_all();
    return;
  }

  // =======================================================================================
  // Compute warps
  // =======================================================================================
  const int ctid = tid;  // 0 .. SC_CT-1
  auto load_elem = [&](const char* g0, int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(g0)[i];
    if (DT == LSS_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g0)[i]);
    return __half2float(reinterpret_cast<const __half*>(g0)[i]);
  };
  for (int j = 0;; ++j) {
    const int s = j & 1;
    if (!mbar_wait_bounded(&ctl->full[s], (uint32_t)((j >> 1) & 1)) && ctid == 0)
      atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
    const ItemDesc d = ctl->desc[s];
    if (d.mode == ITEM_END) break;
    ItemScratch* sc = &ctl->sc[s];
    if (d.mode != ITEM_SKIP) {
      const int row = d.row, lo = d.slice * TS;
      const int n = min(V, lo + TS) - lo;
      const int n4 = (n + 3) >> 2;
      float* tile = reinterpret_cast<float*>(smem + s * stage_bytes);
      const float4* t4 = reinterpret_cast<const float4*>(tile);
      const char* g0 = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
      const int nbulk = d.nb / ES;

      // ---- the slice: plain loads of what the bulk copy skipped, 16-bit widening, padding
      float tailv = 0.0f;
      const int ntail = n - nbulk;
      if (DT == LSS_DTYPE_F32 || nbulk == 0) {
        for (int i = nbulk + ctid; i < n; i += SC_CT) tile[i] = load_elem(g0, i);
      } else if (ctid < ntail) {
        tailv = load_elem(g0, nbulk + ctid);
      }
      if (DT != LSS_DTYPE_F32 && nbulk > 0) {
        // Widen in place, back to front: chunk c's f32 writes only overwrite 16-bit data of
        // chunks >= 2c, which earlier iterations consumed.
        const uint16_t* h = reinterpret_cast<const uint16_t*>(tile);
        constexpr int W = SC_CT * 8;
        const int nch = (nbulk + W - 1) / W;
        for (int c = nch - 1; c >= 0; --c) {
          const int i0 = c * W + ctid * 8;
          float v[8];
          const bool act = i0 < nbulk;
          if (act) {
            const uint4 raw = *reinterpret_cast<const uint4*>(h + i0);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
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
          }
          sc_sync();
          if (act) {
            float4* dd = reinterpret_cast<float4*>(tile + i0);
            dd[0] = make_float4(v[0], v[1], v[2], v[3]);
            dd[1] = make_float4(v[4], v[5], v[6], v[7]);
          }
        }
        sc_sync();
        if (ctid < ntail) tile[nbulk + ctid] = tailv;
      }
      if (ctid < n4 * 4 - n) tile[n + ctid] = -INFINITY;

      // ---- history ids of this slice into the hash (one atomic per distinct id per warp)
      const bool pen = d.hcount > 0;
      if (pen) {
        const int32_t* hs = reinterpret_cast<const int32_t*>(smem + s * stage_bytes + a.tile_bytes);
        const int H = d.hcount;
        for (int j0 = 0; j0 < H; j0 += SC_CT) {  // warp-uniform trip count
          const int jj = j0 + ctid;
          int id = -1;
          if (jj < H) {
            const int w = jj + d.hlead;
            const int raw = (w >= 0 && w < d.hbn) ? hs[w] : a.hist_ids[d.hb + jj];
            if (raw < 0 || raw >= V) atomicOr(a.err, LSS_FLAG_BAD_HISTORY);
            else if (raw >= lo && raw < lo + n) id = raw - lo;
          }
          if (__ballot_sync(0xffffffffu, id >= 0)) {
            const unsigned same = __match_any_sync(0xffffffffu, id);
            if (id >= 0 && lane == __ffs(same) - 1) {
              uint32_t hh = ((uint32_t)id * 2654435761u) >> SC_HSHIFT;
              bool placed = false;
              for (int probe = 0; probe < SC_HSLOTS; ++probe) {
                const uint32_t old = atomicCAS(&hkeys[hh], HASH_EMPTY, (uint32_t)id);
                if (old == HASH_EMPTY) hlist[atomicAdd(&sc->nslots, 1u)] = (uint16_t)hh;
                if (old == HASH_EMPTY || old == (uint32_t)id) {
                  atomicAdd(&hcnts[hh], (uint32_t)__popc(same));
                  placed = true;
                  break;
                }
                hh = (hh + 1) & (SC_HSLOTS - 1);
              }
              if (!placed) atomicOr(&sc->flags, SUM_HASH);
            }
          }
        }
      }
      sc_sync();  // slice complete, hash built
      if (pen) {
        // Penalties once per unique id; the slots used are emptied for the next item.
        const uint32_t ns = *reinterpret_cast<volatile uint32_t*>(&sc->nslots);
        for (uint32_t i = ctid; i < ns; i += SC_CT) {
          const uint32_t hh = hlist[i];
          const uint32_t id = hkeys[hh];
          tile[id] = penalise(tile[id], d.rep, d.freq, d.pres, (int)hcnts[hh]);
          hkeys[hh] = HASH_EMPTY;
          hcnts[hh] = 0;
        }
        sc_sync();
      }

      if (d.mode == ITEM_GREEDY) {
        // ---- greedy row (sampling.py:132-133): argmax of the raw slice, NaN first
        uint64_t best = 0;
#pragma unroll
        for (int i = 0; i < SC_R; ++i) {
          const int q = i * SC_CT + ctid;
          if (q < n4) {
            const float4 v = t4[q];
            const int ix = lo + 4 * q;
            best = max(best, argmax_code(v.x, ix));
            best = max(best, argmax_code(v.y, ix + 1));
            best = max(best, argmax_code(v.z, ix + 2));
            best = max(best, argmax_code(v.w, ix + 3));
          }
        }
        best = warp_allreduce(best, MaxU64());
        if (lane == 0) atomicMax(&sc->best, (unsigned long long)best);
      } else {
        // ---- slice max of z, values kept in registers
        float4 v[SC_R];
        float wmax = -INFINITY;
#pragma unroll
        for (int i = 0; i < SC_R; ++i) {
          const int q = i * SC_CT + ctid;
          v[i] = q < n4 ? t4[q] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
          wmax = fmax_nan(wmax, fmax_nan(fmax_nan(v[i].x, v[i].y), fmax_nan(v[i].z, v[i].w)));
        }
        wmax = warp_allreduce(wmax, MaxF());
        if (lane == 0) {
          if (!(wmax == wmax) || wmax == INFINITY) atomicOr(&sc->flags, SUM_SPECIAL);
          else atomicMax(&sc->maxk, f2key(wmax));
        }
        const float T = d.T, mp = d.mp;
        const int k = d.k;
        const bool tk_on = k > 0 && k < V;
        const bool mp_on = mp > 0.0f && mp < 1.0f;
        if (tk_on)
          for (int i = ctid; i < NBIN + 1; i += SC_CT) HL[i] = 0u;
        sc_sync();
        const bool special = (*reinterpret_cast<volatile uint32_t*>(&sc->flags) & SUM_SPECIAL) != 0u;
        const float M = key2f(*reinterpret_cast<volatile uint32_t*>(&sc->maxk));
        const float my = __fdiv_rn(M, T);
        float thr = INFINITY;  // candidates: z >= thr
        if (!special && my == INFINITY) {
          if (lane == 0 && warp == 0) atomicOr(&sc->flags, SUM_SPECIAL);  // y overflows
        } else if (!special && M > -INFINITY) {
          const float zmp = mp_on ? z_floor_for(minp_floor_y(my, mp), T) : -INFINITY;
          if (tk_on) {
            // Count histogram of z over the slice (bins of 1/16 nat of y below the slice
            // max, values above the min-p floor), then the bin of the slice's k-th largest.
            const float sb = __fdiv_rn(BIN_PER_NAT, T);
            uint32_t far_c = 0;
#pragma unroll
            for (int i = 0; i < SC_R; ++i) {
              const float zs[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                if (!(zs[q] >= zmp) || zs[q] == -INFINITY) continue;
                const float dd = __fmul_rn(__fsub_rn(M, zs[q]), sb);
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
              // Two bins of slack below the k-th largest cover values whose y ties with it.
              float zw = __fsub_rn(M, __fdiv_rn((float)(bk + 2), sb));
              zw = __fsub_rn(zw, fabsf(zw) * 2.384185791015625e-07f + 1e-37f);
              thr = fmaxf(zw, zmp);
            } else if (total > (uint32_t)k) {
              if (lane == 0 && warp == 0) atomicOr(&sc->flags, SUM_FAR);  // k-th largest > 16 nats down
            } else {
              thr = mp_on ? zmp : -FLT_MAX;  // fewer than k values: every finite value above the floor
            }
          } else if (mp_on) {
            thr = zmp;
          } else {
            thr = -FLT_MAX;  // small vocabulary: every finite value is a candidate
          }
        }
        // ---- candidates into the item's segment
        if (thr < INFINITY) {
          uint64_t* out = a.cand + ((int64_t)row * S + d.slice) * a.SEG;
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
    }
    // ---- release the stage; the last warp of the item writes its summary
    fence_proxy_async();  // this warp's accesses to the stage precede the next bulk copy
    __syncwarp();
    if (lane == 0) {
      if (d.mode != ITEM_SKIP) {
        __threadfence_block();
        const uint32_t prev = atomicAdd(&sc->done, 1u);
        if (prev == (uint32_t)(SC_CW - 1)) {
          __threadfence_block();
          volatile ItemScratch* vs = sc;
          const uint64_t av = d.mode == ITEM_GREEDY ? (uint64_t)vs->best : (uint64_t)vs->maxk;
          uint4 sm;
          sm.x = (uint32_t)av;
          sm.y = (uint32_t)(av >> 32);
          sm.z = vs->cnt;
          sm.w = vs->flags;
          a.summ[(int64_t)d.row * S + d.slice] = sm;
          vs->best = 0ull;
          vs->maxk = 0u;
          vs->flags = 0u;
          vs->cnt = 0u;
          vs->nslots = 0u;
          vs->done = 0u;
        }
      }
      mbar_arrive_local(&ctl->empty[s]);
    }
  }
}

}  // namespace lss
