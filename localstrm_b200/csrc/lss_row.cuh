// lss_row.cuh — the latency path for batches of a few rows (LocalStrm's prefix-cache and
// single-request decode, llm_engine.py:823-824 and :989, where sample_next_token runs on one
// [1, V] row): one kernel, one cluster of CL CTAs per row, the whole of sample_next_token
// (sampling.py:118-163) without a round trip through global memory between stages.
//
// CTA r of a row's cluster holds the slice [r TS, (r + 1) TS) of the row in shared memory as
// f32 (one bulk copy; 16-bit logits are widened there).  Per CTA:
//   1. while the copy lands: the row's history ids that fall into the slice, as unique
//      (id, count) pairs in a shared hash table (torch.unique, sampling.py:52); then the
//      penalties applied to those values in place (sampling.py:55-66);
//   2. the slice's max of z, whether it holds NaN, and the max of every group of RW_L lanes'
//      values; cluster barrier; every CTA reads all maxima through distributed shared memory;
//   3. the cut: the exact min-p key from the exact row max (sampling.py:89-94), and for top-k
//      rows a bound from the k-th largest group max (k groups reach it, so k values do);
//   4. the values of y = z / T (sampling.py:146) at or above the cut go to rank 0's candidate
//      buffer; cluster barrier;
//   5. rank 0: the exact k-th largest by radix select, the cut, then the sort / top-p /
//      renormalise / inverse-CDF draw of the resolve kernel (sampling.py:96-113,157-162).
// Greedy rows take the argmax of the raw row (sampling.py:132-133); rows with NaN / +inf or
// nothing finite after scaling take the NaN guard's argmax of y (sampling.py:159-160).  Rows
// whose survivors are not bounded (top-p only on a large vocabulary), whose history exceeds
// RH_CAP ids, or whose candidates overflow FAST_CAP go to the deferred-row kernel, which runs
// after this one; this kernel lists every row of the call in defer_rows (-1: done here).
#pragma once

#include "lss_common.cuh"
#include "lss_resolve.cuh"

namespace lss {

constexpr int RW_MAXCL = 16;            // CTAs per row at most
constexpr int RW_MAXB = 4;              // batches up to this size take the path
constexpr int RW_TILE_MAX = 16384;      // values per CTA at most (64 KB of f32)
constexpr int RW_L = 4;                 // lanes per group of the top-k bound
constexpr int RW_G1 = NT / RW_L;        // groups per CTA

struct RwCtl {
  uint64_t bar;
  uint64_t best;                        // greedy / NaN guard: this CTA's argmax code
  uint32_t zkey, spec;                  // this CTA's max key of z (penalised) and NaN flag
  uint32_t n;                           // rank 0: candidates sent
  uint32_t nh;                          // history pairs in this slice
  uint32_t hflags;
  uint32_t pad[3];
  uint32_t bins[260];
  uint32_t gk[RW_G1];                   // this CTA's group maxima (keys of z)
  uint32_t allk[RW_MAXCL * RW_G1];      // every group max of the row
  uint64_t G[FAST_CAP];                 // rank 0: candidates (key(y) << 32 | ~index)
  float E[FAST_CAP];
  uint32_t hkeys[RH_SLOTS], hcnts[RH_SLOTS];
  uint16_t hslot[RH_CAP];
};

// Dynamic shared memory: the f32 tile, for 16-bit logits the staged copy, then the control block.
__host__ __device__ constexpr size_t rw_tile_bytes(int TS) { return ((size_t)TS * 4 + 127) & ~(size_t)127; }
__host__ __device__ constexpr size_t rw_stage_bytes(int TS, int es) {
  return es == 4 ? 0 : (((size_t)TS * es + 127) & ~(size_t)127);
}
__host__ __device__ constexpr size_t rw_smem_bytes(int TS, int es) {
  return rw_tile_bytes(TS) + rw_stage_bytes(TS, es) + sizeof(RwCtl);
}

template <int DT>
__global__ void __launch_bounds__(NT, 1) lss_row_kernel(const RowArgs a, int TS) {
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  extern __shared__ __align__(128) unsigned char rwm[];
  cg::cluster_group cl = cg::this_cluster();
  const int CL = (int)cl.num_blocks();
  const int me = (int)cl.block_rank();
  const int row = blockIdx.x / CL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* tile = reinterpret_cast<float*>(rwm);
  unsigned char* stage = rwm + rw_tile_bytes(TS);
  RwCtl& c = *reinterpret_cast<RwCtl*>(rwm + rw_tile_bytes(TS) + rw_stage_bytes(TS, ES));
  __shared__ uint64_t r64[NWARP];
  __shared__ double rd[NWARP];
  __shared__ uint32_t r32[NWARP];
  __shared__ int ri[NWARP];
  const RedScratch rs{r64, rd, r32, ri};
  const int V = a.V;
  const int lo = me * TS;
  const int n = max(0, min(V, lo + TS) - lo);
  const float T = a.temperature[row];
  const int k = a.top_k[row];
  const float mp = a.min_p[row], tp = a.top_p[row], u = a.uniforms[row];
  const float rp = a.rep[row], fq = a.freq[row], pr = a.pres[row];
  const bool greedy = T <= 0.0f;
  const bool tk_on = k > 0 && k < V;
  const bool mp_on = mp > 0.0f && mp < 1.0f;
  const bool bounded = greedy || tk_on || mp_on || V <= FAST_CAP / 2;
  // This call's status: the error flags start at zero; the deferred-row list has one entry per
  // row of the call (this kernel writes each row's entry, -1 for a row it finished).
  if (blockIdx.x == 0 && tid < 64) a.err[tid] = tid == 2 ? (uint32_t)a.B : 0u;
  // ---- the slice into shared memory: one bulk copy of its 16-byte aligned body, plain loads
  // for the rest
  const char* src = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
  unsigned char* dst = ES == 4 ? reinterpret_cast<unsigned char*>(tile) : stage;
  const uint32_t nb = (reinterpret_cast<uintptr_t>(src) & 15) == 0 ? (uint32_t)((n * ES) & ~15) : 0u;
  if (tid == 0) {
    c.n = 0u;
    c.nh = 0u;
    c.hflags = 0u;
    mbar_init(&c.bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_expect_tx(&c.bar, nb);
    if (nb > 0) bulk_g2s(dst, src, nb, &c.bar);
  }
  for (int i = (int)nb / ES + tid; i < n; i += NT) {
    if (ES == 4) reinterpret_cast<float*>(dst)[i] = reinterpret_cast<const float*>(src)[i];
    else reinterpret_cast<uint16_t*>(dst)[i] = reinterpret_cast<const uint16_t*>(src)[i];
  }
  // ---- 1. history pairs of this slice, while the copy lands (inputs only)
  const bool hist_on = a.use_hist && !greedy && bounded && (rp != 1.0f || fq != 0.0f || pr != 0.0f);
  int hb = 0, he = 0;
  const bool bad_range = hist_on && !hist_range(a.hist_off, row, a.H, hb, he);
  const int H = he - hb;
  const bool hist_long = H > RH_CAP;
  const uint32_t cap = (H > 0 && !hist_long) ? (uint32_t)next_pow2(max(2 * H, 64)) : 0u;
  if (cap) {
    constexpr int HPT = RH_CAP / NT;
    int idv[HPT];
#pragma unroll
    for (int t = 0; t < HPT; ++t) {
      const int j = t * NT + tid;
      idv[t] = j < H ? a.hist_ids[hb + j] : INT32_MIN;
    }
    for (uint32_t s = tid; s < cap; s += NT) {
      c.hkeys[s] = EMPTY;
      c.hcnts[s] = 0u;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < HPT; ++t) {
      const int id = idv[t];
      bool fresh = false;
      uint32_t slot = 0;
      if (id != INT32_MIN) {
        if (id < 0 || id >= V) {
          if (me == 0) atomicOr(&c.hflags, LSS_FLAG_BAD_HISTORY);
        } else if (id >= lo && id < lo + n) {
          uint32_t h = ((uint32_t)id * 2654435761u) & (cap - 1u);
          for (uint32_t probe = 0; probe < cap; ++probe) {
            const uint32_t old = atomicCAS(&c.hkeys[h], EMPTY, (uint32_t)id);
            if (old == EMPTY || old == (uint32_t)id) {
              atomicAdd(&c.hcnts[h], 1u);
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
        if (lane == leader) base = atomicAdd(&c.nh, (uint32_t)__popc(bal));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (fresh) c.hslot[base + __popc(bal & ((1u << lane) - 1u))] = (uint16_t)slot;
      }
    }
  }
  uint32_t myflags = 0u;
  if (!mbar_wait_bounded(&c.bar, 0)) myflags |= LSS_FLAG_TMA_TIMEOUT;
  __syncthreads();
  if (ES == 2) {  // widen into the f32 tile
    for (int i = tid; i < n; i += NT) {
      const uint16_t h = reinterpret_cast<const uint16_t*>(stage)[i];
      tile[i] = DT == LSS_DTYPE_BF16 ? __uint_as_float((uint32_t)h << 16) : __half2float(__ushort_as_half(h));
    }
    __syncthreads();
  }
  if (cap) {
    for (int i = tid; i < (int)c.nh; i += NT) {
      const uint32_t s = c.hslot[i];
      const int id = (int)c.hkeys[s];
      tile[id - lo] = penalise(tile[id - lo], rp, fq, pr, (int)c.hcnts[s]);
    }
    __syncthreads();
  }
  // ---- 2. maxima (fmaxf passes over NaN, which the flag records; +inf shows up as the max)
  float tmax = -INFINITY;
  bool nan = false;
  uint64_t best = 0;
  const int n4 = n >> 2;  // 16-byte groups of the tile, then the last values one by one
  const float4* t4 = reinterpret_cast<const float4*>(tile);
  for (int q = tid; q < n4; q += NT) {
    const float4 v = t4[q];
    tmax = fmaxf(tmax, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    nan |= (v.x != v.x) | (v.y != v.y) | (v.z != v.z) | (v.w != v.w);
    if (greedy) {
      const int i = lo + 4 * q;
      best = max(best, max(max(argmax_code(v.x, i), argmax_code(v.y, i + 1)),
                           max(argmax_code(v.z, i + 2), argmax_code(v.w, i + 3))));
    }
  }
  for (int i = 4 * n4 + tid; i < n; i += NT) {
    const float z = tile[i];
    tmax = fmaxf(tmax, z);
    nan |= z != z;
    if (greedy) best = max(best, argmax_code(z, lo + i));
  }
  uint32_t gkey = f2key(tmax);
#pragma unroll
  for (int o = 1; o < RW_L; o <<= 1) gkey = max(gkey, __shfl_xor_sync(0xffffffffu, gkey, o));
  if ((lane & (RW_L - 1)) == 0) c.gk[warp * (32 / RW_L) + lane / RW_L] = gkey;
  const uint64_t cm = block_allreduce(((uint64_t)(nan ? 1u : 0u) << 32) | f2key(tmax), MaxU64(), r64);
  if (greedy) best = block_allreduce(best, MaxU64(), r64);
  if (tid == 0) {
    c.zkey = (uint32_t)cm;
    c.spec = (uint32_t)(cm >> 32);
    c.best = best;
  }
  cl.sync();  // every CTA's maxima are visible cluster-wide
  uint64_t rm = 0ull, rb = 0ull;
  if (tid < CL) {
    const RwCtl* rc = cl.map_shared_rank(&c, tid);
    rm = ((uint64_t)rc->spec << 32) | rc->zkey;
    rb = rc->best;
  }
  rm = block_allreduce(rm, MaxU64(), r64);
  const uint32_t zk = (uint32_t)rm, sp = (uint32_t)(rm >> 32);
  const int GK = CL * RW_G1;
  // The group maxima of the row (only top-k rows use them).
  if (tk_on && !greedy)
    for (int t = tid; t < GK; t += NT) c.allk[t] = cl.map_shared_rank(&c, t / RW_G1)->gk[t % RW_G1];
  RwCtl* c0 = cl.map_shared_rank(&c, 0);
  // Rank 0's record of the row: the token and path (when `path` is not 0), the deferred-list
  // entry, the flags.
  auto finish_rank0 = [&](int32_t token, int path, bool defer) {
    if (tid == 0) {
      if (path != 0) {
        a.tokens[row] = token;
        a.row_path[row] = path;
      }
      a.defer_rows[row] = defer ? row : -1;
      const uint32_t fl = myflags | c.hflags | (bad_range ? LSS_FLAG_BAD_HISTORY : 0u);
      if (fl) atomicOr(a.err, fl);
    }
  };
  if (greedy) {
    rb = block_allreduce(rb, MaxU64(), r64);
    cl.sync();  // the maxima have been read
    if (me == 0) finish_rank0((int32_t)(~(uint32_t)rb), LSS_PATH_GREEDY, false);
    else if (tid == 0 && myflags) atomicOr(a.err, myflags);
    return;
  }
  // Rows this kernel leaves to the deferred-row kernel (their penalties were not applied here).
  if (!bounded || hist_long) {
    cl.sync();
    if (me == 0) finish_rank0(0, 0, true);
    else if (tid == 0 && myflags) atomicOr(a.err, myflags);
    return;
  }
  const float my = zk >= KEY_FINITE_MIN ? __fdiv_rn(key2f(zk), T) : -INFINITY;
  const bool special = sp || !(my > -INFINITY && my < INFINITY);
  if (special) {
    // The NaN guard: the argmax of y over the row, NaN first, lowest index.
    uint64_t b = 0;
    for (int i = tid; i < n; i += NT) b = max(b, argmax_code(__fdiv_rn(tile[i], T), lo + i));
    b = block_allreduce(b, MaxU64(), r64);
    if (tid == 0) atomicMax(reinterpret_cast<unsigned long long*>(&c0->best), (unsigned long long)b);
    cl.sync();  // rank 0 holds the row's argmax
    if (me == 0) finish_rank0((int32_t)(~(uint32_t)c.best), LSS_PATH_SPECIAL, false);
    else if (tid == 0 && myflags) atomicOr(a.err, myflags);
    return;
  }
  __syncthreads();  // allk complete
  // ---- 3. the cut: the exact min-p key; for top-k rows the largest 16-bit key prefix that k
  // group maxima reach (no bound when fewer than k groups exist)
  const uint32_t Kmp = mp_on ? minp_key(my, mp) : KEY_FINITE_MIN;
  uint32_t cut0 = Kmp;
  if (tk_on && k <= GK) {
    const uint32_t F = block_kth_largest([&](int i) { return c.allk[i]; }, GK, k, c.bins, 16);
    if (F >= KEY_FINITE_MIN) cut0 = max(cut0, f2key(__fdiv_rn(key2f(F), T)));
  }
  // ---- 4. candidates y >= cut0 to rank 0 (z below zlow cannot reach it)
  const float zlow = z_floor_for(key2f(cut0), T);
  auto is_cand = [&](float z) -> bool {
    if (!(z >= zlow) || z == -INFINITY) return false;
    const float y = __fdiv_rn(z, T);
    return y > -INFINITY && f2key(y) >= cut0;
  };
  uint32_t cnt = 0;
  for (int q = tid; q < n4; q += NT) {
    const float4 v = t4[q];
    if (fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)) >= zlow)
      cnt += (is_cand(v.x) ? 1u : 0u) + (is_cand(v.y) ? 1u : 0u) + (is_cand(v.z) ? 1u : 0u) + (is_cand(v.w) ? 1u : 0u);
  }
  for (int i = 4 * n4 + tid; i < n; i += NT) cnt += is_cand(tile[i]) ? 1u : 0u;
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  uint32_t base = 0;
  if (lane == 31 && incl) base = atomicAdd(&c0->n, incl);
  base = __shfl_sync(0xffffffffu, base, 31) + incl - cnt;
  auto send = [&](float z, int i) {
    if (is_cand(z)) {
      if (base < (uint32_t)FAST_CAP)
        c0->G[base] = ((uint64_t)f2key(__fdiv_rn(z, T)) << 32) | (uint32_t)(~(uint32_t)(lo + i));
      ++base;
    }
  };
  if (cnt) {
    for (int q = tid; q < n4; q += NT) {
      const float4 v = t4[q];
      if (fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)) >= zlow) {
        send(v.x, 4 * q);
        send(v.y, 4 * q + 1);
        send(v.z, 4 * q + 2);
        send(v.w, 4 * q + 3);
      }
    }
    for (int i = 4 * n4 + tid; i < n; i += NT) send(tile[i], i);
  }
  cl.sync();  // rank 0 holds every candidate
  if (me != 0) {
    if (tid == 0 && myflags) atomicOr(a.err, myflags);
    return;
  }
  // ---- 5. rank 0: the exact cut and the resolve
  int nk = (int)c.n;
  if (nk == 0 || nk > FAST_CAP) {
    finish_rank0(0, 0, true);
    return;
  }
  uint32_t cut = Kmp;
  if (tk_on && k <= nk)
    cut = max(cut, block_kth_largest([&](int i) { return (uint32_t)(c.G[i] >> 32); }, nk, k, c.bins));
  if (cut > cut0) {
    constexpr int PER = FAST_CAP / NT;
    uint64_t v[PER];
    uint32_t keep = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid * PER + j;
      v[j] = i < nk ? c.G[i] : 0ull;
      if (i < nk && (uint32_t)(v[j] >> 32) >= cut) keep |= 1u << j;
    }
    uint32_t all;
    const uint32_t at = block_excl_scan((uint32_t)__popc(keep), r32, all);
    __syncthreads();
    uint32_t o = at;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (keep & (1u << j)) c.G[o++] = v[j];
    __syncthreads();
    nk = (int)all;
  }
  finish_rank0(0, 0, false);  // the deferred-list entry and the flags; the resolve writes the token
  const ResolveIn in{my, tk_on, k, tp > 0.0f && tp < 1.0f, tp, u, row, V};
  if (nk <= 32) {
    if (tid < 32) resolve_warp(tid < nk ? c.G[tid] : 0ull, nk, in, a, LSS_PATH_GATHER);
  } else {
    resolve_block<FAST_CAP>(c.G, c.E, nk, in, a, rs, LSS_PATH_GATHER);
  }
}

}  // namespace lss
