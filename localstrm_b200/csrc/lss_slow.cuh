// lss_slow.cuh — K3: the rows the resolve kernel defers (top-p only or no filter on a large
// vocabulary, survivors beyond the gather buffer, histories beyond the scan kernel's hash,
// NaN / +inf / all -inf rows after scaling).
//
// One cluster of CL CTAs per row (persistent over the deferred list): each CTA stages its
// slice in shared memory, applies the penalties, divides by T and the cluster reduces the
// row max.  The survivors of top-k / min-p are gathered into CTA 0 when they fit
// (lss_resolve.cuh); otherwise a cluster-wide radix select over the order-preserving keys of
// y finds the exact cuts (counts for top-k, 2^-40 fixed-point mass for top-p) and the CTA
// whose slice holds the uniform's CDF position finds the token.
#pragma once

#include "lss_common.cuh"
#include "lss_prep.cuh"
#include "lss_resolve.cuh"

namespace lss {

struct __align__(16) SlowCtl {
  uint64_t mbar;
  uint64_t xs[2][MAXCL][4];   // scalar exchange slots, written by peers (double-buffered)
  uint64_t r64[NWARP];
  double rd[NWARP];
  float rf[NWARP];
  uint32_t r32[NWARP];
  int ri[NWARP];
  uint32_t lcount;            // local survivor count
  uint32_t pad[3];
};

template <int CL>
struct SlowLayout {
  static constexpr int LCAP = SLOW_CAP / CL;
  // layout after the tile area: Ctl | lh_cnt[NBIN+1] | lh_mass[NBIN+1] |
  //                             mh_cnt[2][NBIN+1] | mh_mass[2][NBIN+1] | lcand[LCAP]
  static constexpr int CTL = (int)((sizeof(SlowCtl) + 15) & ~15);
  static constexpr int LHC = ((NBIN + 1) * 4 + 15) & ~15;
  static constexpr int LHM = (NBIN + 1) * 8;
  static constexpr int MHC = 2 * LHC;
  static constexpr int MHM = 2 * LHM;
  static constexpr int LC = LCAP * 8;
  static constexpr int EXTRA = CTL + LHC + LHM + MHC + MHM + LC;
};

template <int CL>
struct Row {
  cg::cluster_group cl;
  int me, row, lo, n, n4;
  float* tile;
  SlowCtl* ctl;
  uint32_t* lh_cnt;
  uint64_t* lh_mass;
  uint32_t* mh_cnt;   // [2][NBIN+1]
  uint64_t* mh_mass;  // [2][NBIN+1]
  uint64_t* lcand;
  uint32_t* err;
  int xpar, hpar;

  __device__ Row() : cl(cg::this_cluster()) {}

  // Every CTA publishes four u64 values; afterwards xs[p][r][*] holds rank r's values.
  __device__ int exchange(uint64_t v0, uint64_t v1, uint64_t v2, uint64_t v3) {
    const int p = xpar;
    xpar ^= 1;
    const int t = threadIdx.x;
    if (t < CL * 4) {
      const int r = t >> 2, j = t & 3;
      uint64_t v = j == 0 ? v0 : j == 1 ? v1 : j == 2 ? v2 : v3;
      uint64_t* dst = cl.map_shared_rank(&ctl->xs[p][me][j], r);
      *dst = v;
    }
    cl.sync();
    return p;
  }
  // Adds this CTA's local histogram into every CTA's merged buffer; returns its parity.
  template <bool MASS>
  __device__ int merge_hist() {
    const int p = hpar;
    hpar ^= 1;
    __syncthreads();
    for (int i = threadIdx.x; i < CL * (NBIN + 1); i += NT) {
      const int r = i / (NBIN + 1), b = i - r * (NBIN + 1);
      uint32_t c = lh_cnt[b];
      if (c) {
        atomicAdd(cl.map_shared_rank(&mh_cnt[p * (NBIN + 1) + b], r), c);
        if (MASS) {
          unsigned long long m = lh_mass[b];
          if (m) atomicAdd((unsigned long long*)cl.map_shared_rank(&mh_mass[p * (NBIN + 1) + b], r), m);
        }
      }
    }
    cl.sync();
    return p;
  }
  __device__ void zero_merged(int p) {
    for (int i = threadIdx.x; i < NBIN + 1; i += NT) {
      mh_cnt[p * (NBIN + 1) + i] = 0;
      mh_mass[p * (NBIN + 1) + i] = 0;
    }
  }
  __device__ void zero_local() {
    for (int i = threadIdx.x; i < NBIN + 1; i += NT) {
      lh_cnt[i] = 0;
      lh_mass[i] = 0;
    }
    __syncthreads();
  }
};

// Scan of the NBIN bins of a merged histogram by one warp (every warp of the CTA computes the
// same result): lane l holds bins 8l .. 8l+7 in ascending order, or bins NBIN-1-8l down to
// NBIN-8-8l when `desc`.  Returns the first bin, in scan order, at which base plus the
// inclusive cumulative measure exceeds `target` (reaches it when `ge`), with base plus the
// measure of the bins scanned before it in `before`; -1 when no bin does.  `sum` gets base
// plus the measure of all NBIN bins (the far bin NBIN is not included).
__device__ __forceinline__ int warp_bin_cross(const uint32_t* hc, const uint64_t* hm, bool mass, bool desc,
                                              uint64_t base, uint64_t target, bool ge, uint64_t& before,
                                              uint64_t& sum) {
  static_assert(NBIN == 256, "one warp scans 8 bins per lane");
  const int lane = threadIdx.x & 31;
  uint64_t c8[8];
  uint64_t loc = 0;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int b = desc ? NBIN - 1 - (8 * lane + q) : 8 * lane + q;
    c8[q] = mass ? hm[b] : (uint64_t)hc[b];
    loc += c8[q];
  }
  uint64_t incl = loc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  sum = base + __shfl_sync(0xffffffffu, incl, 31);
  const unsigned hit = __ballot_sync(0xffffffffu, ge ? base + incl >= target : base + incl > target);
  if (!hit) {
    before = sum;
    return -1;
  }
  const int L = __ffs(hit) - 1;
  int qq = 7;
  uint64_t run = base + incl - loc, bef = run;
  bool seen = false;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint64_t nx = run + c8[q];
    if (!seen && (ge ? nx >= target : nx > target)) {
      seen = true;
      qq = q;
      bef = run;
    }
    run = nx;
  }
  const int r = __shfl_sync(0xffffffffu, 8 * lane + qq, L);
  before = __shfl_sync(0xffffffffu, bef, L);
  return desc ? NBIN - 1 - r : r;
}

// Result of a cluster-wide radix select.
struct Sel {
  bool found;     // false when the whole measure is <= target (nothing to cut)
  uint32_t K;     // key of the group that crosses the target
  uint64_t A;     // measure of all elements with key > K
  uint32_t neq;   // elements with key == K
  uint64_t eeq;   // fixed-point mass of one element at K (MASS only)
  uint64_t total; // measure of all candidate elements (key >= floorK)
};

// Finds the key group at which the descending cumulative measure (count, or fixed-point
// mass exp(y - m) * 2^40) of the elements with key >= floorK first exceeds `target`.
// For MASS the target is floor(top_p * total), computed after the first pass.
template <int CL, bool MASS>
__device__ Sel radix_select(Row<CL>& R, uint32_t floorK, float m, uint64_t target_count,
                            float tp) {
  Sel s{};
  const float4* t4 = reinterpret_cast<const float4*>(R.tile);
  // Level 0: value-space bins relative to the max.
  R.zero_local();
  {
    uint32_t far_c = 0;
    uint64_t far_m = 0;
    for (int q = threadIdx.x; q < R.n4; q += NT) {
      float4 v = t4[q];
      float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float y = ys[j];
        uint32_t k = f2key(y);
        if (k < floorK) continue;
        int b = vbin(y, m);
        uint64_t e = MASS ? efix(expf(__fsub_rn(y, m))) : 0;
        if (b < NBIN) {
          atomicAdd(&R.lh_cnt[b], 1u);
          if (MASS && e) atomicAdd((unsigned long long*)&R.lh_mass[b], (unsigned long long)e);
        } else {
          far_c++;
          far_m += e;
        }
      }
    }
    far_c = block_allreduce(far_c, SumU32(), R.ctl->r32);
    if (MASS) far_m = block_allreduce(far_m, SumU64(), R.ctl->r64);
    if (threadIdx.x == 0) {
      R.lh_cnt[NBIN] = far_c;
      R.lh_mass[NBIN] = far_m;
    }
  }
  int p = R.template merge_hist<MASS>();
  const uint32_t* hc = R.mh_cnt + p * (NBIN + 1);
  const uint64_t* hm = R.mh_mass + p * (NBIN + 1);
  uint64_t acc, sum;
  warp_bin_cross(hc, hm, MASS, false, 0, ~0ull, false, acc, sum);
  const uint64_t total = sum + (MASS ? hm[NBIN] : (uint64_t)hc[NBIN]);
  s.total = total;
  uint64_t target = MASS ? (uint64_t)floor((double)total * (double)tp) : target_count;
  if (total <= target) {
    s.found = false;
    __syncthreads();
    R.zero_merged(p);
    return s;
  }
  // First bin (the far bin last) at which the cumulative measure exceeds the target; acc is
  // the measure of the bins before it.
  int b0 = warp_bin_cross(hc, hm, MASS, false, 0, target, false, acc, sum);
  if (b0 < 0) {
    b0 = NBIN;
    acc = sum;
  }
  __syncthreads();
  R.zero_merged(p);
  // Key range that holds bin b0 (widened; the vbin predicate keeps it exact).
  const float span = fmaxf(fabsf(m), 16.0f) * 9.5367431640625e-07f;  // 2^-20 relative slack
  uint32_t lo, hi;
  if (b0 < NBIN) {
    float yhi = __fadd_rn(__fsub_rn(m, (float)b0 / BIN_PER_NAT), span);
    float ylo = __fsub_rn(__fsub_rn(m, (float)(b0 + 1) / BIN_PER_NAT), span);
    hi = min(f2key(yhi), f2key(m));
    lo = max(f2key(ylo), floorK);
  } else {
    float yhi = __fadd_rn(__fsub_rn(m, (float)NBIN / BIN_PER_NAT), span);
    hi = min(f2key(yhi), f2key(m));
    lo = floorK;
  }
  if (lo > hi) lo = hi;
  uint64_t A = acc;
  // Key-space levels.
  for (int level = 0; level < 8; ++level) {
    const uint32_t range = hi - lo;
    const int sh = range < NBIN ? 0 : (32 - __clz(range) - 8);
    R.zero_local();
    for (int q = threadIdx.x; q < R.n4; q += NT) {
      float4 v = t4[q];
      float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float y = ys[j];
        uint32_t k = f2key(y);
        if (k < lo || k > hi || k < floorK) continue;
        if (vbin(y, m) != b0) continue;
        int bb = (int)((k - lo) >> sh);
        atomicAdd(&R.lh_cnt[bb], 1u);
        if (MASS) {
          uint64_t e = efix(expf(__fsub_rn(y, m)));
          if (e) atomicAdd((unsigned long long*)&R.lh_mass[bb], (unsigned long long)e);
        }
      }
    }
    p = R.template merge_hist<MASS>();
    hc = R.mh_cnt + p * (NBIN + 1);
    hm = R.mh_mass + p * (NBIN + 1);
    // Highest bin first; the bins above (range >> sh) hold nothing.
    uint64_t a2, s2;
    const int c = warp_bin_cross(hc, hm, MASS, true, A, target, false, a2, s2);
    uint32_t cnt_c = c >= 0 ? hc[c] : 0;
    uint64_t mass_c = c >= 0 ? hm[c] : 0;
    __syncthreads();
    R.zero_merged(p);
    if (c < 0) {  // cannot happen with exact arithmetic; report and stop
      if (threadIdx.x == 0) atomicOr(R.err, LSS_FLAG_INTERNAL);
      s.found = false;
      return s;
    }
    A = a2;
    const uint32_t nlo = lo + ((uint32_t)c << sh);
    const uint32_t nhi = min(hi, nlo + ((1u << sh) - 1u));
    if (sh == 0) {
      s.found = true;
      s.K = nlo;
      s.A = A;
      s.neq = cnt_c;
      s.eeq = (MASS && cnt_c) ? mass_c / cnt_c : 0;
      return s;
    }
    lo = nlo;
    hi = nhi;
  }
  s.found = false;
  return s;
}

template <int CL, int DT>
__device__ void slow_row(Row<CL>& R, const RowArgs& a, const int row, uint32_t& phase) {
  using SM = SlowLayout<CL>;
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  const int tid = threadIdx.x;
  const int V = a.V;
  float* tile = R.tile;
  SlowCtl* ctl = R.ctl;
  const int lo = R.lo, n = R.n, n4 = R.n4;
  // Rank 0 turns the row's history into per-slice (id, count) segments, using its tile
  // memory as the hash before the slice lands there; the cluster barrier below publishes
  // the segments to every CTA of the cluster.
  if (a.use_hist && R.me == 0) {
    uint32_t* hm = reinterpret_cast<uint32_t*>(tile);
    const bool active = a.temperature[row] > 0.0f &&
                        (a.rep[row] != 1.0f || a.freq[row] != 0.0f || a.pres[row] != 0.0f);
    const PrepOut o{a.seg_off + (int64_t)row * (MAXCL + 1), a.err};
    prep_row<NT>(a, row, active, a.TE, CL, o, hm, BlockSync());
  }
  // The previous row (or the history hash) wrote this tile through the generic proxy; order
  // that before the bulk copy of this row.
  fence_proxy_async();
  __syncthreads();
  // ---- stage this CTA's slice of the row in shared memory
  const char* g0 = reinterpret_cast<const char*>(a.logits) + ((int64_t)row * a.row_stride + lo) * ES;
  const bool bulk = n > 0 && ((reinterpret_cast<uintptr_t>(g0) & 15) == 0);
  const int nbytes = bulk ? ((n * ES) & ~15) : 0;
  const int nbulk = nbytes / ES;
  if (tid == 0 && nbytes > 0) {
    fence_proxy_async();
    mbar_expect_tx(&ctl->mbar, (uint32_t)nbytes);
    constexpr int CH = 32768;
    for (int off = 0; off < nbytes; off += CH)
      bulk_g2s(reinterpret_cast<unsigned char*>(tile) + off, g0 + off, (uint32_t)min(CH, nbytes - off),
               &ctl->mbar);
  }
  // Rank 0 has finished the previous row (its tile held that row's survivors) before any
  // CTA of the cluster touches distributed shared memory for this row.
  R.cl.sync();
  // Elements the bulk copy does not cover (ragged tail / unaligned rows): plain loads.
  auto load_elem = [&](int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(g0)[i];
    if (DT == LSS_DTYPE_BF16)
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g0)[i]);
    return __half2float(reinterpret_cast<const __half*>(g0)[i]);
  };
  float tailv[1];
  const int ntail = n - nbulk;  // < 8 when bulk, else n
  if (DT == LSS_DTYPE_F32 || !bulk) {
    for (int i = nbulk + tid; i < n; i += NT) tile[i] = load_elem(i);
  } else {
    tailv[0] = (tid < ntail) ? load_elem(nbulk + tid) : 0.0f;
  }
  if (nbytes > 0) {
    if (!mbar_wait_bounded(&ctl->mbar, phase & 1u) && tid == 0) atomicOr(a.err, LSS_FLAG_TMA_TIMEOUT);
    ++phase;
  }
  if (DT != LSS_DTYPE_F32 && nbulk > 0) {
    // Widen 16-bit values in place, back to front: chunk c's f32 writes only
    // overwrite 16-bit data of chunks >= 2c, which earlier iterations consumed.
    const uint16_t* h = reinterpret_cast<const uint16_t*>(tile);
    constexpr int W = NT * 8;
    const int nch = (nbulk + W - 1) / W;
    for (int c = nch - 1; c >= 0; --c) {
      const int i0 = c * W + tid * 8;
      float v[8];
      const bool act = i0 < nbulk;  // nbulk is a multiple of 8
      if (act) {
        uint4 raw = *reinterpret_cast<const uint4*>(h + i0);
        uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint16_t l16 = (uint16_t)(w[j] & 0xffffu), h16 = (uint16_t)(w[j] >> 16);
          if (DT == LSS_DTYPE_BF16) {
            v[2 * j] = __uint_as_float((uint32_t)l16 << 16);
            v[2 * j + 1] = __uint_as_float((uint32_t)h16 << 16);
          } else {
            v[2 * j] = __half2float(__ushort_as_half(l16));
            v[2 * j + 1] = __half2float(__ushort_as_half(h16));
          }
        }
      }
      __syncthreads();
      if (act) {
        float4* d = reinterpret_cast<float4*>(tile + i0);
        d[0] = make_float4(v[0], v[1], v[2], v[3]);
        d[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
    __syncthreads();
    if (tid < ntail) tile[nbulk + tid] = tailv[0];
  }
  // Pad to a whole float4 with -inf (never a survivor, never the argmax of a real row).
  if (tid < n4 * 4 - n) tile[n + tid] = -INFINITY;
  __syncthreads();

  const float T = a.temperature[row];
  const bool greedy = T <= 0.0f;
  float4* t4 = reinterpret_cast<float4*>(tile);

  if (greedy) {
    uint64_t best = 0;
    for (int q = tid; q < n4; q += NT) {
      float4 v = t4[q];
      const int i = lo + 4 * q;
      best = max(best, argmax_code(v.x, i));
      best = max(best, argmax_code(v.y, i + 1));
      best = max(best, argmax_code(v.z, i + 2));
      best = max(best, argmax_code(v.w, i + 3));
    }
    best = block_allreduce(best, MaxU64(), ctl->r64);
    const int p = R.exchange(best, 0, 0, 0);
    if (R.me == 0 && tid == 0) {
      uint64_t b = 0;
      for (int r = 0; r < CL; ++r) b = max(b, ctl->xs[p][r][0]);
      a.tokens[row] = (int32_t)(~(uint32_t)b);
      a.row_path[row] = LSS_PATH_GREEDY;
    }
    return;
  }

  // ---- penalties (sampling.py:55-66), then y = z / T (sampling.py:146) and the row max
  if (a.use_hist) {
    apply_patches_global(a, row, R.me, lo, n, tile, 0);
    __syncthreads();
  }
  float lmax = -INFINITY;
  for (int q = tid; q < n4; q += NT) {
    float4 v = t4[q];
    const int i = 4 * q;
    v.x = __fdiv_rn(v.x, T);
    v.y = __fdiv_rn(v.y, T);
    v.z = __fdiv_rn(v.z, T);
    v.w = __fdiv_rn(v.w, T);
    if (i + 3 >= n) {  // keep the -inf padding
      if (i + 1 >= n) v.y = -INFINITY;
      if (i + 2 >= n) v.z = -INFINITY;
      if (i + 3 >= n) v.w = -INFINITY;
    }
    lmax = fmax_nan(lmax, fmax_nan(fmax_nan(v.x, v.y), fmax_nan(v.z, v.w)));
    t4[q] = v;
  }
  lmax = block_allreduce(lmax, MaxF(), ctl->rf);
  int p = R.exchange((uint64_t)__float_as_uint(lmax), 0, 0, 0);
  float m = -INFINITY;
  for (int r = 0; r < CL; ++r) m = fmax_nan(m, __uint_as_float((uint32_t)ctl->xs[p][r][0]));

  if (!(m == m) || m == INFINITY || m == -INFINITY) {
    // NaN guard (sampling.py:159-160): argmax of y with NaN largest, lowest index.
    uint64_t best = 0;
    for (int q = tid; q < n4; q += NT) {
      float4 v = t4[q];
      const int i = lo + 4 * q;
      best = max(best, argmax_code(v.x, i));
      best = max(best, argmax_code(v.y, i + 1));
      best = max(best, argmax_code(v.z, i + 2));
      best = max(best, argmax_code(v.w, i + 3));
    }
    best = block_allreduce(best, MaxU64(), ctl->r64);
    p = R.exchange(best, 0, 0, 0);
    if (R.me == 0 && tid == 0) {
      uint64_t b = 0;
      for (int r = 0; r < CL; ++r) b = max(b, ctl->xs[p][r][0]);
      a.tokens[row] = (int32_t)(~(uint32_t)b);
      a.row_path[row] = LSS_PATH_SPECIAL;
    }
    return;
  }

  // ---- per-row filter parameters
  const int k = a.top_k[row];
  const float mp = a.min_p[row], tp = a.top_p[row];
  const bool tk_on = k > 0 && k < V;
  const bool mp_on = mp > 0.0f && mp < 1.0f;
  const bool tp_on = tp > 0.0f && tp < 1.0f;
  const float u = a.uniforms[row];
  const uint32_t Kmp = mp_on ? minp_key(m, mp) : KEY_FINITE_MIN;

  // ---- top-k window from a value-space count histogram (elements with key >= Kmp)
  bool tk_bind = false;  // top-k cuts inside the min-p survivors
  int bk = NBIN;         // window: vbin <= bk
  bool need_dense = false;
  if (tk_on) {
    R.zero_local();
    uint32_t far_c = 0;
    for (int q = tid; q < n4; q += NT) {
      float4 v = t4[q];
      float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (f2key(ys[j]) < Kmp) continue;
        int b = vbin(ys[j], m);
        if (b < NBIN) atomicAdd(&R.lh_cnt[b], 1u); else far_c++;
      }
    }
    far_c = block_allreduce(far_c, SumU32(), ctl->r32);
    if (tid == 0) R.lh_cnt[NBIN] = far_c;
    const int hp = R.template merge_hist<false>();
    const uint32_t* hc = R.mh_cnt + hp * (NBIN + 1);
    // First bin at which the cumulative count reaches k.
    uint64_t before, sum;
    const int b = warp_bin_cross(hc, R.mh_mass + hp * (NBIN + 1), false, false, 0, (uint64_t)k, true, before, sum);
    if (b >= 0) {
      tk_bind = true;
      bk = b;
    } else if (sum + hc[NBIN] > (uint64_t)k) {
      need_dense = true;  // the k-th largest is more than 16 nats below the max
    }
    __syncthreads();
    R.zero_merged(hp);
  }

  // ---- compaction of the window into a local list: every thread counts what it keeps, a
  // block scan places the threads' runs, and the list is written only when it fits (a CTA
  // over LCAP sends the row to the dense path, which needs no list).
  if (!need_dense) {
    auto keep = [&](float y) {
      return f2key(y) >= Kmp && y > -INFINITY && (!tk_bind || vbin(y, m) <= bk);
    };
    uint32_t mine = 0;
    for (int q = tid; q < n4; q += NT) {
      const float4 v = t4[q];
      mine += (uint32_t)keep(v.x) + (uint32_t)keep(v.y) + (uint32_t)keep(v.z) + (uint32_t)keep(v.w);
    }
    uint32_t ctot;
    uint32_t pos = block_excl_scan(mine, ctl->r32, ctot);
    if (ctot <= (uint32_t)SM::LCAP) {
      for (int q = tid; q < n4; q += NT) {
        const float4 v = t4[q];
        const float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (keep(ys[j])) R.lcand[pos++] = ((uint64_t)f2key(ys[j]) << 32) | (uint32_t)(~(uint32_t)(lo + 4 * q + j));
      }
    }
    if (tid == 0) ctl->lcount = ctot;
    __syncthreads();
  }
  const uint32_t lcount = need_dense ? 0xffffffffu : ctl->lcount;
  p = R.exchange(lcount, 0, 0, 0);
  uint32_t total = 0, before = 0;
  bool overflow = need_dense;
  for (int r = 0; r < CL; ++r) {
    const uint32_t c = (uint32_t)ctl->xs[p][r][0];
    if (c > (uint32_t)SM::LCAP) overflow = true;
    if (r < R.me) before += c;
    total += c;
  }

  if (!overflow) {
    // ---- gather: push the local lists into CTA 0's tile area, then CTA 0 resolves.
    uint64_t* G = reinterpret_cast<uint64_t*>(tile);
    uint64_t* Gdst = R.cl.map_shared_rank(G, 0);
    for (uint32_t i = tid; i < lcount; i += NT) Gdst[before + i] = R.lcand[i];
    R.cl.sync();
    if (R.me != 0) return;

    const ResolveIn in{m, tk_bind, k, tp_on, tp, u, row, V};
    float* E = reinterpret_cast<float*>(tile) + 2 * SLOW_CAP;  // after G[SLOW_CAP]
    const RedScratch rs{ctl->r64, ctl->rd, ctl->r32, ctl->ri};
    resolve_block<SLOW_CAP>(G, E, (int)total, in, a, rs, LSS_PATH_SLOW_GATHER);
    return;
  }

  // ---- dense path: exact cuts by cluster-wide radix select over the whole row
  uint32_t Klo = Kmp;
  if (tk_on) {
    Sel sk = radix_select<CL, false>(R, Kmp, m, (uint64_t)(k - 1), 0.0f);
    if (sk.found && sk.K > Klo) Klo = sk.K;
  }
  bool cut = false;
  uint32_t Kp = 0;
  uint64_t eeq = 0;
  uint32_t rmax = 0;
  if (tp_on) {
    Sel sp = radix_select<CL, true>(R, Klo, m, 0, tp);
    if (sp.found) {
      cut = true;
      Kp = sp.K;
      eeq = sp.eeq;
      const uint64_t target = (uint64_t)floor((double)sp.total * (double)tp);
      uint64_t r = (eeq > 0) ? (target - sp.A) / eeq + 1 : (uint64_t)sp.neq;
      rmax = (uint32_t)(r < (uint64_t)sp.neq ? r : (uint64_t)sp.neq);
    }
  }
  // Per-CTA kept mass (excluding the tie group at the cut) and tie counts.
  uint64_t Mc = 0;
  uint32_t tc = 0;
  for (int q = tid; q < n4; q += NT) {
    float4 v = t4[q];
    float ys[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t key = f2key(ys[j]);
      if (key < Klo || !(ys[j] > -INFINITY)) continue;
      if (cut && key < Kp) continue;
      if (cut && key == Kp) { tc++; continue; }
      Mc += efix(expf(__fsub_rn(ys[j], m)));
    }
  }
  Mc = block_allreduce(Mc, SumU64(), ctl->r64);
  tc = block_allreduce(tc, SumU32(), ctl->r32);
  p = R.exchange(Mc, tc, 0, 0);
  uint64_t Mall[MAXCL];
  uint32_t allow_me = 0;
  uint64_t Sfix = 0, Pme = 0;
  {
    uint32_t tprev = 0;
    for (int r = 0; r < CL; ++r) {
      const uint64_t mr = ctl->xs[p][r][0];
      const uint32_t tr = (uint32_t)ctl->xs[p][r][1];
      uint32_t al = 0;
      if (cut) al = rmax > tprev ? min(rmax - tprev, tr) : 0u;
      tprev += tr;
      Mall[r] = mr + (uint64_t)al * eeq;
      if (r == R.me) allow_me = al;
      if (r < R.me) Pme += Mall[r];
      Sfix += Mall[r];
    }
  }
  uint64_t target = (uint64_t)floor((double)u * (double)Sfix);
  if (target >= Sfix) target = Sfix ? Sfix - 1 : 0;
  // The CTA whose slice holds the target scans it in vocabulary order.
  int owner = CL - 1;
  {
    uint64_t acc = 0;
    for (int r = 0; r < CL; ++r) {
      if (Mall[r] > 0 && target < acc + Mall[r]) { owner = r; break; }
      acc += Mall[r];
    }
    if (Sfix == 0) owner = 0;
  }
  const bool scan_me = (R.me == owner) || a.kept_out || a.probs_out;
  if (scan_me) {
    const float Sf = (float)((double)Sfix / FIX_ONE);
    uint64_t run_base = Pme;
    uint32_t tie_base = 0;
    int found = 0x7fffffff;
    for (int c0 = 0; c0 < n4 * 4; c0 += NT * 4) {
      const int i0 = c0 + tid * 4;
      float ys[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (i0 < n4 * 4) {
        float4 v = t4[i0 >> 2];
        ys[0] = v.x; ys[1] = v.y; ys[2] = v.z; ys[3] = v.w;
      }
      uint32_t keyv[4];
      uint32_t ties = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        keyv[j] = f2key(ys[j]);
        if (cut && keyv[j] == Kp && keyv[j] >= Klo && ys[j] > -INFINITY) ties++;
      }
      uint32_t ttot;
      const uint32_t tpre = block_excl_scan(ties, ctl->r32, ttot) + tie_base;
      uint64_t mloc[4];
      uint64_t msum = 0;
      uint32_t tseen = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bool kept = keyv[j] >= Klo && ys[j] > -INFINITY;
        if (kept && cut) {
          if (keyv[j] < Kp) kept = false;
          else if (keyv[j] == Kp) { kept = (tpre + tseen) < allow_me; tseen++; }
        }
        mloc[j] = kept ? efix(expf(__fsub_rn(ys[j], m))) : 0;
        msum += mloc[j];
        if (kept && (a.kept_out || a.probs_out)) {
          const int64_t o = (int64_t)row * V + lo + i0 + j;
          if (a.kept_out) a.kept_out[o] = 1;
          if (a.probs_out) a.probs_out[o] = __fdiv_rn(expf(__fsub_rn(ys[j], m)), Sf);
        }
      }
      uint64_t mtot;
      const uint64_t mpre = block_excl_scan(msum, ctl->r64, mtot) + run_base;
      if (R.me == owner && found == 0x7fffffff) {
        int f = 0x7fffffff;
        uint64_t run = mpre;
        for (int j = 0; j < 4; ++j) {
          run += mloc[j];
          if (mloc[j] > 0 && run > target) { f = lo + i0 + j; break; }
        }
        f = block_allreduce(f, MinI(), ctl->ri);
        found = f;
      }
      run_base += mtot;
      tie_base += ttot;
    }
    if (R.me == owner && tid == 0) {
      a.tokens[row] = found == 0x7fffffff ? (int32_t)(lo + n - 1) : found;
      a.row_path[row] = LSS_PATH_DENSE;
    }
  }
}

template <int CL, int DT>
__global__ void __launch_bounds__(NT, 2) lss_slow_kernel(const RowArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  pdl_wait();  // the resolve kernel's deferred list is complete and visible
  const int ndefer = (int)a.counters[2];
  const int NC = gridDim.x / CL, cid = blockIdx.x / CL;
  if (cid >= ndefer) return;  // the same for every CTA of the cluster
  using SM = SlowLayout<CL>;
  Row<CL> R;
  R.me = (int)R.cl.block_rank();
  R.xpar = 0;
  R.hpar = 0;
  R.err = a.err;
  const int tid = threadIdx.x;
  R.lo = R.me * a.TE;
  R.n = max(0, min(a.V, R.lo + a.TE) - R.lo);
  R.n4 = (R.n + 3) >> 2;
  R.tile = reinterpret_cast<float*>(smem);
  unsigned char* ex = smem + a.tile_bytes;
  R.ctl = reinterpret_cast<SlowCtl*>(ex);
  R.lh_cnt = reinterpret_cast<uint32_t*>(ex + SM::CTL);
  R.lh_mass = reinterpret_cast<uint64_t*>(ex + SM::CTL + SM::LHC);
  R.mh_cnt = reinterpret_cast<uint32_t*>(ex + SM::CTL + SM::LHC + SM::LHM);
  R.mh_mass = reinterpret_cast<uint64_t*>(ex + SM::CTL + SM::LHC + SM::LHM + SM::MHC);
  R.lcand = reinterpret_cast<uint64_t*>(ex + SM::CTL + SM::LHC + SM::LHM + SM::MHC + SM::MHM);
  // Merged histograms start at zero; every reader zeroes what it read (peers add into them
  // only after a cluster barrier that follows this).
  for (int i = tid; i < 2 * (NBIN + 1); i += NT) {
    R.mh_cnt[i] = 0;
    R.mh_mass[i] = 0;
  }
  if (tid == 0) {
    mbar_init(&R.ctl->mbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  uint32_t phase = 0;
  for (int i = cid; i < ndefer; i += NC) {
    R.row = a.defer_rows[i];
    if (R.row < 0) continue;  // a row the latency path finished (the same for the whole cluster)
    slow_row<CL, DT>(R, a, R.row, phase);
    __syncthreads();
  }
}

}  // namespace lss
