// lss_sampler.cu — batched token sampler for B200 (sm_100a): the one translation unit of
// liblss.so.  It holds the C ABI of include/lsampler.h and the host-side launch logic; the
// kernels live in the headers it includes:
//   lss_prep.cuh   K0  history (id, count) pairs per 1,024-logit segment; K3's per-row preparation
//   lss_stream.cuh K1  persistent streaming pass over the logits (the hot path)
//   lss_resolve.cuh K2 per-row gather of K1's candidates and history values, sort / top-k /
//                      top-p / draw
//   lss_slow.cuh   K3  rows K2 defers (dense radix select, NaN guard)
//   lss_shard.cuh      vocabulary-sharded mode: per-shard top-K records, merge and draw
//   lss_common.cuh     keys, PTX wrappers, reductions
// plus lss_argmax_kernel below (the all-greedy seam, llm_engine.py:1139-1141).
// What is computed, per row (LocalStrm src/engine/sampling.py:118-163): greedy argmax of the
// raw row for T <= 0; otherwise penalties (:38-68), y = z / T (:146), top-k / min-p / top-p
// (:71-115), the NaN guard (:159-160) and an inverse-CDF draw from a supplied uniform (:162).
// No tensor cores: this is a memory-bound select/reduce.  Host entry points return int
// statuses and never abort; device-side bounded waits set flags in the workspace header.

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "lsampler.h"
#include "lss_common.cuh"
#include "lss_prep.cuh"
#include "lss_stream.cuh"
#include "lss_resolve.cuh"
#include "lss_slow.cuh"
#include "lss_shard.cuh"
#include "lss_row.cuh"

namespace lss {

// ---------------------------------------------------------------------------
// Batched greedy argmax: CL CTAs per row stream the row with 16-byte loads.
// ---------------------------------------------------------------------------
template <int CL, int DT>
__global__ void __launch_bounds__(NT) lss_argmax_kernel(const void* logits, int64_t row_stride, int V,
                                                        int TE, int32_t* tokens) {
  __shared__ uint64_t scr[NWARP];
  __shared__ uint64_t slots[MAXCL];
  constexpr int ES = DT == LSS_DTYPE_F32 ? 4 : 2;
  cg::cluster_group cl = cg::this_cluster();
  const int me = (int)cl.block_rank();
  const int row = blockIdx.x / CL;
  const int lo = me * TE;
  const int n = max(0, min(V, lo + TE) - lo);
  const char* g0 = reinterpret_cast<const char*>(logits) + ((int64_t)row * row_stride + lo) * ES;
  cl.sync();  // all CTAs of the cluster are running before slots[] is written remotely
  uint64_t best = 0;
  auto val = [&](int i) -> float {
    if (DT == LSS_DTYPE_F32) return reinterpret_cast<const float*>(g0)[i];
    if (DT == LSS_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g0)[i]);
    return __half2float(reinterpret_cast<const __half*>(g0)[i]);
  };
  constexpr int VE = 16 / ES;  // elements per 16-byte vector
  int head = 0;
  if ((reinterpret_cast<uintptr_t>(g0) & 15) != 0) head = n;  // unaligned rows: scalar path
  const int nvec = (n - head) / VE;
  for (int i = threadIdx.x; i < head; i += NT) best = max(best, argmax_code(val(i), lo + i));
  // Eight 16-byte loads per thread requested before any is used.
  constexpr int U = 8;
  for (int q0 = 0; q0 < nvec; q0 += U * NT) {
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int q = q0 + u * NT + (int)threadIdx.x;
      raw[u] = q < nvec ? __ldg(reinterpret_cast<const uint4*>(g0) + q) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int q = q0 + u * NT + (int)threadIdx.x;
      if (q >= nvec) break;
      const int i = lo + q * VE;
      const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
      if (DT == LSS_DTYPE_F32) {
#pragma unroll
        for (int j = 0; j < 4; ++j) best = max(best, argmax_code(__uint_as_float(w[j]), i + j));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float a0, a1;
          if (DT == LSS_DTYPE_BF16) {
            a0 = __uint_as_float(w[j] << 16);
            a1 = __uint_as_float(w[j] & 0xffff0000u);
          } else {
            a0 = __half2float(__ushort_as_half((uint16_t)(w[j] & 0xffffu)));
            a1 = __half2float(__ushort_as_half((uint16_t)(w[j] >> 16)));
          }
          best = max(best, argmax_code(a0, i + 2 * j));
          best = max(best, argmax_code(a1, i + 2 * j + 1));
        }
      }
    }
  }
  for (int i = head + nvec * VE + threadIdx.x; i < n; i += NT) best = max(best, argmax_code(val(i), lo + i));
  best = block_allreduce(best, MaxU64(), scr);
  if (threadIdx.x < CL) *cl.map_shared_rank(&slots[me], (int)threadIdx.x) = best;
  cl.sync();
  if (me == 0 && threadIdx.x == 0) {
    uint64_t b = 0;
    for (int r = 0; r < CL; ++r) b = max(b, slots[r]);
    tokens[row] = (int32_t)(~(uint32_t)b);
  }
}


// ---------------------------------------------------------------------------
// Stop check: the token-id part of check_stop_criteria (sampling.py:182-185), one thread per
// row: the EOS id first, then the row's stop ids.
// ---------------------------------------------------------------------------
__global__ void lss_stop_kernel(const int32_t* tokens, int B, const int32_t* eos_ids, const int32_t* stop_off,
                                const int32_t* stop_ids, int32_t* out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int32_t t = tokens[b];
  int32_t code = LSS_STOP_NONE;
  if (eos_ids && eos_ids[b] >= 0 && t == eos_ids[b]) {
    code = LSS_STOP_EOS;
  } else if (stop_off) {
    for (int i = stop_off[b], e = stop_off[b + 1]; i < e; ++i)
      if (stop_ids[i] == t) {
        code = LSS_STOP_TOKEN;
        break;
      }
  }
  out[b] = code;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
constexpr int TILE_TARGET_BYTES = 80 * 1024;   // second kernel: slice size per CTA
constexpr int TILE_MAX_BYTES = 160 * 1024;     // second kernel: one CTA per SM
constexpr int MAX_VOCAB = MAXCL * (TILE_MAX_BYTES / 4);

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

struct Plan {
  int MAXSL;                  // slices per row the workspace reserves (either logit width)
  int CL, TE;                 // second kernel: CTAs per row, logits per CTA
  int slow_tile, slow_smem;
};

// Streaming kernel: chunks per row for logits of `es` bytes.
static int chunks_per_row(int V, int es) { return (V + ST_CB / es - 1) / (ST_CB / es); }

// Most CTA ranges one row can intersect when B * C chunks are split over at most ST_GCAP CTAs:
// every range holds at least floor(N / G) chunks.
static int max_slices(int B, int C) {
  const int64_t N = (int64_t)std::max(B, 1) * C;
  const int64_t G = std::min<int64_t>(ST_GCAP, N);
  const int64_t P = N / G;
  return (int)std::min<int64_t>(C, (C - 1 + P - 1) / P + 1);
}

static int slow_extra(int CL) {
  switch (CL) {
    case 1: return SlowLayout<1>::EXTRA;
    case 2: return SlowLayout<2>::EXTRA;
    case 4: return SlowLayout<4>::EXTRA;
    default: return SlowLayout<8>::EXTRA;
  }
}

static Plan make_plan(int B, int V) {
  Plan pl{};
  pl.MAXSL = std::max(max_slices(B, chunks_per_row(V, 4)), max_slices(B, chunks_per_row(V, 2)));
  int CL = 1;
  while (CL < MAXCL && round_up((V + CL - 1) / CL, 16) * 4 > TILE_TARGET_BYTES) CL <<= 1;
  pl.CL = CL;
  pl.TE = round_up((V + CL - 1) / CL, 16);
  pl.slow_tile = round_up(std::max(pl.TE * 4, SLOW_CAP * 12), 128);
  pl.slow_smem = pl.slow_tile + slow_extra(CL);
  return pl;
}

// Workspace: header (word 0 error flags, word 2 deferred-row count), row path codes, the
// streaming kernel's slice summaries, candidate segments and chunk maxima, the second kernel's per-slice
// segments of the unique history pairs, the deferred-row list, the pair arrays (ids, counts)
// and the global hash table for rows with long histories.  row_path sits at a fixed offset.
struct WsLayout {
  size_t header, row_path, summ, cand, cmax, seg_off, defer_rows, uniq_ids, uniq_cnt, gkeys, gcnts, total;
};
static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }
static WsLayout ws_layout(int B, int V, int64_t H) {
  WsLayout L{};
  const size_t b = (size_t)std::max(B, 1), h = (size_t)std::max<int64_t>(H, 1);
  const Plan pl = make_plan(std::max(B, 1), std::max(V, 1));
  const size_t slices = b * (size_t)pl.MAXSL;
  size_t o = 0;
  L.header = o; o += 256;
  L.row_path = o; o = align256(o + 4 * b);
  L.summ = o; o = align256(o + 16 * slices);
  L.cand = o; o = align256(o + 8 * slices * (size_t)ST_SEGCAP);
  L.cmax = o; o = align256(o + 4 * b * (size_t)chunks_per_row(std::max(V, 1), 2));
  L.seg_off = o; o = align256(o + 4 * b * (MAXCL + 1));
  L.defer_rows = o; o = align256(o + 4 * b);
  L.uniq_ids = o; o = align256(o + 4 * (h + 4));
  L.uniq_cnt = o; o = align256(o + 4 * (h + 4));
  L.gkeys = o; o = align256(o + 8 * h);
  L.gcnts = o; o = align256(o + 8 * h);
  L.total = o;
  return L;
}

// Per (kernel, device): dynamic shared memory configured and the number of CTAs or clusters
// that fit.
struct KernelCfg {
  int smem[64];
  int count[64];
};

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  return dev;
}

// The per-(kernel, device) caches are filled on first use; one lock serialises that, so host
// threads that make their first calls at the same time do not race on them.
static std::mutex g_cfg_mu;

template <class K>
static cudaError_t prepare_cluster_kernel(K kern, KernelCfg& kc, int CL, int smem, int& nclusters) {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_cfg_mu);
  if (kc.smem[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(CL * 1024), 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CL;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int nc = 0;
    e = cudaOccupancyMaxActiveClusters(&nc, kern, &cfg);
    if (e != cudaSuccess || nc <= 0) {
      cudaGetLastError();
      int nsm = 148;
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
      nc = std::max(1, nsm / CL);
    }
    kc.smem[dev] = smem;
    kc.count[dev] = nc;
  }
  nclusters = kc.count[dev];
  return cudaSuccess;
}

// Persistent grid of the streaming kernel: every CTA that fits (one per SM at this shared
// memory), at most ST_GCAP.
template <class K>
static cudaError_t prepare_stream_kernel(K kern, KernelCfg& kc, int smem, int& nctas) {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_cfg_mu);
  if (kc.smem[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0, nsm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, ST_NT, (size_t)smem);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    if (per_sm <= 0) return cudaErrorInvalidConfiguration;
    kc.smem[dev] = smem;
    kc.count[dev] = std::min(per_sm * nsm, ST_GCAP);
  }
  nctas = kc.count[dev];
  return cudaSuccess;
}

// Launch with programmatic stream serialization (the kernel may start while the previous
// kernel of the stream runs; it waits for it with griddepcontrol.wait), optionally clustered.
template <class... KArgs, class... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem, int cluster,
                              cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(block, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int na = 0;
  at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (cluster > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = (unsigned)cluster;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = (unsigned)na;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <class K>
static cudaError_t launch_clusters(K kern, const RowArgs& a, int CL, int nclusters, int smem, cudaStream_t st) {
  return launch_pdl(kern, (unsigned)(nclusters * CL), (unsigned)NT, (size_t)smem, CL, st, a);
}

// K3 over the deferred-row list (programmatic dependent launch after the kernel before it).
template <int DT>
static cudaError_t launch_slow(const RowArgs& ra, const Plan& pl, int B, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  int ncs = 0;
  switch (pl.CL) {
    case 1: {
      static KernelCfg c{};
      e = prepare_cluster_kernel(lss_slow_kernel<1, DT>, c, 1, pl.slow_smem, ncs);
      if (e == cudaSuccess) e = launch_clusters(lss_slow_kernel<1, DT>, ra, 1, std::min(ncs, B), pl.slow_smem, st);
      break;
    }
    case 2: {
      static KernelCfg c{};
      e = prepare_cluster_kernel(lss_slow_kernel<2, DT>, c, 2, pl.slow_smem, ncs);
      if (e == cudaSuccess) e = launch_clusters(lss_slow_kernel<2, DT>, ra, 2, std::min(ncs, B), pl.slow_smem, st);
      break;
    }
    case 4: {
      static KernelCfg c{};
      e = prepare_cluster_kernel(lss_slow_kernel<4, DT>, c, 4, pl.slow_smem, ncs);
      if (e == cudaSuccess) e = launch_clusters(lss_slow_kernel<4, DT>, ra, 4, std::min(ncs, B), pl.slow_smem, st);
      break;
    }
    default: {
      static KernelCfg c{};
      e = prepare_cluster_kernel(lss_slow_kernel<8, DT>, c, 8, pl.slow_smem, ncs);
      if (e == cudaSuccess) e = launch_clusters(lss_slow_kernel<8, DT>, ra, 8, std::min(ncs, B), pl.slow_smem, st);
      break;
    }
  }
  return e;
}

// K1 (streaming pass), K2 (resolve, one CTA per row), K3 (second kernel over the deferred list).
template <int DT>
static cudaError_t launch_rows(StreamArgs sa, const RowArgs& ra, GatherArgs ga, const Plan& pl, int B,
                               cudaStream_t st, bool scan_only) {
  static KernelCfg stream_cfg{};
  int nctas = 0;
  constexpr int smem = stream_smem_bytes();
  cudaError_t e = prepare_stream_kernel(lss_stream_kernel<DT>, stream_cfg, smem, nctas);
  if (e != cudaSuccess) return e;
  const int G = (int)std::min<int64_t>(nctas, sa.N);
  // Both kernels derive a row's slices from the same split of the N chunks over G CTAs.
  ga.G = G;
  // The first kernel of a call: an ordinary launch, so that it starts after everything before
  // it on the stream (the producer of the logits included) has finished.
  lss_stream_kernel<DT><<<(unsigned)G, (unsigned)ST_NT, (size_t)smem, st>>>(sa);
  e = cudaGetLastError();
  if (e != cudaSuccess || scan_only) return e;
  {
    static int resolve_smem_set[64] = {};
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(g_cfg_mu);
    if (!resolve_smem_set[dev]) {
      e = cudaFuncSetAttribute(lss_resolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, resolve_smem_bytes());
      if (e != cudaSuccess) return e;
      resolve_smem_set[dev] = 1;
    }
  }
  e = launch_pdl(lss_resolve_kernel, (unsigned)B, (unsigned)NT, (size_t)resolve_smem_bytes(), 1, st, ra, ga);
  if (e != cudaSuccess) return e;
  return launch_slow<DT>(ra, pl, B, st);
}

// The latency path for batches of up to RW_MAXB rows: lss_row_kernel (one cluster of up to 16
// CTAs per row, an ordinary launch) then K3 for the rows it leaves.  Returns false (launching
// nothing) when the row does not fit the path or such clusters cannot be resident.
template <int DT>
static bool launch_row_path(const RowArgs& ra, const Plan& pl, int B, int V, cudaStream_t st, cudaError_t& err) {
  constexpr int es = DT == LSS_DTYPE_F32 ? 4 : 2;
  const int CL = (int)std::min<int64_t>(RW_MAXCL, std::max<int64_t>(1, ((int64_t)V + 9599) / 9600));
  const int TS = round_up((V + CL - 1) / CL, 8);
  if (B < 1 || B > RW_MAXB || TS > RW_TILE_MAX) return false;
  const size_t smem = rw_smem_bytes(TS, es);
  static int attr_set[64] = {};
  static int fits[64][RW_MAXCL + 1];
  static bool fits_init = false;
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lock(g_cfg_mu);
    if (!fits_init) {
      for (auto& d : fits)
        for (int& f : d) f = -1;
      fits_init = true;
    }
    if (!attr_set[dev]) {
      err = cudaFuncSetAttribute(lss_row_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)rw_smem_bytes(RW_TILE_MAX, es));
      if (err == cudaSuccess)
        err = cudaFuncSetAttribute(lss_row_kernel<DT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (err != cudaSuccess) {
        cudaGetLastError();
        err = cudaSuccess;
        return false;
      }
      attr_set[dev] = 1;
    }
    if (fits[dev][CL] < 0) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3((unsigned)(CL * RW_MAXB), 1, 1);
      cfg.blockDim = dim3(NT, 1, 1);
      cfg.dynamicSmemBytes = rw_smem_bytes(RW_TILE_MAX, es);
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = (unsigned)CL;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int nc = 0;
      const cudaError_t e = cudaOccupancyMaxActiveClusters(&nc, lss_row_kernel<DT>, &cfg);
      if (e != cudaSuccess) cudaGetLastError();
      fits[dev][CL] = (e == cudaSuccess && nc >= RW_MAXB) ? 1 : 0;
    }
    if (!fits[dev][CL]) return false;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(B * CL), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, lss_row_kernel<DT>, ra, TS);
  if (err == cudaSuccess) err = launch_slow<DT>(ra, pl, B, st);
  return true;
}

template <int CL, int DT>
static cudaError_t launch_argmax(const void* logits, int64_t stride, int B, int V, int TE, int32_t* tok,
                                 cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(B * CL), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lss_argmax_kernel<CL, DT>, logits, stride, V, TE, tok);
}

template <int DT>
static cudaError_t launch_argmax_dt(const void* logits, int64_t stride, int B, int V, int32_t* tok,
                                    cudaStream_t st) {
  // Enough CTAs to cover the machine: split rows until B * CL >= 2 * 148 or slices get small.
  int CL = 1;
  while (CL < MAXCL && B * CL < 296 && (V + CL - 1) / CL > 4096) CL <<= 1;
  const int TE = round_up((V + CL - 1) / CL, 16);
  switch (CL) {
    case 1: return launch_argmax<1, DT>(logits, stride, B, V, TE, tok, st);
    case 2: return launch_argmax<2, DT>(logits, stride, B, V, TE, tok, st);
    case 4: return launch_argmax<4, DT>(logits, stride, B, V, TE, tok, st);
    default: return launch_argmax<8, DT>(logits, stride, B, V, TE, tok, st);
  }
}

}  // namespace lss

using namespace lss;

extern "C" {

int lss_version(void) { return (0 << 16) | (2 << 8) | 0; }

const char* lss_status_string(int s) {
  switch (s) {
    case LSS_OK: return "ok";
    case LSS_ERR_INVALID_ARG: return "invalid argument";
    case LSS_ERR_WORKSPACE: return "workspace missing or too small";
    case LSS_ERR_CUDA: return "CUDA runtime error";
    case LSS_ERR_UNSUPPORTED: return "unsupported size or device";
    case LSS_ERR_DEVICE: return "device reported an error flag";
    case LSS_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch of lss_sample_noalloc";
    default: return "unknown status";
  }
}

int lss_max_vocab(void) { return MAX_VOCAB; }

size_t lss_workspace_bytes(int B, int V, int64_t hist_total) {
  if (B < 0 || V < 1 || hist_total < 0) return 0;
  return ws_layout(B, V, hist_total).total;
}

static int check_common(int B, int V, int64_t hist_total, const int32_t* hist_offsets,
                        const void* workspace, size_t workspace_bytes) {
  if (B < 0 || V < 1 || hist_total < 0 || hist_total > 0x3fffffff) return LSS_ERR_INVALID_ARG;
  if (V > MAX_VOCAB) return LSS_ERR_UNSUPPORTED;
  if (B == 0) return LSS_OK;
  if (hist_total > 0 && !hist_offsets) return LSS_ERR_INVALID_ARG;
  const WsLayout L = ws_layout(B, V, hist_total);
  if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return LSS_ERR_WORKSPACE;
  return LSS_OK;
}

int lss_sample_prepare(int B, int V, const float* temperature, const int32_t* top_k, const float* min_p,
                       const float* repetition_penalty, const float* frequency_penalty,
                       const float* presence_penalty, const int32_t* hist_offsets, const int32_t* hist_ids,
                       int64_t hist_total, void* workspace, size_t workspace_bytes, void* stream) {
  // The history pairs are built by the resolve kernel of lss_sample_rows, which reads them
  // while the streaming kernel runs; this stage checks the arguments and launches nothing.
  (void)stream;
  int rc = check_common(B, V, hist_total, hist_offsets, workspace, workspace_bytes);
  if (rc != LSS_OK || B == 0) return rc;
  if (!temperature || !top_k || !min_p || !repetition_penalty || !frequency_penalty || !presence_penalty)
    return LSS_ERR_INVALID_ARG;
  if (hist_total > 0 && !hist_ids) return LSS_ERR_INVALID_ARG;
  return LSS_OK;
}

static int sample_rows(const void* logits, int dtype, int B, int V, int64_t row_stride, const float* temperature,
                       const int32_t* top_k, const float* top_p, const float* min_p,
                       const float* repetition_penalty, const float* frequency_penalty,
                       const float* presence_penalty, const int32_t* hist_offsets, const int32_t* hist_ids,
                       int64_t hist_total, const float* uniforms, int32_t* tokens_out, uint8_t* kept_out,
                       float* probs_out, void* workspace, size_t workspace_bytes, void* stream, bool scan_only) {
  if (row_stride < V) return LSS_ERR_INVALID_ARG;
  if (dtype != LSS_DTYPE_F32 && dtype != LSS_DTYPE_BF16 && dtype != LSS_DTYPE_F16) return LSS_ERR_INVALID_ARG;
  int rc = check_common(B, V, hist_total, hist_offsets, workspace, workspace_bytes);
  if (rc != LSS_OK || B == 0) return rc;
  if (!logits || !temperature || !top_k || !top_p || !min_p || !repetition_penalty || !frequency_penalty ||
      !presence_penalty || !uniforms || !tokens_out)
    return LSS_ERR_INVALID_ARG;
  if (hist_total > 0 && !hist_ids) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  const WsLayout L = ws_layout(B, V, hist_total);
  const Plan pl = make_plan(B, V);
  if (kept_out && cudaMemsetAsync(kept_out, 0, (size_t)B * V, st) != cudaSuccess) return LSS_ERR_CUDA;
  if (probs_out && cudaMemsetAsync(probs_out, 0, (size_t)B * V * sizeof(float), st) != cudaSuccess)
    return LSS_ERR_CUDA;
  uint32_t* header = reinterpret_cast<uint32_t*>(ws + L.header);
  const int es = dtype == LSS_DTYPE_F32 ? 4 : 2;
  StreamArgs sa{};
  sa.logits = logits;
  sa.row_stride = row_stride;
  sa.B = B;
  sa.V = V;
  sa.C = chunks_per_row(V, es);
  sa.N = (int64_t)B * sa.C;
  sa.MAXSL = pl.MAXSL;
  sa.temperature = temperature;
  sa.top_k = top_k;
  sa.min_p = min_p;
  sa.summ = reinterpret_cast<uint4*>(ws + L.summ);
  sa.cand = reinterpret_cast<uint64_t*>(ws + L.cand);
  sa.cmax = reinterpret_cast<uint32_t*>(ws + L.cmax);
  sa.header = header;
  RowArgs a{};
  a.logits = logits;
  a.row_stride = row_stride;
  a.B = B;
  a.V = V;
  a.TE = pl.TE;
  a.tile_bytes = pl.slow_tile;
  a.use_hist = hist_total > 0 ? 1 : 0;
  a.H = (int)hist_total;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.min_p = min_p;
  a.rep = repetition_penalty;
  a.freq = frequency_penalty;
  a.pres = presence_penalty;
  a.hist_off = hist_offsets;
  a.hist_ids = hist_ids;
  a.uniq_ids = reinterpret_cast<int32_t*>(ws + L.uniq_ids);
  a.uniq_cnt = reinterpret_cast<int32_t*>(ws + L.uniq_cnt);
  a.seg_off = reinterpret_cast<int32_t*>(ws + L.seg_off);
  a.gkeys = reinterpret_cast<uint32_t*>(ws + L.gkeys);
  a.gcnts = reinterpret_cast<uint32_t*>(ws + L.gcnts);
  a.CL = pl.CL;
  a.uniforms = uniforms;
  a.tokens = tokens_out;
  a.kept_out = kept_out;
  a.probs_out = probs_out;
  a.err = header;
  a.counters = header;
  a.defer_rows = reinterpret_cast<int32_t*>(ws + L.defer_rows);
  a.row_path = reinterpret_cast<int32_t*>(ws + L.row_path);
  GatherArgs ga{};
  ga.summ = sa.summ;
  ga.cand = sa.cand;
  ga.MAXSL = pl.MAXSL;
  ga.SEGCAP = ST_SEGCAP;
  ga.C = sa.C;
  ga.N = sa.N;
  ga.G = 1;  // set at launch to the streaming kernel's grid
  ga.CE = ST_CB / es;
  ga.cmax = sa.cmax;
  ga.dtype = dtype;
  cudaError_t e;
  // Batches of a few rows take the latency path (one cluster kernel per call, then K3).
  if (!scan_only && B <= RW_MAXB) {
    bool done = false;
    e = cudaSuccess;
    switch (dtype) {
      case LSS_DTYPE_F32: done = launch_row_path<LSS_DTYPE_F32>(a, pl, B, V, st, e); break;
      case LSS_DTYPE_BF16: done = launch_row_path<LSS_DTYPE_BF16>(a, pl, B, V, st, e); break;
      default: done = launch_row_path<LSS_DTYPE_F16>(a, pl, B, V, st, e); break;
    }
    if (done) {
      if (e != cudaSuccess) {
        cudaGetLastError();
        return LSS_ERR_CUDA;
      }
      return LSS_OK;
    }
  }
  switch (dtype) {
    case LSS_DTYPE_F32: e = launch_rows<LSS_DTYPE_F32>(sa, a, ga, pl, B, st, scan_only); break;
    case LSS_DTYPE_BF16: e = launch_rows<LSS_DTYPE_BF16>(sa, a, ga, pl, B, st, scan_only); break;
    default: e = launch_rows<LSS_DTYPE_F16>(sa, a, ga, pl, B, st, scan_only); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return LSS_ERR_CUDA;
  }
  return LSS_OK;
}

int lss_sample_rows(const void* logits, int dtype, int B, int V, int64_t row_stride,
                    const float* temperature, const int32_t* top_k, const float* top_p,
                    const float* min_p, const float* repetition_penalty, const float* frequency_penalty,
                    const float* presence_penalty, const int32_t* hist_offsets, const int32_t* hist_ids,
                    int64_t hist_total, const float* uniforms, int32_t* tokens_out, uint8_t* kept_out,
                    float* probs_out, void* workspace, size_t workspace_bytes, void* stream) {
  return sample_rows(logits, dtype, B, V, row_stride, temperature, top_k, top_p, min_p, repetition_penalty,
                     frequency_penalty, presence_penalty, hist_offsets, hist_ids, hist_total, uniforms, tokens_out,
                     kept_out, probs_out, workspace, workspace_bytes, stream, false);
}

int lss_scan_pass(const void* logits, int dtype, int B, int V, int64_t row_stride, const float* temperature,
                  const int32_t* top_k, const float* top_p, const float* min_p, const float* repetition_penalty,
                  const float* frequency_penalty, const float* presence_penalty, const int32_t* hist_offsets,
                  const int32_t* hist_ids, int64_t hist_total, const float* uniforms, int32_t* tokens_out,
                  void* workspace, size_t workspace_bytes, void* stream) {
  return sample_rows(logits, dtype, B, V, row_stride, temperature, top_k, top_p, min_p, repetition_penalty,
                     frequency_penalty, presence_penalty, hist_offsets, hist_ids, hist_total, uniforms, tokens_out,
                     nullptr, nullptr, workspace, workspace_bytes, stream, true);
}

int lss_sample(const void* logits, int dtype, int B, int V, int64_t row_stride, const float* temperature,
               const int32_t* top_k, const float* top_p, const float* min_p,
               const float* repetition_penalty, const float* frequency_penalty,
               const float* presence_penalty, const int32_t* hist_offsets, const int32_t* hist_ids,
               int64_t hist_total, const float* uniforms, int32_t* tokens_out, uint8_t* kept_out,
               float* probs_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (row_stride < V) return LSS_ERR_INVALID_ARG;
  if (dtype != LSS_DTYPE_F32 && dtype != LSS_DTYPE_BF16 && dtype != LSS_DTYPE_F16) return LSS_ERR_INVALID_ARG;
  int rc = check_common(B, V, hist_total, hist_offsets, workspace, workspace_bytes);
  if (rc != LSS_OK || B == 0) return rc;
  if (!logits || !temperature || !top_k || !top_p || !min_p || !repetition_penalty || !frequency_penalty ||
      !presence_penalty || !uniforms || !tokens_out)
    return LSS_ERR_INVALID_ARG;
  if (hist_total > 0 && !hist_ids) return LSS_ERR_INVALID_ARG;
  rc = lss_sample_prepare(B, V, temperature, top_k, min_p, repetition_penalty, frequency_penalty,
                          presence_penalty, hist_offsets, hist_ids, hist_total, workspace, workspace_bytes,
                          stream);
  if (rc != LSS_OK) return rc;
  return lss_sample_rows(logits, dtype, B, V, row_stride, temperature, top_k, top_p, min_p,
                         repetition_penalty, frequency_penalty, presence_penalty, hist_offsets, hist_ids,
                         hist_total, uniforms, tokens_out, kept_out, probs_out, workspace, workspace_bytes,
                         stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant: the workspace is a fixed file-scope device array.
// ---------------------------------------------------------------------------
namespace lss {
static __device__ __align__(256) unsigned char g_noalloc_scratch[LSS_NOALLOC_SCRATCH_BYTES];
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch on the current device, looked up once per device.
static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LSS_ERR_CUDA;
  if (dev < 0 || dev >= 64) return LSS_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return LSS_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return LSS_OK;
}
}  // namespace lss

extern "C" {

int lss_sample_noalloc(const void* logits, int dtype, int B, int V, int64_t row_stride,
                       const float* temperature, const int32_t* top_k, const float* top_p,
                       const float* min_p, const float* repetition_penalty,
                       const float* frequency_penalty, const float* presence_penalty,
                       const int32_t* hist_offsets, const int32_t* hist_ids, int64_t hist_total,
                       const float* uniforms, int32_t* tokens_out, uint8_t* kept_out, float* probs_out,
                       void* stream) {
  if (B < 0 || V < 1 || hist_total < 0) return LSS_ERR_INVALID_ARG;
  if (B == 0) return LSS_OK;
  const size_t need = lss_workspace_bytes(B, V, hist_total);
  if (need == 0) return LSS_ERR_INVALID_ARG;
  if (need > (size_t)LSS_NOALLOC_SCRATCH_BYTES) return LSS_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  int rc = lss::noalloc_scratch(&ws);
  if (rc != LSS_OK) return rc;
  return lss_sample(logits, dtype, B, V, row_stride, temperature, top_k, top_p, min_p, repetition_penalty,
                    frequency_penalty, presence_penalty, hist_offsets, hist_ids, hist_total, uniforms,
                    tokens_out, kept_out, probs_out, ws, (size_t)LSS_NOALLOC_SCRATCH_BYTES, stream);
}

int lss_noalloc_read_status(uint32_t* flags_out, void* stream) {
  if (!flags_out) return LSS_ERR_INVALID_ARG;
  void* ws = nullptr;
  int rc = lss::noalloc_scratch(&ws);
  if (rc != LSS_OK) return rc;
  return lss_read_status(ws, flags_out, stream);
}

size_t lss_shard_record_bytes(int K) { return K < 1 ? 0 : shard_record_bytes(K); }

size_t lss_shard_merge_workspace_bytes(int B) {
  if (B < 0) return 0;
  return 256 + (((size_t)(B > 0 ? B : 1) * 4 + 255) & ~(size_t)255);
}

}  // extern "C"

namespace lss {
// Vocabulary-shard step as clusters (lss_shard_cluster_kernel): P CTAs per row, parts of up to
// 64 KB (16 CTAs at most; the per-part phases cost more than the bytes, so fewer, larger parts
// win), about 4K group maxima per row.  Returns false (and
// launches nothing) when the shard row does not fit or no such cluster can be resident.
template <int DT>
static bool launch_shard_cluster(const void* logits, int64_t stride, int B, int Vs, int64_t voff, const float* T,
                                 int K, unsigned char* rec, cudaStream_t st, cudaError_t& err) {
  constexpr int es = DT == LSS_DTYPE_F32 ? 4 : 2;
  const int P = (int)std::min<int64_t>(SC_MAXCL, std::max<int64_t>(1, ((int64_t)Vs * es + 65535) / 65536));
  const int PS = round_up((Vs + P - 1) / P, 8);
  if ((size_t)PS * es > (size_t)SC_PART_MAX) return false;
  int L = 32;
  while (L > 1 && (int64_t)P * (SC_NT / L) < 4LL * K) L >>= 1;
  while (L < 32 && (int64_t)P * (SC_NT / L) > SC_GKMAX) L <<= 1;
  if ((int64_t)P * (SC_NT / L) < K || (int64_t)P * (SC_NT / L) > SC_GKMAX) return false;
  const size_t smem = sc_part_bytes(PS, es) + sizeof(ScCtl);
  const size_t smem_max = (size_t)SC_PART_MAX + sizeof(ScCtl);
  // Per device: attributes set, and per cluster size whether such clusters fit (-1 unknown).
  static int attr_set[64] = {};
  static int fits[64][SC_MAXCL + 1];
  static bool fits_init = false;
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lock(g_cfg_mu);
    if (!fits_init) {
      for (auto& d : fits)
        for (int& f : d) f = -1;
      fits_init = true;
    }
    if (!attr_set[dev]) {
      err = cudaFuncSetAttribute(lss_shard_cluster_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem_max);
      if (err == cudaSuccess)
        err = cudaFuncSetAttribute(lss_shard_cluster_kernel<DT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (err != cudaSuccess) {
        cudaGetLastError();
        err = cudaSuccess;
        return false;
      }
      attr_set[dev] = 1;
    }
    if (fits[dev][P] < 0) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3((unsigned)(P * 64), 1, 1);
      cfg.blockDim = dim3(SC_NT, 1, 1);
      cfg.dynamicSmemBytes = smem_max;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = (unsigned)P;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int nc = 0;
      const cudaError_t e = cudaOccupancyMaxActiveClusters(&nc, lss_shard_cluster_kernel<DT>, &cfg);
      if (e != cudaSuccess) cudaGetLastError();
      fits[dev][P] = (e == cudaSuccess && nc > 0) ? 1 : 0;
    }
    if (!fits[dev][P]) return false;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(B * P), 1, 1);
  cfg.blockDim = dim3(SC_NT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)P;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, lss_shard_cluster_kernel<DT>, logits, stride, Vs, voff, T, K, PS, L, rec);
  return true;
}
}  // namespace lss

extern "C" {

int lss_shard_topk(const void* logits, int dtype, int B, int Vs, int64_t row_stride, int64_t vocab_offset,
                   const float* temperature, int K, void* records_out, void* stream) {
  if (B < 0 || Vs < 1 || row_stride < Vs || vocab_offset < 0 || K < 1 || K > LSS_SHARD_MAX_K)
    return LSS_ERR_INVALID_ARG;
  if (vocab_offset + Vs > 0x7fffffffLL) return LSS_ERR_UNSUPPORTED;
  if (dtype != LSS_DTYPE_F32 && dtype != LSS_DTYPE_BF16 && dtype != LSS_DTYPE_F16) return LSS_ERR_INVALID_ARG;
  if (B == 0) return LSS_OK;
  if (!logits || !temperature || !records_out || (reinterpret_cast<uintptr_t>(records_out) & 15) != 0)
    return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* rec = reinterpret_cast<unsigned char*>(records_out);
  {
    cudaError_t e = cudaSuccess;
    bool launched = false;
    switch (dtype) {
      case LSS_DTYPE_F32:
        launched = launch_shard_cluster<LSS_DTYPE_F32>(logits, row_stride, B, Vs, vocab_offset, temperature, K, rec, st, e);
        break;
      case LSS_DTYPE_BF16:
        launched = launch_shard_cluster<LSS_DTYPE_BF16>(logits, row_stride, B, Vs, vocab_offset, temperature, K, rec, st, e);
        break;
      default:
        launched = launch_shard_cluster<LSS_DTYPE_F16>(logits, row_stride, B, Vs, vocab_offset, temperature, K, rec, st, e);
        break;
    }
    if (launched) {
      if (e != cudaSuccess) {
        cudaGetLastError();
        return LSS_ERR_CUDA;
      }
      return LSS_OK;
    }
  }
  // Shard rows longer than 16 parts of 64 KB: one CTA per row, three passes.
  switch (dtype) {
    case LSS_DTYPE_F32:
      lss_shard_kernel<LSS_DTYPE_F32><<<B, NT, 0, st>>>(logits, row_stride, Vs, vocab_offset, temperature, K, rec);
      break;
    case LSS_DTYPE_BF16:
      lss_shard_kernel<LSS_DTYPE_BF16><<<B, NT, 0, st>>>(logits, row_stride, Vs, vocab_offset, temperature, K, rec);
      break;
    default:
      lss_shard_kernel<LSS_DTYPE_F16><<<B, NT, 0, st>>>(logits, row_stride, Vs, vocab_offset, temperature, K, rec);
      break;
  }
  if (cudaGetLastError() != cudaSuccess) return LSS_ERR_CUDA;
  return LSS_OK;
}

int lss_shard_merge(const void* records, int nshards, int B, int K, int V_total, const float* temperature,
                    const float* top_p, const float* uniforms, int32_t* tokens_out, uint8_t* kept_out,
                    float* probs_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (nshards < 1 || B < 0 || K < 1 || K > LSS_SHARD_MAX_K || V_total < 1) return LSS_ERR_INVALID_ARG;
  if ((int64_t)nshards * K > MERGE_CAP) return LSS_ERR_UNSUPPORTED;
  if (B == 0) return LSS_OK;
  if (!records || !temperature || !top_p || !uniforms || !tokens_out) return LSS_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < lss_shard_merge_workspace_bytes(B) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return LSS_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* ws = reinterpret_cast<unsigned char*>(workspace);
  if (cudaMemsetAsync(ws, 0, 256, st) != cudaSuccess) return LSS_ERR_CUDA;
  if (kept_out && cudaMemsetAsync(kept_out, 0, (size_t)B * V_total, st) != cudaSuccess) return LSS_ERR_CUDA;
  if (probs_out && cudaMemsetAsync(probs_out, 0, (size_t)B * V_total * sizeof(float), st) != cudaSuccess)
    return LSS_ERR_CUDA;
  RowArgs a{};
  a.B = B;
  a.V = V_total;
  a.temperature = temperature;
  a.top_p = top_p;
  a.uniforms = uniforms;
  a.tokens = tokens_out;
  a.kept_out = kept_out;
  a.probs_out = probs_out;
  a.err = reinterpret_cast<uint32_t*>(ws);
  a.counters = reinterpret_cast<uint32_t*>(ws);
  a.row_path = reinterpret_cast<int32_t*>(ws + 256);
  lss_merge_kernel<<<B, NT, 0, st>>>(reinterpret_cast<const unsigned char*>(records), nshards, B, K, a);
  if (cudaGetLastError() != cudaSuccess) return LSS_ERR_CUDA;
  return LSS_OK;
}

int lss_argmax(const void* logits, int dtype, int B, int V, int64_t row_stride, int32_t* tokens_out,
               void* stream) {
  if (B < 0 || V < 1 || row_stride < V) return LSS_ERR_INVALID_ARG;
  if (dtype != LSS_DTYPE_F32 && dtype != LSS_DTYPE_BF16 && dtype != LSS_DTYPE_F16) return LSS_ERR_INVALID_ARG;
  if (B == 0) return LSS_OK;
  if (!logits || !tokens_out) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (dtype) {
    case LSS_DTYPE_F32: e = launch_argmax_dt<LSS_DTYPE_F32>(logits, row_stride, B, V, tokens_out, st); break;
    case LSS_DTYPE_BF16: e = launch_argmax_dt<LSS_DTYPE_BF16>(logits, row_stride, B, V, tokens_out, st); break;
    default: e = launch_argmax_dt<LSS_DTYPE_F16>(logits, row_stride, B, V, tokens_out, st); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return LSS_ERR_CUDA;
  }
  return LSS_OK;
}

int lss_stop_check(const int32_t* tokens, int B, const int32_t* eos_ids, const int32_t* stop_offsets,
                   const int32_t* stop_ids, int32_t* out, void* stream) {
  if (B < 0) return LSS_ERR_INVALID_ARG;
  if (B == 0) return LSS_OK;
  if (!tokens || !out || (stop_offsets && !stop_ids)) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  constexpr int T = 256;
  lss_stop_kernel<<<(unsigned)((B + T - 1) / T), T, 0, st>>>(tokens, B, eos_ids, stop_offsets, stop_ids, out);
  if (cudaGetLastError() != cudaSuccess) return LSS_ERR_CUDA;
  return LSS_OK;
}

int lss_read_status(const void* workspace, uint32_t* flags_out, void* stream) {
  if (!workspace || !flags_out) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return LSS_ERR_CUDA;
  uint32_t f = 0;
  if (cudaMemcpy(&f, workspace, sizeof(f), cudaMemcpyDeviceToHost) != cudaSuccess) return LSS_ERR_CUDA;
  *flags_out = f;
  return f ? LSS_ERR_DEVICE : LSS_OK;
}

int lss_read_row_paths(const void* workspace, int B, int32_t* paths_out, void* stream) {
  if (!workspace || !paths_out || B < 0) return LSS_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return LSS_ERR_CUDA;
  const WsLayout L = ws_layout(B, 1, 0);
  if (B == 0) return LSS_OK;
  if (cudaMemcpy(paths_out, reinterpret_cast<const unsigned char*>(workspace) + L.row_path,
                 sizeof(int32_t) * (size_t)B, cudaMemcpyDeviceToHost) != cudaSuccess)
    return LSS_ERR_CUDA;
  return LSS_OK;
}

}  // extern "C"
