/*
 * lsampler.h — C ABI of the B200 (sm_100a) batched token sampler.
 *
 * The reference, LocalStrm, samples one row at a time in Python:
 *   sample_next_token(logits, params, past_token_ids) -> int      (src/engine/sampling.py:118-163)
 * with its pieces apply_repetition_penalties (sampling.py:38-68) and
 * apply_top_k_top_p_min_p (sampling.py:71-115), and an all-greedy batched seam
 *   torch.argmax(batched_logits, dim=-1)                           (src/engine/llm_engine.py:1139-1141).
 * The reference has no native code and no FFI; the entry points below are what its
 * engine loop (llm_engine.py:1129-1153) would bind, through ctypes, to replace that
 * per-row loop with one [B, V] call.  localstrm_b200/sampling.py is that binding.
 *
 * Conventions
 *  - Every pointer named "device" is CUDA device memory; "stream" is a cudaStream_t
 *    passed as void*.  Calls are stream-ordered and asynchronous; nothing here
 *    synchronises the device except lss_read_status().
 *  - Every function returns an int status (LSS_OK == 0); nothing aborts the process
 *    and nothing throws across the ABI.  lss_status_string() names a status.
 *  - Logits are read-only (the reference clones before mutating, sampling.py:129).
 *    Values arrive as f32, bf16 or f16 and are widened to f32 on load; all arithmetic
 *    is f32 with IEEE rounding, accumulations in f64 or 2^-40 fixed point.
 *  - Per-row parameters are structure-of-arrays device vectors of length B, with the
 *    reference's meaning (SamplingParams, sampling.py:20-35): temperature <= 0 is
 *    greedy on the raw logits (penalties ignored); top_k <= 0 disables top-k;
 *    top_p outside (0,1) disables top-p; min_p outside (0,1) disables min-p;
 *    repetition_penalty == 1 and frequency == presence == 0 disable penalties.
 *  - Histories are CSR: hist_offsets[B+1] (int32, device, non-decreasing, within
 *    [0, hist_total]) into hist_ids (int32, device, hist_total values in [0, V)).
 *    hist_offsets may be NULL when hist_total == 0.  The kernels check every row's offsets
 *    and ids and raise LSS_FLAG_BAD_HISTORY instead of reading outside the arrays.
 *  - uniforms[B] (device, f32 in [0,1)) drive the draw: the token is the first
 *    vocabulary index whose running probability mass exceeds u * total, over the
 *    kept tokens in index order (inverse CDF).  The reference uses
 *    torch.multinomial on its global generator instead (sampling.py:162).
 */
#ifndef LSAMPLER_H
#define LSAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LSS_OK 0
#define LSS_ERR_INVALID_ARG 1   /* a size, pointer or dtype is out of the supported domain */
#define LSS_ERR_WORKSPACE 2     /* workspace pointer NULL or smaller than lss_workspace_bytes() */
#define LSS_ERR_CUDA 3          /* a CUDA runtime call failed (launch or attribute) */
#define LSS_ERR_UNSUPPORTED 4   /* V larger than the largest supported row, or no sm_100 device */
#define LSS_ERR_DEVICE 5        /* lss_read_status: the device reported an error flag */
#define LSS_ERR_SCRATCH_LIMIT 6 /* lss_sample_noalloc: the call needs more than its fixed scratch */

#define LSS_DTYPE_F32 0
#define LSS_DTYPE_BF16 1
#define LSS_DTYPE_F16 2

/* Device-side error flags (lss_read_status). */
#define LSS_FLAG_TMA_TIMEOUT 0x1u     /* a bounded wait for a bulk copy gave up */
#define LSS_FLAG_BAD_HISTORY 0x2u     /* a history id outside [0, V) was ignored, or a row's CSR
                                         offsets lay outside [0, hist_total] or decreased (that
                                         row's history was ignored; rows whose ranges overlap
                                         give unreliable tokens, but nothing is read or written
                                         out of bounds) */
#define LSS_FLAG_INTERNAL 0x4u        /* an internal capacity check failed (result unreliable) */

/* Per-row path codes written to the workspace (lss_read_row_paths). */
#define LSS_PATH_GREEDY 1     /* temperature <= 0: argmax of the raw row */
#define LSS_PATH_SPECIAL 2    /* NaN, +inf or all -inf after scaling: NaN-guard argmax */
#define LSS_PATH_GATHER 3     /* survivors gathered into one CTA and resolved there */
#define LSS_PATH_DENSE 4      /* cluster-wide radix select over the whole row */
#define LSS_PATH_SLOW_GATHER 5 /* survivors gathered and resolved by the second kernel */

/* Library version, (major << 16) | (minor << 8) | patch. */
int lss_version(void);

/* Human-readable name of a status code.  Never NULL. */
const char* lss_status_string(int status);

/* Largest vocabulary size one row may have (fits the shared memory of one cluster). */
int lss_max_vocab(void);

/* Bytes of device workspace that lss_sample needs for B rows, V columns and hist_total
 * history ids in total.  Replaces the per-call torch allocations of the reference
 * (torch.unique / sort / cumsum temporaries, sampling.py:52,98-99). */
size_t lss_workspace_bytes(int B, int V, int64_t hist_total);

/* Batched sampler: one token per row.  Replaces the engine's per-row calls of
 * sample_next_token (llm_engine.py:1145-1153, sampling.py:118-163).
 *   logits      device, [B rows] x [row_stride elements], dtype per LSS_DTYPE_*
 *   tokens_out  device int32 [B]
 *   kept_out    device uint8 [B*V] or NULL: 1 where a token survives the filters
 *   probs_out   device f32  [B*V] or NULL: the final probabilities (0 elsewhere)
 * kept_out / probs_out are the parity view of apply_top_k_top_p_min_p + softmax
 * (sampling.py:149-157); they are zeroed and written only when non-NULL.
 * workspace   device, >= lss_workspace_bytes(B, V, hist_total), 256-byte aligned. */
int lss_sample(const void* logits, int dtype, int B, int V, int64_t row_stride,
               const float* temperature, const int32_t* top_k, const float* top_p,
               const float* min_p, const float* repetition_penalty,
               const float* frequency_penalty, const float* presence_penalty,
               const int32_t* hist_offsets, const int32_t* hist_ids, int64_t hist_total,
               const float* uniforms, int32_t* tokens_out, uint8_t* kept_out,
               float* probs_out, void* workspace, size_t workspace_bytes, void* stream);

/* The two stages of lss_sample, for callers that overlap or time them separately.
 * lss_sample_prepare validates the arguments and clears the workspace status (error flags
 * and the deferred-row count); it must precede lss_sample_rows on the same stream.
 * lss_sample_rows runs the kernels: a streaming pass over the logits (history penalties,
 * sampling.py:52-66, per-slice maxima and candidates), a per-row resolve (temperature,
 * filters, draw) and a second kernel for the rows that need the whole vocabulary.
 * Arguments mean what they mean in lss_sample. */
int lss_sample_prepare(int B, int V, const float* temperature, const int32_t* top_k,
                       const float* min_p, const float* repetition_penalty,
                       const float* frequency_penalty, const float* presence_penalty,
                       const int32_t* hist_offsets, const int32_t* hist_ids, int64_t hist_total,
                       void* workspace, size_t workspace_bytes, void* stream);
int lss_sample_rows(const void* logits, int dtype, int B, int V, int64_t row_stride,
                    const float* temperature, const int32_t* top_k, const float* top_p,
                    const float* min_p, const float* repetition_penalty,
                    const float* frequency_penalty, const float* presence_penalty,
                    const int32_t* hist_offsets, const int32_t* hist_ids, int64_t hist_total,
                    const float* uniforms, int32_t* tokens_out, uint8_t* kept_out,
                    float* probs_out, void* workspace, size_t workspace_bytes, void* stream);

/* Profiling entry point: only the streaming pass of lss_sample_rows (K1: penalties, slice
 * maxima and candidates into the workspace), without the per-row resolve.  It leaves no
 * tokens; it exists so that the pass can be timed on its own.  Arguments as lss_sample_rows.
 * No counterpart in the reference. */
int lss_scan_pass(const void* logits, int dtype, int B, int V, int64_t row_stride,
                  const float* temperature, const int32_t* top_k, const float* top_p,
                  const float* min_p, const float* repetition_penalty,
                  const float* frequency_penalty, const float* presence_penalty,
                  const int32_t* hist_offsets, const int32_t* hist_ids, int64_t hist_total,
                  const float* uniforms, int32_t* tokens_out, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Vocabulary-sharded sampling: each GPU holds columns [vocab_offset, vocab_offset + Vs) of
 * every row (the reference runs one device per row; this is a mode of its own).  Step 1,
 * lss_shard_topk, writes one record per row of the shard: the shard's K largest values of
 * y = z / T as codes (key(y) << 32 | ~global index, value descending, index ascending), then
 * the shard's max of y, the sum of exp(y - max), flags and the number of codes.  The caller
 * gathers the records of all shards shard-major ([nshards][B] records, e.g. one NCCL
 * all-gather) and runs step 2, lss_shard_merge: the reference's top-k with k = K (ties
 * kept), top-p, renormalisation and the inverse-CDF draw over the union of the shards'
 * candidates, which holds the row's K largest.  Penalties and min-p are not applied in this
 * mode.  records_out must be 16-byte aligned; the merge workspace holds the status word
 * (lss_read_status) and the row paths (lss_read_row_paths). */
#define LSS_SHARD_MAX_K 256
size_t lss_shard_record_bytes(int K);
size_t lss_shard_merge_workspace_bytes(int B);
int lss_shard_topk(const void* logits, int dtype, int B, int Vs, int64_t row_stride,
                   int64_t vocab_offset, const float* temperature, int K, void* records_out,
                   void* stream);
int lss_shard_merge(const void* records, int nshards, int B, int K, int V_total,
                    const float* temperature, const float* top_p, const float* uniforms,
                    int32_t* tokens_out, uint8_t* kept_out, float* probs_out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Batched greedy argmax (NaN counts as largest, lowest index wins ties), the
 * all-greedy seam of the engine (llm_engine.py:1139-1141; torch.argmax semantics). */
int lss_argmax(const void* logits, int dtype, int B, int V, int64_t row_stride,
               int32_t* tokens_out, void* stream);

/* lss_sample without a caller-provided workspace; it allocates nothing.
 * No counterpart in the reference: LocalStrm allocates through PyTorch on every call.
 * It exists for callers that must not allocate device memory while they sample: a serving
 * engine that reserved nearly all of the GPU for its paged KV cache at start-up (as
 * LocalStrm's block pool and VRAM preflight do) cannot count on cudaMalloc succeeding in
 * the middle of a decode step, and a cudaMalloc/cudaFree there can also synchronise the
 * device and stall the other streams.
 * Its scratch is one file-scope device array of LSS_NOALLOC_SCRATCH_BYTES (32 MiB) that
 * every GPU which loads this library holds until the process exits.  A call whose
 * lss_workspace_bytes(B, V, hist_total) exceeds that returns LSS_ERR_SCRATCH_LIMIT and
 * launches nothing (256 rows with 2,048-id histories fit).  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture.  All calls on a device share the one
 * array: two calls that overlap on the GPU (different streams, no ordering between them)
 * race on it and give wrong tokens; serialise them.  Everything that must start at zero
 * is cleared by the call itself.  The looked-up address is kept for the life of the process:
 * after cudaDeviceReset on a device (which unloads this library's device code there) do not
 * call lss_sample_noalloc on that device again.  lss_read_status / lss_read_row_paths take a
 * caller workspace and do not apply; lss_noalloc_read_status reads this call's flags. */
#define LSS_NOALLOC_SCRATCH_BYTES (32u << 20)
int lss_sample_noalloc(const void* logits, int dtype, int B, int V, int64_t row_stride,
                       const float* temperature, const int32_t* top_k, const float* top_p,
                       const float* min_p, const float* repetition_penalty,
                       const float* frequency_penalty, const float* presence_penalty,
                       const int32_t* hist_offsets, const int32_t* hist_ids,
                       int64_t hist_total, const float* uniforms, int32_t* tokens_out,
                       uint8_t* kept_out, float* probs_out, void* stream);

/* Device error flags (LSS_FLAG_*) of the last lss_sample_noalloc call on the current device:
 * synchronises `stream`, then reads the status word of the fixed scratch, as lss_read_status
 * does for a caller workspace.  LSS_ERR_DEVICE when a flag is set (the tokens of that call are
 * then unreliable), LSS_OK otherwise.  No counterpart in the reference.  Allocates nothing. */
int lss_noalloc_read_status(uint32_t* flags_out, void* stream);

/* Token-id part of check_stop_criteria (sampling.py:166-196), batched and on the device, so
 * that a decode loop learns which rows stopped without reading every token back:
 *   out[b] = LSS_STOP_EOS    when tokens[b] == eos_ids[b] (eos_ids[b] < 0: no EOS id),
 *            LSS_STOP_TOKEN  else when tokens[b] is one of stop_ids[stop_offsets[b] ..
 *                            stop_offsets[b+1]),
 *            LSS_STOP_NONE   otherwise.
 * The reference checks the EOS id first, then the stop ids (sampling.py:182-185).  The
 * stop-string part (:188-194) needs the tokenizer and stays on the host.  eos_ids may be NULL
 * (no EOS ids); stop_offsets NULL means no stop ids (stop_ids is then ignored).  All pointers
 * are device pointers; asynchronous on `stream`. */
#define LSS_STOP_NONE 0
#define LSS_STOP_EOS 1
#define LSS_STOP_TOKEN 2
int lss_stop_check(const int32_t* tokens, int B, const int32_t* eos_ids, const int32_t* stop_offsets,
                   const int32_t* stop_ids, int32_t* out, void* stream);

/* Synchronises `stream`, then returns the device error flags accumulated in the
 * workspace since lss_sample last cleared them (0 when none). */
int lss_read_status(const void* workspace, uint32_t* flags_out, void* stream);

/* Synchronises `stream`, then copies the per-row path codes (LSS_PATH_*) of the last
 * lss_sample on this workspace into host memory paths_out[B]. */
int lss_read_row_paths(const void* workspace, int B, int32_t* paths_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LSAMPLER_H */
