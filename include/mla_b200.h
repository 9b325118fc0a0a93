/*
 * mla_b200.h -- C ABI of the B200 (sm_100a) MLA decode engine.
 *
 * Computes the weight-absorbed DeepSeek-V2 decode step
 *
 *     O*[b, h, :] = softmax(scale * Q*[b, h, :] . C_b^T) . C_b[:, :512]
 *
 * over a 576-wide latent cache C_b ([N_b, 576]: 512 latent + 64 rope columns).
 *
 * Conventions (all entry points):
 *   - Every pointer is a DEVICE pointer unless its comment says "host".
 *   - All tensors are dense row-major; the caller owns every buffer, including
 *     the workspace (query its size with mla_b200_workspace_size()).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Launches are
 *     asynchronous on that stream; nothing synchronizes the device.
 *   - Return value: MLA_B200_OK or an mla_b200_status code.  Nothing prints,
 *     aborts or traps.  Argument errors are detected before any launch.
 *   - Thread safety: calls may come from several host threads; concurrent
 *     calls must use distinct workspaces.
 *
 * Each entry point names the reference interface it replaces (lechebs/ada-mla,
 * path:line).  The reference's launchers return void, print CUDA errors and use
 * the legacy default stream; these return a status and take a stream.
 */
#ifndef MLA_B200_H
#define MLA_B200_H

#include <stddef.h>
#include <stdint.h>

/* Only these entry points are exported: the library is built with hidden
 * default visibility, so its kernels and its static CUDA runtime never clash
 * with another library's in the same process. */
#if defined(__GNUC__)
#define MLA_B200_API __attribute__((visibility("default")))
#else
#define MLA_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Model constants the reference hard-codes in Python (mla.py:29-34, with the
 * TODO "should be exported by the C++ module") and in KernelTraits
 * (csrc/mla_decode_splitk_fwd.cuh:37-59). */
#define MLA_B200_NUM_HEADS 128 /* reference default head count */
#define MLA_B200_HEAD_DIM 128  /* nope head dim of the un-absorbed model */
#define MLA_B200_HEAD_DIM_C 512 /* latent (value) width = HEAD_DIM_V */
#define MLA_B200_HEAD_DIM_ROPE 64
#define MLA_B200_HEAD_DIM_K 576 /* HEAD_DIM_C + HEAD_DIM_ROPE */
#define MLA_B200_HEAD_DIM_V 512

typedef enum {
    MLA_B200_OK = 0,
    MLA_B200_ERR_INVALID_ARG = 1,   /* bad pointer / shape / alignment */
    MLA_B200_ERR_UNSUPPORTED = 2,   /* shape valid but not implemented */
    MLA_B200_ERR_WORKSPACE = 3,     /* workspace missing or too small */
    MLA_B200_ERR_CUDA = 4,          /* a CUDA runtime call failed */
    MLA_B200_ERR_DEVICE_TIMEOUT = 5, /* a kernel's bounded wait expired */
    MLA_B200_ERR_NO_DEVICE = 6      /* no sm_100 device current */
} mla_b200_status;

/* Output element type for entry points that can emit either. */
typedef enum { MLA_B200_OUT_F16 = 0, MLA_B200_OUT_F32 = 1, MLA_B200_OUT_BF16 = 2 } mla_b200_out_dtype;

/* Human-readable name of a status code (static string). */
MLA_B200_API const char *mla_b200_status_string(int status);

/* Library version, e.g. "0.1.0". */
MLA_B200_API const char *mla_b200_version(void);

/* Value of a model constant by name ("NUM_HEADS", "HEAD_DIM", "HEAD_DIM_C",
 * "HEAD_DIM_ROPE", "HEAD_DIM_K", "HEAD_DIM_V"); -1 for an unknown name.
 * Retires the reference TODO at mla.py:29. */
MLA_B200_API int mla_b200_constant(const char *name);

/* Properties of the current device as the library sees them: SM count and
 * how many 2-CTA clusters of the tensor-core decode kernel can be resident at
 * once (one wave of work items).  Either pointer may be NULL. */
MLA_B200_API int mla_b200_device_info(int *num_sms, int *decode_clusters);

/* Kernel timing hook for benchmarks (no reference counterpart; the reference
 * is timed from Python with triton.testing.do_bench around the whole call).
 * While set on the calling host thread, every decode entry point records
 * `ev_start` immediately before and `ev_stop` immediately after the launch of
 * its main decode kernel, on the stream it launches on (the split-merge and
 * planning kernels fall outside).  During stream capture the records become
 * event-record nodes of the graph, so the kernel can be timed at replay.
 * Both are cudaEvent_t handles created by the caller; pass NULL, NULL to turn
 * the hook off. */
MLA_B200_API int mla_b200_set_kernel_timing(void *ev_start, void *ev_stop);

/* Device-side span of the main tensor-core decode kernel (no reference
 * counterpart).  While set on the calling host thread, the k-th later launch
 * of that kernel (k counting from 0, wrapping after `slots`) records, in
 * span[2k] and span[2k+1], the %globaltimer (ns) at which its first CTA
 * starts work (after its set-up and the wait for the preceding kernel; atomic
 * min) and at which its last CTA ends (atomic max); the caller initialises
 * each pair to {UINT64_MAX, 0} before the launch runs.  The span excludes the
 * launch latency that an event pair around the launch includes.  `span` is a
 * device array of 2 * slots uint64; NULL (or slots <= 0) turns it off.  Under
 * stream capture the pointer is baked into each captured launch. */
MLA_B200_API int mla_b200_set_kernel_span(unsigned long long *span, int slots);

/* ------------------------------------------------------------------------ */
/* Planning                                                                  */
/* ------------------------------------------------------------------------ */

/* Split-count heuristic.  Replaces the constant `num_splits = 4`
 * (csrc/mla_api.cpp:97).  Given `batch` sequences holding `total_tokens`
 * cache rows in all and `num_heads` heads, chooses how many tokens one split
 * (one work item) covers so that the items fill `num_sms` SMs (0 = the current
 * device's count) while keeping the split-partial traffic small.  Writes the
 * chunk length (a multiple of 96 tokens, the kernel's tile) to *chunk_tokens and, for a single
 * sequence, the resulting split count to *num_splits (either may be NULL).
 *
 * This is the schedule of an automatic split of one sequence.  For a batch
 * of several sequences on the fp16 tensor-core path the decode entry points
 * balance the work instead: the batch's 96-row tiles plus a fixed cost per
 * work item are divided evenly among the resident clusters, a sequence being
 * split only where a cluster's share ends; *chunk_tokens is then that share
 * (in tokens, capped at the longest sequence). */
MLA_B200_API int mla_b200_plan(int batch, int num_heads, long long total_tokens, int max_seq_len,
                               int num_sms, int *chunk_tokens, int *num_splits);

/* Bytes of workspace the f16/f32 decode entry points need for this problem
 * (split partials, the work table and the varlen schedule).  `num_splits` <= 0
 * means "as chosen by mla_b200_plan".  For a single sequence pass batch = 1
 * and total_tokens = seq_length. */
MLA_B200_API size_t mla_b200_workspace_size(int batch, int num_heads, long long total_tokens,
                                            int max_seq_len, int num_splits);

/* ------------------------------------------------------------------------ */
/* Decode entry points                                                       */
/* ------------------------------------------------------------------------ */

/* fp16 split-KV decode of ONE sequence, reference semantics.
 * Replaces run_mla_decode_splitk<at::Half> (csrc/mla_decode.hpp:25-34,
 * csrc/mla_decode_splitk_fwd_sm89.cu:26-47 -> mla_decode_splitk_fwd.cuh:941-985).
 *   query [num_heads, 576] fp16, cache [seq_length, 576] fp16,
 *   out   [num_heads, 512] fp16.
 * Softmax scale is the reference's 1/sqrt(HEAD_DIM + HEAD_DIM_ROPE) = 1/sqrt(192)
 * (csrc/mla_decode_splitk_fwd.cuh:446-450).  num_splits <= 0 selects the
 * heuristic; otherwise the sequence is cut into that many splits (tail masked,
 * no multiple-of-64 requirement).  seq_length == 0 yields zeros.  Softmax
 * state is fp32 (the reference keeps it in fp16). */
MLA_B200_API int mla_b200_decode_split_f16(const void *query, const void *cache, void *out,
                                           int num_heads, int seq_length, int num_splits,
                                           void *workspace, size_t workspace_bytes, void *stream);

/* Batched / variable-length fp16 decode (no reference counterpart: the
 * reference has no batch dimension).
 *   query [batch, num_heads, 576] fp16
 *   cache packed [total_tokens, 576] fp16; sequence b owns rows
 *         cu_seqlens[b] .. cu_seqlens[b+1]-1 (cu_seqlens: DEVICE int32 [batch+1],
 *         cu_seqlens[0] = 0, cu_seqlens[batch] = total_tokens), or
 *         cu_seqlens == NULL for a dense [batch, max_seq_len, 576] cache
 *         (then total_tokens must equal batch * max_seq_len).
 *   max_seq_len >= every N_b (used for planning only).
 *   out [batch, num_heads, 512], fp16 or fp32 per out_dtype.
 *   out_lse: optional [batch, num_heads] fp32 natural-log log-sum-exp of the
 *         scaled logits (-inf for an empty sequence); NULL to skip.
 * softmax_scale multiplies Q.C^T (pass 1.0 when the scale is folded into Q). */
MLA_B200_API int mla_b200_decode_batched_f16(const void *query, const void *cache,
                                             const int32_t *cu_seqlens, int batch, int num_heads,
                                             long long total_tokens, int max_seq_len,
                                             float softmax_scale, int num_splits,
                                             void *out, int out_dtype, float *out_lse,
                                             void *workspace, size_t workspace_bytes, void *stream);

/* Batched / variable-length bf16 decode: the same contract as
 * mla_b200_decode_batched_f16 with query and cache in bf16 (no reference
 * counterpart; the reference lists bf16 as future work, README.md:407).  out is
 * bf16 (MLA_B200_OUT_BF16) or fp32 (MLA_B200_OUT_F32); P enters the second
 * GEMM as bf16, accumulation and softmax state are fp32.  num_heads <= 128. */
MLA_B200_API int mla_b200_decode_batched_bf16(const void *query, const void *cache,
                                              const int32_t *cu_seqlens, int batch, int num_heads,
                                              long long total_tokens, int max_seq_len,
                                              float softmax_scale, int num_splits,
                                              void *out, int out_dtype, float *out_lse,
                                              void *workspace, size_t workspace_bytes, void *stream);

/* Paged latent cache (no counterpart in the reference, whose cache is one
 * contiguous [N, 576] tensor, csrc/mla_api.cpp:20).  The cache is a page pool
 * kv_pages [num_pages, page_size, 576] (fp16 for _f16, bf16 for _bf16); token t
 * of sequence b is row t % page_size of page block_table[b * max_blocks_per_seq
 * + t / page_size].  block_table int32 [batch, max_blocks_per_seq] and seq_lens
 * int32 [batch] are device arrays.  page_size is a multiple of 32 (64 and 128
 * are the usual sizes); max_seq_len bounds every seq_lens[b] (longer lengths
 * are clamped to it) and max_seq_len <= max_blocks_per_seq * page_size.  Page
 * rows past a sequence's end may hold any bits (NaN included): they are never
 * part of the result.  A page index outside [0, num_pages) reads zeros.
 * Workspace: mla_b200_workspace_size(batch, num_heads, batch * max_seq_len,
 * max_seq_len, num_splits).  Otherwise the contract of
 * mla_b200_decode_batched_f16 / _bf16 (out_dtype F16 or F32 for _f16, BF16 or
 * F32 for _bf16); num_heads <= 128. */
MLA_B200_API int mla_b200_decode_paged_f16(const void *query, const void *kv_pages,
                                           const int32_t *block_table, const int32_t *seq_lens,
                                           int batch, int num_heads, int num_pages, int page_size,
                                           int max_blocks_per_seq, int max_seq_len,
                                           float softmax_scale, int num_splits, void *out,
                                           int out_dtype, float *out_lse, void *workspace,
                                           size_t workspace_bytes, void *stream);
MLA_B200_API int mla_b200_decode_paged_bf16(const void *query, const void *kv_pages,
                                            const int32_t *block_table, const int32_t *seq_lens,
                                            int batch, int num_heads, int num_pages, int page_size,
                                            int max_blocks_per_seq, int max_seq_len,
                                            float softmax_scale, int num_splits, void *out,
                                            int out_dtype, float *out_lse, void *workspace,
                                            size_t workspace_bytes, void *stream);

/* Multi-token decode (speculative / MTP drafts; no counterpart in the
 * reference): every sequence carries num_tokens queries, query [batch,
 * num_tokens, num_heads, 576], whose own latent rows are the last num_tokens
 * rows of the sequence's cache; draft token i sees the sequence's first
 * len - (num_tokens - 1 - i) tokens (len >= num_tokens).  num_heads <= 128.
 * When num_tokens * num_heads <= 128 the drafts share every cache tile (rows
 * token * num_heads + head fill one 128-row MMA tile: one pass over the
 * cache).  Above that (e.g. 128 heads) each draft token is decoded as its own
 * sequence of num_heads rows over the same cache rows, scheduled next to the
 * sequence's other drafts so their repeated tile reads come from L2.
 * out [batch, num_tokens, num_heads, 512], out_lse [batch, num_tokens,
 * num_heads] or NULL; otherwise the contract of mla_b200_decode_batched_f16 /
 * _bf16.  Workspace: mla_b200_workspace_size_mtp. */
MLA_B200_API size_t mla_b200_workspace_size_mtp(int batch, int num_tokens, int num_heads,
                                                long long total_tokens, int max_seq_len,
                                                int num_splits);
MLA_B200_API int mla_b200_decode_mtp_f16(const void *query, const void *cache,
                                         const int32_t *cu_seqlens, int batch, int num_tokens,
                                         int num_heads, long long total_tokens, int max_seq_len,
                                         float softmax_scale, int num_splits, void *out,
                                         int out_dtype, float *out_lse, void *workspace,
                                         size_t workspace_bytes, void *stream);
MLA_B200_API int mla_b200_decode_mtp_bf16(const void *query, const void *cache,
                                          const int32_t *cu_seqlens, int batch, int num_tokens,
                                          int num_heads, long long total_tokens, int max_seq_len,
                                          float softmax_scale, int num_splits, void *out,
                                          int out_dtype, float *out_lse, void *workspace,
                                          size_t workspace_bytes, void *stream);

/* FP8 latent cache (no counterpart in the reference, which lists fp8 as future
 * work, README.md:407-408).  cache is e4m3 (OCP FP8, bias 7, no infinities)
 * with the layout of mla_b200_decode_batched_f16's cache (dense or packed) and
 * one per-tensor scale: C = cache * kv_scale.  query is fp16.  GEMM1 runs on
 * the fp8 tensor-core path with Q* split into two e4m3 planes (hi + lo, per-row
 * power-of-two scaling); GEMM2 too, with P split into e4m3 hi + lo planes by
 * the softmax; accumulation and softmax state are fp32.  out_dtype MLA_B200_OUT_F16 or MLA_B200_OUT_F32;
 * num_heads <= 128.  Workspace: mla_b200_workspace_size_fp8 (it adds the
 * e4m3 Q* planes, 2 x batch x num_heads x 576 bytes). */
/* The same with one dequantisation scale per cache row instead of one per
 * tensor: C[t] = cache[t] * kv_scales[t], kv_scales [total_tokens] fp32 on the
 * device, indexed like the cache rows (a per-page or per-tile scale is that
 * value repeated over the block's rows); scales must be positive normal
 * floats.  A scale multiplies its column's logit, and its power of two joins the
 * online softmax's exponent; within one 96-row tile the P weights of rows with
 * small scales sit lower by the tile's scale spread, so scales that span more
 * than ~2^5 inside a tile lose P precision (e4m3 subnormals).  Workspace:
 * mla_b200_workspace_size_fp8. */
MLA_B200_API int mla_b200_decode_batched_fp8_scaled(const void *query, const void *cache,
                                                   const float *kv_scales, const int32_t *cu_seqlens,
                                                   int batch, int num_heads, long long total_tokens,
                                                   int max_seq_len, float softmax_scale, int num_splits,
                                                   void *out, int out_dtype, float *out_lse,
                                                   void *workspace, size_t workspace_bytes, void *stream);
MLA_B200_API size_t mla_b200_workspace_size_fp8(int batch, int num_heads, long long total_tokens,
                                                int max_seq_len, int num_splits);
MLA_B200_API int mla_b200_decode_batched_fp8(const void *query, const void *cache, float kv_scale,
                                             const int32_t *cu_seqlens, int batch, int num_heads,
                                             long long total_tokens, int max_seq_len,
                                             float softmax_scale, int num_splits, void *out,
                                             int out_dtype, float *out_lse, void *workspace,
                                             size_t workspace_bytes, void *stream);

/* fp32 fused decode of ONE sequence, reference semantics (scale 1/sqrt(192),
 * 512 output columns).  Replaces run_mla_decode_fused (csrc/mla_decode.hpp:18-23,
 * csrc/mla_decode_fused_fwd_sm89.cu:6-60).  head_dim_c must be 576. */
MLA_B200_API int mla_b200_decode_fused_f32(const float *query, const float *cache, float *out,
                                           int num_heads, int head_dim_c, int seq_length,
                                           void *workspace, size_t workspace_bytes, void *stream);

/* fp32 naive 3-kernel decode, reference semantics: scale 1/sqrt(head_dim_c),
 * ALL head_dim_c output columns, attention matrix materialized in `attn`
 * ([num_heads, seq_length] fp32, caller-owned scratch).  Replaces
 * run_mla_decode_naive (csrc/mla_decode.hpp:10-16, csrc/mla_decode_naive_fwd.cu:4-31).
 * Any head_dim_c >= 1; seq_length >= 1. */
MLA_B200_API int mla_b200_decode_naive_f32(const float *query, const float *cache, float *attn,
                                           float *out, int num_heads, int head_dim_c,
                                           int seq_length, void *stream);

/* Allocation-free variant of mla_b200_decode_split_f16 (no counterpart in the
 * reference, whose launcher always allocates its split buffers with at::empty).
 *
 * Some callers cannot allocate device memory at decode time: a host program
 * that reaches the library through a thin FFI (ctypes, cgo, JNI) with no CUDA
 * allocator of its own, or a serving process whose memory pool has already
 * reserved the whole GPU for its KV cache, where a cudaMalloc would fail or
 * stall.  This entry point takes only the query, the cache and the output; its
 * split scratch lives in a static device array of MLA_B200_NOALLOC_SCRATCH_BYTES
 * inside this library, which every GPU that loads the library keeps until the
 * process exits.  It calls no cudaMalloc, cudaFree or allocating library routine.
 *
 *   - Same inputs, output and semantics as mla_b200_decode_split_f16.
 *   - num_splits <= 0: the split heuristic, reduced until the partials fit the
 *     scratch.  An explicit num_splits whose partials do not fit is rejected
 *     with MLA_B200_ERR_WORKSPACE before anything is launched.
 *   - The first call on each device looks up the scratch array's device
 *     address (cudaGetSymbolAddress) with that device current; make that first
 *     call before any stream capture.
 *   - All calls share the one scratch array.  Nothing in it must start at
 *     zero (each call writes every partial it reads), but calls that overlap on
 *     the GPU -- on different streams, or from different host threads -- race
 *     on it: serialize them. */
#define MLA_B200_NOALLOC_SCRATCH_BYTES (8u << 20)
MLA_B200_API int mla_b200_decode_split_f16_noalloc(const void *query, const void *cache, void *out,
                                                   int num_heads, int seq_length, int num_splits,
                                                   void *stream);

/* ------------------------------------------------------------------------ */
/* The per-head projections on either side of the decode                     */
/* ------------------------------------------------------------------------ */

/* Q absorption (no kernel counterpart in the reference, whose README.md:74-110
 * derives it and leaves it to the caller):
 *   q_star[b, h, 0:512]   = q_nope[b, h, :] . w_uk[h]     (fp32 accumulate)
 *   q_star[b, h, 512:576] = q_rope[b, h, :]
 * q_nope [batch, num_heads, head_dim], q_rope [batch, num_heads, 64],
 * w_uk [num_heads, head_dim, 512], q_star [batch, num_heads, 576], all fp16
 * (_f16) or all bf16 (_bf16), 16-byte aligned; head_dim a multiple of 64.
 * A tcgen05 kernel streams every weight byte from HBM once (swap-AB: weights on
 * the MMA's M side, the batch on N).  It signals programmatic launch
 * completion early, so a decode launched after it may overlap its set-up. */
MLA_B200_API int mla_b200_absorb_q_f16(const void *q_nope, const void *q_rope, const void *w_uk,
                                       void *q_star, int batch, int num_heads, int head_dim,
                                       void *stream);
MLA_B200_API int mla_b200_absorb_q_bf16(const void *q_nope, const void *q_rope, const void *w_uk,
                                        void *q_star, int batch, int num_heads, int head_dim,
                                        void *stream);

/* Per-head value projection of O* (no reference counterpart):
 *   out[b, h, :] = o_star[b, h, :] . w_uv[h]
 * o_star [batch, num_heads, 512], w_uv [num_heads, 512, head_dim_v],
 * out [batch, num_heads, head_dim_v]; fp16 or bf16 throughout; head_dim_v a
 * multiple of 128.  Same kernel as mla_b200_absorb_q_*. */
MLA_B200_API int mla_b200_project_o_f16(const void *o_star, const void *w_uv, void *out, int batch,
                                        int num_heads, int head_dim_v, void *stream);
MLA_B200_API int mla_b200_project_o_bf16(const void *o_star, const void *w_uv, void *out, int batch,
                                         int num_heads, int head_dim_v, void *stream);

/* ------------------------------------------------------------------------ */
/* Log-sum-exp merge of partial results                                      */
/* ------------------------------------------------------------------------ */

/* Merges `num_parts` partial decodes of the same queries over disjoint KV
 * slices (e.g. one per GPU after an all-gather):
 *   part_o   [num_parts, rows, 512] fp32, each normalized by its own sum
 *   part_lse [num_parts, rows] fp32 natural-log LSE (-inf = empty slice)
 *   out      [rows, 512] fp16 or fp32 (out_dtype); out_lse [rows] or NULL.
 * rows = batch * num_heads.  Rows whose slices are all empty yield zeros.
 * Generalises the reference's mla_decode_combine
 * (csrc/mla_decode_splitk_fwd.cuh:894-939) to any part count and layout. */
MLA_B200_API int mla_b200_combine_f32(const float *part_o, const float *part_lse, int num_parts,
                                      long long rows, void *out, int out_dtype, float *out_lse,
                                      void *stream);

/* The same merge read from a packed exchange buffer, the layout one
 * all-gather of every rank's (O, LSE) produces: part g occupies floats
 * [g * part_stride, (g + 1) * part_stride) of `parts`, its O [rows, 512] fp32
 * first and its LSE [rows] fp32 right after (at g * part_stride + rows * 512).
 * part_stride >= rows * 513 and a multiple of 4 (each part's O 16-byte
 * aligned).  Saves the unpacking copies of a split-KV multi-GPU step
 * (no reference counterpart: the reference runs on one GPU). */
MLA_B200_API int mla_b200_combine_packed_f32(const float *parts, int num_parts, long long rows,
                                             long long part_stride, void *out, int out_dtype,
                                             float *out_lse, void *stream);

/* ------------------------------------------------------------------------ */
/* Cross-GPU exchange over NVLink peer memory (no reference counterpart: the   */
/* reference runs on one GPU).  One process per GPU; replaces the all-gather   */
/* of the split-KV step: each rank's packed (O, LSE) [rows * 513 fp32] is      */
/* stored straight into every rank's exchange buffer, then merged there.       */
/* ------------------------------------------------------------------------ */

/* Bytes of one rank's exchange buffer for `world` ranks (<= 16) and `rows`
 * (sequences x heads) rows: a header of one u32 step count per row (padded to
 * 256 bytes), then two parities of [world][stride] 8-byte words, stride =
 * rows * 513 rounded up to even; each word is one fp32 value with the epoch of
 * the step that stored it in its upper half (readers poll for the epoch). */
MLA_B200_API size_t mla_b200_exchange_bytes(int world, long long rows);

/* cudaMalloc + zero of one exchange buffer on the current device (free with
 * mla_b200_exchange_free, after every peer closed its mapping). */
MLA_B200_API int mla_b200_exchange_alloc(int world, long long rows, void **buf);
MLA_B200_API int mla_b200_exchange_free(void *buf);

/* CUDA IPC: the 64-byte handle of an exchange buffer, and its mapping in
 * another process (peer access enabled lazily); close before the owner frees. */
MLA_B200_API int mla_b200_ipc_handle(const void *buf, void *handle_64_bytes);
MLA_B200_API int mla_b200_ipc_open(const void *handle_64_bytes, void **peer_buf);
MLA_B200_API int mla_b200_ipc_close(void *peer_buf);

/* Publish this rank's packed (O, LSE) `part` (rows * 513 fp32, 16-byte
 * aligned) into part `rank` of every rank's buffer: peer_bufs is a HOST array
 * of `world` device pointers (every rank's buffer as mapped in this process,
 * this rank's own at index `rank`).  Stream-ordered, graph-capturable; every
 * rank calls it once per step, in the same order as its merge. */
MLA_B200_API int mla_b200_exchange_put_f32(const float *part, long long rows, void *const *peer_bufs,
                                           int rank, int world, void *stream);

/* Wait until every rank published the step this rank last put, then
 * LSE-merge the `world` parts into out [rows, 512] (MLA_B200_OUT_F16 or _F32)
 * and out_lse [rows] (or null).  The wait is bounded by wait_limit_ns (at most
 * 60 s): on expiry the rows are left unwritten and mla_b200_get_device_error
 * reports MLA_B200_ERR_DEVICE_TIMEOUT (code 4, a peer wait). */
MLA_B200_API int mla_b200_exchange_merge_f32(const void *own_buf, int world, long long rows, void *out,
                                             int out_dtype, float *out_lse,
                                             unsigned long long wait_limit_ns, void *stream);

/* Put and merge in one kernel launch (one block per row): the same result as
 * mla_b200_exchange_put_f32 followed by mla_b200_exchange_merge_f32, one launch
 * fewer.  Its blocks wait on each other, so all `rows` blocks must be resident
 * at once: MLA_B200_ERR_UNSUPPORTED when they do not fit the device (use put +
 * merge then).  A block kept from running by other work on the device makes
 * the wait run out (device error code 4, rows left unwritten). */
MLA_B200_API int mla_b200_exchange_f32(const float *part, long long rows, void *const *peer_bufs, int rank,
                                       int world, void *out, int out_dtype, float *out_lse,
                                       unsigned long long wait_limit_ns, void *stream);

/* One rank's whole split-KV step: the decode of this rank's KV slice (the
 * arguments of mla_b200_decode_batched_f16) followed by ONE kernel that merges
 * the slice's split partials, publishes the merged (O, LSE) into every rank's
 * buffer and LSE-merges the `world` parts into out / out_lse, as
 * mla_b200_exchange_f32 does.  `direct` is rows * 513 fp32 scratch (16-byte
 * aligned) where the decode stores sequences it finishes as one work item.
 * The same result as mla_b200_decode_batched_f16 (OUT_F32 with LSE) followed
 * by mla_b200_exchange_f32, one launch fewer.  MLA_B200_ERR_UNSUPPORTED (before
 * anything is launched) when the exchange kernel's rows do not fit the device
 * at once or n_h > 128; a wait that runs out: device error code 4. */
MLA_B200_API int mla_b200_decode_exchange_f16(const void *query, const void *cache, const int32_t *cu_seqlens,
                                              int batch, int num_heads, long long total_tokens,
                                              int max_seq_len, float softmax_scale, int num_splits,
                                              void *const *peer_bufs, int rank, int world, float *direct,
                                              void *out, int out_dtype, float *out_lse,
                                              unsigned long long wait_limit_ns, void *workspace,
                                              size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ */
/* Device error word                                                         */
/* ------------------------------------------------------------------------ */

/* Every wait inside the kernels is bounded; a wait that expires records a
 * code in a device-side error word and the kernel returns early.  This reads
 * the word (synchronizing `stream`), writes it to *code (0 = none; may be NULL)
 * and clears it.  Returns MLA_B200_ERR_DEVICE_TIMEOUT when it was set. */
MLA_B200_API int mla_b200_get_device_error(int *code, void *stream);

/* The cudaError_t value behind the most recent MLA_B200_ERR_CUDA status this
 * library returned on the calling thread (0 when there was none).  Replaces
 * the reference's printf of cudaGetErrorString after each launch
 * (csrc/mla_decode_splitk_fwd.cuh:965-985, csrc/mla_decode_fused_fwd_sm89.cu:
 * 43-60): a caller can name the failure without the library printing. */
MLA_B200_API int mla_b200_last_cuda_error(void);

/* Self test of the bounded waits (no reference counterpart): launches one
 * thread that waits, through the same wait loop every kernel here uses, on an
 * mbarrier phase that nothing completes, with a limit of limit_ns (at most
 * 100 ms).  The wait gives up, records code 6 in the device error word and
 * returns; the kernel then writes 1 to the device int *done (2 would mean the
 * wait completed).  Read the word with mla_b200_get_device_error afterwards:
 * MLA_B200_ERR_DEVICE_TIMEOUT with code 6, and the context stays usable. */
MLA_B200_API int mla_b200_selftest_wait_timeout(unsigned long long limit_ns, int *done, void *stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MLA_B200_H */
