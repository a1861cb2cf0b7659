/*
 * fp8mla.h -- C ABI of the B200 (sm_100a) fp8_ds_mla sparse-MLA decode library
 * (libfp8mla.so).
 *
 * Every entry point takes plain device pointers, 64-bit sizes and element
 * strides, and a CUDA stream passed as `void*` (a cudaStream_t; NULL = the
 * legacy default stream).  No torch or CUDA types appear in the signatures.
 * Every call returns an int status (FP8MLA_OK = 0, negative on error); the
 * message of the last failure on the calling thread is available from
 * fp8mla_last_error().  Calls are asynchronous with respect to the host
 * unless stated otherwise, and none of them synchronises the stream.
 *
 * fp8_ds_mla row (656 bytes per KV slot), the format this library reads and
 * writes (reference: vllm_fp8kv/fp8_ds_mla_sparse_decode.py:41-47, :68-74):
 *     [  0:512)  512 x float8_e4m3fn   NoPE latent, per-128-tile scaled
 *     [512:528)    4 x float32         per-128-element tile scales (amax/448)
 *     [528:656)   64 x bfloat16        RoPE, stored raw (never quantized)
 */
#ifndef FP8MLA_H
#define FP8MLA_H

#include <stdint.h>

#if defined(__GNUC__)
#define FP8MLA_API __attribute__((visibility("default")))
#else
#define FP8MLA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FP8MLA_OK 0
#define FP8MLA_ERR_INVALID_ARGUMENT (-1) /* shape, dtype, stride or alignment */
#define FP8MLA_ERR_UNSUPPORTED (-2)      /* device is not sm_100 / no kernel  */
#define FP8MLA_ERR_CUDA (-3)             /* a CUDA runtime call failed        */
#define FP8MLA_ERR_WORKSPACE (-4)        /* workspace missing or too small    */

/* ---- element types ------------------------------------------------------- */
#define FP8MLA_DTYPE_BF16 0
#define FP8MLA_DTYPE_F32 1
#define FP8MLA_DTYPE_F16 2

/* ---- row geometry (reference: fp8_ds_mla_sparse_decode.py:68-74) --------- */
#define FP8MLA_NOPE 512
#define FP8MLA_ROPE 64
#define FP8MLA_TILE 128
#define FP8MLA_ROW_BYTES 656
#define FP8MLA_SCALE_OFF 512
#define FP8MLA_ROPE_OFF 528

/* Message of the last failed call on this thread ("" if none). */
FP8MLA_API const char* fp8mla_last_error(void);

/* ABI version of this library (bumped on any signature change). */
FP8MLA_API int fp8mla_abi_version(void);

/*
 * Device-side status word of the current device: 0, or the bits the decode
 * kernels set when a bounded on-chip wait gave up (bit 0 = wait timeout,
 * bits 8.. = which wait).  Synchronises `stream`; `reset` != 0 clears it.
 * Returns FP8MLA_OK and stores the word in *status.  No reference
 * counterpart (the reference's Triton kernels have no on-chip waits).
 */
FP8MLA_API int fp8mla_device_status(unsigned int* status, int reset, void* stream);

/*
 * Number of mbarrier try_wait calls after which a decode kernel's on-chip
 * wait gives up (and sets the device status word).  No reference counterpart.
 */
FP8MLA_API uint32_t fp8mla_wait_limit(void);

/*
 * Exercises the error path of the decode kernels' bounded on-chip waits: a
 * one-warp kernel runs their wait loop on an mbarrier that nothing arrives
 * on, gives up after `iters` (1 .. fp8mla_wait_limit()) try_wait calls and
 * returns, leaving bit 0 and "which wait" = 63 in the device status word
 * (fp8mla_device_status).  *elapsed_ns (if not NULL) receives the loop's
 * duration, so a caller can see how long a full-limit timeout takes.  No GPU
 * fault is involved and the context stays usable.  Synchronises `stream`.
 * For tests and health checks; no reference counterpart.
 */
FP8MLA_API int fp8mla_selftest_wait_timeout(uint32_t iters, uint64_t* elapsed_ns, void* stream);

/*
 * Lowers the limit of the hand-off waits of the small-head decode kernel
 * (decode_ws_kernel: raw rows, key rows and Q between its producer, dequant
 * and compute warps) to `iters` try_wait calls for the decode calls that
 * follow in this process; 0 restores fp8mla_wait_limit().  With a limit of a
 * few calls the waits give up while the copies they wait for are still
 * arriving, so a test can drive the kernel's error path without a fault:
 * the producer stops issuing copies, waits (with the full limit) for those it
 * issued, every warp returns, and the status word carries the timeout.
 * Results of such calls are meaningless.  For tests; no reference
 * counterpart.  Returns FP8MLA_ERR_INVALID_ARGUMENT above the full limit.
 */
FP8MLA_API int fp8mla_selftest_set_wait_limit(uint32_t iters);

/*
 * Split-KV count the decode picks when called with num_splits = 0.
 * Replaces the host heuristic `_choose_num_kv_splits`
 * (tests/fixtures/triton_mla_sparse_kernel_pr47629.py:406-423): a power of two
 * in {1,2,4,8,16}, 1 when T * head_blocks * 4 >= sm_count, at least 128 top-k
 * entries per split, and topk divisible by the count.
 */
FP8MLA_API int fp8mla_choose_num_splits(int64_t T, int64_t H, int64_t G, int64_t topk,
                             int sm_count);

/*
 * Bytes of device workspace fp8mla_sparse_decode needs for this shape and
 * split count (0 when num_splits == 1).  Pass num_splits = 0 to size for the
 * count fp8mla_choose_num_splits() returns on the current device.
 */
FP8MLA_API int64_t fp8mla_decode_workspace_bytes(int64_t T, int64_t H, int64_t G,
                                      int64_t topk, int num_splits);

/*
 * Name of the decode kernel fp8mla_sparse_decode dispatches for this shape
 * ("decode_tc3_kernel" for 128 or 64 heads per kv group with bf16 q,
 * "decode_ws_kernel" for other head counts with bf16 q and a non-empty pool,
 * "decode_mma_kernel" for fp32 q; "+merge_splits_kernel" is appended when the
 * call splits the top-k axis; the name string stays valid until the calling
 * thread's next call).  Host-only; introspection for benchmarks and profiling.
 * No reference counterpart (the reference has one Triton kernel per path).
 */
FP8MLA_API const char* fp8mla_decode_kernel_name(int64_t T, int64_t H, int64_t G,
                                                 int64_t topk, int q_dtype,
                                                 int num_splits);

/*
 * Sparse MLA decode over fp8_ds_mla pages.
 *
 * Replaces the Triton launch behind `fp8_ds_mla_sparse_decode`
 * (vllm_fp8kv/fp8_ds_mla_sparse_decode.py:214-288, kernel :77-211) and the
 * upstream split-KV pair `_sparse_mla_kernel_split` + `_sparse_mla_merge_kernel`
 * (tests/fixtures/triton_mla_sparse_kernel_pr47629.py:232-403).
 *
 *   q        [T, H, 576]   bf16 (q_dtype = FP8MLA_DTYPE_BF16) or fp32
 *                          (FP8MLA_DTYPE_F32, rounded to bf16 on load);
 *                          unit stride on the last dim.
 *   kv       [num_slots, 656] uint8, contiguous, 16-byte aligned.
 *   indices  [T, G, topk]  int32 flat slot indices; entries < 0 or
 *                          >= num_slots are masked: they contribute nothing
 *                          and no address is formed from them (the TMA-staged
 *                          kernels fetch row 0 in their place and discard it).
 *                          Head h reads group h / (H / G).
 *   sm_scale softmax scale WITHOUT the log2(e) factor.
 *   out      [T, H, 512]   same dtype as q.
 *   lse      [T, H] fp32 natural-log LSE, or NULL.  -inf for a row that
 *                          selected nothing (its out row is all zeros).
 *   num_splits  0 = the library's choice: fp8mla_choose_num_splits() (the
 *               upstream table), except that for the paired tcgen05 kernel (bf16
 *               q, 64 or 128 heads per group) a table answer of 1 is raised to
 *               the largest power of two that keeps T*G*splits CTA pairs within
 *               one wave of SM pairs with at least 256 top-k entries per split;
 *               otherwise 1..64 splits of the top-k axis merged by LSE.  Splits
 *               > 1 need `workspace` (fp8mla_decode_workspace_bytes sizes it).
 *
 * Returns FP8MLA_ERR_INVALID_ARGUMENT for shape/stride/alignment violations.
 */
FP8MLA_API int fp8mla_sparse_decode(const void* q, int q_dtype, int64_t T, int64_t H,
                         int64_t q_stride_t, int64_t q_stride_h,
                         const uint8_t* kv, int64_t num_slots,
                         const int32_t* indices, int64_t G, int64_t topk,
                         int64_t idx_stride_t, int64_t idx_stride_g,
                         float sm_scale,
                         void* out, int64_t out_stride_t, int64_t out_stride_h,
                         float* lse, int64_t lse_stride_t,
                         int num_splits, void* workspace,
                         int64_t workspace_bytes, void* stream);

/*
 * The same decode over request-local token positions: the slot of position
 * tok of query token t is
 *   block_table[req_id[t] * bt_stride + tok / block_size] * block_size
 *     + tok % block_size,
 * -1 (masked) when tok < 0 or tok / block_size >= max_blocks, then masked
 * like fp8mla_sparse_decode when outside [0, num_slots).  The conversion runs
 * inside the gather: no [T, topk] slot array is written or read.
 *
 * Replaces the pair the reference runs per fp8 layer
 * (vllm_fp8kv/backend_patch.py:83-89): vLLM's
 * `triton_convert_req_index_to_global_index` (installed
 * vllm/v1/attention/backends/mla/sparse_utils.py:85) followed by
 * `fp8_ds_mla_sparse_decode`.  Bit-identical to fp8mla_convert_req_index then
 * fp8mla_sparse_decode with the same arguments (int32 arithmetic included).
 *
 *   req_id      [T] int32 request of each query token.
 *   block_table [*, bt_stride] int32 page ids; bt_stride >= max_blocks.
 *   token_idx   [T, G, topk] int32 request-local positions (strides
 *               ti_stride_t, ti_stride_g; unit last stride).
 * Other arguments as fp8mla_sparse_decode.  No topk % 128 requirement.
 */
FP8MLA_API int fp8mla_sparse_decode_paged(
    const void* q, int q_dtype, int64_t T, int64_t H, int64_t q_stride_t, int64_t q_stride_h,
    const uint8_t* kv, int64_t num_slots, const int32_t* req_id, const int32_t* block_table,
    int64_t bt_stride, int64_t max_blocks, int64_t block_size, const int32_t* token_idx,
    int64_t G, int64_t topk, int64_t ti_stride_t, int64_t ti_stride_g, float sm_scale, void* out,
    int64_t out_stride_t, int64_t out_stride_h, float* lse, int64_t lse_stride_t, int num_splits,
    void* workspace, int64_t workspace_bytes, void* stream);

/*
 * fp8mla_sparse_decode for callers that cannot allocate device memory.
 * No counterpart in the reference.  Same arguments and behaviour as
 * fp8mla_sparse_decode minus the workspace: the split-KV scratch comes from a
 * fixed 32 MiB array inside this library (held by each GPU that loads it until
 * the process exits) instead of from the caller, and nothing is allocated.
 * Shapes whose split workspace would exceed 32 MiB return
 * FP8MLA_ERR_WORKSPACE.  The array's address is looked up on the first call
 * made on each device, so make that call before any stream capture.  All
 * calls on a device share the array: calls that can overlap on the GPU race
 * and must be serialised by the caller.
 */
FP8MLA_API int fp8mla_sparse_decode_noalloc(const void* q, int q_dtype, int64_t T, int64_t H,
                                            int64_t q_stride_t, int64_t q_stride_h,
                                            const uint8_t* kv, int64_t num_slots,
                                            const int32_t* indices, int64_t G, int64_t topk,
                                            int64_t idx_stride_t, int64_t idx_stride_g,
                                            float sm_scale,
                                            void* out, int64_t out_stride_t, int64_t out_stride_h,
                                            float* lse, int64_t lse_stride_t,
                                            int num_splits, void* stream);

/*
 * fp8_ds_mla cache writer: quantize bf16 latent + rope into 656-byte rows.
 *
 * Replaces vLLM's `concat_and_cache_mla(..., kv_cache_dtype="fp8_ds_mla")`
 * (called at verify/contract.py:100-103), whose behaviour the reference
 * restates in verify/reference.py:68-91 and tests/fakes.py:28-57: per
 * 128-element tile, scale = max(amax / 448, FLT_MIN); latent byte =
 * float8_e4m3fn(x / scale) with round-to-nearest-even (|v| >= 464 rounds to
 * the NaN encoding 0x7F, as torch's cast does); rope copied as raw bf16.
 * The layer's k_scale is not an input: the format ignores it.
 *
 *   kv_c  [N, 512] bf16 bits, row stride kv_c_stride (elements)
 *   k_pe  [N, 64]  bf16 bits, row stride k_pe_stride (elements)
 *   slot_mapping [N] int64; slots < 0 or >= num_slots are skipped.
 *   cache [num_slots, 656] uint8
 */
FP8MLA_API int fp8mla_ds_mla_write(const uint16_t* kv_c, int64_t kv_c_stride,
                        const uint16_t* k_pe, int64_t k_pe_stride,
                        const int64_t* slot_mapping, int64_t N,
                        uint8_t* cache, int64_t num_slots, void* stream);

/*
 * Device e4m3fn decode of n raw bytes into fp16 / bf16 / fp32 (out_dtype).
 * method 0 = the packed hardware conversion, 1 = the integer bit-math the
 * fused decode uses.  Both are exact for every finite byte; 0x7F/0xFF give NaN.
 * Replaces `_dequant_test_kernel` / `dequant_triton_launch`
 * (vllm_fp8kv/fp8_dequant.py:98-113).
 */
FP8MLA_API int fp8mla_dequant_e4m3(const uint8_t* in, int64_t n, void* out,
                        int out_dtype, int method, void* stream);

/*
 * Gather + dequant of n fp8_ds_mla rows by slot into bf16 out[n, 576]
 * (row stride out_stride elements, >= 576, 16-byte aligned):
 * out[r, d] = bf16(float(e4m3 latent[d]) * scale[d / 128]) for d < 512 and the
 * raw rope for d >= 512; slot < 0 or >= num_slots gives a zero row.  It runs
 * the decode kernels' own device dequant (method 1: the packed-multiply form
 * both decode kernels use; 0: the same arithmetic unpacked) so that it can be
 * checked bit for bit.
 * Replaces the IS_FP8 gather + dequant inside `_fp8_ds_mla_sparse_decode_kernel`
 * (vllm_fp8kv/fp8_ds_mla_sparse_decode.py:136-168).
 */
FP8MLA_API int fp8mla_ds_mla_dequant_rows(const uint8_t* kv, int64_t num_slots,
                               const int32_t* slots, int64_t n, uint16_t* out,
                               int64_t out_stride, int method, void* stream);

/*
 * Token-relative top-k -> flat global slot:
 *   out[t, i] = block_table[req_id[t], tok / block_size] * block_size
 *               + tok % block_size,  with tok = token_idx[t, i];
 * -1 when tok < 0 or the block index is outside [0, max_blocks).
 * Replaces vLLM's `triton_convert_req_index_to_global_index`
 * (called at vllm_fp8kv/backend_patch.py:83-89; mirrored in
 * tests/fakes.py:70-82).  topk must be a multiple of 128.
 */
FP8MLA_API int fp8mla_convert_req_index(const int32_t* req_id, const int32_t* block_table,
                             int64_t bt_stride, int64_t max_blocks,
                             const int32_t* token_idx, int64_t ti_stride,
                             int64_t T, int64_t topk, int64_t block_size,
                             int32_t* out, int64_t out_stride, void* stream);

/*
 * DSA indexer read path, fp8 paged MQA logits.  Replaces the logits step the
 * indexer runs before every sparse-MLA decode (reference specification:
 * PORT_PLAN.md:14 and :41, D3; the reference ships no code for it;
 * semantics of vLLM's `fp8_paged_mqa_logits`, whose torch restatement
 * vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:256-354 the tests pin to):
 *
 *   logits[b*next_n + n, s] = scale_s * sum_h relu(q[b,n,h] . k_s) * weights[b*next_n + n, h]
 *
 * for s < context_lens[b] - next_n + n + 1, and -inf for the other positions
 * of the row up to max_model_len.
 *
 *   q            [B, next_n, H, head_dim] e4m3 bytes; a request's rows are
 *                contiguous, requests q_stride_b bytes apart (16-byte aligned).
 *   k_cache      [num_blocks, block_size * (head_dim + 4)] bytes: per block,
 *                block_size x head_dim e4m3 values, then block_size fp32
 *                scales (structure of arrays, 8448 bytes at block_size 64).
 *   weights      [B * next_n, H] fp32 (row stride w_stride), the query scale
 *                folded in.
 *   context_lens [B] int32; block_table [B, bt_stride] int32 block ids
 *                (positions past a valid block, or an id outside
 *                [0, num_blocks), score -inf).
 *   logits       [B * next_n, logits_stride] fp32, columns [0, max_model_len)
 *                written.
 * Supported: H = 64, head_dim = 128, block_size = 64, next_n = 1 or 2.
 */
FP8MLA_API int fp8mla_indexer_paged_logits(const uint8_t* q, int64_t B, int64_t next_n, int64_t H,
                                           int64_t head_dim, int64_t q_stride_b,
                                           const uint8_t* k_cache, int64_t num_blocks,
                                           int64_t block_size, const float* weights,
                                           int64_t w_stride, const int32_t* context_lens,
                                           const int32_t* block_table, int64_t bt_stride,
                                           int64_t max_blocks, float* logits,
                                           int64_t logits_stride, int64_t max_model_len,
                                           void* stream);

/*
 * Top-k positions of each indexer logits row: the step that fills the
 * decode's top-k position buffer (`topk_indices_buffer`, read at the
 * reference's backend_patch.py:79-81; vLLM's `top_k_per_row_decode`).  Row
 * r = b * next_n + n keeps positions [0, limit) with limit =
 * min(max_model_len, context_lens[b] - next_n + n + 1): all of them when
 * limit <= topk, else the topk largest logits (ties at the threshold broken
 * by the lower position).  Kept positions are written in ascending order,
 * then -1 pads the row: out [rows, out_stride] int32, topk columns written.
 * The set equals torch.topk's on untied values; the decode treats it as a set.
 */
FP8MLA_API int fp8mla_indexer_topk(const float* logits, int64_t rows, int64_t logits_stride,
                                   int64_t next_n, const int32_t* context_lens, int32_t* out,
                                   int64_t out_stride, int64_t topk, int64_t max_model_len,
                                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FP8MLA_H */
