// abi.cu -- the extern "C" boundary of libfp8mla.so (declared in include/fp8mla.h):
// argument validation (mirroring the reference's asserts,
// vllm_fp8kv/fp8_ds_mla_sparse_decode.py:231-255), the split-KV heuristic,
// kernel dispatch, and the thread-local error message.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "decode.h"
#include "wait_limit.h"

namespace fp8mla {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FP8MLA_OK;
  return set_error(FP8MLA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

namespace {
// Hand-off wait limit of the small-head kernel (fp8mla_selftest_set_wait_limit).
std::atomic<uint32_t> g_handoff_wait_iters{kMaxWaitIters};

constexpr int kMaxDevices = 64;
struct DevInfo {
  int sms = 0, major = 0, minor = 0;
};
DevInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

const DevInfo* dev_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_dev_once[dev], [dev] {
    cudaDeviceGetAttribute(&g_dev[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&g_dev[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&g_dev[dev].minor, cudaDevAttrComputeCapabilityMinor, dev);
  });
  return &g_dev[dev];
}

int require_sm100() {
  const DevInfo* d = dev_info();
  if (d == nullptr) return set_error(FP8MLA_ERR_CUDA, "no current CUDA device");
  if (d->major != 10 || d->minor != 0)
    return set_error(FP8MLA_ERR_UNSUPPORTED,
                     "libfp8mla is built for sm_100a (B200); current device is sm_%d%d",
                     d->major, d->minor);
  return FP8MLA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int pick_splits(int64_t T, int64_t H, int64_t G, int64_t topk, int sm_count) {
  // tests/fixtures/triton_mla_sparse_kernel_pr47629.py:406-423
  const int64_t hpg = H / G;
  const int64_t bh = hpg < 16 ? hpg : 16;
  const int64_t head_blocks = G * ((hpg + bh - 1) / bh);
  const int64_t baseline = T * head_blocks;
  if (baseline == 0 || baseline * 4 >= sm_count) return 1;
  int64_t ideal = 1;
  const int64_t want = topk / 128 > 1 ? topk / 128 : 1;
  while (ideal < want) ideal <<= 1;
  int64_t max_splits = sm_count / baseline;
  if (max_splits < 1) max_splits = 1;
  int64_t p2 = 1;
  while ((p2 << 1) <= max_splits) p2 <<= 1;
  int64_t n = ideal < p2 ? ideal : p2;
  while (n > 1 && topk % n != 0) n >>= 1;
  return (int)(n < 1 ? 1 : n);
}

// Split count of a call with num_splits = 0.  The upstream table
// (pick_splits) for the general kernel; for the paired tcgen05 kernel (bf16 q,
// 64 or 128 heads per group), when that table gives one split and the pairs
// would leave SMs idle, the largest power of two that keeps T*G*S pairs within
// one wave of SM pairs and at least 4 tiles (256 entries) per split.
int auto_splits(int64_t T, int64_t H, int64_t G, int64_t topk, bool pair_kernel, int sm_count) {
  int S = pick_splits(T, H, G, topk, sm_count);
  if (!pair_kernel || S != 1) return S;
  const int64_t pairs = T * G, wave = sm_count / 2;
  int64_t s = 1;
  while (pairs * (s * 2) <= wave && topk % (s * 2) == 0 && topk / (s * 2) >= 256) s *= 2;
  return (int)s;
}
bool pair_heads(int64_t H, int64_t G) { return G > 0 && (H / G == 128 || H / G == 64); }

// Split workspace: the normalised partials ws_o[T][H][S][512] (elem_bytes
// each: 2 when the output is bf16, 4 when it is fp32), padded to 256 bytes,
// then the split LSEs ws_lse[T][H][S] (fp32).
int64_t ws_o_bytes(int64_t T, int64_t H, int S, int elem_bytes) {
  return ((T * H * S * kNope * elem_bytes + 255) / 256) * 256;
}
int64_t ws_bytes(int64_t T, int64_t H, int S, int elem_bytes) {
  if (S <= 1) return 0;
  return ws_o_bytes(T, H, S, elem_bytes) + T * H * S * 4;
}
}  // namespace

int device_sm_count() {
  const DevInfo* d = dev_info();
  return (d && d->sms > 0) ? d->sms : 148;
}

}  // namespace fp8mla

using namespace fp8mla;

extern "C" {

const char* fp8mla_last_error(void) { return g_last_error; }

int fp8mla_abi_version(void) { return 1; }

int fp8mla_device_status(unsigned int* status, int reset, void* stream) {
  g_last_error[0] = 0;
  if (status == nullptr) return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "status is NULL");
  *status = 0;
  if (int rc = require_sm100()) return rc;
  // each kernel file keeps its own status word
  unsigned int v2 = 0, v3 = 0, v4 = 0;
  int rc = read_device_status_ws(&v2, reset != 0, static_cast<cudaStream_t>(stream));
  if (rc == FP8MLA_OK) rc = read_device_status_tc3(&v3, reset != 0, static_cast<cudaStream_t>(stream));
  if (rc == FP8MLA_OK) rc = read_device_status_idx(&v4, reset != 0, static_cast<cudaStream_t>(stream));
  *status = v2 | v3 | v4;
  return rc;
}

int fp8mla_selftest_wait_timeout(uint32_t iters, uint64_t* elapsed_ns, void* stream) {
  g_last_error[0] = 0;
  if (iters == 0 || iters > fp8mla_wait_limit())
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "iters must be in [1, %u]", fp8mla_wait_limit());
  if (int rc = require_sm100()) return rc;
  return launch_wait_timeout_selftest(iters, elapsed_ns, static_cast<cudaStream_t>(stream));
}

uint32_t fp8mla_wait_limit(void) { return kMaxWaitIters; }

int fp8mla_selftest_set_wait_limit(uint32_t iters) {
  g_last_error[0] = 0;
  if (iters > kMaxWaitIters)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "iters must be in [0, %u]", kMaxWaitIters);
  g_handoff_wait_iters.store(iters == 0 ? kMaxWaitIters : iters);
  return FP8MLA_OK;
}

int fp8mla_choose_num_splits(int64_t T, int64_t H, int64_t G, int64_t topk, int sm_count) {
  if (G <= 0 || H <= 0 || H % G != 0) return 1;
  return pick_splits(T, H, G, topk, sm_count);
}

int64_t fp8mla_decode_workspace_bytes(int64_t T, int64_t H, int64_t G, int64_t topk,
                                      int num_splits) {
  if (num_splits <= 0) {
    if (G <= 0 || H <= 0 || H % G != 0) return 0;
    // sized for the paired kernel's choice, an upper bound of the general one
    num_splits = auto_splits(T, H, G, topk, pair_heads(H, G), device_sm_count());
  }
  if (num_splits > 64) num_splits = 64;
  // sized for fp32 partials: an upper bound for bf16 outputs (their partials
  // are bf16)
  return ws_bytes(T, H, num_splits, 4);
}

const char* fp8mla_decode_kernel_name(int64_t T, int64_t H, int64_t G, int64_t topk, int q_dtype,
                                      int num_splits) {
  if (G <= 0 || H <= 0 || H % G != 0) return "";
  int S = num_splits > 0 ? num_splits
                         : auto_splits(T, H, G, topk, q_dtype == FP8MLA_DTYPE_BF16 && pair_heads(H, G),
                                       device_sm_count());
  if (S > 64) S = 64;
  if (topk > 0 && S > topk) S = (int)topk;
  DecodeArgs a{};
  a.q_dtype = q_dtype;
  a.T = (int)T;
  a.H = (int)H;
  a.G = (int)G;
  a.topk = (int)topk;
  a.hpg = (int)(H / G);
  a.block_h = a.hpg < 16 ? a.hpg : 16;
  a.num_slots = 1;  // names the kernel of a non-empty pool
  a.num_splits = S < 1 ? 1 : S;
  const char* k = decode_tc3_supported(a)  ? "decode_tc3_kernel"
                  : decode_ws_supported(a) ? "decode_ws_kernel"
                                           : "decode_mma_kernel";
  if (a.num_splits == 1) return k;
  static thread_local char buf[64];
  snprintf(buf, sizeof(buf), "%s+merge_splits_kernel", k);
  return buf;
}

}  // extern "C"

namespace {

// Block-table indirection of fp8mla_sparse_decode_paged (null for flat slots).
struct PagedIndex {
  const int32_t* req_id;
  const int32_t* block_table;
  int64_t bt_stride, max_blocks, block_size;
};

int decode_impl(const void* q, int q_dtype, int64_t T, int64_t H, int64_t q_stride_t,
                int64_t q_stride_h, const uint8_t* kv, int64_t num_slots, const int32_t* indices,
                int64_t G, int64_t topk, int64_t idx_stride_t, int64_t idx_stride_g,
                float sm_scale, void* out, int64_t out_stride_t, int64_t out_stride_h, float* lse,
                int64_t lse_stride_t, int num_splits, void* workspace, int64_t workspace_bytes,
                void* stream, const PagedIndex* paged) {
  g_last_error[0] = 0;
  if (q_dtype != FP8MLA_DTYPE_BF16 && q_dtype != FP8MLA_DTYPE_F32)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT,
                     "q must be bf16 (fp32 allowed for testing); got dtype code %d", q_dtype);
  if (T < 0 || H <= 0 || G <= 0 || topk < 0 || num_slots < 0)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "bad sizes T=%lld H=%lld G=%lld topk=%lld",
                     (long long)T, (long long)H, (long long)G, (long long)topk);
  if (H % G != 0)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "h_q=%lld not divisible by kv_groups=%lld",
                     (long long)H, (long long)G);
  if (topk > (1LL << 30) || T > (1LL << 31) / 64)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "topk or T too large");
  if (T == 0) return FP8MLA_OK;
  const int64_t qa = q_dtype == FP8MLA_DTYPE_BF16 ? 8 : 4;
  if (!aligned16(q) || q_stride_t % qa || q_stride_h % qa)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT,
                     "q must be 16-byte aligned with row strides multiple of 16 bytes");
  if (!aligned16(out) || out_stride_t % 8 || out_stride_h % 8)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT,
                     "out must be 16-byte aligned with strides multiple of 8 elements");
  if (num_slots > 0 && !aligned16(kv))
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "kv cache must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;

  int S = num_splits;
  if (S <= 0)
    S = auto_splits(T, H, G, topk, q_dtype == FP8MLA_DTYPE_BF16 && pair_heads(H, G),
                    device_sm_count());
  if (S > 64) S = 64;
  if (topk > 0 && S > topk) S = (int)topk;
  if (S < 1) S = 1;

  DecodeArgs a{};
  a.q = q;
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.q_dtype = q_dtype;
  a.kv = kv;
  a.num_slots = num_slots;
  a.idx = indices;
  a.idx_st = idx_stride_t;
  a.idx_sg = idx_stride_g;
  a.T = (int)T;
  a.H = (int)H;
  a.G = (int)G;
  a.topk = (int)topk;
  a.hpg = (int)(H / G);
  a.block_h = a.hpg < 16 ? a.hpg : 16;
  a.hb_per_group = (a.hpg + a.block_h - 1) / a.block_h;
  a.scale_log2 = sm_scale * kLog2e;
  a.out = out;
  a.out_st = out_stride_t;
  a.out_sh = out_stride_h;
  a.lse = lse;
  a.lse_st = lse_stride_t;
  a.num_splits = S;
  a.split_len = (int)((topk + S - 1) / S);
  a.wait_iters = g_handoff_wait_iters.load();
  if (S > 1) {
    const int elem = q_dtype == FP8MLA_DTYPE_BF16 ? 2 : 4;  // partials in the output dtype
    const int64_t need = ws_bytes(T, H, S, elem);
    if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
      return set_error(FP8MLA_ERR_WORKSPACE,
                       "split-KV with %d splits needs %lld bytes of 16-B aligned workspace, got %lld",
                       S, (long long)need, (long long)workspace_bytes);
    a.ws_o = static_cast<float*>(workspace);
    a.ws_lse = reinterpret_cast<float*>(static_cast<char*>(workspace) + ws_o_bytes(T, H, S, elem));
  }
  if (paged != nullptr) {
    a.req_id = paged->req_id;
    a.block_table = paged->block_table;
    a.bt_stride = paged->bt_stride;
    a.max_blocks = paged->max_blocks;
    a.block_size = (int)paged->block_size;
    a.block_shift = -1;
    for (int k = 0; k < 31; ++k)
      if ((int64_t)1 << k == paged->block_size) a.block_shift = k;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (decode_tc3_supported(a)) return launch_decode_tc3(a, st);
  if (decode_ws_supported(a)) return launch_decode_ws(a, device_sm_count(), st);
  return launch_decode_mma(a, st);
}

}  // namespace

extern "C" {

int fp8mla_sparse_decode(const void* q, int q_dtype, int64_t T, int64_t H, int64_t q_stride_t,
                         int64_t q_stride_h, const uint8_t* kv, int64_t num_slots,
                         const int32_t* indices, int64_t G, int64_t topk, int64_t idx_stride_t,
                         int64_t idx_stride_g, float sm_scale, void* out, int64_t out_stride_t,
                         int64_t out_stride_h, float* lse, int64_t lse_stride_t, int num_splits,
                         void* workspace, int64_t workspace_bytes, void* stream) {
  return decode_impl(q, q_dtype, T, H, q_stride_t, q_stride_h, kv, num_slots, indices, G, topk,
                     idx_stride_t, idx_stride_g, sm_scale, out, out_stride_t, out_stride_h, lse,
                     lse_stride_t, num_splits, workspace, workspace_bytes, stream, nullptr);
}

int fp8mla_sparse_decode_paged(const void* q, int q_dtype, int64_t T, int64_t H,
                               int64_t q_stride_t, int64_t q_stride_h, const uint8_t* kv,
                               int64_t num_slots, const int32_t* req_id,
                               const int32_t* block_table, int64_t bt_stride, int64_t max_blocks,
                               int64_t block_size, const int32_t* token_idx, int64_t G,
                               int64_t topk, int64_t ti_stride_t, int64_t ti_stride_g,
                               float sm_scale, void* out, int64_t out_stride_t,
                               int64_t out_stride_h, float* lse, int64_t lse_stride_t,
                               int num_splits, void* workspace, int64_t workspace_bytes,
                               void* stream) {
  g_last_error[0] = 0;
  if (block_size <= 0 || block_size > (1 << 20) || max_blocks < 0 || bt_stride < max_blocks)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT,
                     "bad block table: block_size=%lld max_blocks=%lld stride=%lld",
                     (long long)block_size, (long long)max_blocks, (long long)bt_stride);
  if (T > 0 && topk > 0 && (req_id == nullptr || (max_blocks > 0 && block_table == nullptr)))
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "req_id and block_table are required");
  const PagedIndex paged{req_id, block_table, bt_stride, max_blocks, block_size};
  return decode_impl(q, q_dtype, T, H, q_stride_t, q_stride_h, kv, num_slots, token_idx, G, topk,
                     ti_stride_t, ti_stride_g, sm_scale, out, out_stride_t, out_stride_h, lse,
                     lse_stride_t, num_splits, workspace, workspace_bytes, stream, &paged);
}

int fp8mla_ds_mla_write(const uint16_t* kv_c, int64_t kv_c_stride, const uint16_t* k_pe,
                        int64_t k_pe_stride, const int64_t* slot_mapping, int64_t N,
                        uint8_t* cache, int64_t num_slots, void* stream) {
  g_last_error[0] = 0;
  if (N < 0 || num_slots < 0 || kv_c_stride < kNope || k_pe_stride < kRope)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "bad writer sizes/strides");
  if (N == 0) return FP8MLA_OK;
  if (num_slots > 0 && !aligned16(cache))
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "cache must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  return launch_ds_mla_write(kv_c, kv_c_stride, k_pe, k_pe_stride, slot_mapping, N, cache,
                             num_slots, static_cast<cudaStream_t>(stream));
}

int fp8mla_dequant_e4m3(const uint8_t* in, int64_t n, void* out, int out_dtype, int method,
                        void* stream) {
  g_last_error[0] = 0;
  if (n < 0 || (method != 0 && method != 1) ||
      (out_dtype != FP8MLA_DTYPE_BF16 && out_dtype != FP8MLA_DTYPE_F16 &&
       out_dtype != FP8MLA_DTYPE_F32))
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "bad dequant arguments");
  if (n == 0) return FP8MLA_OK;
  if (int rc = require_sm100()) return rc;
  return launch_dequant(in, n, out, out_dtype, method, static_cast<cudaStream_t>(stream));
}

int fp8mla_ds_mla_dequant_rows(const uint8_t* kv, int64_t num_slots, const int32_t* slots,
                               int64_t n, uint16_t* out, int64_t out_stride, int method,
                               void* stream) {
  g_last_error[0] = 0;
  if (n < 0 || num_slots < 0 || (method != 0 && method != 1) || out_stride < kDqk)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "bad row-dequant arguments");
  if (n == 0) return FP8MLA_OK;
  if (kv == nullptr || slots == nullptr || out == nullptr)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "null row-dequant pointer");
  if ((reinterpret_cast<uintptr_t>(kv) | reinterpret_cast<uintptr_t>(out) |
       (uintptr_t)(out_stride * 2)) % 16 != 0)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "row dequant needs 16-byte aligned rows");
  if (int rc = require_sm100()) return rc;
  return launch_dequant_rows(kv, num_slots, slots, n, out, out_stride, method,
                             static_cast<cudaStream_t>(stream));
}

int fp8mla_convert_req_index(const int32_t* req_id, const int32_t* block_table,
                             int64_t bt_stride, int64_t max_blocks, const int32_t* token_idx,
                             int64_t ti_stride, int64_t T, int64_t topk, int64_t block_size,
                             int32_t* out, int64_t out_stride, void* stream) {
  g_last_error[0] = 0;
  if (T < 0 || topk < 0 || block_size <= 0 || max_blocks < 0)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "bad index-conversion sizes");
  if (topk % 128 != 0)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT,
                     "NUM_TOPK_TOKENS (%lld) must be divisible by BLOCK_N (128)", (long long)topk);
  if (T * topk == 0) return FP8MLA_OK;
  if (int rc = require_sm100()) return rc;
  return launch_convert_req_index(req_id, block_table, bt_stride, max_blocks, token_idx,
                                  ti_stride, T, topk, block_size, out, out_stride,
                                  static_cast<cudaStream_t>(stream));
}

int fp8mla_indexer_paged_logits(const uint8_t* q, int64_t B, int64_t next_n, int64_t H,
                                int64_t head_dim, int64_t q_stride_b, const uint8_t* k_cache,
                                int64_t num_blocks, int64_t block_size, const float* weights,
                                int64_t w_stride, const int32_t* context_lens,
                                const int32_t* block_table, int64_t bt_stride, int64_t max_blocks,
                                float* logits, int64_t logits_stride, int64_t max_model_len,
                                void* stream) {
  g_last_error[0] = 0;
  if (H != 64 || head_dim != 128 || block_size != 64)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT,
                     "indexer logits take 64 heads of dim 128 over 64-token blocks (got H=%lld, "
                     "dim=%lld, block_size=%lld)", (long long)H, (long long)head_dim,
                     (long long)block_size);
  if (next_n < 1 || next_n > 2)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "next_n must be 1 or 2, got %lld", (long long)next_n);
  if (B < 0 || max_model_len < 0 || num_blocks < 0 || num_blocks >= (1LL << 31) || max_blocks < 0 ||
      bt_stride < max_blocks || logits_stride < max_model_len || w_stride < H ||
      q_stride_b < next_n * H * head_dim)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "bad indexer logits sizes or strides");
  if (B == 0 || max_model_len == 0) return FP8MLA_OK;
  if (num_blocks == 0)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "the indexer key cache is empty");
  if (!aligned16(q) || q_stride_b % 16 != 0 || !aligned16(k_cache))
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT,
                     "q and the key cache must be 16-byte aligned (q rows 16-byte strided)");
  if (int rc = require_sm100()) return rc;
  return launch_indexer_logits(q, B, next_n, q_stride_b, k_cache, num_blocks, weights, w_stride,
                               context_lens, block_table, bt_stride, max_blocks, logits,
                               logits_stride, max_model_len, device_sm_count(),
                               static_cast<cudaStream_t>(stream));
}

int fp8mla_indexer_topk(const float* logits, int64_t rows, int64_t logits_stride, int64_t next_n,
                        const int32_t* context_lens, int32_t* out, int64_t out_stride,
                        int64_t topk, int64_t max_model_len, void* stream) {
  g_last_error[0] = 0;
  if (rows < 0 || next_n < 1 || rows % next_n != 0 || topk < 1 || topk > (1 << 20) ||
      out_stride < topk || max_model_len < 0 || logits_stride < max_model_len ||
      rows > (int64_t)INT32_MAX)
    return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "bad indexer top-k sizes or strides");
  if (rows == 0) return FP8MLA_OK;
  if (int rc = require_sm100()) return rc;
  return launch_indexer_topk(logits, rows, logits_stride, next_n, context_lens, out, out_stride, topk,
                             max_model_len, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
