// decode.h -- internal arguments shared by the decode kernels and the ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fp8mla {

struct DecodeArgs {
  const void* q;
  int64_t q_st, q_sh;
  int q_dtype;
  const uint8_t* kv;
  int64_t num_slots;
  const int32_t* idx;
  int64_t idx_st, idx_sg;
  int T, H, G, topk;
  int hpg;           // heads per kv group (H / G)
  int block_h;       // heads per CTA of the general kernel: min(16, hpg)
  int hb_per_group;  // ceil(hpg / block_h)
  float scale_log2;  // sm_scale * log2(e)
  void* out;
  int64_t out_st, out_sh;
  float* lse;
  int64_t lse_st;
  int num_splits;
  int split_len;     // top-k entries per split (last split may be shorter)
  float* ws_o;       // [T][H][S][512] normalised split outputs: bf16 (as uint16)
                     // when the output is bf16, fp32 when it is fp32
  float* ws_lse;     // [T][H][S] natural-log split LSE
  // Optional block-table indirection (fp8mla_sparse_decode_paged): when
  // block_table is set, idx holds request-local token positions and the slot
  // of position tok of token t is block_table[req_id[t], tok / block_size] *
  // block_size + tok % block_size (-1 for tok < 0 or a block past max_blocks).
  const int32_t* req_id;
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t max_blocks;
  int block_size;
  int block_shift;   // log2(block_size) when it is a power of two, else -1
  // try_wait calls after which a hand-off wait of decode_ws_kernel gives up
  // (the library default, lowered only by fp8mla_selftest_set_wait_limit);
  // its drains before exit keep the full limit
  uint32_t wait_iters;
};

#ifdef __CUDACC__
// The live slot an index entry names, or -1 (masked, past the table, or
// outside [0, num_slots)).  `req` is req_id[t] when a block table is set.
// The block-table step is vLLM's converter with its int32 arithmetic
// (installed vllm/v1/attention/backends/mla/sparse_utils.py:11-78; the
// library's standalone form is convert_req_index_kernel).
// Block of a non-negative position: a shift for power-of-two pages (the
// usual 64), a division otherwise.
__device__ __forceinline__ int32_t block_of(const DecodeArgs& a, int32_t v) {
  return a.block_shift >= 0 ? (v >> a.block_shift) : v / a.block_size;
}
__device__ __forceinline__ int32_t live_slot(const DecodeArgs& a, int32_t req, int32_t v) {
  if (a.block_table != nullptr) {
    if (v < 0) return -1;
    const int32_t blk = block_of(a, v), off = v - blk * a.block_size;
    if (blk >= a.max_blocks) return -1;
    const uint32_t base = (uint32_t)a.block_table[(int64_t)req * a.bt_stride + blk];
    v = (int32_t)(base * (uint32_t)a.block_size + (uint32_t)off);
  }
  return (v >= 0 && (int64_t)v < a.num_slots) ? v : -1;
}
// live_slot split in two for software-pipelined gathers: slot_fetch issues
// the block-table read of a raw index (nothing for flat slots) and
// slot_finish completes the conversion one pipeline step later, so neither
// waits on a load issued in the same step.  slot_finish(slot_fetch(v)) ==
// live_slot(v).
struct SlotPf {
  int32_t v;
  int32_t base;
};
__device__ __forceinline__ SlotPf slot_fetch(const DecodeArgs& a, int32_t req, int32_t v) {
  SlotPf r{v, 0};
  if (a.block_table != nullptr && v >= 0) {
    const int32_t blk = block_of(a, v);
    if (blk < a.max_blocks) r.base = a.block_table[(int64_t)req * a.bt_stride + blk];
  }
  return r;
}
__device__ __forceinline__ int32_t slot_finish(const DecodeArgs& a, SlotPf p) {
  int32_t v = p.v;
  if (a.block_table != nullptr) {
    if (v < 0) return -1;
    const int32_t blk = block_of(a, v), off = v - blk * a.block_size;
    if (blk >= a.max_blocks) return -1;
    v = (int32_t)((uint32_t)p.base * (uint32_t)a.block_size + (uint32_t)off);
  }
  return (v >= 0 && (int64_t)v < a.num_slots) ? v : -1;
}
// Programmatic dependent launch: the decode kernels are launched so that their
// CTAs may start (and do their setup) while the previous kernel of the stream
// finishes.  pdl_wait() blocks until that kernel has completed and its writes
// are visible; no global memory is read or written before it.
// pdl_launch_dependents() lets the next kernel's CTAs be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ int32_t request_of(const DecodeArgs& a, int64_t t) {
  return a.block_table != nullptr ? a.req_id[t] : 0;
}
#endif

// Launch `kern` on `st` with programmatic stream serialization (see pdl_wait).
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

int launch_decode_mma(const DecodeArgs& a, cudaStream_t st);
int launch_merge_splits(const DecodeArgs& a, cudaStream_t st);
int launch_wait_timeout_selftest(uint32_t iters, uint64_t* elapsed_ns, cudaStream_t st);
bool decode_tc3_supported(const DecodeArgs& a);
int launch_decode_tc3(const DecodeArgs& a, cudaStream_t st);
int read_device_status_tc3(unsigned int* status, bool reset, cudaStream_t st);
bool decode_ws_supported(const DecodeArgs& a);
int launch_decode_ws(const DecodeArgs& a, int sms, cudaStream_t st);
int read_device_status_ws(unsigned int* status, bool reset, cudaStream_t st);

int read_device_status_idx(unsigned int* status, bool reset, cudaStream_t st);
int launch_indexer_logits(const uint8_t* q, int64_t B, int64_t next_n, int64_t q_stride_b,
                          const uint8_t* k_cache, int64_t num_blocks, const float* w,
                          int64_t w_stride, const int32_t* ctx, const int32_t* bt, int64_t bt_stride,
                          int64_t max_blocks, float* logits, int64_t logits_stride,
                          int64_t max_len, int sms, cudaStream_t st);
int launch_indexer_topk(const float* logits, int64_t rows, int64_t logits_stride, int64_t next_n,
                        const int32_t* ctx, int32_t* out, int64_t out_stride, int64_t topk,
                        int64_t max_len, cudaStream_t st);

int launch_dequant(const uint8_t* in, int64_t n, void* out, int out_dtype, int method,
                   cudaStream_t st);
int launch_dequant_rows(const uint8_t* kv, int64_t num_slots, const int32_t* slots, int64_t n,
                        uint16_t* out, int64_t out_stride, int method, cudaStream_t st);
int launch_ds_mla_write(const uint16_t* kv_c, int64_t kv_c_stride, const uint16_t* k_pe,
                        int64_t k_pe_stride, const int64_t* slot_mapping, int64_t N,
                        uint8_t* cache, int64_t num_slots, cudaStream_t st);
int launch_convert_req_index(const int32_t* req_id, const int32_t* block_table,
                             int64_t bt_stride, int64_t max_blocks, const int32_t* token_idx,
                             int64_t ti_stride, int64_t T, int64_t topk, int64_t block_size,
                             int32_t* out, int64_t out_stride, cudaStream_t st);

}  // namespace fp8mla
