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
  float* ws_o;       // [T][H][S][512] fp32 normalised split outputs
  float* ws_lse;     // [T][H][S] natural-log split LSE
};

int launch_decode_mma(const DecodeArgs& a, cudaStream_t st);
int launch_merge_splits(const DecodeArgs& a, cudaStream_t st);
int read_device_status(unsigned int* status, bool reset, cudaStream_t st);
int launch_decode_tc(const DecodeArgs& a, cudaStream_t st);
bool decode_tc_supported(const DecodeArgs& a);

int launch_dequant(const uint8_t* in, int64_t n, void* out, int out_dtype, int method,
                   cudaStream_t st);
int launch_ds_mla_write(const uint16_t* kv_c, int64_t kv_c_stride, const uint16_t* k_pe,
                        int64_t k_pe_stride, const int64_t* slot_mapping, int64_t N,
                        uint8_t* cache, int64_t num_slots, cudaStream_t st);
int launch_convert_req_index(const int32_t* req_id, const int32_t* block_table,
                             int64_t bt_stride, int64_t max_blocks, const int32_t* token_idx,
                             int64_t ti_stride, int64_t T, int64_t topk, int64_t block_size,
                             int32_t* out, int64_t out_stride, cudaStream_t st);

}  // namespace fp8mla
