// unit_kernels.cu -- the small kernels around the decode:
//   * e4m3fn byte decode (unit test of the fused decode's dequant),
//   * gather + dequant of fp8_ds_mla rows with the decode's own device dequant,
//   * the fp8_ds_mla cache writer,
//   * the block-table -> flat slot index converter.
// All are HBM-bound integer/byte work; grids are sized in multiples of the SM
// count and every access is coalesced 16-byte or 4-byte traffic.
#include "common.cuh"

namespace fp8mla {

// ============================================================= e4m3 decode
// Reference: vllm_fp8kv/fp8_dequant.py:80-113 (`dequant_bitmath_triton`,
// `_dequant_test_kernel`).  method 0: packed hardware cvt e4m3x2 -> f16x2;
// method 1: the integer bit-math of dequant4_bf16 (scale 1).
template <int kOut>  // FP8MLA_DTYPE_*
__global__ void dequant_e4m3_kernel(const uint8_t* __restrict__ in, int64_t n,
                                    void* __restrict__ out, int method) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint32_t b = in[i];
    float v;
    if (method == 0) {
      uint32_t h2;
      uint16_t pair = (uint16_t)b;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(h2) : "h"(pair));
      __half h = __ushort_as_half((unsigned short)(h2 & 0xFFFFu));
      if (kOut == FP8MLA_DTYPE_F16) {
        static_cast<__half*>(out)[i] = h;
        continue;
      }
      v = __half2float(h);
    } else {
      uint32_t lo, hi;
      dequant4_bf16(b, 1.0f, false, lo, hi);  // exact: every e4m3 value fits bf16
      v = e4m3_to_f32(b);
      if (kOut == FP8MLA_DTYPE_BF16) {
        static_cast<uint16_t*>(out)[i] = (uint16_t)(lo & 0xFFFFu);
        continue;
      }
    }
    if (kOut == FP8MLA_DTYPE_F32) {
      static_cast<float*>(out)[i] = v;
    } else if (kOut == FP8MLA_DTYPE_F16) {
      static_cast<__half*>(out)[i] = __float2half_rn(v);
    } else {
      static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    }
  }
}

// ============================================================= row gather + dequant
// The decode kernels' in-register dequant, run on its own: rows gathered by
// slot (int64 byte offsets; slot -1 or >= num_slots gives a zero row), latent
// bf16(e4m3 * tile scale) through the same device function the decode uses
// (method 1: dequant4_hw_x2, the packed-multiply form both decode kernels use;
// method 0: dequant4_hw, the same arithmetic unpacked), rope copied raw.  Reference: the IS_FP8 gather and
// dequant of vllm_fp8kv/fp8_ds_mla_sparse_decode.py:136-168 (exact fp32 decode,
// times the fp32 tile scale, rounded to the query dtype bf16).
// One thread per 16-byte chunk: chunks 0..31 of a row are latent (16 values,
// tile c/8), chunks 32..39 the rope.
template <int kMethod>
__global__ void dequant_rows_kernel(const uint8_t* __restrict__ kv, int64_t num_slots,
                                    const int32_t* __restrict__ slots, int64_t n,
                                    uint16_t* __restrict__ out, int64_t out_stride) {
  constexpr int kChunks = kNope / 16 + kRope * 2 / 16;  // 32 + 8
  const int64_t total = n * kChunks;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / kChunks;
    const int c = (int)(i - r * kChunks);
    const int32_t slot = slots[r];
    const bool valid = slot >= 0 && (int64_t)slot < num_slots;
    const uint8_t* row = kv + (valid ? (int64_t)slot : 0) * (int64_t)kRowBytes;
    uint16_t* dst = out + r * out_stride;
    if (c < kNope / 16) {
      uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
      if (valid) {
        const uint4 w = *reinterpret_cast<const uint4*>(row + 16 * c);
        const float sc = reinterpret_cast<const float*>(row + kScaleOff)[c / 8];
        if (kMethod == 0) {
          dequant4_hw(w.x, sc, o0.x, o0.y);
          dequant4_hw(w.y, sc, o0.z, o0.w);
          dequant4_hw(w.z, sc, o1.x, o1.y);
          dequant4_hw(w.w, sc, o1.z, o1.w);
        } else {
          dequant4_hw_x2(w.x, sc, o0.x, o0.y);
          dequant4_hw_x2(w.y, sc, o0.z, o0.w);
          dequant4_hw_x2(w.z, sc, o1.x, o1.y);
          dequant4_hw_x2(w.w, sc, o1.z, o1.w);
        }
      }
      reinterpret_cast<uint4*>(dst + 16 * c)[0] = o0;
      reinterpret_cast<uint4*>(dst + 16 * c)[1] = o1;
    } else {
      const int rc = c - kNope / 16;
      const uint4 v = valid ? *reinterpret_cast<const uint4*>(row + kRopeOff + 16 * rc)
                            : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(dst + kNope + 8 * rc) = v;
    }
  }
}

// ============================================================= cache writer
// fp32 -> e4m3fn byte with torch's semantics (round to nearest even; values
// that round past 448, inf and NaN give 0x7F | sign).  Written from the IEEE
// definition; the CPU oracle states the same rule.
__device__ __forceinline__ uint32_t f32_to_e4m3(float x) {
  uint32_t u = __float_as_uint(x);
  uint32_t sign = (u >> 24) & 0x80u;
  uint32_t a = u & 0x7FFFFFFFu;
  uint32_t r;
  if (a >= 0x43F00000u) {  // >= 480, inf, NaN
    r = 0x7Fu;
  } else if (a < 0x3C800000u) {  // < 2^-6: subnormal range, units of 2^-9
    r = (uint32_t)__float2int_rn(__uint_as_float(a) * 512.0f);
  } else {
    uint32_t e = (a >> 23) - 127u + 7u;
    uint32_t mant = a & 0x7FFFFFu;
    uint32_t keep = mant >> 20, rem = mant & 0xFFFFFu;
    keep += (rem > 0x80000u || (rem == 0x80000u && (keep & 1u))) ? 1u : 0u;
    r = (e << 3) + keep;  // a carry out of the mantissa bumps the exponent
  }
  return r | sign;
}

// Two values x0 (low byte), x1 (high byte) -> e4m3fn with the hardware's
// round-to-nearest-even conversion.  Its saturation (to +-448) differs from
// f32_to_e4m3 (0x7F from 464 up) only for |x| >= 464 and it does not keep NaN
// signs; the writer uses it only on tiles with a finite scale (no NaN or inf
// in the tile), where |x / scale| <= 448 * (1 + 2^-24) because
// scale = RN(amax / 448) (or FLT_MIN, larger).
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float x0, float x1) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(r) : "f"(x1), "f"(x0));
  return r;
}

// One warp per token: lane l owns latent elements [16l, 16l+16) (tile l/8),
// reduces amax over its tile with 8-lane shuffles, divides, converts, and
// writes 16 bytes; lanes 0..3 write the 4 scales, lanes 0..7 copy the rope.
// A warp's next token is loaded before the current one is converted.
// Reference semantics: tests/fakes.py:28-57, verify/reference.py:68-91.
struct WriterIn {
  int64_t slot;
  uint32_t w[8];  // 16 bf16 latent values
  uint4 rope;     // lanes 0..7: 8 bf16 rope values
};
__device__ __forceinline__ void writer_load(WriterIn& in, const uint16_t* __restrict__ kv_c,
                                            int64_t kv_c_stride, const uint16_t* __restrict__ k_pe,
                                            int64_t k_pe_stride, const int64_t* __restrict__ slot_mapping,
                                            int64_t tok, int lane, bool vec_c, bool vec_pe) {
  in.slot = slot_mapping[tok];
  const uint16_t* src = kv_c + tok * kv_c_stride + lane * 16;
  if (vec_c) {
    const uint4 a = reinterpret_cast<const uint4*>(src)[0];
    const uint4 b = reinterpret_cast<const uint4*>(src)[1];
    in.w[0] = a.x; in.w[1] = a.y; in.w[2] = a.z; in.w[3] = a.w;
    in.w[4] = b.x; in.w[5] = b.y; in.w[6] = b.z; in.w[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) in.w[j] = (uint32_t)src[2 * j] | ((uint32_t)src[2 * j + 1] << 16);
  }
  in.rope = make_uint4(0, 0, 0, 0);
  if (lane < 8) {
    const uint16_t* r = k_pe + tok * k_pe_stride + lane * 8;
    if (vec_pe) {
      in.rope = *reinterpret_cast<const uint4*>(r);
    } else {
      in.rope.x = (uint32_t)r[0] | ((uint32_t)r[1] << 16);
      in.rope.y = (uint32_t)r[2] | ((uint32_t)r[3] << 16);
      in.rope.z = (uint32_t)r[4] | ((uint32_t)r[5] << 16);
      in.rope.w = (uint32_t)r[6] | ((uint32_t)r[7] << 16);
    }
  }
}

__global__ void __launch_bounds__(256) ds_mla_write_kernel(
    const uint16_t* __restrict__ kv_c, int64_t kv_c_stride, const uint16_t* __restrict__ k_pe,
    int64_t k_pe_stride, const int64_t* __restrict__ slot_mapping, int64_t N,
    uint8_t* __restrict__ cache, int64_t num_slots) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x / 32);
  const bool vec_c = (kv_c_stride % 8) == 0 && (reinterpret_cast<uintptr_t>(kv_c) & 15) == 0;
  const bool vec_pe = (k_pe_stride % 8) == 0 && (reinterpret_cast<uintptr_t>(k_pe) & 15) == 0;
  int64_t tok = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  WriterIn cur, nxt;
  if (tok < N) writer_load(cur, kv_c, kv_c_stride, k_pe, k_pe_stride, slot_mapping, tok, lane, vec_c, vec_pe);
  for (; tok < N; tok += warps_total) {
    if (tok + warps_total < N)
      writer_load(nxt, kv_c, kv_c_stride, k_pe, k_pe_stride, slot_mapping, tok + warps_total, lane,
                  vec_c, vec_pe);
    const int64_t slot = cur.slot;
    if (slot >= 0 && slot < num_slots) {  // else a padding token
      float x[16];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        x[2 * j] = bf16_lo(cur.w[j]);
        x[2 * j + 1] = bf16_hi(cur.w[j]);
      }
      // amax over the tile (NaN sticky, as torch's amax)
      float amax = 0.0f;
      bool nan = false;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float v = fabsf(x[j]);
        nan |= (v != v);
        amax = fmaxf(amax, v);
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
        nan |= __shfl_xor_sync(0xFFFFFFFFu, (int)nan, off) != 0;
      }
      float scale = nan ? __uint_as_float(0x7FC00000u) : __fdiv_rn(amax, 448.0f);
      if (!nan && scale < 1.1754944e-38f) scale = 1.1754944e-38f;
      uint32_t q[4];
      if (scale < INFINITY) {  // finite: no NaN or inf in the tile
#pragma unroll
        for (int j = 0; j < 4; ++j)
          q[j] = f32x2_to_e4m3x2(__fdiv_rn(x[4 * j + 0], scale), __fdiv_rn(x[4 * j + 1], scale)) |
                 (f32x2_to_e4m3x2(__fdiv_rn(x[4 * j + 2], scale), __fdiv_rn(x[4 * j + 3], scale)) << 16);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t b0 = f32_to_e4m3(__fdiv_rn(x[4 * j + 0], scale));
          uint32_t b1 = f32_to_e4m3(__fdiv_rn(x[4 * j + 1], scale));
          uint32_t b2 = f32_to_e4m3(__fdiv_rn(x[4 * j + 2], scale));
          uint32_t b3 = f32_to_e4m3(__fdiv_rn(x[4 * j + 3], scale));
          q[j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
      }
      uint8_t* row = cache + slot * (int64_t)kRowBytes;
      reinterpret_cast<uint4*>(row)[lane] = make_uint4(q[0], q[1], q[2], q[3]);
      if ((lane & 7) == 0) reinterpret_cast<float*>(row + kScaleOff)[lane >> 3] = scale;
      if (lane < 8) reinterpret_cast<uint4*>(row + kRopeOff)[lane] = cur.rope;
    }
    cur = nxt;
  }
}

// ============================================================= index convert
// out[t, i] = block_table[req_id[t], tok / B] * B + tok % B; -1 when tok < 0 or
// the block index is outside [0, max_blocks).  int32 arithmetic, as vLLM's
// converter (installed vllm/v1/attention/backends/mla/sparse_utils.py:11-78).
__global__ void convert_req_index_kernel(const int32_t* __restrict__ req_id,
                                         const int32_t* __restrict__ block_table,
                                         int64_t bt_stride, int64_t max_blocks,
                                         const int32_t* __restrict__ token_idx,
                                         int64_t ti_stride, int64_t T, int64_t topk,
                                         int32_t block_size, int32_t* __restrict__ out,
                                         int64_t out_stride) {
  const int64_t total = T * topk;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
    const int64_t t = e / topk, i = e - t * topk;
    const int32_t tok = token_idx[t * ti_stride + i];
    int32_t r = -1;
    if (tok >= 0) {
      const int32_t blk = tok / block_size, off = tok - blk * block_size;
      if (blk < max_blocks) {
        const uint32_t base = (uint32_t)block_table[(int64_t)req_id[t] * bt_stride + blk];
        r = (int32_t)(base * (uint32_t)block_size + (uint32_t)off);
      }
    }
    out[t * out_stride + i] = r;
  }
}

// ============================================================= launchers
static int grid_for(int64_t work, int block) {
  int64_t sms = device_sm_count();
  int64_t want = (work + block - 1) / block;
  int64_t cap = sms * 16;
  if (want > cap) want = cap;
  return (int)(want < 1 ? 1 : want);
}

int launch_dequant(const uint8_t* in, int64_t n, void* out, int out_dtype, int method,
                   cudaStream_t st) {
  if (n == 0) return FP8MLA_OK;
  const int block = 256;
  const int grid = grid_for(n, block);
  switch (out_dtype) {
    case FP8MLA_DTYPE_F16:
      dequant_e4m3_kernel<FP8MLA_DTYPE_F16><<<grid, block, 0, st>>>(in, n, out, method);
      break;
    case FP8MLA_DTYPE_BF16:
      dequant_e4m3_kernel<FP8MLA_DTYPE_BF16><<<grid, block, 0, st>>>(in, n, out, method);
      break;
    default:
      dequant_e4m3_kernel<FP8MLA_DTYPE_F32><<<grid, block, 0, st>>>(in, n, out, method);
  }
  return check_cuda(cudaGetLastError(), "dequant_e4m3_kernel launch");
}

int launch_dequant_rows(const uint8_t* kv, int64_t num_slots, const int32_t* slots, int64_t n,
                        uint16_t* out, int64_t out_stride, int method, cudaStream_t st) {
  if (n == 0) return FP8MLA_OK;
  const int block = 256;
  const int grid = grid_for(n * 40, block);
  if (method == 0)
    dequant_rows_kernel<0><<<grid, block, 0, st>>>(kv, num_slots, slots, n, out, out_stride);
  else
    dequant_rows_kernel<1><<<grid, block, 0, st>>>(kv, num_slots, slots, n, out, out_stride);
  return check_cuda(cudaGetLastError(), "dequant_rows_kernel launch");
}

int launch_ds_mla_write(const uint16_t* kv_c, int64_t kv_c_stride, const uint16_t* k_pe,
                        int64_t k_pe_stride, const int64_t* slot_mapping, int64_t N,
                        uint8_t* cache, int64_t num_slots, cudaStream_t st) {
  if (N == 0) return FP8MLA_OK;
  const int block = 256;  // 8 tokens per block
  const int grid = grid_for(N * 32, block);
  ds_mla_write_kernel<<<grid, block, 0, st>>>(kv_c, kv_c_stride, k_pe, k_pe_stride,
                                              slot_mapping, N, cache, num_slots);
  return check_cuda(cudaGetLastError(), "ds_mla_write_kernel launch");
}

int launch_convert_req_index(const int32_t* req_id, const int32_t* block_table,
                             int64_t bt_stride, int64_t max_blocks, const int32_t* token_idx,
                             int64_t ti_stride, int64_t T, int64_t topk, int64_t block_size,
                             int32_t* out, int64_t out_stride, cudaStream_t st) {
  if (T * topk == 0) return FP8MLA_OK;
  const int block = 256;
  const int grid = grid_for(T * topk, block);
  convert_req_index_kernel<<<grid, block, 0, st>>>(req_id, block_table, bt_stride, max_blocks,
                                                   token_idx, ti_stride, T, topk,
                                                   (int32_t)block_size, out, out_stride);
  return check_cuda(cudaGetLastError(), "convert_req_index_kernel launch");
}

}  // namespace fp8mla
