// common.cuh -- shared definitions for the sm_100a fp8_ds_mla kernels.
//
// Row format (656 bytes per KV slot; reference vllm_fp8kv/fp8_ds_mla_sparse_decode.py:41-47):
//   [  0:512)  512 x float8_e4m3fn  NoPE latent
//   [512:528)    4 x float32        per-128-element tile scales
//   [528:656)   64 x bfloat16       RoPE, raw
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fp8mla.h"

namespace fp8mla {

constexpr int kNope = 512;
constexpr int kRope = 64;
constexpr int kDqk = kNope + kRope;  // 576
constexpr int kTile = 128;
constexpr int kNTiles = kNope / kTile;  // 4
constexpr int kRowBytes = 656;
constexpr int kScaleOff = 512;
constexpr int kRopeOff = 528;
constexpr int kRowChunks16 = kRowBytes / 16;  // 41 16-byte chunks per row
static_assert(kRowBytes % 16 == 0, "rows must be 16-byte granular");

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------- host errors
// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int device_sm_count();
int device_arch(int* major, int* minor);

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async global->shared copy; src_bytes == 0 zero-fills without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D[16x8] += A[16x16] * B[16x8], bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// ---------------------------------------------------------------- e4m3 decode
// Integer bit-math: the 7 magnitude bits of an e4m3fn byte placed at fp32 bits
// [26:20] with the sign at bit 31 give exactly value * 2^-120, for normals and
// subnormals alike (the 4-bit exponent lands in the low bits of the 8-bit
// field; e4m3 subnormals become fp32 subnormals).  Magnitude 0x7F (NaN in
// e4m3fn) is not representable this way and must be patched by the caller.
//   byte k of `w` -> fp32 bits of (e4m3 value * 2^-120)
template <int k>
__device__ __forceinline__ uint32_t e4m3_scaled_bits(uint32_t w) {
  // move byte k to bits [31:24], arithmetic shift right by 4 puts the
  // magnitude at [26:20]; keep the sign (bit 31) and the 7 magnitude bits.
  uint32_t top;
  if (k == 3)
    top = w & 0xFF000000u;
  else
    top = w << (24 - 8 * k);
  int32_t sh = static_cast<int32_t>(top) >> 4;
  return static_cast<uint32_t>(sh) & 0x87F00000u;
}

// Nonzero iff some byte of w is 0x7F or 0xFF (e4m3fn NaN).
__device__ __forceinline__ uint32_t e4m3_has_nan(uint32_t w) {
  return ((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;
}

// Exact fp32 of one e4m3fn byte (NaN for 0x7F / 0xFF).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  if ((b & 0x7Fu) == 0x7Fu) return __uint_as_float(0x7FC00000u | ((b & 0x80u) << 24));
  float v = __uint_as_float(((b & 0x7Fu) << 20) | ((b & 0x80u) << 24));
  return v * 1.329227995784915872903807060280344576e36f;  // * 2^120, exact
}

// Dequantize 4 e4m3 bytes times a tile scale into 2 packed bf16x2:
//   bf16_rn(fp32_rn(e4m3 * scale)), the value the reference feeds its MMA
//   (fp8_ds_mla_sparse_decode.py:152-164: decode, fp32 multiply, cast).
// `scale_x` must be scale * 2^120 when that is finite (`fused` true), else
// the plain scale (`fused` false, two multiplies).  Both give the same fp32
// product: the real value of (e * 2^-120) * (s * 2^120) equals e * s.
__device__ __forceinline__ void dequant4_bf16(uint32_t w, float scale_x, bool fused,
                                              uint32_t& lo, uint32_t& hi) {
  float f0 = __uint_as_float(e4m3_scaled_bits<0>(w));
  float f1 = __uint_as_float(e4m3_scaled_bits<1>(w));
  float f2 = __uint_as_float(e4m3_scaled_bits<2>(w));
  float f3 = __uint_as_float(e4m3_scaled_bits<3>(w));
  if (!fused) {
    const float two120 = 1.329227995784915872903807060280344576e36f;
    f0 *= two120;
    f1 *= two120;
    f2 *= two120;
    f3 *= two120;
  }
  f0 *= scale_x;
  f1 *= scale_x;
  f2 *= scale_x;
  f3 *= scale_x;
  if (__builtin_expect(e4m3_has_nan(w) != 0, 0)) {
    const float qnan = __uint_as_float(0x7FC00000u);
    if (((w >> 0) & 0x7Fu) == 0x7Fu) f0 = qnan;
    if (((w >> 8) & 0x7Fu) == 0x7Fu) f1 = qnan;
    if (((w >> 16) & 0x7Fu) == 0x7Fu) f2 = qnan;
    if (((w >> 24) & 0x7Fu) == 0x7Fu) f3 = qnan;
  }
  lo = pack_bf16x2(f0, f1);
  hi = pack_bf16x2(f2, f3);
}

// Exact bf16(fp32(e4m3) * scale) of the 4 bytes of w: the hardware e4m3x2 ->
// f16x2 conversion is exact (every e4m3 value, subnormals and NaN included, is
// an f16), f16 -> f32 is exact, then one fp32 multiply and one RNE cast, as in
// the reference (fp8_ds_mla_sparse_decode.py:152-164).
__device__ __forceinline__ void dequant4_hw(uint32_t w, float s, uint32_t& lo, uint32_t& hi) {
  uint32_t h01, h23;
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n"
      " cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
      : "=r"(h01), "=r"(h23)
      : "r"(w));
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  lo = pack_bf16x2(f01.x * s, f01.y * s);
  hi = pack_bf16x2(f23.x * s, f23.y * s);
}

// dequant4_hw with the two products of each pair in one packed fp32 multiply
// (mul.rn.f32x2: each lane is an ordinary round-to-nearest fp32 product, so the
// bits equal dequant4_hw's); fewer issue slots for load warps that are
// instruction-bound.
__device__ __forceinline__ void dequant4_hw_x2(uint32_t w, float s, uint32_t& lo, uint32_t& hi) {
  uint32_t h01, h23;
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n"
      " cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
      : "=r"(h01), "=r"(h23)
      : "r"(w));
  float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  const float2 s2 = make_float2(s, s);
  asm("mul.rn.f32x2 %0, %0, %1;\n"
      : "+l"(reinterpret_cast<uint64_t&>(f01))
      : "l"(reinterpret_cast<const uint64_t&>(s2)));
  asm("mul.rn.f32x2 %0, %0, %1;\n"
      : "+l"(reinterpret_cast<uint64_t&>(f23))
      : "l"(reinterpret_cast<const uint64_t&>(s2)));
  lo = pack_bf16x2(f01.x, f01.y);
  hi = pack_bf16x2(f23.x, f23.y);
}



}  // namespace fp8mla
