/*
 * fp8mla_oracle.c -- CPU restatement of the fp8_ds_mla byte/integer arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, the
 * smoke check and the bench's CPU-baseline leg compare the CUDA library
 * against.  Nothing in the product links or calls it.
 *
 * Each function restates the reference's algorithm (nickus/vllm-fp8kv, which is
 * Python/torch) in plain C, citing the file:line it follows.  Its outputs are
 * pinned against golden vectors produced by the reference itself
 * (tests/golden/make_golden.py).
 *
 * Build: oracle/Makefile -> oracle/_build/libfp8mla_oracle.so
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define NOPE 512
#define ROPE 64
#define TILE 128
#define N_TILES (NOPE / TILE)
#define ROW_BYTES 656
#define SCALE_OFF 512
#define ROPE_OFF 528

static uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static float bits_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/*
 * float8_e4m3fn byte -> fp32 value (exact).  e4m3fn has no infinity; the two
 * encodings with all magnitude bits set (0x7F, 0xFF) are NaN.
 * Semantics of `tensor.view(torch.float8_e4m3fn).float()` used by
 * verify/reference.py:28 and vllm_fp8kv/fp8_dequant.py:47-58.
 */
float oracle_e4m3_to_f32(uint8_t b) {
  int sign = b >> 7;
  int e = (b >> 3) & 0xF;
  int m = b & 0x7;
  float v;
  if ((b & 0x7F) == 0x7F) return sign ? -NAN : NAN;
  if (e == 0)
    v = ldexpf((float)m, -9); /* subnormal: m/8 * 2^-6 */
  else
    v = ldexpf((float)(8 + m), e - 10); /* (1 + m/8) * 2^(e-7) */
  return sign ? -v : v;
}

/*
 * fp32 -> float8_e4m3fn byte, round to nearest even, non-saturating: |x| that
 * rounds past 448 (i.e. |x| > 464) and NaN/inf map to 0x7F | sign, the NaN
 * encoding.  Semantics of `tensor.to(torch.float8_e4m3fn)` used by the writer
 * mirror verify/reference.py:83 and tests/fakes.py:47.  Written from the IEEE
 * round-to-nearest-even definition.
 */
uint8_t oracle_f32_to_e4m3(float x) {
  uint32_t u = f32_bits(x);
  uint8_t sign = (uint8_t)((u >> 24) & 0x80);
  uint32_t a = u & 0x7FFFFFFFu;
  uint8_t r;
  if (a >= 0x43F00000u) { /* >= 480.0f, inf, NaN */
    r = 0x7F;
  } else if (a < 0x3C800000u) { /* below 2^-6: e4m3 subnormal range */
    float s = nearbyintf(bits_f32(a) * 512.0f); /* units of 2^-9, RNE */
    r = (uint8_t)s;                             /* 0..8; 8 == 2^-6 */
  } else {
    int e = (int)(a >> 23) - 127; /* -6 .. 8 */
    uint32_t mant = a & 0x7FFFFFu;
    uint32_t keep = mant >> 20, rem = mant & 0xFFFFFu;
    if (rem > 0x80000u || (rem == 0x80000u && (keep & 1u))) keep++;
    if (keep == 8) {
      keep = 0;
      e++;
    }
    r = (uint8_t)(((e + 7) << 3) | keep); /* e+7 <= 15; 0x7F is NaN */
  }
  return r | sign;
}

/*
 * fp32 -> bf16 bits, round to nearest even; NaN -> 0x7FC0.  Semantics of
 * `tensor.to(torch.bfloat16)` (the `.to(q.dtype)` cast in
 * vllm_fp8kv/fp8_ds_mla_sparse_decode.py:164 and :194).
 */
uint16_t oracle_f32_to_bf16(float x) {
  uint32_t u = f32_bits(x);
  if (isnan(x)) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/*
 * Row parser: (n, 656) uint8 -> (n, 576) fp32 [NoPE * tile scale | RoPE raw].
 * Restates verify/reference.py:22-33 (`ref_dequant_fp8_ds_mla_row`): the NoPE
 * element is e4m3 * scale multiplied in fp32; the rope is bf16 widened.
 */
void oracle_dequant_rows(const uint8_t* rows, int64_t n, float* out) {
  static float lut[256];
  static int lut_ready = 0;
  if (!lut_ready) { /* 256-entry table of oracle_e4m3_to_f32 (benign race: same values) */
    for (int b = 0; b < 256; ++b) lut[b] = oracle_e4m3_to_f32((uint8_t)b);
    lut_ready = 1;
  }
  for (int64_t i = 0; i < n; ++i) {
    const uint8_t* r = rows + i * ROW_BYTES;
    float* o = out + i * (NOPE + ROPE);
    float sc[N_TILES];
    memcpy(sc, r + SCALE_OFF, sizeof(sc));
    for (int d = 0; d < NOPE; ++d) o[d] = lut[r[d]] * sc[d / TILE];
    for (int d = 0; d < ROPE; ++d) {
      uint16_t h;
      memcpy(&h, r + ROPE_OFF + 2 * d, 2);
      o[NOPE + d] = oracle_bf16_to_f32(h);
    }
  }
}

/*
 * fp8_ds_mla writer.  Restates the mirror of vLLM's C++
 * `concat_and_cache_ds_mla_kernel` in tests/fakes.py:28-57 and
 * verify/reference.py:68-91:
 *   scale_t = clamp_min(amax(|x_tile|) / 448, FLT_MIN)    (fp32, NaN sticky)
 *   byte    = e4m3(x / scale_t)                          (fp32 division)
 *   rope    = raw bf16 copy
 * Tokens whose slot is < 0 or >= num_slots are skipped (vLLM's padding slot
 * convention; the Python mirror never passes one).
 */
void oracle_ds_mla_write(const uint16_t* kv_c, int64_t kv_c_stride,
                         const uint16_t* k_pe, int64_t k_pe_stride,
                         const int64_t* slot_mapping, int64_t N,
                         uint8_t* cache, int64_t num_slots) {
  for (int64_t i = 0; i < N; ++i) {
    int64_t slot = slot_mapping[i];
    if (slot < 0 || slot >= num_slots) continue;
    uint8_t* row = cache + slot * ROW_BYTES;
    const uint16_t* x = kv_c + i * kv_c_stride;
    for (int t = 0; t < N_TILES; ++t) {
      float amax = 0.0f;
      int has_nan = 0;
      for (int j = 0; j < TILE; ++j) {
        float v = fabsf(oracle_bf16_to_f32(x[t * TILE + j]));
        if (isnan(v)) has_nan = 1;
        else if (v > amax) amax = v;
      }
      float scale = has_nan ? NAN : amax / 448.0f;
      if (!isnan(scale) && scale < 1.1754944e-38f) scale = 1.1754944e-38f;
      for (int j = 0; j < TILE; ++j)
        row[t * TILE + j] = oracle_f32_to_e4m3(oracle_bf16_to_f32(x[t * TILE + j]) / scale);
      memcpy(row + SCALE_OFF + 4 * t, &scale, 4);
    }
    memcpy(row + ROPE_OFF, k_pe + i * k_pe_stride, ROPE * 2);
  }
}

/*
 * Token-relative -> flat global slot.  Restates the documented contract of
 * vLLM's `triton_convert_req_index_to_global_index` (installed
 * vllm/v1/attention/backends/mla/sparse_utils.py:85-104, mirrored by the
 * reference in tests/fakes.py:70-82): block_table[req, tok // B] * B + tok % B,
 * -1 when tok < 0 or the block index is out of [0, max_blocks).  int32
 * arithmetic as in the Triton kernel.
 */
void oracle_convert_req_index(const int32_t* req_id, const int32_t* block_table,
                              int64_t bt_stride, int64_t max_blocks,
                              const int32_t* token_idx, int64_t ti_stride,
                              int64_t T, int64_t topk, int64_t block_size,
                              int32_t* out, int64_t out_stride) {
  for (int64_t t = 0; t < T; ++t) {
    int32_t req = req_id[t];
    for (int64_t i = 0; i < topk; ++i) {
      int32_t tok = token_idx[t * ti_stride + i];
      int32_t r = -1;
      if (tok >= 0) {
        int32_t blk = tok / (int32_t)block_size;
        int32_t off = tok % (int32_t)block_size;
        if (blk < max_blocks) {
          uint32_t base = (uint32_t)block_table[(int64_t)req * bt_stride + blk];
          r = (int32_t)(base * (uint32_t)block_size + (uint32_t)off);
        }
      }
      out[t * out_stride + i] = r;
    }
  }
}

/*
 * Batch helpers for the tests: vectorised e4m3 <-> fp32 and fp32 -> bf16.
 */
void oracle_e4m3_to_f32_n(const uint8_t* in, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_e4m3_to_f32(in[i]);
}
void oracle_f32_to_e4m3_n(const float* in, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_e4m3(in[i]);
}
void oracle_f32_to_bf16_n(const float* in, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_bf16(in[i]);
}
