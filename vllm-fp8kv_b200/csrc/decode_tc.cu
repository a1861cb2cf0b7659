// decode_tc.cu -- tcgen05/TMEM sparse MLA decode for 128 heads per kv group.
//
// All 128 heads of a kv group share the gathered latent rows, so the heads
// are the MMA M dimension (M = 128, one tcgen05 M-tile):
//   S = Q K^T   M=128 heads, N=32 tokens, K=576 (36 k-steps of 16)
//   O += P V    M=128 heads, N=256 output dims, K=32 tokens
// A 128 x 512 fp32 O fills a whole SM's tensor memory, so each (token, group)
// runs on two CTAs: CTA r accumulates O[:, 256r : 256r+256) and both compute
// the full S (no cross-SM traffic; the second CTA's row reads hit L2).
//
// An MMA that accumulates into the tile the previous MMA wrote waits for it
// (~190 cycles on B200, whatever N), so a single 36-step QK^T chain would leave
// the tensor pipe idle most of the time.  Each tile's QK^T is therefore split
// into 3 independent partial accumulators over disjoint 192-dim slices of
// d=576, issued interleaved, and the previous tile's PV is slipped into the
// same stream as soon as its P is ready; the softmax adds the 3 partials.
//
// Tensor-memory map (512 columns):
//   [  0,256)  O (fp32)
//   [256,448)  2 S buffers x 3 partials x 32 fp32 columns; P (bf16x2) is
//              written over partial 0 of its buffer
//   [448,512)  Q dims [0,128) as the A operand of the TMEM-A MMA (bf16x2)
// Q dims [128,576) live in shared memory (7 x 64-dim 128B-swizzled blocks).
//
// Warp roles (416 threads):
//   warps 0-3   softmax + epilogue: thread i owns head i = TMEM lane i, so the
//               row max / sum / lazy rescale of its O row need no cross-thread
//               reduction.  The reference max is only raised when a tile
//               exceeds it by more than 8 (log2 units); P <= 2^8 keeps its
//               bf16 precision and the final 1/l and LSE use the same max.
//   warp 4      TMEM allocation and the single-thread MMA issuer
//   warps 5-12  gather + dequant: each warp owns 4 of the 32 rows of a tile and
//               loads them straight into registers two tiles ahead (no load is
//               issued for a masked slot), then writes bf16(e4m3 * scale) and
//               the raw rope into a 128B-swizzled tile that is the K-major B
//               operand of QK^T and, read MN-major, the V operand of PV.
// Every mbarrier wait is bounded; a timeout sets g_device_status, the roles
// drain what they issued and the CTA frees its tensor memory and returns.
//
// Reference semantics: vllm_fp8kv/fp8_ds_mla_sparse_decode.py:77-211 (masking,
// dequant, NaN-free online softmax, LSE) and the split/merge contract of
// tests/fixtures/triton_mla_sparse_kernel_pr47629.py:232-403.
#include "common.cuh"
#include "decode.h"
#include "tc_ptx.cuh"

namespace fp8mla {
namespace tc {

namespace {

constexpr int kHeads = 128;
constexpr int kN = 32;             // tokens per tile
constexpr int kChains = 3;         // independent partial-S accumulators per tile
constexpr int kStepsPerChain = 12; // 36 k-steps / 3
constexpr int kKStages = 3;        // dequantized tile stages
constexpr int kDv = 256;           // output dims per CTA
constexpr int kQTmemSteps = 8;     // k-steps 0..7 (q dims 0..127) read A from tensor memory
constexpr int kQSmemBlocks = 7;    // q dims [128,576) as 7 x 64-dim swizzled blocks
constexpr int kKBlocks = 9;        // 576 dims = 9 x 64-dim blocks
constexpr int kKBlockBytes = kN * 128;                // 4096
constexpr int kKTileBytes = kKBlocks * kKBlockBytes;  // 36864
constexpr int kQBlockBytes = kHeads * 128;            // 16384
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kFirstLoadWarp = 5;
constexpr int kLoadWarps = 8;
constexpr int kThreads = (kSoftmaxWarps + 1 + kLoadWarps) * 32;  // 416
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256, kColQ = 448;
constexpr uint32_t kSBufCols = kChains * kN;  // 96
constexpr float kRescaleThreshold = 8.0f;

constexpr uint32_t kIdescQK = idesc_bf16(128, kN, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, kDv, true);

struct Smem {
  uint8_t q[kQSmemBlocks * kQBlockBytes];     // 1024-aligned (offset 0)
  uint8_t k[kKStages][kKTileBytes];           // 1024-aligned
  uint8_t vnib[kKStages][kLoadWarps];         // validity of 4 rows per load warp
  uint64_t kfull[kKStages], kempty[kKStages];
  uint64_t sfull[2], pfull[2], sfree[2];
  uint64_t qready, ofull, drain;
  uint32_t tmem_base;
};
static_assert(offsetof(Smem, k) % 1024 == 0, "swizzle atoms need 1024-B alignment");
static_assert(kKTileBytes % 1024 == 0 && kQBlockBytes % 1024 == 0, "");
static_assert(offsetof(Smem, kfull) % 8 == 0, "");
static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory budget");

// byte offset of the 16-byte chunk `c` (0..7) of row `r` in a 128B-swizzled block
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

// One load-warp lane's share of a row: fp8 chunks p, p+8, p+16, p+24, rope chunk p,
// and the row's 4 tile scales.
struct RowPart {
  uint4 f[4];
  uint4 rope;
  uint4 sc;
};

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) decode_tc_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the dynamic window is only guaranteed 16-B aligned: round up to 1024
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pairs_per_token = a.G * 2;
  const int64_t t = blockIdx.x / pairs_per_token;
  const int grp = (blockIdx.x % pairs_per_token) >> 1;
  const int half = blockIdx.x & 1;
  const int split = blockIdx.y;
  const int beg = split * a.split_len;
  const int end = min(a.topk, beg + a.split_len);
  const int ntiles = end > beg ? (end - beg + kN - 1) / kN : 0;
  const int32_t* idx_row = a.idx + t * a.idx_st + grp * a.idx_sg;
  const int head0 = grp * kHeads;

  const uint32_t sq = smem_u32(s.q);
  const uint32_t sk0 = smem_u32(s.k[0]);
  const uint32_t b_kfull = smem_u32(&s.kfull[0]), b_kempty = smem_u32(&s.kempty[0]);
  const uint32_t b_sfull = smem_u32(&s.sfull[0]), b_pfull = smem_u32(&s.pfull[0]);
  const uint32_t b_sfree = smem_u32(&s.sfree[0]);
  const uint32_t b_qready = smem_u32(&s.qready), b_ofull = smem_u32(&s.ofull);
  const uint32_t b_drain = smem_u32(&s.drain);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(b_kfull + 8 * i, kLoadWarps * 32);
      mbar_init(b_kempty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(b_sfull + 8 * i, 1);
      mbar_init(b_pfull + 8 * i, kSoftmaxWarps * 32);
      mbar_init(b_sfree + 8 * i, 1);
    }
    mbar_init(b_qready, kSoftmaxWarps * 32);
    mbar_init(b_ofull, 1);
    mbar_init(b_drain, 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&s.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp < kSoftmaxWarps) {
    // ================================================= softmax + epilogue
    const int h = threadIdx.x;                       // head within the group = TMEM lane
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    // ---- Q: dims [0,128) -> TMEM (A operand), dims [128,576) -> swizzled smem
    {
      const uint4* qsrc = reinterpret_cast<const uint4*>(
          static_cast<const uint16_t*>(a.q) + t * a.q_st + (int64_t)(head0 + h) * a.q_sh);
#pragma unroll
      for (int c0 = 0; c0 < kQTmemSteps * 8; c0 += 32) {   // 32 packed columns per store
        uint32_t w[32];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const uint4 x = qsrc[c0 / 4 + v];
          w[4 * v] = x.x;
          w[4 * v + 1] = x.y;
          w[4 * v + 2] = x.z;
          w[4 * v + 3] = x.w;
        }
        tmem_st32(trow + kColQ + c0, w);
      }
#pragma unroll
      for (int blk = 0; blk < kQSmemBlocks; ++blk)
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(s.q + blk * kQBlockBytes + swz(h, c)) =
              qsrc[kQTmemSteps * 2 + blk * 8 + c];
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(b_qready);
    }

    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int b = j & 1, ks = j % kKStages;
      ok = warp_wait(b_sfull + 8 * b, (j >> 1) & 1, 1);
      if (!ok) break;
      ok = warp_wait(b_kfull + 8 * ks, (j / kKStages) & 1, 2);  // orders the validity nibbles
      if (!ok) break;
      tc_fence_after();
      const uint32_t sb = trow + kColS + kSBufCols * b;
      uint32_t s0[32], s1[32], s2[32];
      tmem_ld32(sb, s0);
      tmem_ld32(sb + kN, s1);
      tmem_ld32(sb + 2 * kN, s2);
      const uint2 nib = *reinterpret_cast<const uint2*>(s.vnib[ks]);
      uint32_t vmask = 0;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        vmask |= ((nib.x >> (8 * w)) & 0xFu) << (4 * w);
        vmask |= ((nib.y >> (8 * w)) & 0xFu) << (16 + 4 * w);
      }
      tmem_wait_ld();
      float x[32];
      float tmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float sv = __uint_as_float(s0[i]) + __uint_as_float(s1[i]) + __uint_as_float(s2[i]);
        x[i] = ((vmask >> i) & 1u) ? sv * a.scale_log2 : -INFINITY;
        tmax = fmaxf(tmax, x[i]);
      }
      // lazy reference max: raise it only when this tile exceeds it by > threshold
      float alpha = 1.f;
      if (tmax > m_used + kRescaleThreshold || (m_used == -INFINITY && tmax > -INFINITY)) {
        alpha = (m_used == -INFINITY) ? 1.f : ex2_approx(m_used - tmax);
        m_used = tmax;
        l *= alpha;
      }
      // O rows with alpha < 1 need rescaling once PV(j-1) has finished writing O
      if (__any_sync(0xFFFFFFFFu, alpha != 1.f) && j > 0) {
        ok = warp_wait(b_sfree + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1, 3);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < kDv; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(trow + kColO + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(trow + kColO + c0, o);
        }
      }
      // nothing valid yet: every x is -inf, use 0 so exp2(-inf - ref) is 0, not NaN
      const float mref = (m_used == -INFINITY) ? 0.f : m_used;
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float p0 = ex2_approx(x[2 * i] - mref), p1 = ex2_approx(x[2 * i + 1] - mref);
        l += p0 + p1;
        pk[i] = pack_bf16x2(p0, p1);
      }
      tmem_st16(sb, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(b_pfull + 8 * b);
    }

    // ---- epilogue
    const bool have_o = ok && ntiles > 0 && warp_wait(b_ofull, 0, 4);
    if (have_o) tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float lse_v = l > 0.f ? m_used * kLn2 + logf(l) : -INFINITY;
    const int hh = head0 + h;
#pragma unroll 1
    for (int c0 = 0; c0 < kDv; c0 += 32) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld32(trow + kColO + c0, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      const int d = half * kDv + c0;
      if (a.num_splits == 1) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + t * a.out_st +
                                              (int64_t)hh * a.out_sh + d);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            w[u] = pack_bf16x2(__uint_as_float(o[8 * v + 2 * u]) * inv,
                               __uint_as_float(o[8 * v + 2 * u + 1]) * inv);
          dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
        float4* dst = reinterpret_cast<float4*>(
            a.ws_o + ((t * a.H + hh) * a.num_splits + split) * kNope + d);
#pragma unroll
        for (int v = 0; v < 8; ++v)
          dst[v] = make_float4(__uint_as_float(o[4 * v]) * inv, __uint_as_float(o[4 * v + 1]) * inv,
                               __uint_as_float(o[4 * v + 2]) * inv,
                               __uint_as_float(o[4 * v + 3]) * inv);
      }
    }
    if (half == 0) {
      if (a.num_splits == 1) {
        if (a.lse != nullptr) a.lse[t * a.lse_st + hh] = lse_v;
      } else {
        a.ws_lse[(t * a.H + hh) * a.num_splits + split] = lse_v;
      }
    }
  } else if (warp == kMmaWarp) {
    // ================================================= MMA issuer
    if (lane == 0) {
      bool ok = thread_wait(b_qready, 0, 5);
      tc_fence_after();
      const uint32_t tO = tmem + kColO, tQ = tmem + kColQ;
      const uint64_t kdesc0 = sdesc_sw128(sk0, 16, 1024);
      const uint64_t qdesc0 = sdesc_sw128(sq, 16, 1024);
      const uint64_t vdesc0 =
          sdesc_sw128(sk0 + (uint32_t)half * 4u * kKBlockBytes, kKBlockBytes, 1024);
      int pv_next = 0;  // first tile whose PV is not issued yet
      auto issue_pv = [&](int jj) {
        const int bb = jj & 1, kss = jj % kKStages;
        tc_fence_after();
        const uint32_t pa = tmem + kColS + kSBufCols * bb;
        const uint64_t vd = vdesc0 + (uint64_t)((kss * kKTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk)
          mma_ts(tO, pa + 8 * kk, vd + (uint64_t)((kk * 2048) >> 4), kIdescPV,
                 (jj > 0 || kk > 0) ? 1u : 0u);
        mma_commit(b_sfree + 8 * bb);
        mma_commit(b_kempty + 8 * kss);
        pv_next = jj + 1;
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        const int b = j & 1, ks = j % kKStages;
        ok = thread_wait(b_kfull + 8 * ks, (j / kKStages) & 1, 7);
        if (ok && j >= 2) ok = thread_wait(b_sfree + 8 * b, ((j - 2) >> 1) & 1, 8);
        if (!ok) break;
        tc_fence_after();
        const uint32_t tS = tmem + kColS + kSBufCols * b;
        const uint64_t kd = kdesc0 + (uint64_t)((ks * kKTileBytes) >> 4);
#pragma unroll
        for (int i = 0; i < kStepsPerChain; ++i) {
#pragma unroll
          for (int c = 0; c < kChains; ++c) {
            const int kst = c * kStepsPerChain + i;
            const uint64_t bdesc =
                kd + (uint64_t)((((kst >> 2) * kKBlockBytes) + (kst & 3) * 32) >> 4);
            const uint32_t acc = i > 0 ? 1u : 0u;
            if (kst < kQTmemSteps) {
              mma_ts(tS + kN * c, tQ + 8 * kst, bdesc, kIdescQK, acc);
            } else {
              const int qs = kst - kQTmemSteps;
              const uint64_t adesc =
                  qdesc0 + (uint64_t)((((qs >> 2) * kQBlockBytes) + (qs & 3) * 32) >> 4);
              mma_ss(tS + kN * c, adesc, bdesc, kIdescQK, acc);
            }
          }
          // slip the previous tile's PV in as soon as its P is ready
          if ((i & 3) == 3 && pv_next == j - 1 &&
              mbar_test(b_pfull + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1))
            issue_pv(j - 1);
        }
        mma_commit(b_sfull + 8 * b);
        if (pv_next == j - 1) {
          ok = thread_wait(b_pfull + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1, 6);
          if (!ok) break;
          issue_pv(j - 1);
        }
      }
      if (ok && ntiles > 0) {
        ok = thread_wait(b_pfull + 8 * ((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1, 6);
        if (ok) {
          issue_pv(ntiles - 1);
          mma_commit(b_ofull);
        }
      }
      // drain: nothing this thread issued may still touch tensor memory
      mma_commit(b_drain);
      thread_wait(b_drain, 0, 9);
    }
    __syncwarp();
  } else {
    // ================================================= gather + dequant
    const int lw = warp - kFirstLoadWarp;       // 0..7, owns rows 4lw..4lw+3 of each tile
    const int r = lane & 3, p = lane >> 2;      // row within the 4, 16-byte part 0..7
    const int row = lw * 4 + r;
    auto load = [&](int jt, RowPart& P, bool& valid) {
      const int pos = beg + jt * kN + row;
      int64_t slot = -1;
      if (pos < end) {
        const int32_t v = idx_row[pos];
        if (v >= 0 && (int64_t)v < a.num_slots) slot = v;
      }
      valid = slot >= 0;
      if (valid) {
        const uint8_t* src = a.kv + slot * (int64_t)kRowBytes;
#pragma unroll
        for (int i = 0; i < 4; ++i) P.f[i] = ldg_nc_v4(src + (p + 8 * i) * 16);
        P.rope = ldg_nc_v4(src + kRopeOff + 16 * p);
        P.sc = ldg_nc_v4(src + kScaleOff);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) P.f[i] = make_uint4(0, 0, 0, 0);
        P.rope = make_uint4(0, 0, 0, 0);
        P.sc = make_uint4(0, 0, 0, 0);
      }
    };
    bool ok = true;
    auto step = [&](int j, const RowPart& cur, bool vcur, RowPart& nxt2, bool& vnxt2) {
      if (!ok || j >= ntiles) return;
      if (j + 2 < ntiles) load(j + 2, nxt2, vnxt2);
      const int ks = j % kKStages;
      if (j >= kKStages) ok = warp_wait(b_kempty + 8 * ks, ((j / kKStages) + 1) & 1, 10);
      if (!ok) return;
      uint8_t* ktile = s.k[ks];
      const float scl[4] = {__uint_as_float(cur.sc.x), __uint_as_float(cur.sc.y),
                            __uint_as_float(cur.sc.z), __uint_as_float(cur.sc.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c8 = p + 8 * i;                  // fp8 16-byte chunk = dims 16*c8 .. +15
        float sx;
        bool fused;
        prep_scale(scl[i], sx, fused);
        uint4 o0, o1;
        dequant4_bf16(cur.f[i].x, sx, fused, o0.x, o0.y);
        dequant4_bf16(cur.f[i].y, sx, fused, o0.z, o0.w);
        dequant4_bf16(cur.f[i].z, sx, fused, o1.x, o1.y);
        dequant4_bf16(cur.f[i].w, sx, fused, o1.z, o1.w);
        uint8_t* blk = ktile + (c8 >> 2) * kKBlockBytes;
        const uint32_t c0 = (uint32_t)(c8 & 3) * 2u;
        *reinterpret_cast<uint4*>(blk + swz(row, c0)) = o0;
        *reinterpret_cast<uint4*>(blk + swz(row, c0 + 1)) = o1;
      }
      *reinterpret_cast<uint4*>(ktile + 8 * kKBlockBytes + swz(row, p)) = cur.rope;
      const uint32_t vb = __ballot_sync(0xFFFFFFFFu, p == 0 && vcur);  // bits 0..3 = rows 4lw..+3
      if (lane == 0) s.vnib[ks][lw] = (uint8_t)(vb & 0xFu);
      fence_proxy_async_smem();
      mbar_arrive(b_kfull + 8 * ks);
    };
    RowPart A, B, C;
    bool vA = false, vB = false, vC = false;
    if (ntiles > 0) load(0, A, vA);
    if (ntiles > 1) load(1, B, vB);
    for (int j = 0; j < ntiles && ok; j += 3) {
      step(j, A, vA, C, vC);
      step(j + 1, B, vB, A, vA);
      step(j + 2, C, vC, B, vB);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc

bool decode_tc_supported(const DecodeArgs& a) {
  return a.q_dtype == FP8MLA_DTYPE_BF16 && a.hpg == tc::kHeads && a.G >= 1;
}

int launch_decode_tc(const DecodeArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(tc::Smem) + 1024;  // + alignment slack
  cudaError_t e = cudaFuncSetAttribute(tc::decode_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "decode_tc smem attribute");
  dim3 grid((unsigned)(a.T * a.G * 2), a.num_splits);
  tc::decode_tc_kernel<<<grid, tc::kThreads, smem, st>>>(a);
  int rc = check_cuda(cudaGetLastError(), "decode_tc_kernel launch");
  if (rc != FP8MLA_OK || a.num_splits == 1) return rc;
  return launch_merge_splits(a, st);
}

int read_device_status(unsigned int* status, bool reset, cudaStream_t st) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, tc::g_device_status, sizeof(v), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && reset && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(tc::g_device_status, &zero, sizeof(zero), 0,
                                cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  *status = v;
  return check_cuda(e, "device status read");
}

}  // namespace fp8mla
