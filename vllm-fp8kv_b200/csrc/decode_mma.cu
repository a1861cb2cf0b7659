// decode_mma.cu -- split-KV sparse MLA decode over fp8_ds_mla pages for any
// head count (the general path; 128 heads per kv group with bf16 q use the
// paired tcgen05 kernel of decode_tc3.cu), plus the LSE merge of the split
// partials.
//
// One CTA = (query token, block of <= 16 heads, split of the top-k axis).
// Two chunk sizes: with 32-token chunks two CTAs share an SM (~104 KB of
// shared memory, <= 128 registers), so one CTA's gather latency hides behind
// the other's math -- the choice when the grid has at least two CTAs per SM;
// a grid of fewer CTAs takes 64-token chunks (one CTA per SM, half the
// per-token synchronisation).  Per chunk:
//   gather   256/BN threads per row issue the row's 41 x 16-byte cp.async
//            (zero-fill for masked slots: no global read), double-buffered;
//   dequant  one warp per row: e4m3 * tile scale -> bf16 (hardware e4m3x2 ->
//            f16x2, exact fp32 product then RNE, as the reference:
//            decode.py:152-164);
//   QK^T     warp w: 16 tokens (two n8 tiles per loaded Q fragment) over a
//            1/(8/(BN/16)) share of d = 576 (m16n8k16 k-steps); the shares
//            meet in shared memory;
//   softmax  16 threads per head, BN/16 tokens each (exp2 form; a still -inf
//            running max is replaced by 0 so a fully masked chunk contributes
//            nothing: decode.py:178-197);
//   PV       warp w: output dims 64w..+63, V = the dequantized NoPE rows.
// Reference semantics: vllm_fp8kv/fp8_ds_mla_sparse_decode.py:77-211 and the
// split/merge pair of tests/fixtures/triton_mla_sparse_kernel_pr47629.py:232-403.
#include "common.cuh"
#include "decode.h"

namespace fp8mla {

namespace {

constexpr int kBH = 16;         // heads per CTA
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kKStride = 584;   // bf16 per sQ / sK row: 576 + 8 (1168 B = 73 x 16 B)

template <int BN>  // tokens per chunk: 32 or 64
struct Cfg {
  // QK^T: a warp owns 16 tokens (two n8 tiles share each Q fragment it loads)
  // and a 1/kParts share of d = 576; the shares meet in shared memory.
  static constexpr int kTokGroups = BN / 16;
  static constexpr int kParts = kThreads / 32 / kTokGroups;  // d shares
  static constexpr int kPartSteps = kDqk / 16 / kParts;      // k-steps per share
  static constexpr int kPStride = BN + 8;
  static constexpr int kSStride = BN + 1;
  static constexpr int kRowThreads = kThreads / BN;   // gather threads per row
  static constexpr int kMinBlocks = BN == 32 ? 2 : 1;
  static_assert(kThreads / 32 == kTokGroups * kParts && kDqk / 16 % kParts == 0,
                "one warp per (16-token group, d share)");
};

template <int BN>
struct Smem {
  uint16_t q[kBH * kKStride];
  uint16_t k[BN * kKStride];
  uint8_t raw[2][BN * kRowBytes];
  uint16_t p[kBH * Cfg<BN>::kPStride];
  float sp[Cfg<BN>::kParts][kBH * Cfg<BN>::kSStride];  // partial S per d share
  float m_run[kBH], l_run[kBH], alpha[kBH];
  int valid[2][BN];
};
static_assert(2 * (sizeof(Smem<32>) + 1024) <= 228 * 1024, "two 32-token CTAs per SM");
static_assert(sizeof(Smem<64>) <= 227 * 1024, "shared memory budget");
static_assert(offsetof(Smem<32>, raw) % 16 == 0 && offsetof(Smem<64>, raw) % 16 == 0,
              "cp.async destinations must be 16-B aligned");

// Row r = threadIdx.x / kRowThreads of a chunk is gathered by kRowThreads
// threads; `slot` is that row's live slot (-1: masked, no global read).
template <int BN>
__device__ __forceinline__ void issue_gather(Smem<BN>& s, int buf, const DecodeArgs& a,
                                             int32_t slot) {
  constexpr int kRT = Cfg<BN>::kRowThreads;
  const int r = threadIdx.x / kRT, sub = threadIdx.x % kRT;
  const bool ok = slot >= 0;
  const uint8_t* src = a.kv + (ok ? slot : 0) * (int64_t)kRowBytes;
  const uint32_t dst = smem_u32(&s.raw[buf][r * kRowBytes]);
  for (int j = sub; j < kRowChunks16; j += kRT) cp_async16(dst + j * 16, src + j * 16, ok ? 16 : 0);
  if (sub == 0) s.valid[buf][r] = ok;
}

}  // namespace

template <typename QT, typename OT, int BN>
__global__ void __launch_bounds__(kThreads, Cfg<BN>::kMinBlocks)
    decode_mma_kernel(const DecodeArgs a) {
  using C = Cfg<BN>;
  constexpr int kBN = BN, kPStride = C::kPStride, kSStride = C::kSStride;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<BN>& s = *reinterpret_cast<Smem<BN>*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  const int nhb = a.G * a.hb_per_group;                    // head blocks per token
  const int hbi = blockIdx.x % nhb;
  const int grp = hbi / a.hb_per_group;
  const int hb = hbi % a.hb_per_group;
  const int hrow0 = hb * a.block_h;                        // head offset within group
  const int nh = min(a.block_h, a.hpg - hrow0);            // valid heads in this CTA
  const int head0 = grp * a.hpg + hrow0;
  const int64_t t = blockIdx.x / nhb;
  const int split = blockIdx.y;
  const int beg = split * a.split_len;
  const int end = min(a.topk, beg + a.split_len);
  const int32_t* idx_row = a.idx + t * a.idx_st + grp * a.idx_sg;

  const int nchunks = end > beg ? (end - beg + kBN - 1) / kBN : 0;
  if (tid == 0) pdl_launch_dependents();
  pdl_wait();  // the previous kernel of the stream has completed
  const int32_t req = request_of(a, t);
  // Index prefetch: a chunk's raw top-k entry is loaded two chunks before its
  // gather, its block-table entry (if any) read one chunk before, and the
  // slot completed at the gather, so issuing a gather never waits for an
  // index load.
  const int grow = tid / C::kRowThreads;  // this thread's gather row
  auto raw_at = [&](int ch) -> int32_t {
    const int pos = beg + ch * kBN + grow;
    return (ch < nchunks && pos < end) ? idx_row[pos] : -1;
  };
  if (nchunks > 0) issue_gather(s, 0, a, live_slot(a, req, raw_at(0)));
  cp_async_commit();
  if (nchunks > 1) issue_gather(s, 1, a, live_slot(a, req, raw_at(1)));
  cp_async_commit();
  SlotPf slot_n = slot_fetch(a, req, raw_at(2));  // chunk c + 2
  int32_t raw_n = raw_at(3);                      // chunk c + 3

  // ---- Q -> smem (bf16), zero rows for padded heads
  for (int e = tid; e < kBH * (kDqk / 8); e += kThreads) {
    const int row = e / (kDqk / 8), c8 = e % (kDqk / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < nh) {
      const QT* src = static_cast<const QT*>(a.q) + t * a.q_st + (int64_t)(head0 + row) * a.q_sh + c8 * 8;
      if constexpr (sizeof(QT) == 2) {
        v = *reinterpret_cast<const uint4*>(src);
      } else {
        const float4 f0 = reinterpret_cast<const float4*>(src)[0];
        const float4 f1 = reinterpret_cast<const float4*>(src)[1];
        v = make_uint4(pack_bf16x2(f0.x, f0.y), pack_bf16x2(f0.z, f0.w),
                       pack_bf16x2(f1.x, f1.y), pack_bf16x2(f1.z, f1.w));
      }
    }
    *reinterpret_cast<uint4*>(&s.q[row * kKStride + c8 * 8]) = v;
  }
  if (tid < kBH) {
    s.m_run[tid] = -INFINITY;
    s.l_run[tid] = 0.f;
  }

  const int g = lane >> 2, q4 = lane & 3;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  const uint32_t q_base = smem_u32(s.q);
  const uint32_t k_base = smem_u32(s.k);
  const uint32_t p_base = smem_u32(s.p);
  // softmax ownership: head sh, tokens kTPT sp2 .. +kTPT-1 (16 threads per head)
  constexpr int kTPT = kBN / 16;
  const int sh = tid >> 4, sp2 = tid & 15;

  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    cp_async_wait<1>();
    __syncthreads();

    // ---- dequant raw[buf] -> k (bf16): warp per row, lane owns 16 bytes; the
    // warp's rows are unrolled so their load -> convert -> store chains overlap
#pragma unroll
    for (int r = warp; r < kBN; r += kWarps) {
      const uint8_t* row = &s.raw[buf][r * kRowBytes];
      const uint4 w = reinterpret_cast<const uint4*>(row)[lane];
      const float sc = reinterpret_cast<const float*>(row + kScaleOff)[lane >> 3];
      uint4 o0, o1;
      dequant4_hw_x2(w.x, sc, o0.x, o0.y);
      dequant4_hw_x2(w.y, sc, o0.z, o0.w);
      dequant4_hw_x2(w.z, sc, o1.x, o1.y);
      dequant4_hw_x2(w.w, sc, o1.z, o1.w);
      uint4* dst = reinterpret_cast<uint4*>(&s.k[r * kKStride + lane * 16]);
      dst[0] = o0;
      dst[1] = o1;
      if (lane < 8)
        reinterpret_cast<uint4*>(&s.k[r * kKStride + kNope])[lane] =
            reinterpret_cast<const uint4*>(row + kRopeOff)[lane];
    }
    // validity of this thread's softmax tokens, read before the gather of
    // chunk c + 2 reuses the flag buffer
    bool vt[kTPT];
#pragma unroll
    for (int u = 0; u < kTPT; ++u) vt[u] = s.valid[buf][kTPT * sp2 + u] != 0;
    __syncthreads();
    if (c + 2 < nchunks) issue_gather(s, buf, a, slot_finish(a, slot_n));
    cp_async_commit();
    slot_n = slot_fetch(a, req, raw_n);
    raw_n = raw_at(c + 4);

    // ---- partial S = Q K^T: tokens 16(w % groups)..+15, d share w / groups
    {
      const int n0 = (warp % C::kTokGroups) * 16, k0 = (warp / C::kTokGroups) * C::kPartSteps;
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      // ldmatrix rows: lane l -> Q row l & 15, column half l >> 4; K token
      // n0 + 8 (l >> 4) + (l & 7), column half (l >> 3) & 1
      const uint32_t qa0 = q_base + (((lane & 15) * kKStride + (lane >> 4) * 8) << 1);
      const uint32_t kb0 =
          k_base + (((n0 + ((lane >> 4) << 3) + (lane & 7)) * kKStride + ((lane >> 3) & 1) * 8) << 1);
#pragma unroll 3
      for (int kk = k0; kk < k0 + C::kPartSteps; ++kk) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ldmatrix_x4(qa0 + kk * 32, a0, a1, a2, a3);
        ldmatrix_x4(kb0 + kk * 32, b0, b1, b2, b3);
        mma_bf16_16816(sacc[0], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(sacc[1], a0, a1, a2, a3, b2, b3);
      }
      float* sp = s.sp[warp / C::kTokGroups];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int col = n0 + 8 * t + q4 * 2;
        sp[g * kSStride + col] = sacc[t][0];
        sp[g * kSStride + col + 1] = sacc[t][1];
        sp[(g + 8) * kSStride + col] = sacc[t][2];
        sp[(g + 8) * kSStride + col + 1] = sacc[t][3];
      }
    }
    __syncthreads();

    // ---- online softmax (exp2 form): 16 threads per head, kTPT tokens each
    {
      const int i0 = sh * kSStride + kTPT * sp2;
      const bool hv = sh < nh;
      float x[kTPT];
      float mt = -INFINITY;
#pragma unroll
      for (int u = 0; u < kTPT; ++u) {
        float sv = s.sp[0][i0 + u];
#pragma unroll
        for (int part = 1; part < C::kParts; ++part) sv += s.sp[part][i0 + u];
        x[u] = (vt[u] && hv) ? sv * a.scale_log2 : -INFINITY;
        mt = fmaxf(mt, x[u]);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xFFFFFFFFu, mt, o));
      const float m_old = s.m_run[sh];
      const float mn = fmaxf(m_old, mt);
      const float safe = (mn == -INFINITY) ? 0.f : mn;
      float ps = 0.f;
#pragma unroll
      for (int u = 0; u < kTPT; u += 2) {
        const float p0 = exp2f(x[u] - safe), p1 = exp2f(x[u + 1] - safe);
        *reinterpret_cast<uint32_t*>(&s.p[sh * kPStride + kTPT * sp2 + u]) = pack_bf16x2(p0, p1);
        ps += p0 + p1;
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, o);
      if (sp2 == 0) {
        const float al = exp2f(m_old - safe);
        s.alpha[sh] = al;
        s.l_run[sh] = s.l_run[sh] * al + ps;
        s.m_run[sh] = mn;
      }
    }
    __syncthreads();

    // ---- O = alpha O + P V for this warp's 64 output dims
    {
      const float al0 = s.alpha[g], al1 = s.alpha[g + 8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[i][0] *= al0;
        acc[i][1] *= al0;
        acc[i][2] *= al1;
        acc[i][3] *= al1;
      }
      const int d0 = warp * 64;
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(p_base + (((lane & 15) * kPStride + kk * 16 + (lane >> 4) * 8) << 1), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          uint32_t b0, b1, b2, b3;
          const int tok = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          ldmatrix_x4_trans(k_base + ((tok * kKStride + d0 + nt * 8 + (lane >> 4) * 8) << 1), b0, b1, b2, b3);
          mma_bf16_16816(acc[nt], a0, a1, a2, a3, b0, b1);
          mma_bf16_16816(acc[nt + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  const float l[2] = {s.l_run[g], s.l_run[g + 8]};
  const float mr[2] = {s.m_run[g], s.m_run[g + 8]};
  const int d0 = warp * 64 + q4 * 2;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = g + half * 8;
    if (row >= nh) continue;
    const int h = head0 + row;
    const float inv = l[half] > 0.f ? 1.f / l[half] : 1.f;
    const float lse_v = l[half] > 0.f ? mr[half] * kLn2 + logf(l[half]) : -INFINITY;
    if (a.num_splits == 1) {
      OT* o = static_cast<OT*>(a.out) + t * a.out_st + (int64_t)h * a.out_sh + d0;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float v0 = acc[nt][half * 2] * inv, v1 = acc[nt][half * 2 + 1] * inv;
        if constexpr (sizeof(OT) == 2) {
          *reinterpret_cast<uint32_t*>(o + nt * 8) = pack_bf16x2(v0, v1);
        } else {
          *reinterpret_cast<float2*>(o + nt * 8) = make_float2(v0, v1);
        }
      }
      if (a.lse != nullptr && warp == 0 && q4 == 0) a.lse[t * a.lse_st + h] = lse_v;
    } else {
      const int64_t base = ((t * a.H + h) * a.num_splits + split);
      if constexpr (sizeof(OT) == 2) {  // bf16 output: bf16 partials (half the traffic)
        uint16_t* o = reinterpret_cast<uint16_t*>(a.ws_o) + base * kNope + d0;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<uint32_t*>(o + nt * 8) =
              pack_bf16x2(acc[nt][half * 2] * inv, acc[nt][half * 2 + 1] * inv);
      } else {
        float* o = a.ws_o + base * kNope + d0;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<float2*>(o + nt * 8) =
              make_float2(acc[nt][half * 2] * inv, acc[nt][half * 2 + 1] * inv);
      }
      if (warp == 0 && q4 == 0) a.ws_lse[base] = lse_v;
    }
  }
}

// LSE merge of split partials: out = sum_s w_s o_s / sum_s w_s with
// w_s = exp(lse_s - max lse); an all-empty row gives zeros and LSE -inf.
// Partials are bf16 for a bf16 output (each is normalised, so bf16 keeps its
// relative precision; the sum is fp32) and fp32 for an fp32 output.
// Reference: tests/fixtures/triton_mla_sparse_kernel_pr47629.py:331-403.
template <typename OT>
__global__ void __launch_bounds__(128) merge_splits_kernel(const DecodeArgs a) {
  const int64_t th = blockIdx.x;  // t * H + h
  const int64_t t = th / a.H, h = th % a.H;
  const int S = a.num_splits;
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();  // the decode kernel's partials are complete
  const float* lse_s = a.ws_lse + th * S;
  float m = -INFINITY;
  for (int i = 0; i < S; ++i) m = fmaxf(m, lse_s[i]);
  const int d = threadIdx.x * 4;
  float4 accv = make_float4(0.f, 0.f, 0.f, 0.f);
  float denom = 0.f;
  if (m != -INFINITY) {
    for (int i = 0; i < S; ++i) {
      const float w = expf(lse_s[i] - m);
      denom += w;
      float4 o;
      if constexpr (sizeof(OT) == 2) {
        const uint2 p = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(a.ws_o) +
                                                        (th * S + i) * kNope + d);
        o = make_float4(__uint_as_float(p.x << 16), __uint_as_float(p.x & 0xFFFF0000u),
                        __uint_as_float(p.y << 16), __uint_as_float(p.y & 0xFFFF0000u));
      } else {
        o = *reinterpret_cast<const float4*>(a.ws_o + (th * S + i) * kNope + d);
      }
      accv.x += w * o.x;
      accv.y += w * o.y;
      accv.z += w * o.z;
      accv.w += w * o.w;
    }
  }
  const float inv = denom > 0.f ? 1.f / denom : 1.f;
  OT* o = static_cast<OT*>(a.out) + t * a.out_st + h * a.out_sh + d;
  if constexpr (sizeof(OT) == 2) {
    reinterpret_cast<uint2*>(o)[0] =
        make_uint2(pack_bf16x2(accv.x * inv, accv.y * inv), pack_bf16x2(accv.z * inv, accv.w * inv));
  } else {
    reinterpret_cast<float4*>(o)[0] = make_float4(accv.x * inv, accv.y * inv, accv.z * inv, accv.w * inv);
  }
  if (a.lse != nullptr && threadIdx.x == 0)
    a.lse[t * a.lse_st + h] = denom > 0.f ? m + logf(denom) : -INFINITY;
}

int launch_decode_mma(const DecodeArgs& a, cudaStream_t st) {
  // head blocks of one token are adjacent in x so they re-hit the same rows in L2
  dim3 grid((unsigned)(a.T * a.G * a.hb_per_group), a.num_splits);
  // 32-token chunks pay off once the grid can keep two CTAs on every SM
  const bool small_chunks = (int64_t)grid.x * grid.y >= 2 * (int64_t)device_sm_count();
  int rc = FP8MLA_OK;
  auto go = [&](auto kern, size_t smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "decode_mma smem attribute");
    return check_cuda(launch_pdl(kern, grid, dim3(kThreads), smem, st, a), "decode_mma_kernel launch");
  };
  const size_t s32 = sizeof(Smem<32>), s64 = sizeof(Smem<64>);
  if (a.q_dtype == FP8MLA_DTYPE_BF16)
    rc = small_chunks ? go(decode_mma_kernel<__nv_bfloat16, __nv_bfloat16, 32>, s32)
                      : go(decode_mma_kernel<__nv_bfloat16, __nv_bfloat16, 64>, s64);
  else
    rc = small_chunks ? go(decode_mma_kernel<float, float, 32>, s32)
                      : go(decode_mma_kernel<float, float, 64>, s64);
  if (rc != FP8MLA_OK || a.num_splits == 1) return rc;
  return launch_merge_splits(a, st);
}

int launch_merge_splits(const DecodeArgs& a, cudaStream_t st) {
  dim3 mgrid((unsigned)(a.T * a.H));
  const cudaError_t e =
      a.q_dtype == FP8MLA_DTYPE_BF16
          ? launch_pdl(merge_splits_kernel<__nv_bfloat16>, mgrid, dim3(128), 0, st, a)
          : launch_pdl(merge_splits_kernel<float>, mgrid, dim3(128), 0, st, a);
  return check_cuda(e, "merge_splits_kernel launch");
}

}  // namespace fp8mla
