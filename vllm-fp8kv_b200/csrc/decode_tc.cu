// decode_tc.cu -- tcgen05/TMEM sparse MLA decode for 128 heads per kv group.
//
// All 128 heads of a kv group share the gathered latent rows, so the heads
// are the MMA M dimension (M = 128, one tcgen05 M-tile):
//   S = Q K^T   M=128 heads, N=64 tokens, K=576 (36 k-steps of 16)
//   O += P V    M=128 heads, N=256 output dims, K=64 tokens (4 k-steps)
// A 128 x 512 fp32 O fills a whole SM's tensor memory, so each (token, group)
// runs on two CTAs: CTA h accumulates O[:, 256h : 256h+256) and both compute
// the full S (no cross-SM traffic; the second CTA's row reads hit L2).
//
// Throughput model (B200, one SM): tcgen05.mma issued as straight-line code
// runs back to back whatever the accumulator; an M=128 kind::f16 MMA costs
// max(N/2 cycles of math, bytes read from shared memory / 128 B per cycle).
// An N=32 QK^T step re-reads 4 KB of Q for 1 KB of K and runs at a third of
// the math rate; N=64 with a third of Q held in tensor memory (TMEM-A MMA, no
// shared-memory read for A) brings a 64-token tile to ~1.5K cycles of QK^T.
//
// Tensor-memory map (512 columns):
//   [  0,256)  O (fp32)
//   [256,384)  2 S buffers x 64 fp32 columns; P (bf16x2, 32 columns) is
//              written over the first half of its buffer
//   [384,512)  Q dims [0,256) as the A operand of the TMEM-A MMA (bf16x2)
// Shared memory (216 KB):
//   q   Q dims [256,576): 5 x 64-dim 128B-swizzled blocks (128 rows)
//   v   3-deep ring of this CTA's V blocks: tile dims [256h, 256h+256) as
//       4 x 64-dim swizzled blocks of 64 rows -- the K-major B operand of
//       QK^T and, read MN-major, the V operand of PV.  A slot is released
//       when the tile's PV completes.
//   nv  the tile's other 5 blocks (the other latent half and the rope),
//       single-buffered: released as soon as the tile's QK^T completes.
// QK^T issues the V-block k-steps first, so the loaders refill `nv` while
// the pipe runs the previous tile's PV and this tile's first 16 k-steps.
//
// Warp roles (416 threads):
//   warps 0-3   softmax + epilogue: thread i owns head i = TMEM lane i, so the
//               row max / sum / lazy rescale of its O row need no cross-thread
//               reduction.  The reference max is only raised when a tile
//               exceeds it by more than 8 (log2 units); P <= 2^8 keeps its
//               bf16 precision and the final 1/l and LSE use the same max.
//               S is read from tensor memory twice, 32 columns at a time (the
//               max, then the exponentials): small code and few registers.
//   warp 4      TMEM allocation and the single-thread MMA issuer
//   warps 5-12  gather + dequant: each warp owns 8 of the 64 rows of a tile
//               (4 lanes per row) and loads them straight into registers one
//               tile ahead, their slots two tiles ahead (no load is issued for
//               a masked slot), then writes bf16(e4m3 * scale) and the raw rope
//               into the swizzled blocks.
// Pipe order per tile j: QK(j) [V blocks, then nv blocks], PV(j-1).
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
constexpr int kN = 64;              // tokens per tile
constexpr int kKSteps = 36;         // 576 / 16
constexpr int kDv = 256;            // output dims per CTA
constexpr int kQTmemSteps = 16;     // k-steps 0..15 (q dims 0..255) read A from tensor memory
constexpr int kQSmemBlocks = 5;     // q dims [256,576) as 5 x 64-dim swizzled blocks
constexpr int kBlkBytes = kN * 128;                 // 8192: one 64-dim block of a tile
constexpr int kVBlocks = 4;                         // this CTA's latent half
constexpr int kNvBlocks = 5;                        // other latent half + rope
constexpr int kVSlotBytes = kVBlocks * kBlkBytes;   // 32768
constexpr int kVStages = 3;
constexpr int kQBlockBytes = kHeads * 128;          // 16384
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kFirstLoadWarp = 5;
constexpr int kLoadWarps = 8;
constexpr int kLoadThreads = kLoadWarps * 32;
constexpr int kThreads = (kSoftmaxWarps + 1 + kLoadWarps) * 32;  // 416
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256, kColQ = 384;
constexpr uint32_t kSBufCols = kN;  // 64
constexpr float kRescaleThreshold = 8.0f;

constexpr uint32_t kIdescQK = idesc_bf16(128, kN, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, kDv, true);

struct Smem {
  uint8_t q[kQSmemBlocks * kQBlockBytes];   // 1024-aligned (offset 0)
  uint8_t v[kVStages][kVSlotBytes];         // 1024-aligned
  uint8_t nv[kNvBlocks * kBlkBytes];        // 1024-aligned
  uint8_t vbits[kVStages][kLoadWarps];      // validity of the 8 rows of each load warp
  uint64_t vfull[kVStages], vempty[kVStages];
  uint64_t nvfull, nvempty;
  uint64_t sfull[2], pfull[2], sfree[2];
  uint64_t qready, ofull, drain;
  uint32_t tmem_base;
};
static_assert(offsetof(Smem, v) % 1024 == 0 && offsetof(Smem, nv) % 1024 == 0,
              "swizzle atoms need 1024-B alignment");
static_assert(offsetof(Smem, vfull) % 8 == 0, "");
static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory budget");

// byte offset of the 16-byte chunk `c` (0..7) of row `r` in a 128B-swizzled block
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

// Block `bi` (0..8) of a tile for CTA half H: V blocks live in the ring slot,
// the rest in the nv buffer.
template <int H>
__host__ __device__ constexpr bool is_v_block(int bi) {
  return bi >= 4 * H && bi < 4 * H + 4;
}
template <int H>
__host__ __device__ constexpr int nv_index(int bi) {
  return bi < 4 * H ? bi : bi - 4;
}

// One load-warp lane's share of a row: fp8 chunks p + 4i (i = 0..7, chunk i
// lands in tile block i), rope chunks p and p + 4, and the row's 4 tile scales.
struct RowPart {
  uint4 f[8];
  uint4 rope[2];
  uint4 sc;
};

struct Ctx {
  const DecodeArgs* a;
  const int32_t* idx_row;
  int32_t req;  // request of this token (block-table indirection only)
  int beg, end, ntiles;
  uint32_t tmem;
  uint32_t sq, sv0, snv;
  uint32_t b_vfull, b_vempty, b_nvfull, b_nvempty;
  uint32_t b_sfull, b_pfull, b_sfree, b_qready, b_ofull, b_drain;
};

// ------------------------------------------------------------------ MMA issuer
// QK^T k-steps of one tile whose B block is (PartV ? a V block : an nv block),
// in ascending k order.  Everything is unrolled: straight-line tcgen05.mma.
template <int H, bool PartV>
__device__ __forceinline__ void issue_qk_part(uint32_t tS, uint32_t tQ, uint64_t qdesc0,
                                              uint64_t vdesc, uint64_t nvdesc) {
  
  constexpr int kFirst = 16 * H;  // first k-step issued for the tile (its V blocks)
#pragma unroll
  for (int kst = 0; kst < kKSteps; ++kst) {
    const int bi = kst >> 2;
    if (is_v_block<H>(bi) != PartV) continue;
    const uint32_t acc = kst == kFirst ? 0u : 1u;
    const uint32_t boff = (PartV ? (bi - 4 * H) : nv_index<H>(bi)) * kBlkBytes + (kst & 3) * 32;
    const uint64_t bdesc = (PartV ? vdesc : nvdesc) + (uint64_t)(boff >> 4);
    if (kst < kQTmemSteps) {
      mma_ts(tS, tQ + 8 * kst, bdesc, kIdescQK, acc);
    } else {
      const int qs = kst - kQTmemSteps;
      const uint64_t adesc = qdesc0 + (uint64_t)(((qs >> 2) * kQBlockBytes + (qs & 3) * 32) >> 4);
      mma_ss(tS, adesc, bdesc, kIdescQK, acc);
    }
  }
}

// Spin (without suspending) on an mbarrier phase the tensor pipe completes;
// bounded like every other wait.
__device__ __forceinline__ bool thread_spin(uint32_t bar, uint32_t parity, uint32_t where) {
  for (uint32_t it = 0; it < (kMaxWaitIters << 4); ++it)
    if (mbar_test(bar, parity)) return true;
  atomicOr(&g_device_status, kStatusWaitTimeout | (where << 8));
  return false;
}

template <int H>
__device__ void mma_role(const Ctx& c) {
  bool ok = thread_wait(c.b_qready, 0, 5);
  tc_fence_after();
  const uint32_t tO = c.tmem + kColO, tQ = c.tmem + kColQ;
  const uint64_t qdesc0 = sdesc_sw128(c.sq, 16, 1024);
  const uint64_t vdesc0 = sdesc_sw128(c.sv0, 16, 1024);
  const uint64_t nvdesc = sdesc_sw128(c.snv, 16, 1024);
  // V read MN-major: 64-dim blocks kBlkBytes apart (LBO), 8-token groups 1 KB apart (SBO)
  const uint64_t pvdesc0 = sdesc_sw128(c.sv0, kBlkBytes, 1024);
  auto issue_pv = [&](int jj) {
    const int bb = jj & 1, vs = jj % kVStages;
    tc_fence_after();
    const uint32_t pa = c.tmem + kColS + kSBufCols * bb;
    const uint64_t vd = pvdesc0 + (uint64_t)((vs * kVSlotBytes) >> 4);
#pragma unroll
    for (int kk = 0; kk < kN / 16; ++kk)
      mma_ts(tO, pa + 8 * kk, vd + (uint64_t)((kk * 16 * 128) >> 4), kIdescPV,
             (jj > 0 || kk > 0) ? 1u : 0u);
    mma_commit(c.b_sfree + 8 * bb);
    mma_commit(c.b_vempty + 8 * vs);
  };
  for (int j = 0; j < c.ntiles && ok; ++j) {
    const int b = j & 1, vs = j % kVStages;
    ok = thread_wait(c.b_vfull + 8 * vs, (j / kVStages) & 1, 7);
    // S buffer b last held P(j-2): PV(j-2) must have finished reading it
    if (ok && j >= 2) ok = thread_spin(c.b_sfree + 8 * b, ((j - 2) >> 1) & 1, 8);
    if (!ok) break;
    tc_fence_after();
    const uint32_t tS = c.tmem + kColS + kSBufCols * b;
    const uint64_t vdesc = vdesc0 + (uint64_t)((vs * kVSlotBytes) >> 4);
    issue_qk_part<H, true>(tS, tQ, qdesc0, vdesc, nvdesc);
    ok = thread_wait(c.b_nvfull, j & 1, 11);
    if (!ok) break;
    tc_fence_after();
    issue_qk_part<H, false>(tS, tQ, qdesc0, vdesc, nvdesc);
    mma_commit(c.b_sfull + 8 * b);
    mma_commit(c.b_nvempty);
    if (j >= 1) {
      ok = thread_wait(c.b_pfull + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1, 6);
      if (!ok) break;
      issue_pv(j - 1);
    }
  }
  if (ok && c.ntiles > 0) {
    const int jl = c.ntiles - 1;
    ok = thread_wait(c.b_pfull + 8 * (jl & 1), (jl >> 1) & 1, 6);
    if (ok) {
      issue_pv(jl);
      mma_commit(c.b_ofull);
    }
  }
  // drain: nothing this thread issued may still touch tensor memory
  mma_commit(c.b_drain);
  thread_wait(c.b_drain, 0, 9);
}

// ------------------------------------------------------------------ gather + dequant
template <int H>
__device__ void load_role(const Ctx& c, Smem& s, int lw, int lane) {
  const DecodeArgs& a = *c.a;
  const int r = lane & 7, p = lane >> 3;  // row within the warp's 8, quarter 0..3
  const int row = lw * 8 + r;
  // the live slot of this lane's row of tile jt, or -1 (masked, out of range, past the end)
  auto slot_of = [&](int jt) -> int32_t {
    const int pos = c.beg + jt * kN + row;
    return pos < c.end ? live_slot(a, c.req, c.idx_row[pos]) : -1;
  };
  auto load = [&](int32_t slot, RowPart& P, bool& valid) {
    valid = slot >= 0;
    if (valid) {
      const uint8_t* src = a.kv + slot * (int64_t)kRowBytes;
#pragma unroll
      for (int i = 0; i < 8; ++i) P.f[i] = ldg_v4(src + (p + 4 * i) * 16);
      P.rope[0] = ldg_v4(src + kRopeOff + 16 * p);
      P.rope[1] = ldg_v4(src + kRopeOff + 16 * (p + 4));
      P.sc = ldg_v4(src + kScaleOff);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) P.f[i] = make_uint4(0, 0, 0, 0);
      P.rope[0] = P.rope[1] = make_uint4(0, 0, 0, 0);
      P.sc = make_uint4(0, 0, 0, 0);
    }
  };
  // dequantize chunk i (64-dim block i, 16 dims at 16p) of the row into `blk`
  auto put = [&](const RowPart& P, int i, uint8_t* blk) {
    const float sc = (i >> 1) == 0   ? __uint_as_float(P.sc.x)
                     : (i >> 1) == 1 ? __uint_as_float(P.sc.y)
                     : (i >> 1) == 2 ? __uint_as_float(P.sc.z)
                                     : __uint_as_float(P.sc.w);
    uint4 o0, o1;
    dequant4_hw_x2(P.f[i].x, sc, o0.x, o0.y);
    dequant4_hw_x2(P.f[i].y, sc, o0.z, o0.w);
    dequant4_hw_x2(P.f[i].z, sc, o1.x, o1.y);
    dequant4_hw_x2(P.f[i].w, sc, o1.z, o1.w);
    *reinterpret_cast<uint4*>(blk + swz(row, 2 * p)) = o0;
    *reinterpret_cast<uint4*>(blk + swz(row, 2 * p + 1)) = o1;
  };
  bool ok = true;
  // slots are read one step before their rows: the index load's latency hides
  // behind a tile of dequant instead of stalling the row loads
  int32_t slot_next = c.ntiles > 1 ? slot_of(1) : -1;
  auto step = [&](int j, const RowPart& cur, bool vcur, RowPart& nxt, bool& vnxt) {
    if (!ok || j >= c.ntiles) return;
    const int32_t slot1 = slot_next;
    if (j + 2 < c.ntiles) slot_next = slot_of(j + 2);
    if (j + 1 < c.ntiles) load(slot1, nxt, vnxt);
    const int vs = j % kVStages;
    // V blocks of tile j -> ring slot vs (free once PV(j-3) completed)
    if (j >= kVStages) ok = warp_wait(c.b_vempty + 8 * vs, ((j / kVStages) + 1) & 1, 10);
    if (!ok) return;
    uint8_t* vslot = s.v[vs];
#pragma unroll
    for (int i = 4 * H; i < 4 * H + 4; ++i) put(cur, i, vslot + (i - 4 * H) * kBlkBytes);
    const uint32_t vb = __ballot_sync(0xFFFFFFFFu, p == 0 && vcur);  // bits 0..7 = rows 8lw..+7
    if (lane == 0) s.vbits[vs][lw] = (uint8_t)(vb & 0xFFu);
    fence_proxy_async_smem();
    mbar_arrive(c.b_vfull + 8 * vs);
    // the other blocks -> nv (free once QK(j-1) completed)
    if (j >= 1) ok = warp_wait(c.b_nvempty, (j - 1) & 1, 12);
    if (!ok) return;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (!is_v_block<H>(i)) put(cur, i, s.nv + nv_index<H>(i) * kBlkBytes);
    uint8_t* rope = s.nv + nv_index<H>(8) * kBlkBytes;
    *reinterpret_cast<uint4*>(rope + swz(row, p)) = cur.rope[0];
    *reinterpret_cast<uint4*>(rope + swz(row, p + 4)) = cur.rope[1];
    fence_proxy_async_smem();
    mbar_arrive(c.b_nvfull);
  };
  RowPart A, B;
  bool vA = false, vB = false;
  if (c.ntiles > 0) load(slot_of(0), A, vA);
  for (int j = 0; j < c.ntiles && ok; j += 2) {
    step(j, A, vA, B, vB);
    step(j + 1, B, vB, A, vA);
  }
}

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
  const int head0 = grp * kHeads;

  Ctx c;
  c.a = &a;
  c.beg = split * a.split_len;
  c.end = min(a.topk, c.beg + a.split_len);
  c.ntiles = c.end > c.beg ? (c.end - c.beg + kN - 1) / kN : 0;
  c.idx_row = a.idx + t * a.idx_st + grp * a.idx_sg;
  c.req = request_of(a, t);
  c.sq = smem_u32(s.q);
  c.sv0 = smem_u32(s.v[0]);
  c.snv = smem_u32(s.nv);
  c.b_vfull = smem_u32(&s.vfull[0]);
  c.b_vempty = smem_u32(&s.vempty[0]);
  c.b_nvfull = smem_u32(&s.nvfull);
  c.b_nvempty = smem_u32(&s.nvempty);
  c.b_sfull = smem_u32(&s.sfull[0]);
  c.b_pfull = smem_u32(&s.pfull[0]);
  c.b_sfree = smem_u32(&s.sfree[0]);
  c.b_qready = smem_u32(&s.qready);
  c.b_ofull = smem_u32(&s.ofull);
  c.b_drain = smem_u32(&s.drain);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(c.b_vfull + 8 * i, kLoadThreads);
      mbar_init(c.b_vempty + 8 * i, 1);
    }
    mbar_init(c.b_nvfull, kLoadThreads);
    mbar_init(c.b_nvempty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(c.b_sfull + 8 * i, 1);
      mbar_init(c.b_pfull + 8 * i, kSoftmaxWarps * 32);
      mbar_init(c.b_sfree + 8 * i, 1);
    }
    mbar_init(c.b_qready, kSoftmaxWarps * 32);
    mbar_init(c.b_ofull, 1);
    mbar_init(c.b_drain, 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&s.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem = s.tmem_base;
  const uint32_t tmem = c.tmem;

  if (warp < kSoftmaxWarps) {
    // ================================================= softmax + epilogue
    const int h = threadIdx.x;                       // head within the group = TMEM lane
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    // ---- Q: dims [0,256) -> TMEM (A operand), dims [256,576) -> swizzled smem
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
        for (int cc = 0; cc < 8; ++cc)
          *reinterpret_cast<uint4*>(s.q + blk * kQBlockBytes + swz(h, cc)) =
              qsrc[kQTmemSteps * 2 + blk * 8 + cc];
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(c.b_qready);
    }

    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < c.ntiles && ok; ++j) {
      const int b = j & 1, vs = j % kVStages;
      ok = warp_wait(c.b_sfull + 8 * b, (j >> 1) & 1, 1);
      if (!ok) break;
      ok = warp_wait(c.b_vfull + 8 * vs, (j / kVStages) & 1, 2);  // orders the validity bits
      if (!ok) break;
      tc_fence_after();
      const uint32_t sb = trow + kColS + kSBufCols * b;
      const uint2 vbw = *reinterpret_cast<const uint2*>(s.vbits[vs]);  // bit k = token k
      // pass 1: the tile max (rolled over the two 32-token halves: small code)
      float tmax = -INFINITY;
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t sv[32];
        tmem_ld32(sb + 32 * hf, sv);
        tmem_wait_ld();
        const uint32_t vm = hf ? vbw.y : vbw.x;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if ((vm >> i) & 1u) tmax = fmaxf(tmax, __uint_as_float(sv[i]) * a.scale_log2);
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
        ok = warp_wait(c.b_sfree + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1, 3);
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
      // pass 2: P for tokens 32hf..+31 over packed columns 16hf..+15 (their S was read)
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t sv[32];
        tmem_ld32(sb + 32 * hf, sv);
        tmem_wait_ld();
        const uint32_t vm = hf ? vbw.y : vbw.x;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = ((vm >> (2 * i)) & 1u) ? __uint_as_float(sv[2 * i]) * a.scale_log2 : -INFINITY;
          const float x1 =
              ((vm >> (2 * i + 1)) & 1u) ? __uint_as_float(sv[2 * i + 1]) * a.scale_log2 : -INFINITY;
          const float p0 = ex2_approx(x0 - mref), p1 = ex2_approx(x1 - mref);
          l += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        tmem_st16(sb + 16 * hf, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(c.b_pfull + 8 * b);
    }

    // ---- epilogue
    const bool have_o = ok && c.ntiles > 0 && warp_wait(c.b_ofull, 0, 4);
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
      if (half == 0)
        mma_role<0>(c);
      else
        mma_role<1>(c);
    }
    __syncwarp();
  } else {
    // ================================================= gather + dequant
    const int lw = warp - kFirstLoadWarp;  // 0..7
    if (half == 0)
      load_role<0>(c, s, lw, lane);
    else
      load_role<1>(c, s, lw, lane);
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
