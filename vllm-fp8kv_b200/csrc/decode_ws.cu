// decode_ws.cu -- sparse MLA decode over fp8_ds_mla pages for bf16 q in head
// blocks of <= 16 heads (small head counts; 64 or 128 heads per kv group take
// the paired tcgen05 kernel of decode_tc3.cu, fp32 q the kernel of
// decode_mma.cu): persistent, warp-specialised, rows gathered by TMA.
//
// One CTA per SM walks units u = blockIdx.x, blockIdx.x + gridDim.x, ...; a
// unit is (query token, head block of one kv group, top-k split).  A unit's
// top-k rows are taken in 32-token chunks, numbered over all of the CTA's
// units, so the rings below run across unit boundaries (the next unit's rows
// and Q arrive while the current one finishes):
//   warp 0      producer.  Lane i takes index i of a chunk (copied into a
//               shared ring eight chunks ahead with cp.async) and converts it
//               to a slot; lanes 0-7 each issue one TMA tile::gather4 of four
//               whole 656-byte rows into a stage of the raw ring (masked rows
//               fetch row 0 and are flagged invalid).  At each unit start it
//               bulk-copies the unit's Q rows into the Q buffer.
//   warps 1-7   dequant.  Raw ring -> bf16 key rows of a two-stage K ring
//               (e4m3 * tile scale in fp32, RNE to bf16; rope copied raw),
//               invalid rows written as zeros, validity flags alongside.
//   warps 8-15  compute (mma.sync m16n8k16).  S = Q K^T with warp w owning
//               tokens 16 (w % 2).. +15 over a quarter of d = 576, its Q
//               fragments held in registers for the whole unit (the quarters
//               meet in shared memory); online softmax in the exp2 form;
//               O += P V with warp w owning 64 output dims; the unit's
//               epilogue (output, or a bf16 split partial and its LSE).
// Hand-offs are mbarriers with bounded waits; the compute warps also meet
// twice per chunk on a named barrier of their own.
//
// Reference semantics: vllm_fp8kv/fp8_ds_mla_sparse_decode.py:77-211 (masking,
// dequant, NaN-free online softmax, LSE) and the split/merge contract of
// tests/fixtures/triton_mla_sparse_kernel_pr47629.py:232-403.
#include <cuda.h>

#include "common.cuh"
#include "decode.h"
#include "tc_ptx.cuh"
#include "tma_map.h"

namespace fp8mla {
namespace ws {

using namespace fp8mla::tc;

namespace {

constexpr int kBN = 32;                       // tokens per chunk
constexpr int kBH = 16;                       // heads per unit
constexpr int kRawStages = 5;
constexpr int kGroupBytes = 2688;             // 4 rows (2624 B) padded to a multiple of 128
constexpr int kRawStageBytes = 8 * kGroupBytes;
constexpr int kChunkTx = kBN * kRowBytes;     // bytes a chunk's eight gather4 deliver
constexpr int kKStride = 584;                 // bf16 per K / Q row: 576 + 8 (bank spread)
constexpr int kRowStrideB = kKStride * 2;     // 1168 B
constexpr int kKStages = 2;
constexpr int kQBufs = 1;                     // Q moves to registers at each unit start
constexpr int kPStride = kBN + 8;             // bf16 per P row
constexpr int kDequantWarps = 7;  // 16 warps in all: 128 registers a thread
constexpr int kRowsPerDequantWarp = (kBN + kDequantWarps - 1) / kDequantWarps;  // at most
constexpr int kComputeWarps = 8;
constexpr int kTokGroups = kBN / 16;                // QK: 16 tokens per warp ...
constexpr int kDParts = kComputeWarps / kTokGroups; // ... and a quarter of d = 576
constexpr int kPartSteps = kDqk / 16 / kDParts;     // k-steps per share
constexpr int kOutDims = kNope / kComputeWarps;     // PV: output dims per warp
constexpr int kOutTiles = kOutDims / 8;
constexpr int kIdxAhead = 8;                  // chunks of indices in flight (cp.async)
constexpr int kIdxSlots = kIdxAhead + 1;
constexpr int kFirstCompute = 1 + kDequantWarps;
constexpr int kThreads = (kFirstCompute + kComputeWarps) * 32;

struct Smem {
  uint8_t raw[kRawStages][kRawStageBytes];    // 128-B aligned gather4 destinations
  uint16_t q[kQBufs][kBH * kKStride];
  uint16_t k[kKStages][kBN * kKStride];
  uint16_t p[kBH * kPStride];
  float sp[kDParts][kBH][kBN + 1];            // partial S per d share
  float alpha[kBH];                           // this chunk's O rescale per head
  float m_fin[kBH], l_fin[kBH];               // a unit's final max and sum per head
  int32_t sidx[kIdxSlots][kBN];
  uint8_t valid[kRawStages][kBN];
  uint8_t kvalid[kKStages][kBN];
  uint64_t raw_full[kRawStages], raw_empty[kRawStages];
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t q_full[kQBufs], q_empty[kQBufs];
};
static_assert(offsetof(Smem, q) % 16 == 0 && offsetof(Smem, k) % 16 == 0 &&
                  offsetof(Smem, p) % 16 == 0 && offsetof(Smem, raw_full) % 8 == 0,
              "alignment");
static_assert(sizeof(Smem) + 128 <= 227 * 1024, "shared memory budget");

struct Unit {
  int64_t t;
  int head0, nh, split, beg, end, nch;
  const int32_t* idx_row;
};

__device__ __forceinline__ Unit unit_of(const DecodeArgs& a, int u) {
  const int nhb = a.G * a.hb_per_group;
  Unit x;
  x.split = u % a.num_splits;
  const int rest = u / a.num_splits;
  const int hbi = rest % nhb;
  x.t = rest / nhb;
  const int grp = hbi / a.hb_per_group, hb = hbi % a.hb_per_group;
  const int hrow0 = hb * a.block_h;
  x.nh = min(a.block_h, a.hpg - hrow0);
  x.head0 = grp * a.hpg + hrow0;
  x.beg = x.split * a.split_len;
  x.end = min(a.topk, x.beg + a.split_len);
  x.nch = x.end > x.beg ? (x.end - x.beg + kBN - 1) / kBN : 0;
  x.idx_row = a.idx + x.t * a.idx_st + (int64_t)grp * a.idx_sg;
  return x;
}

// Bounded warp wait after which every lane has acquired the phase itself.
__device__ __forceinline__ bool warp_acquire(uint32_t bar, uint32_t parity, uint32_t where,
                                             uint32_t iters) {
  const bool ok = warp_wait_n(bar, parity, where, iters);
  if (ok) (void)mbar_try_wait(bar, parity);
  return ok;
}

// The compute warps' own barrier (id 1; the other warps never use it).
__device__ __forceinline__ void named_sync_ws() {
  asm volatile("bar.sync 1, %0;\n" ::"n"(kComputeWarps * 32) : "memory");
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                              uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ------------------------------------------------------------------ producer (warp 0)
// Walks the CTA's (unit, chunk) sequence; `ahead` runs kIdxAhead chunks in
// front of it, copying each chunk's 32 raw indices into a shared-memory ring
// with 4-byte cp.async (no register waits on index loads).
struct ChunkCursor {
  int u, c;
  Unit x;
  __device__ __forceinline__ void settle(const DecodeArgs& a, int nunits) {
    while (u < nunits && c >= x.nch) {
      u += gridDim.x;
      c = 0;
      if (u < nunits) x = unit_of(a, u);
    }
  }
};

__device__ void producer(const DecodeArgs& a, Smem& s, const CUtensorMap* tm, int nunits, int lane) {
  ChunkCursor ahead;
  ahead.u = blockIdx.x;
  ahead.c = 0;
  ahead.x = unit_of(a, ahead.u);
  ahead.settle(a, nunits);
  auto fetch_idx = [&](int slot) {
    if (ahead.u < nunits) {
      const int pos = ahead.x.beg + ahead.c * kBN + lane;
      if (pos < ahead.x.end) cp_async4(smem_u32(&s.sidx[slot][lane]), ahead.x.idx_row + pos);
      ++ahead.c;
      ahead.settle(a, nunits);
    }
    cp_async_commit();
  };
#pragma unroll 1
  for (int i = 0; i < kIdxAhead; ++i) fetch_idx(i);

  // g: raw stages armed so far (chunk count), qc: Q buffers armed so far.
  // A stage (buffer) is armed again only after its release was seen, which
  // implies its previous copies landed; when a release wait gives up, the
  // producer stops arming altogether.  So at the end only the last
  // kRawStages stages and kQBufs buffers can still have copies in flight.
  int g = 0, qc = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
    const Unit x = unit_of(a, u);
    if (x.nch == 0) continue;
    const int32_t req = request_of(a, x.t);
    // the unit's Q rows -> the Q buffer, once the compute warps are done with it
    const int qb = qc % kQBufs;
    const uint32_t qfull = smem_u32(&s.q_full[qb]);
    if (qc >= kQBufs) ok = warp_wait_n(smem_u32(&s.q_empty[qb]), ((qc / kQBufs) + 1) & 1, 20, a.wait_iters);
    if (!ok) break;
    if (lane == 0) mbar_arrive_expect_tx(qfull, (uint32_t)x.nh * kDqk * 2);
    __syncwarp();
    if (lane < x.nh)
      bulk_copy_g2s(smem_u32(&s.q[qb][lane * kKStride]),
                    static_cast<const uint16_t*>(a.q) + x.t * a.q_st + (int64_t)(x.head0 + lane) * a.q_sh,
                    kDqk * 2, qfull);
    ++qc;
    for (int c = 0; c < x.nch; ++c) {
      // chunk g's indices (copy group g) have landed; lane i owns row i
      cp_async_wait<kIdxAhead - 1>();
      const int pos = x.beg + c * kBN + lane;
      const int32_t raw = pos < x.end ? s.sidx[g % kIdxSlots][lane] : -1;
      fetch_idx((g + kIdxAhead) % kIdxSlots);  // the slot read one chunk ago
      const int32_t slot = live_slot(a, req, raw);
      const int st = g % kRawStages;
      if (g >= kRawStages)
        ok = warp_wait_n(smem_u32(&s.raw_empty[st]), ((g / kRawStages) + 1) & 1, 21, a.wait_iters);
      if (!ok) break;
      s.valid[st][lane] = slot >= 0 ? 1 : 0;
      const int32_t row = slot >= 0 ? slot : 0;  // masked: a valid row, flagged invalid
      const uint32_t bar = smem_u32(&s.raw_full[st]);
      // the flags (generic stores) are released by the arrive below
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(bar, kChunkTx);
      __syncwarp();
      const int32_t r0 = __shfl_sync(0xFFFFFFFFu, row, (4 * lane) & 31);
      const int32_t r1 = __shfl_sync(0xFFFFFFFFu, row, (4 * lane + 1) & 31);
      const int32_t r2 = __shfl_sync(0xFFFFFFFFu, row, (4 * lane + 2) & 31);
      const int32_t r3 = __shfl_sync(0xFFFFFFFFu, row, (4 * lane + 3) & 31);
      if (lane < 8) tma_gather4(smem_u32(&s.raw[st][lane * kGroupBytes]), tm, 0, r0, r1, r2, r3, bar);
      ++g;
    }
  }
  cp_async_wait<0>();  // no index copy may outlive the CTA
  // nor a TMA copy: the stages and Q buffers armed last have landed before the
  // producer returns, even after a timed-out wait (in a normal run these
  // phases completed long ago and the waits return at once).  These waits
  // keep the full limit whatever the hand-off limit is.
  for (int x = g > kRawStages ? g - kRawStages : 0; x < g; ++x)
    (void)warp_wait(smem_u32(&s.raw_full[x % kRawStages]), (x / kRawStages) & 1, 26);
  for (int x = qc > kQBufs ? qc - kQBufs : 0; x < qc; ++x)
    (void)warp_wait(smem_u32(&s.q_full[x % kQBufs]), (x / kQBufs) & 1, 27);
}

// ------------------------------------------------------------------ dequant (warps 1-8)
__device__ void dequant(const DecodeArgs& a, Smem& s, int nunits, int dw, int lane) {
  int g = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
    const int nch = unit_of(a, u).nch;
    for (int c = 0; c < nch; ++c, ++g) {
      const int st = g % kRawStages, ks = g % kKStages;
      if (ok) ok = warp_acquire(smem_u32(&s.raw_full[st]), (g / kRawStages) & 1, 22, a.wait_iters);
      const uint8_t* rs = s.raw[st];
      uint8_t* kst = reinterpret_cast<uint8_t*>(s.k[ks]);
      // all of this warp's rows are loaded before any is converted, so their
      // shared-memory loads and conversion chains overlap.  Lane l converts
      // bytes [8l, 8l+8) and [256+8l, 256+8l+8): each of the two 16-byte
      // stores per row is contiguous across the warp.
      uint2 w0[kRowsPerDequantWarp], w1[kRowsPerDequantWarp];
      float sc0[kRowsPerDequantWarp], sc1[kRowsPerDequantWarp];
      uint4 rope[kRowsPerDequantWarp];
      bool vrow[kRowsPerDequantWarp];
#pragma unroll
      for (int i = 0; i < kRowsPerDequantWarp; ++i) {
        const int r = dw + kDequantWarps * i;
        if (r < kBN) {
          const uint8_t* row = rs + (r >> 2) * kGroupBytes + (r & 3) * kRowBytes;
          vrow[i] = s.valid[st][r] != 0;
          w0[i] = reinterpret_cast<const uint2*>(row)[lane];
          w1[i] = reinterpret_cast<const uint2*>(row + 256)[lane];
          const float* scl = reinterpret_cast<const float*>(row + kScaleOff);
          sc0[i] = scl[lane >> 4];
          sc1[i] = scl[2 + (lane >> 4)];
          rope[i] = lane < 8 ? reinterpret_cast<const uint4*>(row + kRopeOff)[lane] : make_uint4(0, 0, 0, 0);
        }
      }
      // the raw stage is consumed (its values are in registers): hand it back
      // to the producer, then wait for the K stage
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.raw_empty[st]));
      if (g >= kKStages && ok)
        ok = warp_wait_n(smem_u32(&s.k_empty[ks]), ((g / kKStages) + 1) & 1, 23, a.wait_iters);
#pragma unroll
      for (int i = 0; i < kRowsPerDequantWarp; ++i) {
        const int r = dw + kDequantWarps * i;
        if (r < kBN) {
          uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
          if (vrow[i]) {
            dequant4_hw_x2(w0[i].x, sc0[i], o0.x, o0.y);
            dequant4_hw_x2(w0[i].y, sc0[i], o0.z, o0.w);
            dequant4_hw_x2(w1[i].x, sc1[i], o1.x, o1.y);
            dequant4_hw_x2(w1[i].y, sc1[i], o1.z, o1.w);
          }
          uint4* dst = reinterpret_cast<uint4*>(kst + r * kRowStrideB);
          dst[lane] = o0;
          dst[32 + lane] = o1;
          if (lane < 8)
            reinterpret_cast<uint4*>(kst + r * kRowStrideB + kNope * 2)[lane] =
                vrow[i] ? rope[i] : make_uint4(0, 0, 0, 0);
          if (lane == 0) s.kvalid[ks][r] = vrow[i] ? 1 : 0;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.k_full[ks]));
    }
  }
}

// ------------------------------------------------------------------ compute warps
// QK: warp w owns tokens 16 (w % 2).. +15 and k-steps 9 (w / 2).. +8 of
// d = 576; its Q fragments stay in registers for the whole unit, so each
// chunk reads K once and Q not at all.  Softmax: thread t owns head t / 16 and
// tokens 2 (t % 16), +1.  PV: warp w owns output dims 64 w.. +63.
__device__ void compute(const DecodeArgs& a, Smem& s, int nunits, int cw, int lane) {
  const int gq = lane >> 2, q4 = lane & 3;  // mma fragment row group / column pair
  const int tg = cw % kTokGroups, dp = cw / kTokGroups;
  const int n0 = 16 * tg;                   // this warp's tokens in S
  const int k0 = dp * kPartSteps;           // and its share of d (k-steps)
  const int d0 = kOutDims * cw;             // this warp's output dims
  const int ct = cw * 32 + lane;            // softmax: head sh, tokens 2 sp2, +1
  const int sh = ct >> 4, sp2 = ct & 15;
  const uint32_t p_base = smem_u32(s.p);
  int g = 0, qc = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
    const Unit x = unit_of(a, u);
    float acc[kOutTiles][4];
#pragma unroll
    for (int i = 0; i < kOutTiles; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;   // head sh (shared by its 16 threads)
    if (x.nch > 0) {
      const int qb = qc % kQBufs;
      if (ok) ok = warp_acquire(smem_u32(&s.q_full[qb]), (qc / kQBufs) & 1, 24, a.wait_iters);
      uint32_t qf[kPartSteps][4];
      {
        const uint32_t qa0 = smem_u32(s.q[qb]) + (((lane & 15) * kKStride + (lane >> 4) * 8) << 1);
#pragma unroll
        for (int i = 0; i < kPartSteps; ++i)
          ldmatrix_x4(qa0 + (k0 + i) * 32, qf[i][0], qf[i][1], qf[i][2], qf[i][3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.q_empty[qb]));  // Q now lives in registers
      ++qc;
      for (int c = 0; c < x.nch; ++c, ++g) {
        const int ks = g % kKStages;
        if (ok) ok = warp_acquire(smem_u32(&s.k_full[ks]), (g / kKStages) & 1, 25, a.wait_iters);
        const uint32_t k_base = smem_u32(s.k[ks]);
        // ---- partial S: two n8 tiles (tokens n0..n0+15) over this warp's k-steps
        float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        // B rows: lane l -> token n0 + 8 (l >> 4) + (l & 7), k half (l >> 3) & 1
        const uint32_t kb0 =
            k_base + (((n0 + ((lane >> 4) << 3) + (lane & 7)) * kKStride + ((lane >> 3) & 1) * 8) << 1);
#pragma unroll
        for (int i = 0; i < kPartSteps; ++i) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kb0 + (k0 + i) * 32, b0, b1, b2, b3);
          mma_bf16_16816(sa[0], qf[i][0], qf[i][1], qf[i][2], qf[i][3], b0, b1);
          mma_bf16_16816(sa[1], qf[i][0], qf[i][1], qf[i][2], qf[i][3], b2, b3);
        }
#pragma unroll
        for (int t2 = 0; t2 < 2; ++t2) {
          const int col = n0 + 8 * t2 + 2 * q4;
          s.sp[dp][gq][col] = sa[t2][0];
          s.sp[dp][gq][col + 1] = sa[t2][1];
          s.sp[dp][gq + 8][col] = sa[t2][2];
          s.sp[dp][gq + 8][col + 1] = sa[t2][3];
        }
        named_sync_ws();
        // ---- online softmax (exp2 form; a still -inf maximum is replaced by
        // 0, so a fully masked chunk contributes nothing)
        {
          float x0 = 0.f, x1 = 0.f;
#pragma unroll
          for (int p = 0; p < kDParts; ++p) {
            x0 += s.sp[p][sh][2 * sp2];
            x1 += s.sp[p][sh][2 * sp2 + 1];
          }
          x0 = s.kvalid[ks][2 * sp2] != 0 ? x0 * a.scale_log2 : -INFINITY;
          x1 = s.kvalid[ks][2 * sp2 + 1] != 0 ? x1 * a.scale_log2 : -INFINITY;
          float mt = fmaxf(x0, x1);
#pragma unroll
          for (int o = 1; o < 16; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xFFFFFFFFu, mt, o));
          const float mn = fmaxf(m_run, mt);
          const float safe = mn == -INFINITY ? 0.f : mn;
          const float p0 = exp2f(x0 - safe), p1 = exp2f(x1 - safe);
          *reinterpret_cast<uint32_t*>(&s.p[sh * kPStride + 2 * sp2]) = pack_bf16x2(p0, p1);
          float ps = p0 + p1;
#pragma unroll
          for (int o = 1; o < 16; o <<= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, o);
          const float al = exp2f(m_run - safe);
          l_run = l_run * al + ps;
          m_run = mn;
          if (sp2 == 0) s.alpha[sh] = al;
        }
        named_sync_ws();
        // ---- O = alpha O + P V over this warp's output dims
        {
          const float al0 = s.alpha[gq], al1 = s.alpha[gq + 8];
#pragma unroll
          for (int i = 0; i < kOutTiles; ++i) {
            acc[i][0] *= al0;
            acc[i][1] *= al0;
            acc[i][2] *= al1;
            acc[i][3] *= al1;
          }
        }
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(p_base + (((lane & 15) * kPStride + kk * 16 + (lane >> 4) * 8) << 1), a0, a1, a2, a3);
          const int tok = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int nt = 0; nt < kOutTiles; nt += 2) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(k_base + ((tok * kKStride + d0 + nt * 8 + (lane >> 4) * 8) << 1), b0, b1,
                              b2, b3);
            mma_bf16_16816(acc[nt], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(acc[nt + 1], a0, a1, a2, a3, b2, b3);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&s.k_empty[ks]));
      }
    }
    // ---- epilogue: rows gq and gq+8 of the unit's heads
    if (sp2 == 0) {
      s.m_fin[sh] = m_run;
      s.l_fin[sh] = l_run;
    }
    named_sync_ws();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = gq + 8 * h;
      const float l = s.l_fin[row], mr = s.m_fin[row];
      if (row >= x.nh) continue;
      const int hd = x.head0 + row;
      const float inv = l > 0.f ? 1.f / l : 1.f;
      const float lse_v = l > 0.f ? mr * kLn2 + logf(l) : -INFINITY;
      uint16_t* o;
      if (a.num_splits == 1) {
        o = static_cast<uint16_t*>(a.out) + x.t * a.out_st + (int64_t)hd * a.out_sh;
        if (a.lse != nullptr && cw == 0 && q4 == 0) a.lse[x.t * a.lse_st + hd] = lse_v;
      } else {
        const int64_t base = (x.t * a.H + hd) * a.num_splits + x.split;
        o = reinterpret_cast<uint16_t*>(a.ws_o) + base * kNope;
        if (cw == 0 && q4 == 0) a.ws_lse[base] = lse_v;
      }
#pragma unroll
      for (int nt = 0; nt < kOutTiles; ++nt)
        *reinterpret_cast<uint32_t*>(o + d0 + nt * 8 + 2 * q4) =
            pack_bf16x2(acc[nt][2 * h] * inv, acc[nt][2 * h + 1] * inv);
    }
    named_sync_ws();  // m_fin / l_fin are rewritten by the next unit
  }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    decode_ws_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap tm) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = ((raw_base + 127u) & ~127u) - raw_base;
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + pad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nunits = a.T * a.G * a.hb_per_group * a.num_splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(smem_u32(&s.raw_full[i]), 1);
      mbar_init(smem_u32(&s.raw_empty[i]), kDequantWarps);
    }
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(smem_u32(&s.k_full[i]), kDequantWarps);
      mbar_init(smem_u32(&s.k_empty[i]), kComputeWarps);
    }
    for (int i = 0; i < kQBufs; ++i) {
      mbar_init(smem_u32(&s.q_full[i]), 1);
      mbar_init(smem_u32(&s.q_empty[i]), kComputeWarps);
    }
    mbar_init_fence();
  }
  // Q buffers start zeroed: a unit with fewer than 16 heads leaves its padding
  // rows finite (they are computed and never stored)
  for (int i = threadIdx.x; i < kQBufs * kBH * kKStride / 8; i += kThreads)
    reinterpret_cast<uint4*>(s.q)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();  // the zeros before any bulk copy into the buffers
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();  // the previous kernel of the stream has completed: global memory from here on

  if (warp == 0) {
    producer(a, s, &tm, nunits, lane);
  } else if (warp < kFirstCompute) {
    dequant(a, s, nunits, warp - 1, lane);
  } else {
    compute(a, s, nunits, warp - kFirstCompute, lane);
  }
}

}  // namespace ws

bool decode_ws_supported(const DecodeArgs& a) {
  return a.q_dtype == FP8MLA_DTYPE_BF16 && a.num_slots > 0 && a.num_slots < (1ll << 31) &&
         a.block_h <= ws::kBH && a.T > 0;
}

int launch_decode_ws(const DecodeArgs& a, int sms, cudaStream_t st) {
  // the pool as [num_slots] rows of 82 uint64: one gather4 box = 4 whole rows
  CUtensorMap tm;
  if (int rc = encode_row_map(&tm, a.kv, a.num_slots, kRowBytes / 8)) return rc;
  const size_t smem = sizeof(ws::Smem) + 128;
  cudaError_t e = cudaFuncSetAttribute(ws::decode_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "decode_ws smem attribute");
  const int64_t units = (int64_t)a.T * a.G * a.hb_per_group * a.num_splits;
  const unsigned grid = (unsigned)(units < sms ? units : sms);
  int rc = check_cuda(launch_pdl(ws::decode_ws_kernel, dim3(grid), dim3(ws::kThreads), smem, st, a, tm),
                      "decode_ws_kernel launch");
  if (rc != FP8MLA_OK || a.num_splits == 1) return rc;
  return launch_merge_splits(a, st);
}

int read_device_status_ws(unsigned int* status, bool reset, cudaStream_t st) {
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
