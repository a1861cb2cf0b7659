// decode_sh.cu -- sparse MLA decode for head blocks of <= 16 heads of one kv
// group (bf16 q) on one SM, with tcgen05 MMAs in the swapped orientation:
// tokens and output dims on M, heads on N.
//
//   S^T = K Q^T      M=64 tokens, N=16 heads, K=576 (36 k-steps).  A = the
//                    tile's bf16 key rows in shared memory (K-major), B = Q^T
//   O^T += V^T P^T   M=128 output dims (four MMAs cover the 512), N=16 heads,
//                    K=64 tokens (4 k-steps).  A = the same key rows read
//                    MN-major (V is the first 512 dims of K), B = P^T
// In the usual orientation a 16-head block fills an M=128 MMA with 112 rows
// of padding; swapped, every MMA row is a real token or output dim, and an
// MMA costs about its shared-memory operand bytes / 128 B per cycle.
//
// One CTA per SM walks units u = blockIdx.x, blockIdx.x + gridDim.x, ...; a
// unit is (query token, head block of one kv group, top-k split), as in the
// split/merge contract below.  A unit's top-k rows are taken in 64-token
// tiles numbered over all of the CTA's units, so every ring runs across unit
// boundaries.
//
// Warp roles (512 threads; warp w runs on SM sub-partition w % 4):
//   warps 0-3   softmax + epilogue.  S^T of an M=64 MMA sits in lanes
//               [32w, 32w+16) of sub-partition w (token 16w + i in lane
//               32w + i), so lanes 0-15 of softmax warp w own tokens
//               [16w, 16w+16) of a tile; all 32 lanes of a warp own output
//               dims in the epilogue (O^T lane = dim).
//   warp 4      tensor memory allocation; lane 0 issues every MMA and each
//               unit's Q^T load (a 3-D TMA box per 64 dims, landing swizzled)
//   warps 5, 8, 12
//               producers: top-k entries -> slots (block table included for
//               the paged entry point, software-pipelined) -> tile::gather4
//               of whole 656-B rows into a 5-stage raw ring of 16-row
//               stages.  The four gather4 of a stage are spread over the
//               three warps: one warp issues about one gather4 per 300
//               cycles (2.3 TB/s over 148 SMs, measured), and the rate grows
//               with the number of issuing warps.
//   warps 6, 7, 9-11, 13-15
//               dequant: raw rows -> bf16 key rows of the two-stage KV ring
//               (e4m3 * tile scale in fp32, RNE to bf16; rope copied), masked
//               rows written as zeros, a validity byte per token
//   (sub-partition 0, which issues the MMAs, carries no dequant work)
// MMA order per tile g: QK(g), then PV(g-1), so softmax(g) overlaps PV(g-1)
// and QK(g+1) overlaps the dequant of tile g+2.  At a unit's first tile the
// order is Q^T load, PV(g-1), QK(g), so the load overlaps the previous unit's
// last softmax and PV.
//
// Tensor memory (256 columns): O^T of two units [0,128) (64 columns each:
// four 128-dim blocks x 16 heads), S^T of two tiles [128,160).
// Shared memory (about 225 KB):
//   kv   2 stages: 64 tokens x 576 dims, 9 swizzled blocks of 64 rows   144 KB
//   q    Q^T: 16 heads x 576 dims, 9 swizzled blocks of 16 rows          18 KB
//   p    2 buffers: P^T (bf16) of 16 heads x 64 tokens                    4 KB
//   raw  5 stages: 16 rows as gathered by TMA                            52.5 KB
// Every wait is bounded; after a failed wait a role stops, and the producer
// and the MMA issuer drain what they issued (full limit) before returning.
// The softmax warps meet through mbarriers, never bar.sync, so a warp that
// stops cannot leave the others blocked.  No load uses cluster multicast.
//
// Reference semantics: vllm_fp8kv/fp8_ds_mla_sparse_decode.py:77-211 (masking,
// dequant, NaN-free online softmax, LSE) and the split/merge contract of
// tests/fixtures/triton_mla_sparse_kernel_pr47629.py:232-403.
#include <cuda.h>

#include "common.cuh"
#include "decode.h"
#include "tc_cluster.cuh"
#include "tc_ptx.cuh"
#include "tma_map.h"

namespace fp8mla {
namespace sh {

using namespace fp8mla::tc;

namespace {

constexpr int kBH = 16;             // heads per unit (MMA N)
constexpr int kTileN = 64;          // tokens per tile (QK M)
constexpr int kKSteps = kDqk / 16;  // 36
constexpr int kStageRows = 16;      // rows per raw stage
constexpr int kStagesPerTile = kTileN / kStageRows;  // 4
constexpr int kRawStages = 5;
constexpr int kGroupBytes = 2688;   // 4 whole rows (2624 B) padded to a multiple of 128
constexpr int kRawStageBytes = (kStageRows / 4) * kGroupBytes;
constexpr int kKVBlockBytes = kTileN * 128;          // 64 rows of a 64-dim block
constexpr int kKVStageBytes = 9 * kKVBlockBytes;
constexpr int kKVStages = 2;
constexpr int kQBlockBytes = kBH * 128;
constexpr int kPBytes = kBH * 128;  // 16 heads x 64 tokens bf16
constexpr int kPBufs = 2;
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kProducerWarps = 3;  // warps 5, 8, 12
constexpr int kDequantWarps = 8;
constexpr int kThreads = 16 * 32;
// dequant index of warp w (6, 7, 9-11, 13-15 -> 0-7)
__device__ __forceinline__ int dequant_index(int w) {
  return w < 8 ? w - 6 : w < 12 ? (w == 8 ? -1 : w - 7) : (w == 12 ? -1 : w - 8);
}
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColO = 0, kColS = 128;
constexpr float kRescaleThreshold = 8.0f;
// rows of a raw stage per dequant warp
constexpr int kRowsPerWarp = kStageRows / kDequantWarps;  // 2

// kind::f16 instruction descriptors (fp32 accumulate, bf16 A and B)
constexpr uint32_t kIdescQK = idesc_bf16(kTileN, kBH, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, kBH, false) | (1u << 15);  // A MN-major

struct Smem {
  uint8_t kv[kKVStages][kKVStageBytes];  // 1024-aligned (offset 0)
  uint8_t q[9 * kQBlockBytes];
  uint8_t p[kPBufs][kPBytes];
  uint8_t raw[kRawStages][kRawStageBytes];  // gather4 destinations (128-B aligned)
  float pmax[2][kSoftmaxWarps][kBH];         // per-warp tile max, by tile parity
  float lpart[2][kSoftmaxWarps][kBH];        // per-warp row sums, by unit parity
  float mfin[2][kBH];                        // a unit's final max, by unit parity
  uint8_t rvalid[kRawStages][kStageRows];    // producer: row live
  uint8_t tvalid[kKVStages][kTileN];         // dequant: token of the KV stage live
  uint64_t raw_full[kRawStages], raw_empty[kRawStages];
  uint64_t kvfull[kKVStages], kvempty[kKVStages];
  uint64_t sfull[2], pfull[kPBufs], pvdone[2];
  uint64_t xch[2], fin;
  uint64_t qfull, qempty, ofull[2], oempty[2], drain;
  uint32_t tmem_base;
};
static_assert(offsetof(Smem, kv) == 0 && offsetof(Smem, q) % 1024 == 0 &&
                  offsetof(Smem, p) % 1024 == 0 && kKVStageBytes % 1024 == 0,
              "swizzle atoms need 1024-B alignment");
static_assert(offsetof(Smem, raw) % 128 == 0 && kRawStageBytes % 128 == 0, "TMA destinations");
static_assert(offsetof(Smem, raw_full) % 8 == 0, "");
static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

struct Unit {
  int64_t t;
  int head0, nh, split, beg, end, nt;
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
  x.nt = x.end > x.beg ? (x.end - x.beg + kTileN - 1) / kTileN : 0;
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

// A raw stage's position in the CTA's sequence: unit u, tile t, stage q.
struct Pos {
  int u, t, q;
  Unit x;
  int32_t req;
};
__device__ __forceinline__ void pos_settle(Pos& p, const DecodeArgs& a, int nunits) {
  while (p.u < nunits && p.t >= p.x.nt) {
    p.u += gridDim.x;
    p.t = 0;
    p.q = 0;
    if (p.u < nunits) {
      p.x = unit_of(a, p.u);
      p.req = request_of(a, p.x.t);
    }
  }
}
__device__ __forceinline__ void pos_init(Pos& p, const DecodeArgs& a, int nunits) {
  p.u = blockIdx.x;
  p.t = 0;
  p.q = 0;
  if (p.u < nunits) {
    p.x = unit_of(a, p.u);
    p.req = request_of(a, p.x.t);
  }
  pos_settle(p, a, nunits);
}
__device__ __forceinline__ void pos_next(Pos& p, const DecodeArgs& a, int nunits) {
  if (p.u >= nunits) return;
  if (++p.q == kStagesPerTile) {
    p.q = 0;
    ++p.t;
    pos_settle(p, a, nunits);
  }
}
// Lane i < 16: the raw top-k entry of row i of stage p (-1 past the unit or
// the sequence).
__device__ __forceinline__ int32_t pos_raw(const Pos& p, int nunits, int lane) {
  if (p.u >= nunits || lane >= kStageRows) return -1;
  const int pos = p.x.beg + p.t * kTileN + p.q * kStageRows + lane;
  return pos < p.x.end ? p.x.idx_row[pos] : -1;
}

// ------------------------------------------------------------------ producers (warps 5, 8, 12)
// Every producer warp walks the whole stage sequence and converts the
// stage's 16 entries (lanes 0-15); gather group k (rows 4k..4k+3) of stage
// g4 is issued by warp (4 g4 + k) % 3.  Index pipeline: raw entries three
// stages ahead and the block-table read of the next stage (paged), so no
// stage waits on a load issued in its own step.
__device__ void producer(const DecodeArgs& a, Smem& s, const CUtensorMap* tm, int nunits, int pw,
                         int lane) {
  Pos cur, nx, ah;
  pos_init(cur, a, nunits);
  nx = cur;
  pos_next(nx, a, nunits);
  ah = nx;
  int32_t r1 = pos_raw(nx, nunits, lane);  // stage +1
  pos_next(ah, a, nunits);
  int32_t r2 = pos_raw(ah, nunits, lane);  // stage +2
  pos_next(ah, a, nunits);
  int32_t r3 = pos_raw(ah, nunits, lane);  // stage +3
  pos_next(ah, a, nunits);                 // ah: stage +4
  SlotPf f = slot_fetch(a, cur.req, pos_raw(cur, nunits, lane));
  int g4 = 0;
  bool ok = true;
  while (cur.u < nunits) {
    const int32_t slot = slot_finish(a, f);
    f = slot_fetch(a, nx.req, r1);
    r1 = r2;
    r2 = r3;
    r3 = pos_raw(ah, nunits, lane);
    cur = nx;
    pos_next(nx, a, nunits);
    pos_next(ah, a, nunits);
    const int st = g4 % kRawStages;
    if (g4 >= kRawStages)
      ok = warp_wait_n(smem_u32(&s.raw_empty[st]), ((g4 / kRawStages) + 1) & 1, 16, a.wait_iters);
    if (!ok) break;
    const int k0 = (pw - (4 * g4) % kProducerWarps + kProducerWarps) % kProducerWarps;  // first group
    const int ngroups = k0 + kProducerWarps < kStageRows / 4 ? 2 : 1;
    const int gk = lane >> 2;  // group of row `lane`
    if (lane < kStageRows && (gk == k0 || gk == k0 + kProducerWarps))
      s.rvalid[st][lane] = slot >= 0 ? 1 : 0;
    const int32_t row = slot >= 0 ? slot : 0;  // masked: a valid row, flagged invalid
    const int src = (4 * lane) & 15;
    const int32_t g0 = __shfl_sync(0xFFFFFFFFu, row, src);
    const int32_t g1 = __shfl_sync(0xFFFFFFFFu, row, src + 1);
    const int32_t g2 = __shfl_sync(0xFFFFFFFFu, row, src + 2);
    const int32_t g3 = __shfl_sync(0xFFFFFFFFu, row, src + 3);
    const uint32_t bar = smem_u32(&s.raw_full[st]);
    __syncwarp();  // the flags (generic stores) are released by the arrive below
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)ngroups * 4 * kRowBytes);
    __syncwarp();
    if (lane < kStageRows / 4 && (lane == k0 || lane == k0 + kProducerWarps))
      tma_gather4(smem_u32(s.raw[st]) + lane * kGroupBytes, tm, 0, g0, g1, g2, g3, bar);
    ++g4;
  }
  // the stages armed last have landed before the producer returns, even after
  // a failed wait (full limit)
  for (int x = g4 > kRawStages ? g4 - kRawStages : 0; x < g4; ++x)
    (void)warp_wait(smem_u32(&s.raw_full[x % kRawStages]), (x / kRawStages) & 1, 17);
}

// ------------------------------------------------------------------ dequant
// Warp dw takes rows 2 dw, 2 dw + 1 of every raw stage (8 rows of a tile).
// Lane l converts latent bytes [8l, 8l+8) and [256+8l, 256+8l+8) and copies
// rope bytes [4l, 4l+4), so every 8-lane phase of a 16-byte store fills one
// 128-byte swizzled row.  All four stages of a tile are read into registers
// (and handed back) before the warp waits for its KV stage, so the raw ring
// keeps refilling while PV(g-2) still holds the stage.
__device__ void dequant(const DecodeArgs& a, Smem& s, int nunits, int dw, int lane) {
  constexpr int kRows = kStagesPerTile * kRowsPerWarp;  // 8
  int g = 0, g4 = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
    const int nt = unit_of(a, u).nt;
    for (int t = 0; t < nt && ok; ++t, ++g) {
      const int ks = g % kKVStages;
      uint8_t* kst = s.kv[ks];
      uint2 w0[kRows], w1[kRows];
      float sc0[kRows], sc1[kRows];
      uint32_t rope[kRows];
      uint32_t vbits = 0;
#pragma unroll
      for (int q = 0; q < kStagesPerTile; ++q) {
        const int st = (g4 + q) % kRawStages;
        ok = warp_acquire(smem_u32(&s.raw_full[st]), ((g4 + q) / kRawStages) & 1, 18, a.wait_iters);
        if (!ok) break;
        const uint8_t* rs = s.raw[st];
#pragma unroll
        for (int e = 0; e < kRowsPerWarp; ++e) {
          const int r = kRowsPerWarp * dw + e, i = q * kRowsPerWarp + e;
          const uint8_t* row = rs + (r >> 2) * kGroupBytes + (r & 3) * kRowBytes;
          if (s.rvalid[st][r] != 0) vbits |= 1u << i;
          w0[i] = reinterpret_cast<const uint2*>(row)[lane];
          w1[i] = reinterpret_cast<const uint2*>(row + 256)[lane];
          const float* scl = reinterpret_cast<const float*>(row + kScaleOff);
          sc0[i] = scl[lane >> 4];
          sc1[i] = scl[2 + (lane >> 4)];
          rope[i] = reinterpret_cast<const uint32_t*>(row + kRopeOff)[lane];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&s.raw_empty[st]));  // stage in registers
      }
      g4 += kStagesPerTile;
      if (!ok) break;
      // the KV stage: released by PV(g-2)
      if (g >= kKVStages)
        ok = warp_wait_n(smem_u32(&s.kvempty[ks]), ((g / kKVStages) + 1) & 1, 19, a.wait_iters);
      if (!ok) break;
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int tr = (i / kRowsPerWarp) * kStageRows + kRowsPerWarp * dw + (i % kRowsPerWarp);
        const bool v = (vbits >> i) & 1u;
        uint4 o0 = make_uint4(0, 0, 0, 0), o1 = make_uint4(0, 0, 0, 0);
        if (v) {
          dequant4_hw_x2(w0[i].x, sc0[i], o0.x, o0.y);
          dequant4_hw_x2(w0[i].y, sc0[i], o0.z, o0.w);
          dequant4_hw_x2(w1[i].x, sc1[i], o1.x, o1.y);
          dequant4_hw_x2(w1[i].y, sc1[i], o1.z, o1.w);
        }
        *reinterpret_cast<uint4*>(kst + (lane >> 3) * kKVBlockBytes + swz(tr, lane & 7)) = o0;
        *reinterpret_cast<uint4*>(kst + (4 + (lane >> 3)) * kKVBlockBytes + swz(tr, lane & 7)) = o1;
        *reinterpret_cast<uint32_t*>(kst + 8 * kKVBlockBytes + swz(tr, lane >> 2) + 4 * (lane & 3)) =
            v ? rope[i] : 0u;
        if (lane == 0) s.tvalid[ks][tr] = v ? 1 : 0;
      }
      fence_proxy_async_smem();  // generic stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.kvfull[ks]));
    }
  }
}

// ------------------------------------------------------------------ MMA issuer (warp 4, lane 0)
__device__ void mma_role(const DecodeArgs& a, Smem& s, int nunits, uint32_t tmem,
                         const CUtensorMap* tm_q) {
  const uint32_t iters = a.wait_iters;
  const uint64_t qd0 = sdesc_sw128(smem_u32(s.q), 16, 1024);
  const uint64_t kd0 = sdesc_sw128(smem_u32(s.kv[0]), 16, 1024);
  const uint64_t vd0 = sdesc_sw128(smem_u32(s.kv[0]), kKVBlockBytes, 1024);
  const uint64_t pd0 = sdesc_sw128(smem_u32(s.p[0]), 16, 1024);
  // the tile whose PV is still to be issued: global tile g, tile t of the
  // kk-th live unit, last tile of that unit or not
  int pg = -1, pt = 0, pkk = 0;
  bool plast = false;
  auto issue_pv = [&]() -> bool {
    const int ks = pg % kKVStages, pb = pg % kPBufs, ob = pkk & 1;
    if (!thread_wait_n(smem_u32(&s.pfull[pb]), (pg / kPBufs) & 1, 22, iters)) return false;
    // the first PV of a unit overwrites O^T buffer ob: the epilogue of the unit
    // two back has read it
    if (pt == 0 && pkk >= 2 &&
        !thread_wait_n(smem_u32(&s.oempty[ob]), ((pkk - 2) >> 1) & 1, 23, iters))
      return false;
    tc_fence_after();
#pragma unroll
    for (int kq = 0; kq < kTileN / 16; ++kq)
#pragma unroll
      for (int blk = 0; blk < 4; ++blk)
        mma_ss(tmem + kColO + 64 * ob + 16 * blk,
               vd0 + (uint64_t)((ks * kKVStageBytes + blk * 2 * kKVBlockBytes + kq * 16 * 128) >> 4),
               pd0 + (uint64_t)((pb * kPBytes + kq * 32) >> 4), kIdescPV, (pt > 0 || kq > 0) ? 1u : 0u);
    mma_commit(smem_u32(&s.kvempty[ks]));
    mma_commit(smem_u32(&s.pvdone[pg & 1]));
    if (plast) mma_commit(smem_u32(&s.ofull[ob]));
    return true;
  };
  bool ok = true, q_pending = false;  // a Q^T load issued and not yet seen landed
  int g = 0, kk = 0, q_phase = 0;     // qfull phase of the last Q^T load
  for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
    const Unit x = unit_of(a, u);
    const int nt = x.nt;
    if (nt == 0) continue;
    for (int t = 0; t < nt; ++t, ++g) {
      if (t == 0) {
        // Q^T of this unit, once the previous unit's QKs are complete
        if (kk > 0) ok = thread_wait_n(smem_u32(&s.qempty), (kk - 1) & 1, 20, iters);
        if (!ok) break;
        mbar_arrive_expect_tx(smem_u32(&s.qfull), 9 * kQBlockBytes);
        q_pending = true;
        q_phase = kk;
#pragma unroll 1
        for (int b = 0; b < 9; ++b)
          tma_load_3d(smem_u32(s.q) + b * kQBlockBytes, tm_q, 64 * b, x.head0, (int32_t)x.t,
                      smem_u32(&s.qfull));
        if (pg >= 0) ok = issue_pv();  // the previous unit's last PV while Q^T lands
        pg = -1;
        if (ok) ok = thread_wait_n(smem_u32(&s.qfull), kk & 1, 31, iters);
        if (ok) q_pending = false;
      }
      const int ks = g % kKVStages;
      if (ok) ok = thread_wait_n(smem_u32(&s.kvfull[ks]), (g / kKVStages) & 1, 21, iters);
      if (!ok) break;
      tc_fence_after();
      const uint32_t dS = tmem + kColS + 16 * (g & 1);
#pragma unroll
      for (int kst = 0; kst < kKSteps; ++kst)
        mma_ss(dS,
               kd0 + (uint64_t)((ks * kKVStageBytes + (kst >> 2) * kKVBlockBytes + (kst & 3) * 32) >> 4),
               qd0 + (uint64_t)((((kst >> 2) * kQBlockBytes) + (kst & 3) * 32) >> 4), kIdescQK,
               kst > 0 ? 1u : 0u);
      mma_commit(smem_u32(&s.sfull[g & 1]));
      if (t == nt - 1) mma_commit(smem_u32(&s.qempty));  // Q^T free for the next unit
      if (pg >= 0) ok = issue_pv();
      if (!ok) break;
      pg = g;
      pt = t;
      pkk = kk;
      plast = t == nt - 1;
    }
    ++kk;
  }
  if (ok && pg >= 0) (void)issue_pv();
  // drain: no Q^T copy may outlive the CTA, nor any MMA run when tensor
  // memory is freed
  if (q_pending) (void)thread_wait(smem_u32(&s.qfull), q_phase & 1, 26);
  mma_commit(smem_u32(&s.drain));
  (void)thread_wait(smem_u32(&s.drain), 0, 24);
}

// ------------------------------------------------------------------ softmax + epilogue (warps 0-3)
// Reduce-scatter of v[16] over the 16 lanes of each half-warp: afterwards lane
// i holds op over those lanes of element (i & 15).
template <bool kMax>
__device__ __forceinline__ float reduce16(const float (&v)[16], int lane) {
  float a8[8], a4[4], a2[2];
  const bool b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1, b1 = (lane >> 1) & 1, b0 = lane & 1;
  auto op = [](float x, float y) { return kMax ? fmaxf(x, y) : x + y; };
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = b3 ? v[i] : v[i + 8], keep = b3 ? v[i + 8] : v[i];
    a8[i] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 8));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b2 ? a8[i] : a8[i + 4], keep = b2 ? a8[i + 4] : a8[i];
    a4[i] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 4));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b1 ? a4[i] : a4[i + 2], keep = b1 ? a4[i + 2] : a4[i];
    a2[i] = op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 2));
  }
  const float send = b0 ? a2[0] : a2[1], keep = b0 ? a2[1] : a2[0];
  return op(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 1));
}

__device__ __forceinline__ uint16_t bf16_bits(float x) {
  return (uint16_t)(pack_bf16x2(x, 0.f) & 0xFFFFu);
}

__device__ void softmax_role(const DecodeArgs& a, Smem& s, int nunits, int w, int lane,
                             uint32_t tmem) {
  const uint32_t iters = a.wait_iters;
  const int L = threadIdx.x;             // 0..127: O^T lane (output dim within a block)
  const bool tl = lane < 16;             // lane holds a token of the M=64 S^T
  const int tok = 16 * w + (lane & 15);  // that token within the tile
  const uint32_t trow = tmem + ((uint32_t)(32 * w) << 16);

  auto dst_row = [&](const Unit& x, int h) -> uint16_t* {
    const int hd = x.head0 + h;
    return a.num_splits == 1
               ? static_cast<uint16_t*>(a.out) + x.t * a.out_st + (int64_t)hd * a.out_sh
               : reinterpret_cast<uint16_t*>(a.ws_o) + ((x.t * a.H + hd) * a.num_splits + x.split) * kNope;
  };
  auto put_lse = [&](const Unit& x, int h, float v) {
    const int hd = x.head0 + h;
    if (a.num_splits == 1) {
      if (a.lse != nullptr) a.lse[x.t * a.lse_st + hd] = v;
    } else {
      a.ws_lse[(x.t * a.H + hd) * a.num_splits + x.split] = v;
    }
  };
  // epilogue of the kk-th live unit x: O^T / l -> output rows (or the split's
  // partial), LSE; then O^T buffer kk & 1 is released
  auto epilogue = [&](const Unit& x, int kk) -> bool {
    const int ob = kk & 1;
    if (!warp_wait_n(smem_u32(&s.ofull[ob]), (kk >> 1) & 1, 29, iters)) return false;
    tc_fence_after();
    float inv[kBH];
    float lmine = 0.f;
#pragma unroll
    for (int h = 0; h < kBH; ++h) {
      const float l = s.lpart[ob][0][h] + s.lpart[ob][1][h] + s.lpart[ob][2][h] + s.lpart[ob][3][h];
      inv[h] = l > 0.f ? 1.f / l : 0.f;
      if (h == (L & 15)) lmine = l;
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t o[32];
      tmem_ld32(trow + kColO + 64 * ob + 32 * half, o);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int h = i & 15, d = 128 * (2 * half + (i >> 4)) + L;
        if (h < x.nh) dst_row(x, h)[d] = bf16_bits(__uint_as_float(o[i]) * inv[h]);
      }
    }
    if (L < x.nh) put_lse(x, L, lmine > 0.f ? s.mfin[ob][L] * kLn2 + logf(lmine) : -INFINITY);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&s.oempty[ob]));
    return true;
  };

  bool ok = true, pend = false;
  Unit px;
  int pkk = 0, g = 0, kk = 0;
  float m[kBH], l[kBH];
  for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
    const Unit x = unit_of(a, u);
    if (x.nt == 0) {  // an empty split: zero partial, LSE -inf
#pragma unroll 1
      for (int h = 0; h < x.nh; ++h) {
        uint16_t* d = dst_row(x, h);
        for (int c = L; c < kNope; c += 128) d[c] = 0;
      }
      if (L < x.nh) put_lse(x, L, -INFINITY);
      continue;
    }
    const int ob = kk & 1;
#pragma unroll
    for (int h = 0; h < kBH; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.f;
    }
    for (int t = 0; t < x.nt; ++t, ++g) {
      const int sb = g & 1;
      ok = warp_wait_n(smem_u32(&s.sfull[sb]), (g >> 1) & 1, 25, iters);
      if (ok) ok = warp_acquire(smem_u32(&s.kvfull[sb]), (g >> 1) & 1, 26, iters);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[16];
      tmem_ld16(trow + kColS + 16 * sb, sv);
      tmem_wait_ld();
      const bool valid = tl && s.tvalid[sb][tok] != 0;
      float (&xs)[kBH] = reinterpret_cast<float(&)[kBH]>(sv);  // scores, log2 domain
#pragma unroll
      for (int h = 0; h < kBH; ++h) xs[h] = valid ? __uint_as_float(sv[h]) * a.scale_log2 : -INFINITY;
      // tile max per head: this warp's 16 tokens, then the four warps
      const float wm = reduce16<true>(xs, lane);
      if (tl) s.pmax[sb][w][lane] = wm;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.xch[sb]));
      ok = warp_wait_n(smem_u32(&s.xch[sb]), (g >> 1) & 1, 27, iters);
      if (!ok) break;
      const int hl = lane & 15;
      const float tmine = fmaxf(fmaxf(s.pmax[sb][0][hl], s.pmax[sb][1][hl]),
                                fmaxf(s.pmax[sb][2][hl], s.pmax[sb][3][hl]));
      float al[kBH];
      bool any = false;
#pragma unroll
      for (int h = 0; h < kBH; ++h) {
        const float tmx = __shfl_sync(0xFFFFFFFFu, tmine, h);
        al[h] = 1.f;
        if (tmx > m[h] + kRescaleThreshold || (m[h] == -INFINITY && tmx > -INFINITY)) {
          al[h] = m[h] == -INFINITY ? 1.f : ex2_approx(m[h] - tmx);
          m[h] = tmx;
          l[h] *= al[h];
          any |= al[h] != 1.f;
        }
      }
      if (any && t > 0) {
        // O^T columns of the rescaled heads, once PV(g-1) has written them
        ok = warp_wait_n(smem_u32(&s.pvdone[(g - 1) & 1]), ((g - 1) >> 1) & 1, 28, iters);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int blk = 0; blk < 4; ++blk) {
          uint32_t o[16];
          tmem_ld16(trow + kColO + 64 * ob + 16 * blk, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * al[i]);
          tmem_st16(trow + kColO + 64 * ob + 16 * blk, o);
        }
        tmem_wait_st();
      }
      // P^T: row h = head, 64 tokens per 128-byte swizzled row.  Buffer g & 1
      // was last read by PV(g-2), issued before QK(g): sfull(g) implies it is done.
      uint8_t* pbuf = s.p[g & 1];
#pragma unroll
      for (int h = 0; h < kBH; ++h) {
        const float p = valid ? ex2_approx(xs[h] - (m[h] == -INFINITY ? 0.f : m[h])) : 0.f;
        l[h] += p;
        if (tl)
          *reinterpret_cast<uint16_t*>(pbuf + h * 128 + ((((tok >> 3) ^ (h & 7))) << 4) + (tok & 7) * 2) =
              bf16_bits(p);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.pfull[g & 1]));
      if (pend && t == 0) {
        // the previous unit's epilogue, now that this unit's first PV can go
        ok = epilogue(px, pkk);
        pend = false;
        if (!ok) break;
      }
    }
    if (!ok) break;
    // the unit's row sums: this warp's 16 token lanes, per head
    const float lr = reduce16<false>(l, lane);
    if (tl) s.lpart[ob][w][lane] = lr;
    if (w == 0 && lane == 0) {
#pragma unroll
      for (int h = 0; h < kBH; ++h) s.mfin[ob][h] = m[h];
    }
    pend = true;
    px = x;
    pkk = kk;
    ++kk;
  }
  if (ok && pend) {
    // the last unit: every warp's row sums are written before any reads them
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&s.fin));
    if (warp_wait_n(smem_u32(&s.fin), 0, 30, iters)) (void)epilogue(px, pkk);
  }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    decode_sh_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap tm,
                     const __grid_constant__ CUtensorMap tm_q) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + pad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nunits = a.T * a.G * a.hb_per_group * a.num_splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(smem_u32(&s.raw_full[i]), kProducerWarps);
      mbar_init(smem_u32(&s.raw_empty[i]), kDequantWarps);
    }
    for (int i = 0; i < kKVStages; ++i) {
      mbar_init(smem_u32(&s.kvfull[i]), kDequantWarps);
      mbar_init(smem_u32(&s.kvempty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s.sfull[i]), 1);
      mbar_init(smem_u32(&s.pfull[i]), kSoftmaxWarps);
      mbar_init(smem_u32(&s.pvdone[i]), 1);
      mbar_init(smem_u32(&s.xch[i]), kSoftmaxWarps);
      mbar_init(smem_u32(&s.ofull[i]), 1);
      mbar_init(smem_u32(&s.oempty[i]), kSoftmaxWarps);
    }
    mbar_init(smem_u32(&s.fin), kSoftmaxWarps);
    mbar_init(smem_u32(&s.qfull), 1);
    mbar_init(smem_u32(&s.qempty), 1);
    mbar_init(smem_u32(&s.drain), 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&s.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();  // barriers initialised, tensor memory allocated
  tc_fence_after();
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();  // the previous kernel of the stream has completed: global memory from here on
  const uint32_t tmem = s.tmem_base;

  if (warp < kSoftmaxWarps) {
    softmax_role(a, s, nunits, warp, lane, tmem);
  } else if (warp == kMmaWarp) {
    if (lane == 0) mma_role(a, s, nunits, tmem, &tm_q);
    __syncwarp();
  } else if (warp == 5 || warp == 8 || warp == 12) {
    producer(a, s, &tm, nunits, warp == 5 ? 0 : warp == 8 ? 1 : 2, lane);
  } else {
    dequant(a, s, nunits, dequant_index(warp), lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace sh

bool decode_sh_supported(const DecodeArgs& a) {
  // Q^T comes by TMA: token and head strides must not overlap the rows
  const bool q_rows = a.q_sh >= kDqk && (a.T == 1 || a.q_st >= (int64_t)a.H * a.q_sh);
  return a.q_dtype == FP8MLA_DTYPE_BF16 && a.num_slots > 0 && a.num_slots < (1ll << 31) &&
         a.block_h <= sh::kBH && a.T > 0 && q_rows;
}

int launch_decode_sh(const DecodeArgs& a, int sms, cudaStream_t st) {
  // the pool as [num_slots] rows of 82 uint64: one gather4 box = 4 whole rows
  CUtensorMap tm, tm_q;
  if (int rc = encode_row_map(&tm, a.kv, a.num_slots, kRowBytes / 8)) return rc;
  if (int rc = encode_q_map(&tm_q, a.q, a.T, a.H, a.q_st, a.q_sh)) return rc;
  const size_t smem = sizeof(sh::Smem) + 1024;  // + alignment slack
  cudaError_t e = cudaFuncSetAttribute(sh::decode_sh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "decode_sh smem attribute");
  const int64_t units = (int64_t)a.T * a.G * a.hb_per_group * a.num_splits;
  const unsigned grid = (unsigned)(units < sms ? units : sms);
  int rc = check_cuda(launch_pdl(sh::decode_sh_kernel, dim3(grid), dim3(sh::kThreads), smem, st, a, tm, tm_q),
                      "decode_sh_kernel launch");
  if (rc != FP8MLA_OK || a.num_splits == 1) return rc;
  return launch_merge_splits(a, st);
}

int read_device_status_sh(unsigned int* status, bool reset, cudaStream_t st) {
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
