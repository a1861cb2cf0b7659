// decode_tc3.cu -- sparse MLA decode for 64 or 128 heads per kv group on a
// pair of SMs (a 2-CTA cluster) sharing cta_group::2 tcgen05 MMAs, with the
// selected rows staged in shared memory by TMA.
//
// The MMA side is decode_tc2.cu's: the pair splits the heads (CTA c owns
// heads [64c, 64c+64) and their S and O in its tensor memory), tiles are 64
// tokens, and
//   S = Q K^T   M=128 heads, N=64 tokens, K=576 (36 k-steps); B is split by N:
//               CTA c supplies the rows of its 32 "own" tokens [32c, 32c+32)
//   O += P V    M=128, N=256 dims (two MMAs), K=64 tokens; B is split by N:
//               CTA c supplies latent tiles c and c+2 (its "PV half")
// What changes is how rows reach shared memory.  A producer warp turns each
// top-k entry into a slot and issues TMA tile::gather4 copies (four rows per
// instruction) into a ring of raw fp8 stages; the dequant warps read those
// stages from shared memory instead of issuing global loads of their own, so
// the bytes in flight are bounded by the ring, not by L1, and no dequant warp
// waits on a global load.  A raw stage holds half a tile for this CTA: 16 own
// rows whole (656 B: latent, scales, rope) and the PV half of 16 rows of the
// other CTA (tiles c and c+2, 128 B each, and the 16 B of scales), fetched
// through three tensor maps over the pool (whole rows, 128-byte tiles,
// scales).  A masked slot fetches row 0 and is flagged invalid: its K and V
// rows are written as zeros and its score is replaced by -inf in the softmax
// (validity bits per tile), so a fully masked row still gives P = 0 and
// LSE = -inf.
//
// Tensor memory (512 columns, both CTAs), as decode_tc2.cu:
//   [  0,256)  O, dims [0,256) MMA in [0,128), dims [256,512) MMA in [128,256)
//   [256,320)  2 S buffers x 32 fp32 columns
//   [320,512)  Q dims [0,384), the A operand of 24 k-steps (lanes L and L^64
//              hold the same head)
// Shared memory (about 225 KB):
//   q    Q dims [384,576): 3 x 64-dim swizzled blocks of 64 rows      24 KB
//   k    2 stages: own 32 tokens x 576 dims, 9 blocks of 32 rows      72 KB
//   v    2 stages: 64 tokens x PV-half dims, 4 blocks of 64 rows      64 KB
//   p    2 stages: P (bf16) of 64 heads x 64 tokens                   16 KB
//   raw  3 half-tile stages of gathered fp8 rows                      45 KB
//
// Warp roles (448 threads per CTA):
//   warps 0-3   softmax + epilogue (thread L = TMEM lane L)
//   warp 4      TMEM allocation in both CTAs; lane 0 of the even CTA issues
//               every MMA of the pair
//   warps 5-12  dequant: part A = the PV half of the 64 tile rows (V stage,
//               and the K stage for own rows), part B = the other half and
//               the rope of the 32 own rows (K stage)
//   warp 13     producer: indices -> slots (block table included for the
//               paged entry point) -> gather4 into the raw ring
// Barriers that gate the issuing thread live in the even CTA and count
// arrivals of both CTAs; pair-MMA completion reaches both CTAs through a
// multicast commit.  Every wait is bounded; after a failed wait a role stops,
// and the producer waits (with the full limit) for the copies it issued, so
// none outlives the CTA.  No load uses cluster multicast.
//
// Reference semantics: vllm_fp8kv/fp8_ds_mla_sparse_decode.py:77-211 (masking,
// dequant, NaN-free online softmax, LSE) and the split/merge contract of
// tests/fixtures/triton_mla_sparse_kernel_pr47629.py:232-403.
#include "common.cuh"
#include "decode.h"
#include "tc_cluster.cuh"
#include "tc_ptx.cuh"
#include "tma_map.h"

namespace fp8mla {
namespace tc3 {

using namespace fp8mla::tc;

namespace {

constexpr int kHeads = 128;        // per kv group = per pair
constexpr int kN = 64;             // tokens per tile
constexpr int kOwn = kN / 2;       // tokens per tile whose whole row a CTA gathers
constexpr int kKSteps = 36;        // 576 / 16
constexpr int kQTmemSteps = 24;    // q dims [0,384) from tensor memory
constexpr int kQSmemBlocks = 3;    // q dims [384,576)
constexpr int kQBlockBytes = 64 * 128;    // 64 rows (this CTA's heads)
constexpr int kKBlockBytes = kOwn * 128;  // 4096: 32 own rows of a 64-dim block
constexpr int kKStageBytes = 9 * kKBlockBytes;
constexpr int kKStages = 2;
constexpr int kVBlockBytes = kN * 128;    // 8192: 64 rows of a 64-dim block
constexpr int kVStageBytes = 4 * kVBlockBytes;
constexpr int kVStages = 2;
constexpr int kPStageBytes = 64 * 128;    // 64 heads x 64 tokens bf16
constexpr int kPStages = 2;
// raw ring: a stage is half a tile of this CTA's rows
constexpr int kHalfRows = kOwn / 2;              // 16 own rows + 16 rows of the other CTA
constexpr int kOwnGroupBytes = 2688;             // 4 whole rows (2624 B), 128-B multiple
constexpr int kOthGroupBytes = 1152;             // 4 rows: tile c 512 | tile c+2 512 | scales 64 (+64)
constexpr int kOthBase = 4 * kOwnGroupBytes;     // 10752
constexpr int kRawStageBytes = kOthBase + 4 * kOthGroupBytes;  // 15360
constexpr int kRawStages = 3;
constexpr uint32_t kRawTx = kHalfRows * kRowBytes + kHalfRows * (2 * kTile + 16);  // 14848
constexpr int kVMaskSlots = 4;
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kFirstLoadWarp = 5;
constexpr int kLoadWarps = 8;
constexpr int kProducerWarp = kFirstLoadWarp + kLoadWarps;  // 13
constexpr int kThreads = (kProducerWarp + 1) * 32;          // 448
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256, kColQ = 320;
constexpr uint32_t kSBufCols = kN / 2;  // 32
constexpr float kRescaleThreshold = 8.0f;

constexpr uint32_t kIdescQK = idesc_bf16(128, kN, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, 256, true);

struct Smem {
  uint8_t q[kQSmemBlocks * kQBlockBytes];  // 1024-aligned (offset 0)
  uint8_t k[kKStages][kKStageBytes];
  uint8_t v[kVStages][kVStageBytes];
  uint8_t p[kPStages][kPStageBytes];
  uint8_t raw[kRawStages][kRawStageBytes];  // gather4 destinations (128-B aligned)
  float pmax[2][128];                       // partial tile max, by tile parity
  float lsum[128];                          // partial row sums (epilogue)
  uint8_t rvalid[kRawStages][2 * kHalfRows];  // per raw row: own 0..15, other 16..31
  uint32_t vmask[kVMaskSlots][2];           // tile rows [0,32) and [32,64) live bits
  uint64_t raw_full[kRawStages], raw_empty[kRawStages];
  uint64_t tfull[kKStages];                 // even CTA: tile j's K and V in both CTAs
  uint64_t kempty[kKStages], vempty[kVStages];
  uint64_t sfull[2], pfull[kPStages], pempty[kPStages];
  uint64_t xch[2];
  uint64_t vfull[kVMaskSlots];              // this CTA: tile's validity bits written
  uint64_t qready, ofull, drain;
  uint32_t tmem_base;
};
static_assert(offsetof(Smem, k) % 1024 == 0 && offsetof(Smem, v) % 1024 == 0 &&
                  offsetof(Smem, p) % 1024 == 0 && kKStageBytes % 1024 == 0,
              "swizzle atoms need 1024-B alignment");
static_assert(offsetof(Smem, raw) % 128 == 0 && kRawStageBytes % 128 == 0, "TMA destinations");
static_assert(offsetof(Smem, raw_full) % 8 == 0, "");
static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

struct Rows {
  uint4 a[4], asc;
  uint4 b[2], brope, bsc;
};

struct Ctx {
  const DecodeArgs* a;
  const int32_t* idx_row;
  int32_t req;
  int beg, end, ntiles;
  uint32_t rank;
  uint32_t tmem;
  uint32_t sq, sk0, sv0, sp0;
  uint32_t b_tfull, b_kempty, b_vempty, b_sfull, b_pfull, b_pempty;
  uint32_t b_xch, b_qready, b_ofull, b_drain;
  uint32_t b_rawfull, b_rawempty, b_vfull;
};

// ------------------------------------------------------------------ MMA issuer (even CTA)
__device__ __forceinline__ void issue_qk(uint32_t tS, uint32_t tQ, uint64_t qdesc0, uint64_t kdesc) {
#pragma unroll
  for (int kst = 0; kst < kKSteps; ++kst) {
    const uint64_t bdesc =
        kdesc + (uint64_t)((((kst >> 2) * kKBlockBytes) + (kst & 3) * 32) >> 4);
    if (kst < kQTmemSteps) {
      mma_pair_ts(tS, tQ + 8 * kst, bdesc, kIdescQK, kst > 0 ? 1u : 0u);
    } else {
      const int qs = kst - kQTmemSteps;
      const uint64_t adesc =
          qdesc0 + (uint64_t)((((qs >> 2) * kQBlockBytes) + (qs & 3) * 32) >> 4);
      mma_pair_ss(tS, adesc, bdesc, kIdescQK, 1u);
    }
  }
}

__device__ void mma_role(const Ctx& c) {
  bool ok = thread_wait_cluster(c.b_qready, 0, 35);
  tc_fence_after();
  const uint32_t tQ = c.tmem + kColQ;
  const uint64_t qdesc0 = sdesc_sw128(c.sq, 16, 1024);
  const uint64_t kdesc0 = sdesc_sw128(c.sk0, 16, 1024);
  const uint64_t pdesc0 = sdesc_sw128(c.sp0, 16, 1024);
  const uint64_t vdesc0 = sdesc_sw128(c.sv0, kVBlockBytes, 1024);
  auto issue_pv = [&](int jj) {
    const int ps = jj % kPStages, vs = jj % kVStages;
    const uint64_t pd = pdesc0 + (uint64_t)((ps * kPStageBytes) >> 4);
    const uint64_t vd = vdesc0 + (uint64_t)((vs * kVStageBytes) >> 4);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk)
        mma_pair_ss(c.tmem + kColO + 128 * hf, pd + (uint64_t)((kk * 32) >> 4),
                    vd + (uint64_t)((hf * 2 * kVBlockBytes + kk * 16 * 128) >> 4), kIdescPV,
                    (jj > 0 || kk > 0) ? 1u : 0u);
    mma_commit_pair(c.b_pempty + 8 * ps);
    mma_commit_pair(c.b_vempty + 8 * vs);
  };
  for (int j = 0; j < c.ntiles && ok; ++j) {
    const int b = j & 1, ks = j % kKStages;
    ok = thread_wait_cluster(c.b_tfull + 8 * ks, (j / kKStages) & 1, 37);
    if (!ok) break;
    tc_fence_after();
    issue_qk(c.tmem + kColS + kSBufCols * b, tQ, qdesc0,
             kdesc0 + (uint64_t)((ks * kKStageBytes) >> 4));
    mma_commit_pair(c.b_sfull + 8 * b);
    mma_commit_pair(c.b_kempty + 8 * ks);
    if (j >= 1) {
      const int jp = j - 1;
      ok = thread_wait_cluster(c.b_pfull + 8 * (jp % kPStages), (jp / kPStages) & 1, 36);
      if (!ok) break;
      tc_fence_after();
      issue_pv(jp);
    }
  }
  if (ok && c.ntiles > 0) {
    const int jl = c.ntiles - 1;
    ok = thread_wait_cluster(c.b_pfull + 8 * (jl % kPStages), (jl / kPStages) & 1, 36);
    if (ok) {
      tc_fence_after();
      issue_pv(jl);
      mma_commit_pair(c.b_ofull);
    }
  }
  // drain: nothing this thread issued may still touch either CTA's memory
  mma_commit_pair(c.b_drain);
  thread_wait_cluster(c.b_drain, 0, 39);
}

// ------------------------------------------------------------------ producer
// Half-stage hs (tile hs >> 1, half hs & 1) holds own rows [16h, 16h+16) of
// this CTA's 32 and the other CTA's rows [16h, 16h+16) of its 32.  Lane i < 16
// takes own row i, lane 16 + i the other CTA's row i.
template <bool kPaged>
__device__ void producer(const Ctx& c, Smem& s, const CUtensorMap* tm_row, const CUtensorMap* tm_tile,
                         const CUtensorMap* tm_scale, int lane) {
  const DecodeArgs& a = *c.a;
  const int cr = (int)c.rank;
  const int nhs = 2 * c.ntiles;
  // tile row of this lane's entry in half-stage hs
  const int rsub = lane & 15;
  const int rbase = lane < 16 ? kOwn * cr : kOwn * (1 - cr);
  auto raw_at = [&](int hs) -> int32_t {
    if (hs >= nhs) return -1;
    const int pos = c.beg + (hs >> 1) * kN + rbase + 16 * (hs & 1) + rsub;
    return pos < c.end ? c.idx_row[pos] : -1;
  };
  // index pipeline: raw entries two half-stages ahead (flat), or three ahead
  // with the block-table read two ahead (paged), so no step waits on a load
  int32_t r1 = raw_at(0), r2 = raw_at(1);
  SlotPf f1{-1, 0};
  if constexpr (kPaged) {
    f1 = slot_fetch(a, c.req, r1);
    r1 = r2;
    r2 = raw_at(2);
  }
  // gather4 assignment: lanes 0-3 whole own rows (group g = lane), lanes 4-15
  // the other CTA's rows (group g = (lane-4)/3; tile c, tile c+2, scales)
  const int og = (lane - 4) / 3, kind = (lane - 4) % 3;
  const int src = lane < 4 ? 4 * lane : 16 + 4 * og;
  uint32_t dst_off = 0;
  const CUtensorMap* tm = tm_row;
  int32_t x = 0;
  if (lane < 4) {
    dst_off = lane * kOwnGroupBytes;
  } else if (lane < 16) {
    dst_off = kOthBase + og * kOthGroupBytes + kind * 512;
    tm = kind < 2 ? tm_tile : tm_scale;
    x = kind < 2 ? 16 * (cr + 2 * kind) : 64;
  }
  bool ok = true;
  int armed = 0;
  for (int hs = 0; hs < nhs; ++hs) {
    int32_t slot;
    if constexpr (kPaged) {
      slot = slot_finish(a, f1);
      f1 = slot_fetch(a, c.req, r1);
      r1 = r2;
      r2 = raw_at(hs + 3);
    } else {
      slot = live_slot(a, c.req, r1);
      r1 = r2;
      r2 = raw_at(hs + 2);
    }
    const int st = hs % kRawStages;
    if (hs >= kRawStages)
      ok = warp_wait(c.b_rawempty + 8 * st, ((hs / kRawStages) + 1) & 1, 40);
    if (!ok) break;
    s.rvalid[st][lane] = slot >= 0 ? 1 : 0;
    const int32_t row = slot >= 0 ? slot : 0;  // masked: a valid row, flagged invalid
    const int32_t g0 = __shfl_sync(0xFFFFFFFFu, row, src & 31);
    const int32_t g1 = __shfl_sync(0xFFFFFFFFu, row, (src + 1) & 31);
    const int32_t g2 = __shfl_sync(0xFFFFFFFFu, row, (src + 2) & 31);
    const int32_t g3 = __shfl_sync(0xFFFFFFFFu, row, (src + 3) & 31);
    const uint32_t bar = c.b_rawfull + 8 * st;
    __syncwarp();  // the flags (generic stores) are released by the arrive below
    if (lane == 0) mbar_arrive_expect_tx(bar, kRawTx);
    __syncwarp();
    if (lane < 16) tma_gather4(smem_u32(s.raw[st]) + dst_off, tm, x, g0, g1, g2, g3, bar);
    ++armed;
  }
  // the stages armed last have landed before the producer returns, even
  // after a failed wait (full limit)
  for (int xh = armed > kRawStages ? armed - kRawStages : 0; xh < armed; ++xh)
    (void)warp_wait(c.b_rawfull + 8 * (xh % kRawStages), (xh / kRawStages) & 1, 41);
}

// ------------------------------------------------------------------ dequant
__device__ void dequant_role(const Ctx& c, Smem& s, int lw, int lane) {
  const int cr = (int)c.rank;
  // part A: tile row rowA, lane quarter pA: PV-half chunks pA + 4i
  const int rowA = lw * 8 + (lane & 7), pA = lane >> 3;
  const bool ownA = (rowA >> 5) == cr;
  const int oA = rowA & 31, hA = oA >> 4, iA = oA & 15;
  // part B: own row rowB (own index), lane eighth qB
  const int rowB = lw * 4 + (lane >> 3), qB = lane & 7;
  const int hB = rowB >> 4, iB = rowB & 15;
  // byte offsets inside a raw stage
  const uint32_t offA = ownA ? (uint32_t)((iA >> 2) * kOwnGroupBytes + (iA & 3) * kRowBytes)
                             : (uint32_t)(kOthBase + (iA >> 2) * kOthGroupBytes + (iA & 3) * kTile);
  const uint32_t offB = (uint32_t)((iB >> 2) * kOwnGroupBytes + (iB & 3) * kRowBytes);
  const uint32_t offAsc = ownA ? offA + kScaleOff
                               : (uint32_t)(kOthBase + (iA >> 2) * kOthGroupBytes + 1024 + (iA & 3) * 16);
  auto deq = [&](const uint4& w, float sc, uint4& o0, uint4& o1) {
    dequant4_hw_x2(w.x, sc, o0.x, o0.y);
    dequant4_hw_x2(w.y, sc, o0.z, o0.w);
    dequant4_hw_x2(w.z, sc, o1.x, o1.y);
    dequant4_hw_x2(w.w, sc, o1.z, o1.w);
  };
  auto pick = [](const uint4& sc, int tile) -> float {
    return __uint_as_float(tile == 0 ? sc.x : tile == 1 ? sc.y : tile == 2 ? sc.z : sc.w);
  };
  const uint4 z4 = make_uint4(0, 0, 0, 0);
  bool ok = true;
  for (int j = 0; j < c.ntiles && ok; ++j) {
    const int hs0 = 2 * j, hs1 = 2 * j + 1;
    const int stA = (hs0 + hA) % kRawStages, stB = (hs0 + hB) % kRawStages;
    ok = warp_wait(c.b_rawfull + 8 * (hs0 % kRawStages), (hs0 / kRawStages) & 1, 42);
    if (ok) ok = warp_wait(c.b_rawfull + 8 * (hs1 % kRawStages), (hs1 / kRawStages) & 1, 42);
    if (!ok) break;
    // every lane acquires the two stages' copies itself before reading them
    (void)mbar_try_wait(c.b_rawfull + 8 * (hs0 % kRawStages), (hs0 / kRawStages) & 1);
    (void)mbar_try_wait(c.b_rawfull + 8 * (hs1 % kRawStages), (hs1 / kRawStages) & 1);
    Rows R;
    const uint8_t* ra = s.raw[stA];
    const bool vA = s.rvalid[stA][(ownA ? 0 : 16) + iA] != 0;
    const bool vB = s.rvalid[stB][iB] != 0;
    if (vA) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tile = cr + 2 * (i >> 1);
        const int chunk = pA + 4 * (i & 1);
        // own rows: tile t at 128 t; other rows: tile c at 0, tile c+2 at 512
        const uint32_t o = ownA ? offA + 128 * tile + 16 * chunk : offA + 512 * (i >> 1) + 16 * chunk;
        R.a[i] = *reinterpret_cast<const uint4*>(ra + o);
      }
      R.asc = *reinterpret_cast<const uint4*>(ra + offAsc);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) R.a[i] = z4;
      R.asc = z4;
    }
    if (vB) {
      const uint8_t* rb = s.raw[stB] + offB;
      R.b[0] = *reinterpret_cast<const uint4*>(rb + 128 * (1 - cr) + 16 * qB);
      R.b[1] = *reinterpret_cast<const uint4*>(rb + 128 * (3 - cr) + 16 * qB);
      R.brope = *reinterpret_cast<const uint4*>(rb + kRopeOff + 16 * qB);
      R.bsc = *reinterpret_cast<const uint4*>(rb + kScaleOff);
    } else {
      R.b[0] = R.b[1] = R.brope = R.bsc = z4;
    }
    // the tile's live bits: lanes 0-7 hold part-A rows [8 lw, 8 lw + 8)
    const uint32_t bits = __ballot_sync(0xFFFFFFFFu, vA) & 0xFFu;
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(c.b_rawempty + 8 * (hs0 % kRawStages));
      mbar_arrive(c.b_rawempty + 8 * (hs1 % kRawStages));
    }
    const int ks = j % kKStages, vs = j % kVStages;
    if (j >= kKStages) ok = warp_wait_cluster(c.b_kempty + 8 * ks, ((j / kKStages) + 1) & 1, 43);
    if (ok && j >= kVStages) ok = warp_wait_cluster(c.b_vempty + 8 * vs, ((j / kVStages) + 1) & 1, 44);
    if (!ok) break;
    // live bits of tile j into slot j % 4: its previous reader, the softmax of
    // tile j - 4, handed over P(j - 4) before PV(j - 4) was issued, and that
    // precedes QK(j - 2), whose completion the K-stage wait above saw
    if (lane == 0) reinterpret_cast<uint8_t*>(s.vmask[j % kVMaskSlots])[lw] = (uint8_t)bits;
    uint8_t* kst = s.k[ks];
    uint8_t* vst = s.v[vs];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tile = cr + 2 * (i >> 1);
      uint4 o0, o1;
      deq(R.a[i], pick(R.asc, tile), o0, o1);
      uint8_t* vb = vst + i * kVBlockBytes;
      *reinterpret_cast<uint4*>(vb + swz(rowA, 2 * pA)) = o0;
      *reinterpret_cast<uint4*>(vb + swz(rowA, 2 * pA + 1)) = o1;
      if (ownA) {
        uint8_t* kb = kst + (2 * tile + (i & 1)) * kKBlockBytes;
        const int r = rowA - kOwn * cr;
        *reinterpret_cast<uint4*>(kb + swz(r, 2 * pA)) = o0;
        *reinterpret_cast<uint4*>(kb + swz(r, 2 * pA + 1)) = o1;
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int tile = (1 - cr) + 2 * i;
      uint4 o0, o1;
      deq(R.b[i], pick(R.bsc, tile), o0, o1);
      uint8_t* kb = kst + (2 * tile + (qB >> 2)) * kKBlockBytes;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3))) = o0;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3) + 1)) = o1;
    }
    *reinterpret_cast<uint4*>(kst + 8 * kKBlockBytes + swz(rowB, qB)) = R.brope;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(c.b_vfull + 8 * (j % kVMaskSlots));  // this CTA's softmax: live bits
      mbar_arrive_cluster(c.b_tfull + 8 * ks, 0);       // the issuing CTA: K and V rows
    }
  }
}

}  // namespace

template <bool kPaged>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    decode_tc3_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap tm_row,
                      const __grid_constant__ CUtensorMap tm_tile,
                      const __grid_constant__ CUtensorMap tm_scale) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x / (2 * a.G);
  const int grp = (blockIdx.x >> 1) % a.G;
  const int split = blockIdx.y;
  const uint32_t rank = cluster_rank();  // == blockIdx.x & 1
  const int head0 = grp * a.hpg + 64 * (int)rank;
  const int nh = max(0, min(64, a.hpg - 64 * (int)rank));  // real heads of this CTA

  Ctx c;
  c.a = &a;
  c.rank = rank;
  c.beg = split * a.split_len;
  c.end = min(a.topk, c.beg + a.split_len);
  c.ntiles = c.end > c.beg ? (c.end - c.beg + kN - 1) / kN : 0;
  c.idx_row = a.idx + t * a.idx_st + grp * a.idx_sg;
  c.req = 0;
  c.sq = smem_u32(s.q);
  c.sk0 = smem_u32(s.k[0]);
  c.sv0 = smem_u32(s.v[0]);
  c.sp0 = smem_u32(s.p[0]);
  c.b_tfull = smem_u32(&s.tfull[0]);
  c.b_kempty = smem_u32(&s.kempty[0]);
  c.b_vempty = smem_u32(&s.vempty[0]);
  c.b_sfull = smem_u32(&s.sfull[0]);
  c.b_pfull = smem_u32(&s.pfull[0]);
  c.b_pempty = smem_u32(&s.pempty[0]);
  c.b_xch = smem_u32(&s.xch[0]);
  c.b_qready = smem_u32(&s.qready);
  c.b_ofull = smem_u32(&s.ofull);
  c.b_drain = smem_u32(&s.drain);
  c.b_rawfull = smem_u32(&s.raw_full[0]);
  c.b_rawempty = smem_u32(&s.raw_empty[0]);
  c.b_vfull = smem_u32(&s.vfull[0]);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(c.b_rawfull + 8 * i, 1);
      mbar_init(c.b_rawempty + 8 * i, kLoadWarps);
    }
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(c.b_tfull + 8 * i, 2 * kLoadWarps);
      mbar_init(c.b_kempty + 8 * i, 1);
    }
    for (int i = 0; i < kVStages; ++i) mbar_init(c.b_vempty + 8 * i, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(c.b_sfull + 8 * i, 1);
      mbar_init(c.b_xch + 8 * i, kSoftmaxWarps);
    }
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(c.b_pfull + 8 * i, 2 * kSoftmaxWarps);
      mbar_init(c.b_pempty + 8 * i, 1);
    }
    for (int i = 0; i < kVMaskSlots; ++i) mbar_init(c.b_vfull + 8 * i, kLoadWarps);
    mbar_init(c.b_qready, 2 * kSoftmaxWarps);
    mbar_init(c.b_ofull, 1);
    mbar_init(c.b_drain, 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(smem_u32(&s.tmem_base), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, tensor memory allocated
  tc_fence_after();
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();  // the previous kernel of the stream has completed: global memory from here on
  c.req = request_of(a, t);
  c.tmem = s.tmem_base;
  const uint32_t tmem = c.tmem;

  if (warp < kSoftmaxWarps) {
    // ================================================= softmax + epilogue
    const int L = threadIdx.x;          // TMEM lane
    const int m = L & 63, hh = L >> 6;  // head within the CTA, token half of a tile
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    {
      // Q dims [0,384) -> TMEM (lanes L and L^64 both hold head m), dims
      // [384,576) -> swizzled smem (thread hh writes chunks [4hh, 4hh+4) of
      // each block); padding rows are zero
      const bool hv = m < nh;
      const uint4* qsrc = reinterpret_cast<const uint4*>(
          static_cast<const uint16_t*>(a.q) + t * a.q_st + (int64_t)(hv ? head0 + m : 0) * a.q_sh);
      const uint4 z4 = make_uint4(0, 0, 0, 0);
      {
        uint4 x[12];
#pragma unroll
        for (int blk = 0; blk < kQSmemBlocks; ++blk)
#pragma unroll
          for (int i = 0; i < 4; ++i) x[4 * blk + i] = hv ? qsrc[kQTmemSteps * 2 + blk * 8 + 4 * hh + i] : z4;
#pragma unroll
        for (int blk = 0; blk < kQSmemBlocks; ++blk)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<uint4*>(s.q + blk * kQBlockBytes + swz(m, 4 * hh + i)) = x[4 * blk + i];
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        constexpr int kChunks = kQTmemSteps;  // 16-B chunks per half: 96 columns
        uint4 x[kChunks];
#pragma unroll
        for (int v = 0; v < kChunks; ++v) x[v] = hv ? qsrc[half * kChunks + v] : z4;
#pragma unroll
        for (int c0 = 0; c0 < kChunks * 4; c0 += 32) {
          uint32_t w[32];
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            w[4 * v] = x[c0 / 4 + v].x;
            w[4 * v + 1] = x[c0 / 4 + v].y;
            w[4 * v + 2] = x[c0 / 4 + v].z;
            w[4 * v + 3] = x[c0 / 4 + v].w;
          }
          tmem_st32(trow + kColQ + half * kChunks * 4 + c0, w);
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(c.b_qready, 0);
    }

    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < c.ntiles && ok; ++j) {
      const int b = j & 1, ps = j % kPStages;
      ok = warp_wait_cluster(c.b_sfull + 8 * b, (j >> 1) & 1, 31);
      if (ok) ok = warp_wait(c.b_vfull + 8 * (j % kVMaskSlots), (j / kVMaskSlots) & 1, 30);
      if (!ok) break;
      (void)mbar_try_wait(c.b_vfull + 8 * (j % kVMaskSlots), (j / kVMaskSlots) & 1);
      const uint32_t live = s.vmask[j % kVMaskSlots][hh];  // tokens [32 hh, 32 hh + 32)
      tc_fence_after();
      uint32_t sv[32];
      tmem_ld32(trow + kColS + kSBufCols * b, sv);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (!((live >> i) & 1u)) sv[i] = __float_as_uint(-INFINITY);
      float pm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) pm = fmaxf(pm, __uint_as_float(sv[i]));
      pm *= a.scale_log2;
      s.pmax[b][L] = pm;
      __syncwarp();
      if (lane == 0) mbar_arrive(c.b_xch + 8 * b);
      ok = warp_wait(c.b_xch + 8 * b, (j >> 1) & 1, 34);
      if (!ok) break;
      const float tmax = fmaxf(pm, s.pmax[b][L ^ 64]);
      float alpha = 1.f;
      if (tmax > m_used + kRescaleThreshold || (m_used == -INFINITY && tmax > -INFINITY)) {
        alpha = (m_used == -INFINITY) ? 1.f : ex2_approx(m_used - tmax);
        m_used = tmax;
        l *= alpha;
      }
      if (__any_sync(0xFFFFFFFFu, alpha != 1.f) && j > 0) {
        // O rows are rescaled once PV(j-1) has finished writing them
        const int jp = j - 1;
        ok = warp_wait_cluster(c.b_pempty + 8 * (jp % kPStages), (jp / kPStages) & 1, 33);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < 256; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(trow + kColO + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(trow + kColO + c0, o);
        }
        tmem_wait_st();
      }
      const float mref = (m_used == -INFINITY) ? 0.f : m_used;
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(sv[2 * i]), a.scale_log2, -mref));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sv[2 * i + 1]), a.scale_log2, -mref));
        l += p0 + p1;
        pk[i] = pack_bf16x2(p0, p1);
      }
      // P stage ps was last read by PV(j-2), which was issued before QK(j):
      // its completion is implied by sfull(j)
      uint8_t* prow = s.p[ps];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4)
        *reinterpret_cast<uint4*>(prow + swz(m, 4 * hh + q4)) =
            make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(c.b_pfull + 8 * ps, 0);
    }

    // ---- epilogue: the two threads of a head add their row sums
    s.lsum[L] = l;
    named_sync(1, kSoftmaxWarps * 32);
    const float lt = l + s.lsum[L ^ 64];
    const bool have_o = ok && c.ntiles > 0 && warp_wait_cluster(c.b_ofull, 0, 32);
    if (have_o) tc_fence_after();
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    const float lse_v = lt > 0.f ? m_used * kLn2 + logf(lt) : -INFINITY;
    const int hh_glob = head0 + m;
    auto store32 = [&](const uint32_t (&o)[32], int c0) {
      const int d = 256 * (c0 >> 7) + 128 * hh + (c0 & 127);
      uint4* dst = a.num_splits == 1
                       ? reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + t * a.out_st +
                                                  (int64_t)hh_glob * a.out_sh + d)
                       : reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.ws_o) +
                                                  ((t * a.H + hh_glob) * a.num_splits + split) * kNope + d);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          w[u] = pack_bf16x2(__uint_as_float(o[8 * v + 2 * u]) * inv,
                             __uint_as_float(o[8 * v + 2 * u + 1]) * inv);
        dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    };
#pragma unroll 1
    for (int c0 = 0; c0 < 256; c0 += 64) {
      uint32_t o0[32], o1[32];
      if (have_o) {
        tmem_ld32(trow + kColO + c0, o0);
        tmem_ld32(trow + kColO + c0 + 32, o1);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o0[i] = o1[i] = 0u;
      }
      if (m < nh) {
        store32(o0, c0);
        store32(o1, c0 + 32);
      }
    }
    if (hh == 0 && m < nh) {
      if (a.num_splits == 1) {
        if (a.lse != nullptr) a.lse[t * a.lse_st + hh_glob] = lse_v;
      } else {
        a.ws_lse[(t * a.H + hh_glob) * a.num_splits + split] = lse_v;
      }
    }
  } else if (warp == kMmaWarp) {
    if (rank == 0 && lane == 0) mma_role(c);
    __syncwarp();
  } else if (warp == kProducerWarp) {
    producer<kPaged>(c, s, &tm_row, &tm_tile, &tm_scale, lane);
  } else {
    dequant_role(c, s, warp - kFirstLoadWarp, lane);
  }

  // both CTAs: no MMA of the pair may still run, no arrival may still target
  // the other CTA, before tensor memory is freed and the CTAs exit
  tc_fence_before();
  cluster_sync_all();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace tc3

bool decode_tc3_supported(const DecodeArgs& a) {
  return a.q_dtype == FP8MLA_DTYPE_BF16 && (a.hpg == tc3::kHeads || a.hpg == tc3::kHeads / 2) &&
         a.G >= 1 && a.num_slots > 0 && a.num_slots < (1ll << 31);
}

int read_device_status_tc3(unsigned int* status, bool reset, cudaStream_t st) {
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

int launch_decode_tc3(const DecodeArgs& a, cudaStream_t st) {
  CUtensorMap maps[3];
  if (int rc = encode_row_map(&maps[0], a.kv, a.num_slots, kRowBytes / 8)) return rc;
  if (int rc = encode_row_map(&maps[1], a.kv, a.num_slots, kTile / 8)) return rc;
  if (int rc = encode_row_map(&maps[2], a.kv, a.num_slots, 2)) return rc;
  const size_t smem = sizeof(tc3::Smem) + 1024;  // + alignment slack
  auto go = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "decode_tc3 smem attribute");
    dim3 grid((unsigned)(a.T * a.G * 2), a.num_splits);
    return check_cuda(launch_pdl(kern, grid, dim3(tc3::kThreads), smem, st, a, maps[0], maps[1], maps[2]),
                      "decode_tc3_kernel launch");
  };
  const int rc = a.block_table != nullptr ? go(tc3::decode_tc3_kernel<true>)
                                          : go(tc3::decode_tc3_kernel<false>);
  if (rc != FP8MLA_OK || a.num_splits == 1) return rc;
  return launch_merge_splits(a, st);
}

}  // namespace fp8mla
