// decode_tc3.cu -- sparse MLA decode for 64 or 128 heads per kv group on a
// pair of SMs (a 2-CTA cluster) sharing cta_group::2 tcgen05 MMAs, with each
// CTA's own rows staged in shared memory by TMA.
//
// The pair splits the heads, not the output dims: CTA c owns heads
// [64c, 64c+64) and its TMEM holds their S and O.  A tile is 64 tokens and one
// MMA spans both SMs:
//   S = Q K^T   M=128 heads (64 per CTA), N=64 tokens, K=576 (36 k-steps); B
//               is split by N: CTA c supplies the rows of its 32 "own" tokens
//               [32c, 32c+32) of the tile, all 576 dims
//   O += P V    M=128 heads, N=256 dims (two MMAs for the 512), K=64 tokens; B
//               is split by N: CTA c supplies dims [128c, 128c+128) of each
//               MMA, i.e. latent tiles c and c+2 (its "PV half"), all 64 tokens
// So each CTA needs per tile its 32 own rows whole (656 B) and the PV half of
// the other 32 rows (2 x 128 fp8 bytes + scales): the pair reads 59 KB of rows
// per tile instead of 84 KB for two CTAs that each gather the whole tile.
// Accumulator layout of an M=128 cta_group::2 MMA (measured): per CTA, lanes
// [0,64) hold the CTA's 64 rows x columns [0, N/2), lanes [64,128) the same
// rows x columns [N/2, N).  So softmax thread L (TMEM lane L) owns head
// (L & 63) and tokens [32 (L >> 6), +32) of a tile; the two threads of a head
// exchange their partial max through shared memory once per tile.
//
// Rows reach shared memory two ways.  A CTA's 32 own rows per tile (656 B
// each, 21 KB) come whole by TMA: a producer warp turns top-k entries into
// slots and issues 8 tile::gather4 copies (four rows each) into a 2-stage
// raw ring, so those bytes bypass L1 and no warp waits for them.  The PV
// half of the other CTA's 32 rows (272 B each) is loaded into registers by
// the dequant warps that handle those rows, one tile ahead, issued right
// after the step's proxy fence so that no fence waits on loads in flight.
// A masked slot fetches row 0 (TMA) or nothing (registers) and is flagged
// invalid: its K and V rows are zeros and its score is replaced by -inf in
// the softmax (validity bits per tile), so a fully masked row still gives
// P = 0 and LSE = -inf.
//
// K and V of a tile are signalled separately: QK(j) waits for the K rows
// only, PV(j) for the V rows, so with two V stages the dequant of tile j
// never waits for PV(j-2) before QK(j) can start.
//
// Tensor memory (512 columns, both CTAs):
//   [  0,256)  O, dims [0,256) MMA in [0,128), dims [256,512) MMA in [128,256)
//   [256,320)  2 S buffers x 32 fp32 columns
//   [320,512)  Q dims [0,384), the A operand of 24 k-steps (lanes L and L^64
//              hold the same head)
// Shared memory (about 221 KB):
//   q    Q dims [384,576): 3 x 64-dim swizzled blocks of 64 rows      24 KB
//   k    2 stages: own 32 tokens x 576 dims, 9 blocks of 32 rows      72 KB
//   v    2 stages: 64 tokens x PV-half dims, 4 blocks of 64 rows      64 KB
//   p    2 stages: P (bf16) of 64 heads x 64 tokens                   16 KB
//   raw  2 stages: the tile's 32 own rows as gathered by TMA          42 KB
//
// Warp roles (512 threads per CTA; warp w runs on SM sub-partition w % 4):
//   warps 0-3   softmax (thread L = TMEM lane L), row sums and LSE
//   all warps   epilogue: warp w stores O columns [64 (w / 4), +64) of TMEM
//               lanes [32 (w % 4), +32)
//   warp 4      TMEM allocation in both CTAs; lane 0 of the even CTA issues
//               every MMA of the pair
//   warp 15     producer: indices -> slots (block table included for the
//               paged entry point) -> gather4 of own rows into the raw ring
//   warps 5-7, 9-11, 13-14
//               dequant: part A = the PV half of the 64 tile rows (V stage,
//               and the K stage for own rows; the other CTA's rows loaded
//               into registers here), part B = the other half and the rope
//               of the 32 own rows (K stage)
//   warps 8, 12 idle: sub-partition 0, which issues the MMAs, runs only the
//               issuing thread and softmax warp 0 (c2 88.0 vs 89.1 us per
//               call with a dequant warp there; 82.6 vs 83.9 with the
//               producer there)
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
static_assert(kKStages == 2 && kVStages == kPStages, "S / K and P / V completions share barriers");
// raw ring: a stage is one tile's 32 own rows, 8 gather4 groups of 4 rows
constexpr int kGroupBytes = 2688;         // 4 whole rows (2624 B), 128-B multiple
constexpr int kRawStageBytes = 8 * kGroupBytes;
constexpr int kRawStages = 2;
constexpr uint32_t kRawTx = kOwn * kRowBytes;  // 20992
constexpr int kMaskSlots = 4;
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kLoadWarps = 8;
constexpr int kProducerWarp = 15;
constexpr int kIdleWarp0 = 8, kIdleWarp1 = 12;
constexpr int kThreads = 16 * 32;  // 512
// dequant index of warp w (5-7, 9-11, 13-14 -> 0-7)
__device__ __forceinline__ int dequant_index(int w) { return w < 8 ? w - 5 : w < 12 ? w - 6 : w - 7; }
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
  float inv[128];                           // 1 / row sum per TMEM lane (epilogue)
  uint32_t epi_ok[kSoftmaxWarps];           // softmax warp q finished every tile
  uint8_t rvalid[kRawStages][kOwn];         // own row live (producer's flags)
  uint32_t vmask[kMaskSlots][2];            // tile rows [0,32) and [32,64) live bits
  uint64_t raw_full[kRawStages], raw_empty[kRawStages];
  uint64_t kready[kKStages], vready[kVStages];  // even CTA: tile j's K / V rows in both CTAs
  // one commit per MMA group: QK(j) done frees K stage j % 2 and fills S
  // buffer j % 2; PV(j) done frees P and V stage j % 2
  uint64_t sfull[2], pfull[kPStages], pempty[kPStages];
  uint64_t xch[2];
  uint64_t mfull[kMaskSlots];               // this CTA: the tile's live bits written
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

struct Ctx {
  const DecodeArgs* a;
  const int32_t* idx_row;
  int32_t req;
  int beg, end, ntiles;
  uint32_t rank;
  uint32_t tmem;
  uint32_t sq, sk0, sv0, sp0;
  uint32_t b_kready, b_vready, b_kempty, b_vempty, b_sfull, b_pfull, b_pempty;
  uint32_t b_xch, b_qready, b_ofull, b_drain;
  uint32_t b_rawfull, b_rawempty, b_mfull;
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
  // PV(jj): waits for P(jj) (softmax of both CTAs) and V(jj) (dequant of
  // both).  Every dequant warp writes and fences V(jj) before its K(jj + 1)
  // arrival, so once QK(jj + 1) has been issued V(jj) is known to be in place:
  // only the last tile waits for its V barrier (whose earlier phases have all
  // completed by then, so the parity names the right one).
  auto issue_pv = [&](int jj) -> bool {
    const int ps = jj % kPStages, vs = jj % kVStages;
    if (!thread_wait_cluster(c.b_pfull + 8 * ps, (jj / kPStages) & 1, 36)) return false;
    if (jj == c.ntiles - 1 && !thread_wait_cluster(c.b_vready + 8 * vs, (jj / kVStages) & 1, 38))
      return false;
    tc_fence_after();
    const uint64_t pd = pdesc0 + (uint64_t)((ps * kPStageBytes) >> 4);
    const uint64_t vd = vdesc0 + (uint64_t)((vs * kVStageBytes) >> 4);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk)
        mma_pair_ss(c.tmem + kColO + 128 * hf, pd + (uint64_t)((kk * 32) >> 4),
                    vd + (uint64_t)((hf * 2 * kVBlockBytes + kk * 16 * 128) >> 4), kIdescPV,
                    (jj > 0 || kk > 0) ? 1u : 0u);
    mma_commit_pair(c.b_pempty + 8 * ps);  // = V stage vs empty
    return true;
  };
  for (int j = 0; j < c.ntiles && ok; ++j) {
    const int b = j & 1, ks = j % kKStages;
    ok = thread_wait_cluster(c.b_kready + 8 * ks, (j / kKStages) & 1, 37);
    if (!ok) break;
    tc_fence_after();
    issue_qk(c.tmem + kColS + kSBufCols * b, tQ, qdesc0,
             kdesc0 + (uint64_t)((ks * kKStageBytes) >> 4));
    mma_commit_pair(c.b_sfull + 8 * b);  // = K stage ks empty
    if (j >= 1) ok = issue_pv(j - 1);
  }
  if (ok && c.ntiles > 0) {
    ok = issue_pv(c.ntiles - 1);
    if (ok) mma_commit_pair(c.b_ofull);
  }
  // drain: nothing this thread issued may still touch either CTA's memory
  mma_commit_pair(c.b_drain);
  thread_wait_cluster(c.b_drain, 0, 39);
}

// ------------------------------------------------------------------ producer
// Tile j's own rows: lane i takes own row i (tile row 32c + i); lanes 0-7 each
// gather four of them.
template <bool kPaged>
__device__ void producer(const Ctx& c, Smem& s, const CUtensorMap* tm, int lane) {
  const DecodeArgs& a = *c.a;
  const int cr = (int)c.rank;
  auto raw_at = [&](int j) -> int32_t {
    if (j >= c.ntiles) return -1;
    const int pos = c.beg + j * kN + kOwn * cr + lane;
    return pos < c.end ? c.idx_row[pos] : -1;
  };
  // index pipeline: raw entries two tiles ahead (flat), or three ahead with
  // the block-table read two ahead (paged), so no step waits on a load
  int32_t r1 = raw_at(0), r2 = raw_at(1);
  SlotPf f1{-1, 0};
  if constexpr (kPaged) {
    f1 = slot_fetch(a, c.req, r1);
    r1 = r2;
    r2 = raw_at(2);
  }
  bool ok = true;
  int armed = 0;
  for (int j = 0; j < c.ntiles; ++j) {
    int32_t slot;
    if constexpr (kPaged) {
      slot = slot_finish(a, f1);
      f1 = slot_fetch(a, c.req, r1);
      r1 = r2;
      r2 = raw_at(j + 3);
    } else {
      slot = live_slot(a, c.req, r1);
      r1 = r2;
      r2 = raw_at(j + 2);
    }
    const int st = j % kRawStages;
    if (j >= kRawStages) ok = warp_wait(c.b_rawempty + 8 * st, ((j / kRawStages) + 1) & 1, 40);
    if (!ok) break;
    s.rvalid[st][lane] = slot >= 0 ? 1 : 0;
    const int32_t row = slot >= 0 ? slot : 0;  // masked: a valid row, flagged invalid
    const int src = (4 * lane) & 31;
    const int32_t g0 = __shfl_sync(0xFFFFFFFFu, row, src);
    const int32_t g1 = __shfl_sync(0xFFFFFFFFu, row, src + 1);
    const int32_t g2 = __shfl_sync(0xFFFFFFFFu, row, src + 2);
    const int32_t g3 = __shfl_sync(0xFFFFFFFFu, row, src + 3);
    const uint32_t bar = c.b_rawfull + 8 * st;
    __syncwarp();  // the flags (generic stores) are released by the arrive below
    if (lane == 0) mbar_arrive_expect_tx(bar, kRawTx);
    __syncwarp();
    if (lane < 8) tma_gather4(smem_u32(s.raw[st]) + lane * kGroupBytes, tm, 0, g0, g1, g2, g3, bar);
    ++armed;
  }
  // the stages armed last have landed before the producer returns, even
  // after a failed wait (full limit)
  for (int x = armed > kRawStages ? armed - kRawStages : 0; x < armed; ++x)
    (void)warp_wait(c.b_rawfull + 8 * (x % kRawStages), (x / kRawStages) & 1, 41);
}

// ------------------------------------------------------------------ dequant
template <bool kPaged>
__device__ void dequant_role(const Ctx& c, Smem& s, int lw, int lane) {
  const DecodeArgs& a = *c.a;
  const int cr = (int)c.rank;
  // part A: tile row rowA, lane quarter pA: PV-half chunks pA + 4i.  A warp's
  // eight part-A rows are all own rows or all rows of the other CTA.
  const int rowA = lw * 8 + (lane & 7), pA = lane >> 3;
  const bool ownA = (rowA >> 5) == cr;
  const int oA = rowA & 31;
  // part B: own row rowB (own index), lane eighth qB
  const int rowB = lw * 4 + (lane >> 3), qB = lane & 7;
  const uint32_t offA = (uint32_t)((oA >> 2) * kGroupBytes + (oA & 3) * kRowBytes);
  const uint32_t offB = (uint32_t)((rowB >> 2) * kGroupBytes + (rowB & 3) * kRowBytes);
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

  // ---- the other CTA's rows (warps with !ownA): slots and register loads
  // one tile ahead.  Lane i < 8 converts the index of part-A row lw*8 + i; the
  // slot reaches the lanes of that row by shuffle.
  auto raw_at = [&](int j) -> int32_t {
    if (ownA || lane >= 8 || j >= c.ntiles) return -1;
    const int pos = c.beg + j * kN + lw * 8 + lane;
    return pos < c.end ? c.idx_row[pos] : -1;
  };
  uint4 A[4], Asc;
  bool vAnext = false;
  auto load_other = [&](int32_t sl) {
    const int32_t sa = __shfl_sync(0xFFFFFFFFu, sl, lane & 7);
    vAnext = sa >= 0;
    if (sa >= 0) {
      const uint8_t* src = a.kv + sa * (int64_t)kRowBytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tile = cr + 2 * (i >> 1);
        A[i] = ldg_v4(src + 128 * tile + 16 * (pA + 4 * (i & 1)));
      }
      Asc = ldg_v4(src + kScaleOff);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) A[i] = z4;
      Asc = z4;
    }
  };
  int32_t n1 = -1, n2 = -1;  // flat: raw entries of tiles j+1, j+2; paged: tiles j+2, j+3
  SlotPf nf{-1, 0};           // paged: block-table read of tile j+1
  if (!ownA) {
    const int32_t s0 = live_slot(a, c.req, raw_at(0));
    if (c.ntiles > 0) load_other(s0);
    if constexpr (kPaged) {
      nf = slot_fetch(a, c.req, raw_at(1));
      n1 = raw_at(2);
      n2 = raw_at(3);
    } else {
      n1 = raw_at(1);
      n2 = raw_at(2);
    }
  }
  bool ok = true;
  for (int j = 0; j < c.ntiles && ok; ++j) {
    const int st = j % kRawStages;
    ok = warp_wait(c.b_rawfull + 8 * st, (j / kRawStages) & 1, 42);
    if (!ok) break;
    (void)mbar_try_wait(c.b_rawfull + 8 * st, (j / kRawStages) & 1);  // every lane acquires
    const uint8_t* rs = s.raw[st];
    bool vA;
    if (ownA) {
      vA = s.rvalid[st][oA] != 0;
      if (vA) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tile = cr + 2 * (i >> 1);
          A[i] = *reinterpret_cast<const uint4*>(rs + offA + 128 * tile + 16 * (pA + 4 * (i & 1)));
        }
        Asc = *reinterpret_cast<const uint4*>(rs + offA + kScaleOff);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) A[i] = z4;
        Asc = z4;
      }
    } else {
      vA = vAnext;
    }
    const bool vB = s.rvalid[st][rowB] != 0;
    uint4 B0 = z4, B1 = z4, Brope = z4, Bsc = z4;
    if (vB) {
      const uint8_t* rb = rs + offB;
      B0 = *reinterpret_cast<const uint4*>(rb + 128 * (1 - cr) + 16 * qB);
      B1 = *reinterpret_cast<const uint4*>(rb + 128 * (3 - cr) + 16 * qB);
      Brope = *reinterpret_cast<const uint4*>(rb + kRopeOff + 16 * qB);
      Bsc = *reinterpret_cast<const uint4*>(rb + kScaleOff);
    }
    // the tile's live bits: lanes 0-7 hold part-A rows [8 lw, 8 lw + 8)
    const uint32_t bits = __ballot_sync(0xFFFFFFFFu, vA) & 0xFFu;
    // part A in bf16 (used for the own rows' K and for V)
    uint4 Ab[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) deq(A[i], pick(Asc, cr + 2 * (i >> 1)), Ab[2 * i], Ab[2 * i + 1]);
    __syncwarp();
    if (lane == 0) mbar_arrive(c.b_rawempty + 8 * st);  // the raw stage is in registers

    // ---- K rows: part A own rows, part B
    const int ks = j % kKStages, vs = j % kVStages;
    if (j >= kKStages) ok = warp_wait_cluster(c.b_kempty + 8 * ks, ((j / kKStages) + 1) & 1, 43);
    if (!ok) break;
    // live bits of tile j into slot j % 4: its previous reader, the softmax of
    // tile j - 4, handed over P(j - 4) before PV(j - 4) was issued, and that
    // precedes QK(j - 2), whose completion the K-stage wait above saw
    if (lane == 0) reinterpret_cast<uint8_t*>(s.vmask[j % kMaskSlots])[lw] = (uint8_t)bits;
    uint8_t* kst = s.k[ks];
    if (ownA) {
      const int r = rowA - kOwn * cr;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tile = cr + 2 * (i >> 1);
        uint8_t* kb = kst + (2 * tile + (i & 1)) * kKBlockBytes;
        *reinterpret_cast<uint4*>(kb + swz(r, 2 * pA)) = Ab[2 * i];
        *reinterpret_cast<uint4*>(kb + swz(r, 2 * pA + 1)) = Ab[2 * i + 1];
      }
    }
    {
      uint4 o0, o1;
      deq(B0, pick(Bsc, 1 - cr), o0, o1);
      uint8_t* kb = kst + (2 * (1 - cr) + (qB >> 2)) * kKBlockBytes;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3))) = o0;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3) + 1)) = o1;
      deq(B1, pick(Bsc, 3 - cr), o0, o1);
      kb = kst + (2 * (3 - cr) + (qB >> 2)) * kKBlockBytes;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3))) = o0;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3) + 1)) = o1;
    }
    *reinterpret_cast<uint4*>(kst + 8 * kKBlockBytes + swz(rowB, qB)) = Brope;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(c.b_mfull + 8 * (j % kMaskSlots));  // this CTA's softmax: live bits
      mbar_arrive_cluster(c.b_kready + 8 * ks, 0);    // the issuing CTA: K rows
    }

    // ---- V rows: part A, all 64 rows
    if (j >= kVStages) ok = warp_wait_cluster(c.b_vempty + 8 * vs, ((j / kVStages) + 1) & 1, 44);
    if (!ok) break;
    uint8_t* vst = s.v[vs];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint8_t* vb = vst + i * kVBlockBytes;
      *reinterpret_cast<uint4*>(vb + swz(rowA, 2 * pA)) = Ab[2 * i];
      *reinterpret_cast<uint4*>(vb + swz(rowA, 2 * pA + 1)) = Ab[2 * i + 1];
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(c.b_vready + 8 * vs, 0);

    // ---- the other CTA's rows of tile j+1: issued after the fences above,
    // so no fence of this warp waits for them
    if (!ownA && j + 1 < c.ntiles) {
      int32_t s1;
      if constexpr (kPaged) {
        s1 = slot_finish(a, nf);
        nf = slot_fetch(a, c.req, n1);
        n1 = n2;
        n2 = raw_at(j + 4);
      } else {
        s1 = live_slot(a, c.req, n1);
        n1 = n2;
        n2 = raw_at(j + 3);
      }
      load_other(s1);
    }
  }
}

}  // namespace

template <bool kPaged>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    decode_tc3_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap tm_row) {
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
  c.b_kready = smem_u32(&s.kready[0]);
  c.b_vready = smem_u32(&s.vready[0]);
  c.b_sfull = smem_u32(&s.sfull[0]);
  c.b_pfull = smem_u32(&s.pfull[0]);
  c.b_pempty = smem_u32(&s.pempty[0]);
  c.b_kempty = c.b_sfull;
  c.b_vempty = c.b_pempty;
  c.b_xch = smem_u32(&s.xch[0]);
  c.b_qready = smem_u32(&s.qready);
  c.b_ofull = smem_u32(&s.ofull);
  c.b_drain = smem_u32(&s.drain);
  c.b_rawfull = smem_u32(&s.raw_full[0]);
  c.b_rawempty = smem_u32(&s.raw_empty[0]);
  c.b_mfull = smem_u32(&s.mfull[0]);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(c.b_rawfull + 8 * i, 1);
      mbar_init(c.b_rawempty + 8 * i, kLoadWarps);
    }
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(c.b_kready + 8 * i, 2 * kLoadWarps);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(c.b_vready + 8 * i, 2 * kLoadWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(c.b_sfull + 8 * i, 1);
      mbar_init(c.b_xch + 8 * i, kSoftmaxWarps);
    }
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(c.b_pfull + 8 * i, 2 * kSoftmaxWarps);
      mbar_init(c.b_pempty + 8 * i, 1);
    }
    for (int i = 0; i < kMaskSlots; ++i) mbar_init(c.b_mfull + 8 * i, kLoadWarps);
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
    // ================================================= softmax
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
      if (ok) ok = warp_wait(c.b_mfull + 8 * (j % kMaskSlots), (j / kMaskSlots) & 1, 30);
      if (!ok) break;
      (void)mbar_try_wait(c.b_mfull + 8 * (j % kMaskSlots), (j / kMaskSlots) & 1);
      const uint32_t live = s.vmask[j % kMaskSlots][hh];  // tokens [32 hh, 32 hh + 32)
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

    // ---- epilogue: the two threads of a head add their row sums; the
    // output rows are stored below by all warps
    s.lsum[L] = l;
    named_sync(1, kSoftmaxWarps * 32);
    const float lt = l + s.lsum[L ^ 64];
    const float lse_v = lt > 0.f ? m_used * kLn2 + logf(lt) : -INFINITY;
    s.inv[L] = lt > 0.f ? 1.f / lt : 0.f;
    if (lane == 0) s.epi_ok[warp] = ok ? 1u : 0u;
    const int hh_glob = head0 + m;
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
    producer<kPaged>(c, s, &tm_row, lane);
  } else if (warp != kIdleWarp0 && warp != kIdleWarp1) {
    dequant_role<kPaged>(c, s, dequant_index(warp), lane);
  }

  // ---- epilogue over all 16 warps: warp w normalises and stores columns
  // [64 (w / 4), +64) of the O rows in TMEM lanes [32 (w % 4), +32) (a warp
  // reaches the lanes of its sub-partition only), once PV(last) is complete
  named_sync(2, kThreads);  // the softmax warps' 1 / l and status are in place
  {
    const int qd = warp & 3;
    const int L = 32 * qd + lane;
    const int m = L & 63, hh = L >> 6;
    const bool have_o = s.epi_ok[qd] != 0 && c.ntiles > 0 && warp_wait_cluster(c.b_ofull, 0, 32);
    if (have_o) tc_fence_after();
    const float inv = s.inv[L];
    const int hh_glob = head0 + m;
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
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
    const int c0 = 64 * (warp >> 2);
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

namespace {
// Self-test of the bounded-wait error path: one warp runs the decode kernels'
// wait loop (warp_wait_n) on an mbarrier that nothing arrives on.  It gives
// up after `iters` try_wait calls, records the timeout (bits 8.. =
// kSelftestWhere) in this file's status word and the kernel returns: no
// fault, the context stays usable.
constexpr unsigned int kSelftestWhere = 63;
__device__ unsigned long long g_selftest_ns = 0;
__global__ void __launch_bounds__(32) wait_timeout_selftest_kernel(uint32_t iters) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(smem_u32(&bar), 1);
    tc::mbar_init_fence();
  }
  __syncwarp();
  unsigned long long t0, t1;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  (void)tc::warp_wait_n(smem_u32(&bar), 0, kSelftestWhere, iters);
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
  if (threadIdx.x == 0) g_selftest_ns = t1 - t0;
}
}  // namespace

int launch_wait_timeout_selftest(uint32_t iters, uint64_t* elapsed_ns, cudaStream_t st) {
  wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(iters);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  unsigned long long ns = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&ns, g_selftest_ns, sizeof(ns));
  if (elapsed_ns != nullptr) *elapsed_ns = ns;
  return check_cuda(e, "wait timeout self-test");
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
  // the pool as [num_slots] rows of 82 uint64: one gather4 box = 4 whole rows
  CUtensorMap map;
  if (int rc = encode_row_map(&map, a.kv, a.num_slots, kRowBytes / 8)) return rc;
  const size_t smem = sizeof(tc3::Smem) + 1024;  // + alignment slack
  auto go = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "decode_tc3 smem attribute");
    dim3 grid((unsigned)(a.T * a.G * 2), a.num_splits);
    return check_cuda(launch_pdl(kern, grid, dim3(tc3::kThreads), smem, st, a, map),
                      "decode_tc3_kernel launch");
  };
  const int rc = a.block_table != nullptr ? go(tc3::decode_tc3_kernel<true>)
                                          : go(tc3::decode_tc3_kernel<false>);
  if (rc != FP8MLA_OK || a.num_splits == 1) return rc;
  return launch_merge_splits(a, st);
}

}  // namespace fp8mla
