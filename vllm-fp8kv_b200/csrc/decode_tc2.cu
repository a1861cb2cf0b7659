// decode_tc2.cu -- sparse MLA decode for 128 heads per kv group on a pair of
// SMs (a 2-CTA cluster) sharing cta_group::2 tcgen05 MMAs.
//
// The pair splits the heads, not the output dims: CTA c owns heads
// [64c, 64c+64) and its TMEM holds their S and O.  One MMA spans both SMs:
//   S = Q K^T   M=128 heads (64 per CTA), N=64 tokens, K=576 (36 k-steps) plus
//               one mask k-step (S = -inf for masked tokens)
//               B is split by N: CTA c supplies the rows of tokens [32c, 32c+32)
//               of the 64-token tile (its "own" tokens), all 576 dims.
//   O += P V    M=128 heads, N=256 dims (two MMAs for the 512), K=64 tokens
//               B is split by N: CTA c supplies dims [128c, 128c+128) of each
//               MMA, i.e. latent tiles c and c+2 (its "PV half"), all 64 tokens.
// So each CTA gathers per tile: its 32 own rows whole (656 B) and the PV half
// of the other 32 rows (2 x 128 fp8 bytes + scales).  Nothing crosses between
// the SMs but the tensor cores' own operand exchange and mbarrier arrivals:
// per tile each SM dequantizes 24 K values (instead of 32 K) and the pair
// reads 59 KB of rows (instead of 84 KB for two CTAs that each gather the
// whole tile).
//
// Accumulator layout of an M=128 cta_group::2 MMA (measured): per CTA, lanes
// [0,64) hold the CTA's 64 rows x columns [0, N/2), lanes [64,128) the same
// rows x columns [N/2, N).  So softmax thread L (TMEM lane L) owns head
// (L & 63) and tokens [32 (L >> 6), +32) of a tile; the two threads of a head
// exchange their partial max through shared memory once per tile.
//
// Tensor memory (512 columns, both CTAs):
//   [  0,128)  O, dims [0,256) MMA    [128,256)  O, dims [256,512) MMA
//   [256,320)  2 S buffers x 32 fp32 columns
//   [320,512)  Q dims [0,384) as the A operand of the TMEM-A MMA (24 k-steps,
//              8 bf16x2 columns each; lanes L and L^64 hold the same head)
// Shared memory (224 KB):
//   q   Q dims [384,576) and the mask column: 4 x 64-dim swizzled blocks (64 rows)
//   k   2 stages: own tokens x 576 dims + mask column, 10 x 64-dim blocks of 32
//       rows (QK B)
//   v   3 stages: 64 tokens x PV-half dims, 4 x 64-dim blocks of 64 rows,
//       read MN-major as the PV B operand
//   p   2 stages: P (bf16) of this CTA's 64 heads x 64 tokens (PV A operand)
// S and P do not alias, so a QK may overwrite an S buffer as soon as the
// softmax that read it has handed over its P; a K stage is free once its QK
// completes, a V and a P stage once their PV completes.
//
// Warp roles (416 threads per CTA):
//   warps 0-3   softmax + epilogue (thread L = TMEM lane L)
//   warp 4      TMEM allocation in both CTAs; lane 0 of the even CTA issues
//               every MMA of the pair
//   warps 5-12  gather + dequant: part A = the PV half of the 64 rows (4 lanes
//               per row, 8 rows per warp), part B = the other half and the
//               rope of the 32 own rows (8 lanes per row, 4 rows per warp);
//               registers hold the next tile's rows while this tile is
//               written, slots are read two tiles ahead (with a block table,
//               the kPaged instantiation: raw positions three tiles ahead,
//               block-table entries two ahead).
// Barriers that gate the issuing thread (tile data, P, Q) live in the even
// CTA and count arrivals of both CTAs (one per warp; the odd CTA's by remote
// arrive); completion of pair MMAs is signalled to both CTAs by a multicast
// commit.  Every wait is bounded (g_device_status records a timeout, the roles
// drain what they issued and both CTAs free their tensor memory).
//
// Reference semantics: vllm_fp8kv/fp8_ds_mla_sparse_decode.py:77-211 (masking,
// dequant, NaN-free online softmax, LSE) and the split/merge contract of
// tests/fixtures/triton_mla_sparse_kernel_pr47629.py:232-403.
#include "common.cuh"
#include "decode.h"
#include "tc_ptx.cuh"
#include "tc_cluster.cuh"

namespace fp8mla {
namespace tc2 {

using namespace fp8mla::tc;

namespace {

constexpr int kHeads = 128;        // per kv group = per pair
constexpr int kN = 64;             // tokens per tile
constexpr int kOwn = kN / 2;       // tokens per tile whose whole row a CTA gathers
constexpr int kKSteps = 36;        // 576 / 16
// One extra k-step carries the mask: K column 576 is 0 for a live token and
// -inf for a masked one, Q column 576 is 1 (the rest of the k-step is 0), so
// the MMA itself makes S = -inf for masked tokens and the softmax needs no
// validity bits.
constexpr int kMaskBlock = 9;      // K block / Q block index holding column 576
constexpr int kQTmemSteps = 24;    // q dims [0,384) from tensor memory
constexpr int kQSmemBlocks = 4;    // q dims [384,576) and the mask column
constexpr int kQBlockBytes = 64 * 128;   // 64 rows (this CTA's heads)
constexpr int kKBlockBytes = kOwn * 128;  // 4096: 32 own rows of a 64-dim block
constexpr int kKStageBytes = 10 * kKBlockBytes;  // 9 data blocks + the mask block
constexpr int kKStages = 2;
constexpr int kVBlockBytes = kN * 128;    // 8192: 64 rows of a 64-dim block
constexpr int kVStageBytes = 4 * kVBlockBytes;
constexpr int kVStages = 3;
constexpr int kPStageBytes = 64 * 128;    // 64 heads x 64 tokens bf16
constexpr int kPStages = 2;
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kFirstLoadWarp = 5;
constexpr int kLoadWarps = 8;
constexpr int kThreads = (kSoftmaxWarps + 1 + kLoadWarps) * 32;  // 416
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
  float pmax[2][128];                      // partial tile max, by tile parity
  float lsum[128];                         // partial row sums (epilogue)
  uint64_t tfull[kVStages];                // even CTA: tile j's rows in both CTAs
  uint64_t kempty[kKStages], vempty[kVStages];
  uint64_t sfull[2], pfull[kPStages], pempty[kPStages];
  uint64_t xch[2];                         // partial-max exchange, by tile parity
  uint64_t qready, ofull, drain;
  uint32_t tmem_base;
};
static_assert(offsetof(Smem, k) % 1024 == 0 && offsetof(Smem, v) % 1024 == 0 &&
                  offsetof(Smem, p) % 1024 == 0 && kKStageBytes % 1024 == 0,
              "swizzle atoms need 1024-B alignment");
static_assert(offsetof(Smem, tfull) % 8 == 0, "");
static_assert(sizeof(Smem) + 1024 <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

// One load lane's share of a tile: part A (PV half of row rowA: 4 fp8 chunks
// + the scale chunk), part B (own row rowB: 2 fp8 chunks, 1 rope chunk and
// the scale chunk).
struct Rows {
  uint4 a[4], asc;
  uint4 b[2], brope, bsc;
};

struct Ctx {
  const DecodeArgs* a;
  const int32_t* idx_row;
  int32_t req;
  int beg, end, ntiles;
  uint32_t rank;  // 0 = the CTA that issues the pair's MMAs
  uint32_t tmem;
  uint32_t sq, sk0, sv0, sp0;
  uint32_t b_tfull, b_kempty, b_vempty, b_sfull, b_pfull, b_pempty;
  uint32_t b_xch, b_qready, b_ofull, b_drain;
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
  // the mask k-step: Q block 3 / K block 9, first 16 columns
  mma_pair_ss(tS, qdesc0 + (uint64_t)((3 * kQBlockBytes) >> 4),
              kdesc + (uint64_t)((kMaskBlock * kKBlockBytes) >> 4), kIdescQK, 1u);
}

__device__ void mma_role(const Ctx& c) {
  bool ok = thread_wait_cluster(c.b_qready, 0, 5);
  tc_fence_after();
  const uint32_t tQ = c.tmem + kColQ;
  const uint64_t qdesc0 = sdesc_sw128(c.sq, 16, 1024);
  const uint64_t kdesc0 = sdesc_sw128(c.sk0, 16, 1024);
  const uint64_t pdesc0 = sdesc_sw128(c.sp0, 16, 1024);
  // V read MN-major: the CTA's two 64-dim blocks of an MMA kVBlockBytes apart
  // (LBO), 8-token groups 1 KB apart (SBO)
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
    const int b = j & 1, ks = j % kKStages, ts = j % kVStages;
    ok = thread_wait_cluster(c.b_tfull + 8 * ts, (j / kVStages) & 1, 7);
    if (!ok) break;
    tc_fence_after();
    issue_qk(c.tmem + kColS + kSBufCols * b, tQ, qdesc0,
             kdesc0 + (uint64_t)((ks * kKStageBytes) >> 4));
    mma_commit_pair(c.b_sfull + 8 * b);
    mma_commit_pair(c.b_kempty + 8 * ks);
    if (j >= 1) {
      const int jp = j - 1;
      ok = thread_wait_cluster(c.b_pfull + 8 * (jp % kPStages), (jp / kPStages) & 1, 6);
      if (!ok) break;
      tc_fence_after();
      issue_pv(jp);
    }
  }
  if (ok && c.ntiles > 0) {
    const int jl = c.ntiles - 1;
    ok = thread_wait_cluster(c.b_pfull + 8 * (jl % kPStages), (jl / kPStages) & 1, 6);
    if (ok) {
      tc_fence_after();
      issue_pv(jl);
      mma_commit_pair(c.b_ofull);
    }
  }
  // drain: nothing this thread issued may still touch either CTA's memory
  mma_commit_pair(c.b_drain);
  thread_wait_cluster(c.b_drain, 0, 9);
}

// ------------------------------------------------------------------ gather + dequant
// kPaged: the index entries are request-local positions resolved through the
// block table; the index pipeline then runs one tile deeper (raw entry three
// tiles ahead, block-table read two ahead, slot one ahead) so that no step
// waits on the two dependent loads of a position.
template <bool kPaged>
__device__ void load_role(const Ctx& c, Smem& s, int lw, int lane) {
  const DecodeArgs& a = *c.a;
  const int cr = (int)c.rank;
  // part A: row rowA of the tile, lane quarter pA: PV-half chunks pA + 4i
  const int rowA = lw * 8 + (lane & 7), pA = lane >> 3;
  // part B: own row rowB (tile row kOwn*cr + rowB), lane eighth qB
  const int rowB = lw * 4 + (lane >> 3), qB = lane & 7;
  const bool ownA = (rowA >> 5) == cr;
  // A warp's tile rows are 8 part-A rows and 4 own part-B rows: lane i < 8
  // converts the index of part-A row lw*8 + i, lane 8 + i (i < 4) that of own
  // row lw*4 + i, and the slots reach the lanes that gather them by shuffle.
  const int irow = lane < 8 ? lw * 8 + lane : (lane < 12 ? kOwn * cr + lw * 4 + (lane - 8) : -1);
  auto raw_at = [&](int jt) -> int32_t {
    const int pos = c.beg + jt * kN + irow;
    return (irow >= 0 && pos < c.end) ? c.idx_row[pos] : -1;
  };
  auto slot_at = [&](int jt) -> int32_t { return live_slot(a, c.req, raw_at(jt)); };
  auto share = [&](int32_t sl, int32_t& sa, int32_t& sb) {
    sa = __shfl_sync(0xFFFFFFFFu, sl, lane & 7);         // part-A row of this lane
    sb = __shfl_sync(0xFFFFFFFFu, sl, 8 + (lane >> 3));  // own part-B row of this lane
  };
  // vb: own row rowB is live (its mask column is 0, else -inf)
  auto load = [&](int32_t sa, int32_t sb, Rows& R, bool& vb) {
    vb = sb >= 0;
    if (sa >= 0) {
      const uint8_t* src = a.kv + sa * (int64_t)kRowBytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tile = cr + 2 * (i >> 1);
        R.a[i] = ldg_v4(src + 128 * tile + 16 * (pA + 4 * (i & 1)));
      }
      R.asc = ldg_v4(src + kScaleOff);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) R.a[i] = make_uint4(0, 0, 0, 0);
      R.asc = make_uint4(0, 0, 0, 0);
    }
    if (sb >= 0) {
      const uint8_t* src = a.kv + sb * (int64_t)kRowBytes;
      R.b[0] = ldg_v4(src + 128 * (1 - cr) + 16 * qB);
      R.b[1] = ldg_v4(src + 128 * (3 - cr) + 16 * qB);
      R.brope = ldg_v4(src + kRopeOff + 16 * qB);
      R.bsc = ldg_v4(src + kScaleOff);
    } else {
      R.b[0] = R.b[1] = R.brope = R.bsc = make_uint4(0, 0, 0, 0);
    }
  };
  auto deq = [&](const uint4& w, float sc, uint4& o0, uint4& o1) {
    dequant4_hw_x2(w.x, sc, o0.x, o0.y);
    dequant4_hw_x2(w.y, sc, o0.z, o0.w);
    dequant4_hw_x2(w.z, sc, o1.x, o1.y);
    dequant4_hw_x2(w.w, sc, o1.z, o1.w);
  };
  auto pick = [](const uint4& sc, int tile) -> float {
    return __uint_as_float(tile == 0 ? sc.x : tile == 1 ? sc.y : tile == 2 ? sc.z : sc.w);
  };
  bool ok = true;
  // at step j >= 1: slots of tile j+1 (read one step ahead); tiles 0 and 1
  // are loaded before step 0, with the first three tiles' indices read at once
  int32_t nI = -1;       // flat: slot of tile j+1; paged: raw entry of tile j+2
  SlotPf fI{-1, 0};       // paged: block-table read of tile j+1 (at step j >= 1)
  auto step = [&](int j, const Rows& cur, bool vownB, Rows& nxt, bool& vnxt) {
    if (!ok || j >= c.ntiles) return;
    if (j >= 1) {
      int32_t s1;
      if constexpr (kPaged) {
        s1 = slot_finish(a, fI);
        fI = slot_fetch(a, c.req, nI);
        nI = raw_at(j + 3);
      } else {
        s1 = nI;
        if (j + 2 < c.ntiles) nI = slot_at(j + 2);
      }
      int32_t sa1, sb1;
      share(s1, sa1, sb1);
      if (j + 1 < c.ntiles) load(sa1, sb1, nxt, vnxt);
    }
    const int ks = j % kKStages, vs = j % kVStages;
    if (j >= kKStages) ok = warp_wait_cluster(c.b_kempty + 8 * ks, ((j / kKStages) + 1) & 1, 10);
    if (ok && j >= kVStages)
      ok = warp_wait_cluster(c.b_vempty + 8 * vs, ((j / kVStages) + 1) & 1, 12);
    if (!ok) return;
    uint8_t* kst = s.k[ks];
    uint8_t* vst = s.v[vs];
    // part A -> V stage (and the K stage for own rows)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tile = cr + 2 * (i >> 1);
      uint4 o0, o1;
      deq(cur.a[i], pick(cur.asc, tile), o0, o1);
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
    // part B -> K stage: the other two latent tiles and the rope of own row rowB
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int tile = (1 - cr) + 2 * i;
      uint4 o0, o1;
      deq(cur.b[i], pick(cur.bsc, tile), o0, o1);
      uint8_t* kb = kst + (2 * tile + (qB >> 2)) * kKBlockBytes;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3))) = o0;
      *reinterpret_cast<uint4*>(kb + swz(rowB, 2 * (qB & 3) + 1)) = o1;
    }
    *reinterpret_cast<uint4*>(kst + 8 * kKBlockBytes + swz(rowB, qB)) = cur.brope;
    // mask column of own row rowB: bf16 0 (live) or -inf (masked); the other
    // 15 columns of the k-step (chunk 1 and the rest of chunk 0) stay 0
    if (qB < 2)
      *reinterpret_cast<uint4*>(kst + kMaskBlock * kKBlockBytes + swz(rowB, qB)) =
          make_uint4(qB == 0 && !vownB ? 0xFF80u : 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(c.b_tfull + 8 * vs, 0);  // the issuing CTA's tile barrier
  };
  Rows A, B;
  bool vA = false, vB = false;
  {
    const int32_t s0 = slot_at(0), s1 = slot_at(1);
    if constexpr (kPaged) {
      fI = slot_fetch(a, c.req, raw_at(2));
      nI = raw_at(3);
    } else {
      nI = slot_at(2);
    }
    int32_t s0A, s0B, s1A, s1B;
    share(s0, s0A, s0B);
    share(s1, s1A, s1B);
    if (c.ntiles > 0) load(s0A, s0B, A, vA);
    if (c.ntiles > 1) load(s1A, s1B, B, vB);
  }
  for (int j = 0; j < c.ntiles && ok; j += 2) {
    step(j, A, vA, B, vB);
    step(j + 1, B, vB, A, vA);
  }
}

}  // namespace

template <bool kPaged>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    decode_tc2_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x / (2 * a.G);
  const int grp = (blockIdx.x >> 1) % a.G;
  const int split = blockIdx.y;
  const uint32_t rank = cluster_rank();  // == blockIdx.x & 1
  // 128 heads per group, or 64: then the odd CTA's rows are padding (zero Q,
  // nothing stored) and the even CTA holds every head
  const int head0 = grp * a.hpg + 64 * (int)rank;
  const int nh = max(0, min(64, a.hpg - 64 * (int)rank));  // real heads of this CTA

  Ctx c;
  c.a = &a;
  c.rank = rank;
  c.beg = split * a.split_len;
  c.end = min(a.topk, c.beg + a.split_len);
  c.ntiles = c.end > c.beg ? (c.end - c.beg + kN - 1) / kN : 0;
  c.idx_row = a.idx + t * a.idx_st + grp * a.idx_sg;
  c.req = 0;  // read after pdl_wait below
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

  if (threadIdx.x == 0) {
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(c.b_tfull + 8 * i, 2 * kLoadWarps);
      mbar_init(c.b_vempty + 8 * i, 1);
    }
    for (int i = 0; i < kKStages; ++i) mbar_init(c.b_kempty + 8 * i, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(c.b_sfull + 8 * i, 1);
      mbar_init(c.b_xch + 8 * i, kSoftmaxWarps);
    }
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(c.b_pfull + 8 * i, 2 * kSoftmaxWarps);
      mbar_init(c.b_pempty + 8 * i, 1);
    }
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
      // Q dims [0,384) -> TMEM (lane L and L^64 both hold head m), dims [384,576)
      // -> swizzled smem (thread hh writes chunks [4hh, 4hh+4) of each block);
      // padding rows are zero
      const bool hv = m < nh;
      const uint4* qsrc = reinterpret_cast<const uint4*>(
          static_cast<const uint16_t*>(a.q) + t * a.q_st + (int64_t)(hv ? head0 + m : 0) * a.q_sh);
      const uint4 z4 = make_uint4(0, 0, 0, 0);
      // three load rounds (was seven): dims [384,576) (this thread's 12
      // chunks) to smem, then dims [0,384) (48 chunks) to tensor memory in
      // two halves
      {
        uint4 x[12];
#pragma unroll
        for (int blk = 0; blk < kQSmemBlocks - 1; ++blk)
#pragma unroll
          for (int i = 0; i < 4; ++i) x[4 * blk + i] = hv ? qsrc[kQTmemSteps * 2 + blk * 8 + 4 * hh + i] : z4;
#pragma unroll
        for (int blk = 0; blk < kQSmemBlocks - 1; ++blk)
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
      if (hh == 0) {  // mask k-step of Q: bf16 1.0 in column 576, zeros in 577..591
        *reinterpret_cast<uint4*>(s.q + 3 * kQBlockBytes + swz(m, 0)) = make_uint4(0x3F80u, 0, 0, 0);
        *reinterpret_cast<uint4*>(s.q + 3 * kQBlockBytes + swz(m, 1)) = make_uint4(0, 0, 0, 0);
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
      ok = warp_wait_cluster(c.b_sfull + 8 * b, (j >> 1) & 1, 1);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32];
      tmem_ld32(trow + kColS + kSBufCols * b, sv);
      tmem_wait_ld();
      float pm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) pm = fmaxf(pm, __uint_as_float(sv[i]));  // masked: -inf
      pm *= a.scale_log2;
      s.pmax[b][L] = pm;
      __syncwarp();
      if (lane == 0) mbar_arrive(c.b_xch + 8 * b);
      ok = warp_wait(c.b_xch + 8 * b, (j >> 1) & 1, 14);  // bounded, unlike a named barrier
      if (!ok) break;
      const float tmax = fmaxf(pm, s.pmax[b][L ^ 64]);
      // lazy reference max (same decision in both threads of a head)
      float alpha = 1.f;
      if (tmax > m_used + kRescaleThreshold || (m_used == -INFINITY && tmax > -INFINITY)) {
        alpha = (m_used == -INFINITY) ? 1.f : ex2_approx(m_used - tmax);
        m_used = tmax;
        l *= alpha;
      }
      if (__any_sync(0xFFFFFFFFu, alpha != 1.f) && j > 0) {
        // O rows are rescaled once PV(j-1) has finished writing them
        const int jp = j - 1;
        ok = warp_wait_cluster(c.b_pempty + 8 * (jp % kPStages), (jp / kPStages) & 1, 3);
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
      // P stage ps was last read by PV(j-2), which was issued before QK(j): its
      // completion is implied by sfull(j) (a commit arrives once every earlier
      // MMA of the issuing thread has completed)
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
    const bool have_o = ok && c.ntiles > 0 && warp_wait_cluster(c.b_ofull, 0, 4);
    if (have_o) tc_fence_after();
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    const float lse_v = lt > 0.f ? m_used * kLn2 + logf(lt) : -INFINITY;
    const int hh_glob = head0 + m;
    // O column c of MMA hf holds dim 256 hf + 128 hh + (c mod 128)
    auto store32 = [&](const uint32_t (&o)[32], int c0) {
      const int d = 256 * (c0 >> 7) + 128 * hh + (c0 & 127);
      uint4* dst = a.num_splits == 1
                       ? reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + t * a.out_st +
                                                  (int64_t)hh_glob * a.out_sh + d)
                       // bf16 partials (the output is bf16), merged in fp32 by merge_splits_kernel
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
    // two 32-column tensor-memory loads in flight per wait
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
      if (m < nh) {  // padding rows store nothing (the loads above are warp-collective)
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
    // ================================================= MMA issuer (even CTA)
    if (rank == 0 && lane == 0) mma_role(c);
    __syncwarp();
  } else {
    // ================================================= gather + dequant
    load_role<kPaged>(c, s, warp - kFirstLoadWarp, lane);
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

}  // namespace tc2

bool decode_tc_supported(const DecodeArgs& a) {
  return a.q_dtype == FP8MLA_DTYPE_BF16 && (a.hpg == tc2::kHeads || a.hpg == tc2::kHeads / 2) &&
         a.G >= 1;
}

int launch_decode_tc2(const DecodeArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(tc2::Smem) + 1024;  // + alignment slack
  auto go = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "decode_tc2 smem attribute");
    dim3 grid((unsigned)(a.T * a.G * 2), a.num_splits);
    return check_cuda(launch_pdl(kern, grid, dim3(tc2::kThreads), smem, st, a),
                      "decode_tc2_kernel launch");
  };
  const int rc = a.block_table != nullptr ? go(tc2::decode_tc2_kernel<true>)
                                          : go(tc2::decode_tc2_kernel<false>);
  if (rc != FP8MLA_OK || a.num_splits == 1) return rc;
  return launch_merge_splits(a, st);
}

namespace {
// Self-test of the bounded-wait error path: one warp runs the decode kernels'
// wait loop (warp_wait_n) on an mbarrier that nothing arrives on.  It gives
// up after `iters` try_wait calls, records the timeout (bits 8.. =
// kSelftestWhere) and the kernel returns: no fault, the context stays usable.
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
