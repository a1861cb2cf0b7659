// indexer.cu -- the read path of the sparse-MLA models' token indexer on
// sm_100a: fp8 paged MQA logits (tcgen05, kind::f8f6f4) and the per-row top-k
// that fills the decode's top-k position buffer.
//
// Key cache (vLLM's indexer cache, structure of arrays per block): a block of
// 64 tokens is 64 x 128 e4m3 bytes followed by 64 fp32 scales, 8448 bytes
// (reference PORT_PLAN.md:14 and trap 3).  Queries are e4m3 too, [B, next_n,
// 64 heads, 128]; their scale is folded into `weights` by the caller.
//
//   logits[b*next_n + n, s] = scale_s * sum_h relu(q[b,n,h] . k_s) * w[b*next_n + n, h]
//   for s < context_len_b - next_n + n + 1, and -inf elsewhere
//
// (vLLM 0.22's restatement of DeepGEMM's reference,
// vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:256-354, which the oracle and
// the golden vectors follow.)  The reference repository has no code for this
// path, only its specification.
//
// Logits kernel: one CTA handles a chunk of one request's context in tiles of
// 128 tokens (two blocks).  The products are one MMA per 32 dims with the
// tokens as M (128) and the request's next_n x 64 query heads as N:
// D[token][head] = k_token . q_head, exact e4m3 x e4m3 products accumulated in
// fp32, so that each epilogue thread (TMEM lane = token) reduces its own row
// over the heads without talking to other threads.
//   warps 0-3  epilogue: relu, weights, sum, scale, mask, store (coalesced)
//   warp 4     producer: block ids from the block table, TMA copies of each
//              block's values (one 3-D box, 128-byte swizzled) and a bulk copy
//              of its 64 scales into a ring of five stages (four when
//              next_n is 2); the epilogue warps release a stage
//   warp 5     tensor memory allocation; lane 0 issues the MMAs
// Two accumulator buffers in tensor memory let the epilogue of tile t overlap
// the MMAs of tile t+1.  Every wait is bounded (status word, as the decode).
//
// Top-k: a 2-CTA cluster per logits row (one CTA per row for rows above
// 92,160 positions).  Logits map to order-preserving 32-bit keys, kept in
// shared memory (each CTA its half of the row); three histogram passes (11, 11
// and 10 bits, the two CTAs' counts added through distributed shared memory)
// find the k-th largest key exactly; a final pass in position order writes
// every position above it and the lowest-positioned ties, ascending, then -1
// padding.
#include "common.cuh"
#include "decode.h"
#include "tc_cluster.cuh"
#include "tc_ptx.cuh"
#include "tma_map.h"

namespace fp8mla {
namespace idx {

using namespace fp8mla::tc;

namespace {

constexpr int kDim = 128;                 // index head dim (bytes per fp8 key row)
constexpr int kHeads = 64;                // index heads per query token
constexpr int kBlock = 64;                // tokens per cache block
constexpr int kPageBytes = kBlock * (kDim + 4);   // 8448
constexpr int kTileTokens = 128;          // MMA M: two blocks
constexpr int kStageBytes = kTileTokens * kDim;   // 16 KB of values
// The logits kernel is built for NN = 1 (decode) and NN = 2 (next_n 2) query
// tokens per request (N = 64 NN query heads <= 128; the C ABI refuses larger
// next_n): with one token's query rows the key ring has five stages in the
// shared memory that two CTAs per SM leave, with two tokens' four.
template <int NN>
constexpr int stages_for() { return NN == 1 ? 5 : 4; }
constexpr int kThreads = 6 * 32;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;

// kind::f8f6f4 instruction descriptor: fp32 accumulate, A and B e4m3 (format
// code 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int NN>
struct Smem {
  static constexpr int kStages = stages_for<NN>();
  uint8_t kv[kStages][kStageBytes];        // 1024-aligned: swizzled operand tiles
  uint8_t q[2][NN * kHeads * kDim];        // 1024-aligned: N rows of 128 B, swizzled, by item parity
  float scale[kStages][kTileTokens];
  float w[2][NN * kHeads];                 // by item parity
  uint8_t pvalid[kStages][2];              // block p of the stage's tile was loaded
  uint64_t full[kStages], empty[kStages];
  uint64_t tfull[2], tempty[2];
  uint64_t qfull[2], qempty[2], drain;
  uint32_t tmem_base;
};
static_assert(offsetof(Smem<1>, q) % 1024 == 0 && offsetof(Smem<2>, q) % 1024 == 0,
              "swizzle atoms need 1024-B alignment");
static_assert(offsetof(Smem<1>, full) % 8 == 0 && offsetof(Smem<2>, full) % 8 == 0, "");
static_assert(2 * (sizeof(Smem<1>) + 1024) <= 228 * 1024 && 2 * (sizeof(Smem<2>) + 1024) <= 228 * 1024,
              "two CTAs per SM");

struct Args {
  const uint8_t* q;          // [B, next_n, 64, 128] e4m3, contiguous per request
  int64_t q_stride_b;        // bytes between requests
  const uint8_t* k_cache;    // [num_blocks, 8448]
  int64_t num_blocks;
  const float* w;            // [B * next_n, 64], row stride w_stride
  int64_t w_stride;
  const int32_t* ctx;        // [B]
  const int32_t* bt;         // [B, bt_stride]
  int64_t bt_stride, max_blocks;
  float* logits;             // [B * next_n, logits_stride]
  int64_t logits_stride, max_len;
  int next_n;
  int tiles_per_item;        // tiles of a work item (a chunk of one request's context)
  int chunks_per_req;        // items per request
  int items;                 // B * chunks_per_req
};

// The epilogue warps' own barrier (id 1; the other warps never use it).
__device__ __forceinline__ void named_sync_epi() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

__device__ __forceinline__ uint32_t swz128(uint32_t r, uint32_t c) {  // row r, 16-B chunk c
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

__device__ __forceinline__ void mma_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tma_load_page(uint32_t dst, const CUtensorMap* tm, int32_t block,
                                              uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(dst),
      "l"(tm), "r"(0), "r"(0), "r"(block), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

}  // namespace

namespace {

// ------------------------------------------------------------------ logits
// Persistent: CTA x walks items u = x, x + gridDim.x, ...; an item is
// tiles_per_item tiles of one request's context.  Every role walks the same
// sequence; the stage ring and the accumulator buffers run across items (i
// counts the CTA's computed tiles), the query rows and head weights are
// double-buffered by item parity (k counts the CTA's items).
struct Item {
  int b, t0, ntiles, ncomp, ctx;
};
__device__ __forceinline__ Item item_of(const Args& a, int u) {
  Item it;
  it.b = u / a.chunks_per_req;
  it.t0 = (u % a.chunks_per_req) * a.tiles_per_item;
  const int total_tiles = (int)((a.max_len + kTileTokens - 1) / kTileTokens);
  it.ntiles = max(0, min(a.tiles_per_item, total_tiles - it.t0));
  it.ctx = max(0, a.ctx[it.b]);
  // tiles with a token below the context are computed; the rest are -inf
  const int ctx_tiles = (int)(((int64_t)it.ctx + kTileTokens - 1) / kTileTokens);
  it.ncomp = max(0, min(it.ntiles, ctx_tiles - it.t0));
  return it;
}

template <int NN>
__device__ void producer(const Args& a, Smem<NN>& s, const CUtensorMap* tm) {
  constexpr int kStages = Smem<NN>::kStages;
  int i = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < a.items && ok; u += gridDim.x) {
    const Item it = item_of(a, u);
    for (int ii = 0; ii < it.ncomp; ++ii, ++i) {
      const int st = i % kStages, t = it.t0 + ii;
      if (i >= kStages) ok = thread_wait(smem_u32(&s.empty[st]), ((i / kStages) + 1) & 1, 50);
      if (!ok) break;
      int32_t bid[2];
      uint32_t bytes = 0;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int64_t pos = 2 * (int64_t)t + p;  // block of the request
        bid[p] = -1;
        if ((int64_t)t * kTileTokens + p * kBlock < it.ctx && pos < a.max_blocks) {
          const int32_t v = a.bt[(int64_t)it.b * a.bt_stride + pos];
          if (v >= 0 && v < a.num_blocks) bid[p] = v;
        }
        s.pvalid[st][p] = bid[p] >= 0 ? 1 : 0;
        if (bid[p] >= 0) bytes += kBlock * kDim + kBlock * 4;
      }
      const uint32_t bar = smem_u32(&s.full[st]);
      mbar_arrive_expect_tx(bar, bytes);  // releases the flags above
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (bid[p] < 0) continue;
        tma_load_page(smem_u32(s.kv[st]) + p * kBlock * kDim, tm, bid[p], bar);
        bulk_g2s(smem_u32(&s.scale[st][p * kBlock]),
                 a.k_cache + (int64_t)bid[p] * kPageBytes + kBlock * kDim, kBlock * 4, bar);
      }
    }
  }
  // no copy may outlive the CTA: the stages armed last have landed (full limit)
  for (int x = i > kStages ? i - kStages : 0; x < i; ++x)
    (void)thread_wait(smem_u32(&s.full[x % kStages]), (x / kStages) & 1, 51);
}

template <int NN>
__device__ void mma_issuer(const Args& a, Smem<NN>& s, uint32_t tmem, int N) {
  constexpr int kStages = Smem<NN>::kStages;
  const uint32_t idesc = idesc_e4m3(kTileTokens, N);
  int i = 0, k = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < a.items && ok; u += gridDim.x, ++k) {
    const int ncomp = item_of(a, u).ncomp;
    const int qb = k & 1;
    ok = thread_wait(smem_u32(&s.qfull[qb]), (k >> 1) & 1, 52);
    if (!ok) break;
    tc_fence_after();
    const uint64_t qdesc = sdesc_sw128(smem_u32(s.q[qb]), 16, 1024);
    for (int ii = 0; ii < ncomp && ok; ++ii, ++i) {
      const int st = i % kStages, buf = i & 1;
      ok = thread_wait(smem_u32(&s.full[st]), (i / kStages) & 1, 53);
      if (ok && i >= 2) ok = thread_wait(smem_u32(&s.tempty[buf]), ((i >> 1) + 1) & 1, 54);
      if (!ok) break;
      tc_fence_after();
      const uint64_t adesc = sdesc_sw128(smem_u32(s.kv[st]), 16, 1024);
#pragma unroll
      for (int kk = 0; kk < kDim / 32; ++kk)  // 32 e4m3 values = 32 bytes per k-step
        mma_f8(tmem + buf * N, adesc + (uint64_t)((kk * 32) >> 4), qdesc + (uint64_t)((kk * 32) >> 4),
               idesc, kk > 0 ? 1u : 0u);
      // the stage is released by the epilogue warps, which read its scales
      // after they have seen this commit (so the MMAs are done with it)
      mma_commit(smem_u32(&s.tfull[buf]));
    }
    // this item's query buffer is free once its MMAs complete (at once when
    // it had none)
    mma_commit(smem_u32(&s.qempty[qb]));
  }
  // drain: no MMA may still run when tensor memory is freed
  mma_commit(smem_u32(&s.drain));
  (void)thread_wait(smem_u32(&s.drain), 0, 55);
}

// The request's query rows (swizzled K-major operand) and head weights into
// buffer qb; announced on qfull[qb] after every epilogue warp's stores.
template <int NN>
__device__ void load_query(const Args& a, Smem<NN>& s, int b, int qb, int N, int lane) {
  const int nn = a.next_n;
  const uint4* qsrc = reinterpret_cast<const uint4*>(a.q + (int64_t)b * a.q_stride_b);
  for (int c = threadIdx.x; c < N * (kDim / 16); c += 128) {
    const int row = c >> 3, chunk = c & 7;
    *reinterpret_cast<uint4*>(s.q[qb] + swz128(row, chunk)) = qsrc[c];
  }
  for (int c = threadIdx.x; c < N; c += 128)
    s.w[qb][c] = a.w[((int64_t)b * nn + c / kHeads) * a.w_stride + (c % kHeads)];
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) mbar_arrive(smem_u32(&s.qfull[qb]));
}

template <int NN>
__device__ void epilogue(const Args& a, Smem<NN>& s, uint32_t tmem, int N) {
  constexpr int kStages = Smem<NN>::kStages;
  constexpr int kMaxNextN = NN;  // query tokens per request, at most
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = threadIdx.x;  // TMEM lane = token of the tile
  const int nn = a.next_n;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  bool ok = true;
  int i = 0, k = 0;
  if ((int)blockIdx.x < a.items) load_query(a, s, item_of(a, blockIdx.x).b, 0, N, lane);
  for (int u = blockIdx.x; u < a.items; u += gridDim.x, ++k) {
    const Item it = item_of(a, u);
    // the next item's query rows and weights into the other buffer, once the
    // MMAs of the item before this one (its last user) are complete and every
    // epilogue warp has finished that item's tiles (its weights)
    const int un = u + gridDim.x;
    named_sync_epi();
    if (un < a.items) {
      if (k >= 1 && ok) ok = warp_wait(smem_u32(&s.qempty[(k + 1) & 1]), ((k - 1) >> 1) & 1, 58);
      load_query(a, s, item_of(a, un).b, (k + 1) & 1, N, lane);
    }
    // every epilogue warp reaches these barriers twice per item whatever `ok`
    // is (a warp whose wait gave up keeps walking the items without work)
    named_sync_epi();  // s.w[k & 1] (stored one item ago) is read below
    const float* wk = s.w[k & 1];
    for (int ii = 0; ii < it.ntiles; ++ii) {
      const int64_t tok = (int64_t)(it.t0 + ii) * kTileTokens + r;
      float v[kMaxNextN];
#pragma unroll
      for (int n = 0; n < kMaxNextN; ++n) v[n] = -INFINITY;
      if (ii < it.ncomp) {
        const int st = i % kStages, buf = i & 1;
        ++i;
        if (ok) ok = warp_wait(smem_u32(&s.tfull[buf]), ((i - 1) >> 1) & 1, 56);
        if (ok) ok = warp_wait(smem_u32(&s.full[st]), ((i - 1) / kStages) & 1, 57);
        if (ok) {
          (void)mbar_try_wait(smem_u32(&s.full[st]), ((i - 1) / kStages) & 1);  // every lane acquires
          tc_fence_after();
          float acc[kMaxNextN];
#pragma unroll
          for (int n = 0; n < kMaxNextN; ++n) {
            acc[n] = 0.f;
            if (n < nn) {
              uint32_t d0[32], d1[32];
              tmem_ld32(trow + buf * N + n * kHeads, d0);
              tmem_ld32(trow + buf * N + n * kHeads + 32, d1);
              tmem_wait_ld();
              const float* w = wk + n * kHeads;
#pragma unroll
              for (int h = 0; h < 32; ++h) {
                acc[n] = fmaf(fmaxf(__uint_as_float(d0[h]), 0.f), w[h], acc[n]);
                acc[n] = fmaf(fmaxf(__uint_as_float(d1[h]), 0.f), w[32 + h], acc[n]);
              }
            }
          }
          const float sc = s.scale[st][r];
          const bool live = s.pvalid[st][r >> 6] != 0;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(smem_u32(&s.tempty[buf]));  // accumulator buffer read
            mbar_arrive(smem_u32(&s.empty[st]));    // scales and flags read
          }
#pragma unroll
          for (int n = 0; n < kMaxNextN; ++n)
            if (n < nn && live && tok < (int64_t)it.ctx - nn + n + 1) v[n] = acc[n] * sc;
        }
      }
      if (tok < a.max_len) {
#pragma unroll
        for (int n = 0; n < kMaxNextN; ++n)
          if (n < nn) a.logits[((int64_t)it.b * nn + n) * a.logits_stride + tok] = v[n];
      }
    }
  }
}

}  // namespace

template <int NN>
__global__ void __launch_bounds__(kThreads, 1)
    indexer_logits_kernel(const Args a, const __grid_constant__ CUtensorMap tm) {
  constexpr int kStages = Smem<NN>::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
  Smem<NN>& s = *reinterpret_cast<Smem<NN>*>(smem_raw + pad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = kHeads * a.next_n;
  const uint32_t tmem_cols = N <= 64 ? 128u : 256u;  // two accumulator buffers

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&s.full[i]), 1);
      mbar_init(smem_u32(&s.empty[i]), 4);  // the 4 epilogue warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s.tfull[i]), 1);
      mbar_init(smem_u32(&s.tempty[i]), 4);
      mbar_init(smem_u32(&s.qfull[i]), 4);
      mbar_init(smem_u32(&s.qempty[i]), 1);
    }
    mbar_init(smem_u32(&s.drain), 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&s.tmem_base), tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();  // the previous kernel of the stream has completed: global memory from here on
  const uint32_t tmem = s.tmem_base;

  if (warp < 4) {
    epilogue(a, s, tmem, N);
  } else if (warp == kProducerWarp) {
    if (lane == 0) producer(a, s, &tm);
    __syncwarp();
  } else {
    if (lane == 0) mma_issuer(a, s, tmem, N);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// ------------------------------------------------------------------ top-k
constexpr int kTopkThreads = 1024;

__device__ __forceinline__ uint32_t sortable_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive scan of v over 1024 threads; returns this thread's
// prefix and writes the total to *total (every thread).
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* warp_sums, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const uint32_t before = (warp > 0 ? warp_sums[warp - 1] : 0u) + (x - v);
  *total = warp_sums[31];
  __syncthreads();  // warp_sums is reused by the next call
  return before;
}

// A row is split over a 2-CTA cluster; each CTA keeps up to this many of its
// positions' keys in shared memory (192 KB), so the row is read from global
// memory once.  Longer rows take the single-CTA kernel, which re-reads the
// row for each pass (from L2).
constexpr int kSmemKeys = 46 * 1024;
constexpr int kCand = 4096;  // compacted candidates of the first pass (16 KB)
constexpr int64_t kRound = (int64_t)kTopkThreads * 32;  // positions of one write round
static_assert(kSmemKeys <= 2 * kRound, "a CTA's positions take at most two write rounds");

// Positions of a row per CTA of the pair: half the row, rounded up to whole
// 1024-position warp ranges; CTA c takes [c * half, c * half + half).
__host__ __device__ constexpr int64_t pair_half(int64_t lim) {
  return (((lim + 1) / 2) + 1023) & ~(int64_t)1023;
}
// Longest row the pair keeps resident.
constexpr int64_t kPairMaxLen = 2 * (int64_t)kSmemKeys - 2048;
static_assert(pair_half(kPairMaxLen) <= kSmemKeys, "");

// Store v to the 32-bit word at shared::cta address `local` of cluster CTA `rank`.
__device__ __forceinline__ void st_dsmem(uint32_t local, uint32_t rank, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;\n" ::"r"(mapa(local, rank)), "r"(v) : "memory");
}

// Top-k of one row on a CTA pair (rows up to kPairMaxLen).  Each CTA loads and
// converts its half of the row; the three histogram passes add the two CTAs'
// counts through distributed shared memory, so both choose the same bins;
// each CTA compacts and counts its own candidates; CTA 1 writes its positions
// after CTA 0's (its base is CTA 0's totals).
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTopkThreads)
    indexer_topk_pair_kernel(const float* logits, int64_t logits_stride, int next_n,
                             const int32_t* ctx, int32_t* out, int64_t out_stride, int k,
                             int64_t max_len) {
  extern __shared__ uint32_t skeys[];  // keys of this CTA's positions
  __shared__ uint32_t hist[2048];      // this CTA's counts
  __shared__ uint32_t hpeer[2][2048];  // the peer CTA's counts, by pass parity
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sel[2];          // chosen bin, keys above it (this pass)
  __shared__ uint32_t cand[kCand];     // this CTA's positions in the first pass's bin
  __shared__ uint32_t ncand;
  __shared__ uint32_t gabove[32], cgt[32], ceq[32];  // per warp range
  __shared__ uint32_t tot_ge[2];       // CTA 1: CTA 0's keys above / equal to the k-th key
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  const uint32_t peer = cluster_rank() ^ 1u;
  const int64_t r = blockIdx.x >> 1;
  const int b = (int)(r / next_n), n = (int)(r % next_n);
  const int64_t lim = min(max_len, (int64_t)ctx[b] - next_n + n + 1);
  const float* row = logits + r * logits_stride;
  int32_t* o = out + r * out_stride;
  if (lim <= k) {  // every position kept, then padding (both CTAs leave here)
    if (peer == 1)
      for (int i = threadIdx.x; i < k; i += kTopkThreads) o[i] = i < lim ? i : -1;
    return;
  }
  const int64_t half = pair_half(lim), base = (int64_t)(peer ^ 1u) * half;
  const int64_t nloc = max((int64_t)0, min(lim - base, half));  // positions [base, base + nloc)
  const float* rowl = row + base;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // each CTA stores its counts of the first nbins bins into its peer's
  // hpeer[b], and one cluster barrier completes the stores.  The buffers
  // alternate by pass: the peer stores into hpeer[b] again two passes later,
  // after the barrier of the pass in between, which follows this CTA's last
  // read of it.
  auto merge = [&](int nbins, int b) {
    __syncthreads();  // this CTA's histogram is complete
    for (int i = threadIdx.x; i < nbins; i += kTopkThreads) st_dsmem(smem_u32(&hpeer[b][i]), peer, hist[i]);
    cluster_sync_all();
  };
  // The bin holding the `rem`-th largest counted key (bins taken from the
  // top): thread t owns nbins / 1024 bins and one block scan orders the
  // threads.  Leaves the bin and the count above it in sel[0], sel[1].
  auto select_bin = [&](int nbins, uint32_t rem, int b) {
    const uint32_t* hp = hpeer[b];
    const int per = nbins / kTopkThreads;
    const int hi = nbins - per * (int)threadIdx.x;
    uint32_t sum = 0;
    for (int bi = hi - 1; bi >= hi - per; --bi) sum += hist[bi] + hp[bi];
    uint32_t tot;
    const uint32_t ex = block_excl_scan(sum, warp_sums, &tot);
    if (ex < rem && ex + sum >= rem) {
      uint32_t above = ex;
      int bi = hi - 1;
      for (; bi > hi - per; --bi) {
        if (above + hist[bi] + hp[bi] >= rem) break;
        above += hist[bi] + hp[bi];
      }
      sel[0] = (uint32_t)bi;
      sel[1] = above;
    }
    __syncthreads();
  };
  // ---- this CTA's positions into shared memory (16-byte cp.async copies,
  // all of a thread's in flight at once; unaligned rows and the ragged tail
  // element by element), converted to keys in place while the first pass's
  // histogram (top 11 bits) is counted
  for (int i = threadIdx.x; i < 2048; i += kTopkThreads) hist[i] = 0;
  __syncthreads();
  const int64_t n4 = (reinterpret_cast<uintptr_t>(rowl) & 15u) == 0 ? nloc >> 2 : 0;
  for (int64_t i = threadIdx.x; i < n4; i += kTopkThreads)
    cp_async16(smem_u32(&skeys[4 * i]), rowl + 4 * i, 16);
  cp_async_commit();
  for (int64_t i = 4 * n4 + threadIdx.x; i < nloc; i += kTopkThreads) {
    const uint32_t key = sortable_key(rowl[i]);
    skeys[i] = key;
    atomicAdd(&hist[key >> 21], 1u);
  }
  cp_async_wait<0>();
  __syncthreads();
  for (int64_t i = threadIdx.x; i < n4; i += kTopkThreads) {
    uint4 v = reinterpret_cast<const uint4*>(skeys)[i];
    v = make_uint4(sortable_key(__uint_as_float(v.x)), sortable_key(__uint_as_float(v.y)),
                   sortable_key(__uint_as_float(v.z)), sortable_key(__uint_as_float(v.w)));
    reinterpret_cast<uint4*>(skeys)[i] = v;
    atomicAdd(&hist[v.x >> 21], 1u);
    atomicAdd(&hist[v.y >> 21], 1u);
    atomicAdd(&hist[v.z >> 21], 1u);
    atomicAdd(&hist[v.w >> 21], 1u);
  }
  merge(2048, 0);
  uint32_t remaining = (uint32_t)k;
  select_bin(2048, remaining, 0);
  const uint32_t bin0 = sel[0];
  const bool fits = hist[bin0] <= (uint32_t)kCand;  // this CTA's keys of the bin fit the list
  uint32_t prefix = bin0 << 21, pmask = 0x7FFu << 21;
  remaining -= sel[1];
  // ---- the write pass's mapping: warp w owns local positions [wspan w,
  // wspan (w + 1)) in groups of 128, lane l positions 4 l .. 4 l + 3 of a
  // group (one 16-byte shared-memory load).  Per warp: the keys above the
  // bin and in it; then the bin's positions into the candidates at the
  // warp's offset (a block scan, no atomics)
  const int G4 = (int)((nloc + 4095) / 4096);  // groups per warp, <= 12
  const int wspan = 128 * G4;
  const int wb = warp * wspan;
  const int nl = (int)nloc;
  // group gi's four keys of this lane and how many of them are positions < nloc
  auto load4 = [&](int gi, uint32_t (&kk)[4]) -> int {
    const int p0 = wb + 128 * gi + 4 * lane;
    if (p0 >= nl) {
      kk[0] = kk[1] = kk[2] = kk[3] = 0u;
      return 0;
    }
    const uint4 v = *reinterpret_cast<const uint4*>(&skeys[p0]);  // p0 + 4 <= the CTA's share
    kk[0] = v.x;
    kk[1] = v.y;
    kk[2] = v.z;
    kk[3] = v.w;
    return min(4, nl - p0);
  };
  // exclusive prefix over the warp's lanes, and the warp's total
  auto warp_excl = [&](uint32_t v, uint32_t& total) -> uint32_t {
    uint32_t x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, off);
      if (lane >= off) x += y;
    }
    total = __shfl_sync(0xFFFFFFFFu, x, 31);
    return x - v;
  };
  {
    uint32_t ga = 0, gb = 0;
    for (int gi = 0; gi < G4; ++gi) {
      uint32_t kk[4];
      const int nv = load4(gi, kk);
      uint32_t ca = 0, cb = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t top = kk[q] >> 21;
        ca += (q < nv && top > bin0) ? 1u : 0u;
        cb += (q < nv && top == bin0) ? 1u : 0u;
      }
      ga += __reduce_add_sync(0xFFFFFFFFu, ca);
      gb += __reduce_add_sync(0xFFFFFFFFu, cb);
    }
    if (lane == 0) gabove[warp] = ga;
    if (fits) {
      uint32_t tot;
      uint32_t cbase = block_excl_scan(lane == 0 ? gb : 0u, warp_sums, &tot);
      cbase = __shfl_sync(0xFFFFFFFFu, cbase, 0);
      if (threadIdx.x == 0) ncand = tot;
      for (int gi = 0; gi < G4; ++gi) {
        uint32_t kk[4];
        const int nv = load4(gi, kk);
        uint32_t m = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) m |= (q < nv && (kk[q] >> 21) == bin0) ? 1u << q : 0u;
        uint32_t wt;
        uint32_t at = cbase + warp_excl((uint32_t)__popc(m), wt);
        const uint32_t p0 = (uint32_t)(wb + 128 * gi + 4 * lane);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if ((m >> q) & 1u) cand[at++] = p0 + q;
        cbase += wt;
      }
    }
  }
  __syncthreads();
  // ---- the two refining passes over the bin's keys (or, when this CTA's did
  // not fit, over its whole half)
  const int nc = fits ? (int)ncand : 0;
#pragma unroll 1
  for (int pass = 1; pass < 3; ++pass) {
    const int shift = pass == 1 ? 10 : 0;
    const int nbins = pass == 2 ? 1024 : 2048;
    for (int i = threadIdx.x; i < nbins; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    if (fits) {
      for (int c = threadIdx.x; c < nc; c += kTopkThreads) {
        const uint32_t key = skeys[cand[c]];
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & (nbins - 1)], 1u);
      }
    } else {
      for (int64_t i = threadIdx.x; i < nloc; i += kTopkThreads) {
        const uint32_t key = skeys[i];
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & (nbins - 1)], 1u);
      }
    }
    merge(nbins, pass & 1);
    select_bin(nbins, remaining, pass & 1);
    prefix |= sel[0] << shift;
    pmask |= (uint32_t)(nbins - 1) << shift;
    remaining -= sel[1];
    __syncthreads();  // sel and hist are rewritten by the next pass
  }
  // ---- per warp range, keys above the k-th key and keys equal to it: the
  // bin's share from the candidates, or a counting pass over the half
  if (threadIdx.x < 32) {
    cgt[threadIdx.x] = 0;
    ceq[threadIdx.x] = 0;
  }
  __syncthreads();
  if (fits) {
    for (int c = threadIdx.x; c < nc; c += kTopkThreads) {
      const uint32_t pos = cand[c], key = skeys[pos];
      const int ww = (int)pos / wspan;
      if (key > prefix) atomicAdd(&cgt[ww], 1u);
      else if (key == prefix) atomicAdd(&ceq[ww], 1u);
    }
  } else {
    uint32_t cg = 0, ce = 0;
    for (int gi = 0; gi < G4; ++gi) {
      uint32_t kk[4];
      const int nv = load4(gi, kk);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        cg += (q < nv && kk[q] > prefix && (kk[q] >> 21) == bin0) ? 1u : 0u;
        ce += (q < nv && kk[q] == prefix) ? 1u : 0u;
      }
    }
    cg = __reduce_add_sync(0xFFFFFFFFu, cg);
    ce = __reduce_add_sync(0xFFFFFFFFu, ce);
    if (lane == 0) {
      cgt[warp] = cg;
      ceq[warp] = ce;
    }
  }
  __syncthreads();
  // ---- CTA 1's output starts after CTA 0's: CTA 0 stores its totals into
  // CTA 1's shared memory, and one cluster barrier (release / acquire)
  // completes the stores before CTA 1 reads them or CTA 0 exits
  if (warp == 0 && peer == 1) {
    uint32_t tg = gabove[lane] + cgt[lane], te = ceq[lane];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      tg += __shfl_xor_sync(0xFFFFFFFFu, tg, off);
      te += __shfl_xor_sync(0xFFFFFFFFu, te, off);
    }
    if (lane == 0) {
      st_dsmem(smem_u32(&tot_ge[0]), 1, tg);
      st_dsmem(smem_u32(&tot_ge[1]), 1, te);
    }
  }
  cluster_sync_all();
  const uint32_t base_g = peer == 0 ? tot_ge[0] : 0u, base_e = peer == 0 ? tot_ge[1] : 0u;
  // ---- write: ascending positions above the k-th key and the first
  // `remaining` equal to it (lim > k: exactly k in all).  This CTA's counts
  // are below 2^16 (<= 46 K positions), so one packed scan orders the warps.
  {
    const uint32_t cg = gabove[warp] + cgt[warp], ce = ceq[warp];
    uint32_t tot;
    const uint32_t ex = block_excl_scan(lane == 0 ? ((cg << 16) | ce) : 0u, warp_sums, &tot);
    const uint32_t exw = __shfl_sync(0xFFFFFFFFu, ex, 0);
    uint32_t g = base_g + (exw >> 16), e = base_e + (exw & 0xFFFFu);
    for (int gi = 0; gi < G4; ++gi) {
      uint32_t kk[4];
      const int nv = load4(gi, kk);
      uint32_t mg = 0, me = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        mg |= (q < nv && kk[q] > prefix) ? 1u << q : 0u;
        me |= (q < nv && kk[q] == prefix) ? 1u << q : 0u;
      }
      // lanes in order, then a lane's four positions in order (counts of a
      // group are at most 128, so the two counts share one scan)
      uint32_t wt;
      const uint32_t ex4 = warp_excl(((uint32_t)__popc(mg) << 16) | (uint32_t)__popc(me), wt);
      uint32_t gg = g + (ex4 >> 16), ee = e + (ex4 & 0xFFFFu);
      const int64_t p0 = base + wb + 128 * gi + 4 * lane;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if ((mg >> q) & 1u) {
          o[gg + min(ee, remaining)] = (int32_t)(p0 + q);
          ++gg;
        } else if ((me >> q) & 1u) {
          if (ee < remaining) o[gg + ee] = (int32_t)(p0 + q);
          ++ee;
        }
      }
      g += wt >> 16;
      e += wt & 0xFFFFu;
    }
  }
}

__global__ void __launch_bounds__(kTopkThreads)
    indexer_topk_kernel(const float* logits, int64_t logits_stride, int next_n, const int32_t* ctx,
                        int32_t* out, int64_t out_stride, int k, int64_t max_len) {
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sel[2];  // chosen bin, keys above it (this pass)
  __shared__ uint32_t cand[kCand];  // the first pass's chosen-bin keys
  __shared__ uint32_t ncand;
  if (threadIdx.x == 0) pdl_launch_dependents();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const int b = (int)(r / next_n), n = (int)(r % next_n);
  const int64_t lim = min(max_len, (int64_t)ctx[b] - next_n + n + 1);
  const float* row = logits + r * logits_stride;
  int32_t* o = out + r * out_stride;
  if (lim <= k) {  // every position kept, then padding
    for (int i = threadIdx.x; i < k; i += kTopkThreads) o[i] = i < lim ? i : -1;
    return;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  // every pass reads the row (from L2)
  auto key_at = [&](int64_t i) -> uint32_t { return sortable_key(row[i]); };
  // radix select of the k-th largest key: 11 + 11 + 10 bits.  After the first
  // pass the keys of the chosen bin (usually a few percent of the row) are
  // compacted, and the later passes count only them; a bin of more than
  // kCand keys keeps the full scans.
  uint32_t prefix = 0, pmask = 0, remaining = (uint32_t)k;
  bool use_cand = false;
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 21 : pass == 1 ? 10 : 0;
    const int nbins = pass == 2 ? 1024 : 2048;
    for (int i = threadIdx.x; i < nbins; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    if (use_cand) {
      for (int i = threadIdx.x; i < (int)ncand; i += kTopkThreads) {
        const uint32_t key = cand[i];
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & (nbins - 1)], 1u);
      }
    } else {
      for (int64_t i = threadIdx.x; i < lim; i += kTopkThreads) {
        const uint32_t key = key_at(i);
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & (nbins - 1)], 1u);
      }
    }
    __syncthreads();
    // the bin holding the remaining-th largest key: thread t owns `per` bins,
    // taken from the top, and one block scan orders the threads
    {
      const int per = nbins / kTopkThreads;
      const int hi = nbins - per * (int)threadIdx.x;
      uint32_t sum = 0;
      for (int bi = hi - 1; bi >= hi - per; --bi) sum += hist[bi];
      uint32_t tot;
      const uint32_t ex = block_excl_scan(sum, warp_sums, &tot);
      if (ex < remaining && ex + sum >= remaining) {
        uint32_t above = ex;
        int bi = hi - 1;
        for (; bi > hi - per; --bi) {
          if (above + hist[bi] >= remaining) break;
          above += hist[bi];
        }
        sel[0] = (uint32_t)bi;
        sel[1] = above;
      }
    }
    __syncthreads();
    const uint32_t bin = sel[0];
    prefix |= bin << shift;
    pmask |= (uint32_t)(nbins - 1) << shift;
    remaining -= sel[1];
    if (pass == 0 && hist[bin] <= (uint32_t)kCand) {
      // compact the chosen bin's keys (warp-aggregated appends)
      if (threadIdx.x == 0) ncand = 0;
      __syncthreads();
      const int lane = threadIdx.x & 31;
      const int64_t nr = (lim + 31) & ~(int64_t)31;
      for (int64_t i = threadIdx.x; i < nr; i += kTopkThreads) {
        const uint32_t key = i < lim ? key_at(i) : 0u;
        const bool m = i < lim && (key & pmask) == prefix;
        const uint32_t bal = __ballot_sync(0xFFFFFFFFu, m);
        uint32_t base = 0;
        if (lane == 0 && bal != 0) base = atomicAdd(&ncand, (uint32_t)__popc(bal));
        base = __shfl_sync(0xFFFFFFFFu, base, 0);
        if (m) cand[base + __popc(bal & ((1u << lane) - 1u))] = key;
      }
      use_cand = true;
    }
    __syncthreads();  // sel, hist and the candidates are read by the next pass
  }
  // prefix is the k-th largest key; `remaining` of the keys equal to it are
  // kept (the lowest positions), every key above it too.  Warp w takes
  // positions [1024 w, 1024 w + 1024) of each round, lane l position 32 j + l
  // at step j (coalesced reads); ballots order the lanes, one block scan the
  // warps.
  uint32_t base_g = 0, base_e = 0;
  for (int64_t start = 0; start < lim; start += kRound) {
    const int64_t wb = start + (int64_t)warp * 1024;
    uint32_t cg = 0, ce = 0;
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
      const int64_t i = wb + 32 * j + lane;
      const uint32_t key = i < lim ? key_at(i) : 0u;
      cg += __popc(__ballot_sync(0xFFFFFFFFu, i < lim && key > prefix));
      ce += __popc(__ballot_sync(0xFFFFFFFFu, i < lim && key == prefix));
    }
    uint32_t tot;
    const uint32_t ex = block_excl_scan(lane == 0 ? ((cg << 16) | ce) : 0u, warp_sums, &tot);
    const uint32_t exw = __shfl_sync(0xFFFFFFFFu, ex, 0);
    uint32_t g = base_g + (exw >> 16), e = base_e + (exw & 0xFFFFu);
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
      const int64_t i = wb + 32 * j + lane;
      const uint32_t key = i < lim ? key_at(i) : 0u;
      const bool isg = i < lim && key > prefix, ise = i < lim && key == prefix;
      const uint32_t bg = __ballot_sync(0xFFFFFFFFu, isg), be = __ballot_sync(0xFFFFFFFFu, ise);
      const uint32_t gb = g + __popc(bg & lt), eb = e + __popc(be & lt);
      if (isg) o[gb + min(eb, remaining)] = (int32_t)i;
      else if (ise && eb < remaining) o[gb + eb] = (int32_t)i;
      g += __popc(bg);
      e += __popc(be);
    }
    base_g += tot >> 16;
    base_e += tot & 0xFFFFu;
  }
}

}  // namespace idx

// ------------------------------------------------------------------ host
int read_device_status_idx(unsigned int* status, bool reset, cudaStream_t st) {
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

int launch_indexer_logits(const uint8_t* q, int64_t B, int64_t next_n, int64_t q_stride_b,
                          const uint8_t* k_cache, int64_t num_blocks, const float* w,
                          int64_t w_stride, const int32_t* ctx, const int32_t* bt, int64_t bt_stride,
                          int64_t max_blocks, float* logits, int64_t logits_stride,
                          int64_t max_len, int sms, cudaStream_t st) {
  CUtensorMap tm;
  if (int rc = encode_indexer_page_map(&tm, k_cache, num_blocks, idx::kBlock, idx::kDim)) return rc;
  idx::Args a{};
  a.q = q;
  a.q_stride_b = q_stride_b;
  a.k_cache = k_cache;
  a.num_blocks = num_blocks;
  a.w = w;
  a.w_stride = w_stride;
  a.ctx = ctx;
  a.bt = bt;
  a.bt_stride = bt_stride;
  a.max_blocks = max_blocks;
  a.logits = logits;
  a.logits_stride = logits_stride;
  a.max_len = max_len;
  a.next_n = (int)next_n;
  // items of 8 tiles (1024 tokens), fewer when the batch would leave CTA
  // slots idle (two CTAs fit an SM); a persistent grid of at most two CTAs per
  // SM walks them
  const int64_t total_tiles = (max_len + idx::kTileTokens - 1) / idx::kTileTokens;
  int64_t tpi = 8;
  while (tpi > 2 && B * ((total_tiles + tpi - 1) / tpi) < 2 * (int64_t)sms) tpi >>= 1;
  a.tiles_per_item = (int)tpi;
  a.chunks_per_req = (int)((total_tiles + tpi - 1) / tpi);
  const int64_t items = B * (int64_t)a.chunks_per_req;
  if (items > INT32_MAX) return set_error(FP8MLA_ERR_INVALID_ARGUMENT, "too many indexer work items");
  a.items = (int)items;
  if (a.items == 0) return FP8MLA_OK;
  const dim3 grid((unsigned)std::min<int64_t>(items, 2 * (int64_t)sms));
  auto launch = [&](auto kern, size_t smem) -> int {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "indexer logits smem attribute");
    return check_cuda(launch_pdl(kern, grid, dim3(idx::kThreads), smem, st, a, tm),
                      "indexer_logits_kernel launch");
  };
  if (next_n == 1) return launch(idx::indexer_logits_kernel<1>, sizeof(idx::Smem<1>) + 1024);
  return launch(idx::indexer_logits_kernel<2>, sizeof(idx::Smem<2>) + 1024);
}

int launch_indexer_topk(const float* logits, int64_t rows, int64_t logits_stride, int64_t next_n,
                        const int32_t* ctx, int32_t* out, int64_t out_stride, int64_t topk,
                        int64_t max_len, cudaStream_t st) {
  if (max_len <= idx::kPairMaxLen) {
    const size_t smem = (size_t)idx::pair_half(max_len) * sizeof(uint32_t);
    cudaError_t e = cudaFuncSetAttribute(idx::indexer_topk_pair_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(idx::kSmemKeys * sizeof(uint32_t)));
    if (e != cudaSuccess) return check_cuda(e, "indexer top-k smem attribute");
    return check_cuda(launch_pdl(idx::indexer_topk_pair_kernel, dim3((unsigned)(2 * rows)),
                                 dim3(idx::kTopkThreads), smem, st, logits, logits_stride,
                                 (int)next_n, ctx, out, out_stride, (int)topk, max_len),
                      "indexer_topk_pair_kernel launch");
  }
  return check_cuda(launch_pdl(idx::indexer_topk_kernel, dim3((unsigned)rows),
                               dim3(idx::kTopkThreads), 0, st, logits, logits_stride, (int)next_n,
                               ctx, out, out_stride, (int)topk, max_len),
                    "indexer_topk_kernel launch");
}

}  // namespace fp8mla
