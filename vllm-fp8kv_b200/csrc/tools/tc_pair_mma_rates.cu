// tc_pair_mma_rates.cu -- microbenchmark for the paired (cta_group::2) tcgen05.mma the decode uses:
// (1) the accumulator layout of an M=128 MMA over a 2-CTA cluster, checked value by value
//     (D[m][n] = (m+1) + 256 n, read back from both CTAs' tensor memory), and
// (2) the throughput of straight-line pair MMAs (kind::f16, bf16 in, fp32 accumulate, K=16) by N
//     and by A source; the even CTA's thread 0 issues 16 unrolled MMAs per iteration.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -o tc_pair_mma_rates tc_pair_mma_rates.cu
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cuda_runtime.h>
#include "../common.cuh"
#include "../tc_ptx.cuh"
#include "../tc_cluster.cuh"
using namespace fp8mla;
using namespace fp8mla::tc;

constexpr int kBlk = 16384;
struct __align__(1024) Smem {
  uint8_t buf[12 * kBlk];
  uint64_t bar;
  uint32_t tmem;
};
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }
__device__ __forceinline__ void put_bf16(uint8_t* blk, int row, int k, float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  *reinterpret_cast<__nv_bfloat16*>(blk + swz(row, k >> 3) + (k & 7) * 2) = b;
}

// ---- layout: D[m][n] = (m + 1) + 256 n for global row m, column n
template <int N>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1) layout_k(float* out) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t base = smem_u32(sm);
  Smem& s = *reinterpret_cast<Smem*>(sm + (((base + 1023u) & ~1023u) - base));
  const uint32_t r = cluster_rank();
  for (int i = threadIdx.x; i < 2 * kBlk / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(s.buf)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  uint8_t* A = s.buf;            // 64 rows
  uint8_t* B = s.buf + kBlk;     // N/2 rows
  if (threadIdx.x < 64) {
    put_bf16(A, threadIdx.x, 0, (float)(64 * r + threadIdx.x + 1));
    put_bf16(A, threadIdx.x, 1, 256.f);
  }
  if (threadIdx.x < N / 2) {
    put_bf16(B, threadIdx.x, 0, 1.f);
    put_bf16(B, threadIdx.x, 1, (float)(r * (N / 2) + threadIdx.x));
  }
  const uint32_t bar = smem_u32(&s.bar);
  if (threadIdx.x == 0) { mbar_init(bar, 1); mbar_init_fence(); }
  if (threadIdx.x < 32) { tmem_alloc_pair(smem_u32(&s.tmem), 256); tmem_relinquish_pair(); }
  fence_proxy_async_smem();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  if (r == 0 && threadIdx.x == 0) {
    const uint32_t sa = smem_u32(s.buf);
    mma_pair_ss(tmem, sdesc_sw128(sa, 16, 1024), sdesc_sw128(sa + kBlk, 16, 1024), idesc_bf16(128, N, false), 0u);
    mma_commit_pair(bar);
  }
  const bool ok = warp_wait_cluster(bar, 0, 1);
  tc_fence_after();
  const int w = threadIdx.x >> 5;
  for (int c0 = 0; c0 < N / 2; c0 += 32) {
    uint32_t v[32];
    tmem_ld32(tmem + ((uint32_t)(32 * w) << 16) + c0, v);
    tmem_wait_ld();
    for (int i = 0; i < 32; ++i)
      out[((size_t)r * 128 + threadIdx.x) * 128 + c0 + i] = ok ? __uint_as_float(v[i]) : -1.f;
  }
  tc_fence_before();
  cluster_sync_all();
  if (threadIdx.x < 32) { tc_fence_after(); tmem_dealloc_pair(tmem, 256); }
}

// ---- rates: the leader issues 16 unrolled MMAs per iteration into one accumulator
template <int N, bool TS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1) rate_k(int iters, long long* out) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t base = smem_u32(sm);
  Smem& s = *reinterpret_cast<Smem*>(sm + (((base + 1023u) & ~1023u) - base));
  const uint32_t r = cluster_rank();
  for (int i = threadIdx.x; i < (int)sizeof(s.buf) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(s.buf)[i] = make_uint4(0x3C003C00u, 0, 0x3C003C00u, 0);
  const uint32_t bar = smem_u32(&s.bar);
  if (threadIdx.x == 0) { mbar_init(bar, 1); mbar_init_fence(); }
  if (threadIdx.x < 32) { tmem_alloc_pair(smem_u32(&s.tmem), 512); tmem_relinquish_pair(); }
  fence_proxy_async_smem();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  long long t0 = clock64();
  if (r == 0 && threadIdx.x == 0) {
    constexpr uint32_t idesc = idesc_bf16(128, N, false);
    const uint32_t sa = smem_u32(s.buf);
    const uint64_t a0 = sdesc_sw128(sa, 16, 1024), b0 = sdesc_sw128(sa + 4 * kBlk, 16, 1024);
    const uint32_t tA = tmem + 448;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint64_t bd = b0 + (uint64_t)((((k >> 2) * kBlk) + (k & 3) * 32) >> 4);
        if (TS) mma_pair_ts(tmem, tA + 8 * (k & 7), bd, idesc, 1u);
        else mma_pair_ss(tmem, a0 + (uint64_t)((((k >> 2) * kBlk) + (k & 3) * 32) >> 4), bd, idesc, 1u);
      }
    }
    mma_commit_pair(bar);
  }
  if (threadIdx.x == 0) {
    const bool ok = thread_wait_cluster(bar, 0, 1);
    out[r] = ok ? clock64() - t0 : -1;
  }
  tc_fence_before();
  cluster_sync_all();
  if (threadIdx.x < 32) { tc_fence_after(); tmem_dealloc_pair(tmem, 512); }
}

template <int N>
int layout(float* d) {
  const int smem = sizeof(Smem) + 1024;
  cudaFuncSetAttribute(layout_k<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaMemset(d, 0, 2 * 128 * 128 * 4);
  layout_k<N><<<2, 128, smem>>>(d);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) { printf("layout N=%d error %s\n", N, cudaGetErrorString(e)); exit(1); }
  static float h[2 * 128 * 128];
  cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  int bad = 0, shown = 0;
  for (int r = 0; r < 2; ++r)
    for (int L = 0; L < 128; ++L)
      for (int c = 0; c < N / 2; ++c) {
        const float v = h[((size_t)r * 128 + L) * 128 + c];
        // expected by the "2x2" layout: lanes [0,64) hold columns [0,N/2), lanes [64,128) [N/2,N)
        const int m = 64 * r + (L & 63), n = c + (L >= 64 ? N / 2 : 0);
        const float want = (float)(m + 1) + 256.f * n;
        if (v != want) {
          ++bad;
          if (shown < 6) {
            const int iv = (int)v;
            printf("  N=%d cta %d lane %3d col %3d: got %.0f (m=%d n=%d) want m=%d n=%d\n", N, r, L, c, v,
                   (iv & 255) - 1, iv >> 8, m, n);
            ++shown;
          }
        }
      }
  printf("layout N=%3d: %s (%d mismatches of %d)\n", N, bad ? "DIFFERS" : "2x2 as expected", bad, 2 * 128 * N / 2);
  return bad;
}

template <int N, bool TS>
void rate(long long* d) {
  const int smem = sizeof(Smem) + 1024, iters = 64;
  cudaFuncSetAttribute(rate_k<N, TS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  rate_k<N, TS><<<2, 128, smem>>>(2, d);
  rate_k<N, TS><<<2, 128, smem>>>(iters, d);
  cudaError_t e = cudaDeviceSynchronize();
  long long clk[2];
  cudaMemcpy(clk, d, sizeof(clk), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) { printf("rate error %s\n", cudaGetErrorString(e)); exit(1); }
  const double n = 16.0 * iters;
  printf("2SM M=128 N=%3d A=%s | %6.1f cycles/MMA (peer %6.1f)  %6.0f MACs/cycle per SM\n", N, TS ? "tmem" : "smem",
         clk[0] / n, clk[1] / n, n * 64.0 * N * 16 / clk[0]);
}

int main() {
  float* f; long long* d;
  cudaMalloc(&f, 2 * 128 * 128 * 4);
  cudaMalloc(&d, 16);
  int bad = layout<64>(f) + layout<128>(f) + layout<256>(f);
  rate<32, false>(d); rate<32, true>(d);
  rate<64, false>(d); rate<64, true>(d);
  rate<128, false>(d); rate<128, true>(d);
  rate<256, false>(d); rate<256, true>(d);
  return bad ? 2 : 0;
}
