// tc_mma_rates.cu -- microbenchmark: tcgen05.mma kind::f16 throughput vs N, number of independent
// accumulator chains, and A source (smem vs tmem).  One CTA, thread 0 issues.
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "../common.cuh"
#include "../tc_ptx.cuh"
using namespace fp8mla;
using namespace fp8mla::tc;

struct __align__(1024) SmemB {
  uint8_t a[128 * 128];     // A: 128 rows x 128 B (one 64-dim K block), SW128
  uint8_t b[256 * 128];     // B: 256 rows x 128 B, SW128
  uint64_t bar;
  uint32_t tmem;
};

__global__ void __launch_bounds__(128, 1) mma_bench(int N, int chains, int ts, int iters,
                                                    long long* out_clk) {
  // out_clk[0] = SM cycles, out_clk[1] = nanoseconds (globaltimer) for the same interval
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t base = smem_u32(sm);
  const uint32_t pad = ((base + 1023u) & ~1023u) - base;
  SmemB& s = *reinterpret_cast<SmemB*>(sm + pad);
  for (int i = threadIdx.x; i < (int)sizeof(s.a) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(s.a)[i] = make_uint4(0, 0, 0, 0);
  for (int i = threadIdx.x; i < (int)sizeof(s.b) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(s.b)[i] = make_uint4(0, 0, 0, 0);
  const uint32_t bar = smem_u32(&s.bar);
  if (threadIdx.x == 0) { mbar_init(bar, 1); mbar_init_fence(); }
  if (threadIdx.x < 32) { tmem_alloc(smem_u32(&s.tmem), 512); tmem_relinquish(); }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_bf16(128, N, false);
    const uint32_t sa = smem_u32(s.a), sb = smem_u32(s.b);
    uint64_t ad[4], bd[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ad[k] = sdesc_sw128(sa + k * 32, 16, 1024);
      bd[k] = sdesc_sw128(sb + k * 32, 16, 1024);
    }
    uint32_t dcol[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) dcol[c] = tmem + c * N;
    const uint32_t acol = tmem + 448;
    uint64_t g0, g1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));
    long long t0 = clock64();
    if (ts) {
      for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (c < chains) mma_ts(dcol[c], acol, bd[k], idesc, 1u);
      }
    } else {
      for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (c < chains) mma_ss(dcol[c], ad[k], bd[k], idesc, 1u);
      }
    }
    mma_commit(bar);
    bool ok = thread_wait(bar, 0, 1);
    long long t1 = clock64();
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g1));
    out_clk[0] = ok ? (t1 - t0) : -1;
    out_clk[1] = (long long)(g1 - g0);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) { tc_fence_after(); tmem_dealloc(tmem, 512); }
}

int main() {
  long long* d_clk;
  cudaMalloc(&d_clk, 2 * sizeof(long long));
  const int smem = sizeof(SmemB) + 1024;
  cudaFuncSetAttribute(mma_bench, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int iters = 256;
  printf("N chains ts | clk/MMA  MACs/clk  ns/MMA  SM-MHz\n");
  int cfg[][2] = {{32, 1}, {32, 2}, {32, 4}, {32, 6}, {32, 8}, {64, 1}, {64, 2}, {64, 4},
                  {64, 6}, {128, 1}, {128, 2}, {128, 3}, {256, 1}};
  for (int ts = 0; ts < 2; ++ts)
    for (auto& c : cfg) {
      int N = c[0], ch = c[1];
      mma_bench<<<1, 128, smem>>>(N, ch, ts, 4, d_clk);  // warm
      mma_bench<<<1, 128, smem>>>(N, ch, ts, iters, d_clk);
      cudaError_t e = cudaDeviceSynchronize();
      long long r[2] = {0, 0};
      cudaMemcpy(r, d_clk, sizeof(r), cudaMemcpyDeviceToHost);
      const long long clk = r[0];
      if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); return 1; }
      const double n_mma = (double)iters * 4 * ch;
      const double macs = n_mma * 128.0 * N * 16;
      printf("%3d %d %d | %8.1f  %8.0f  %6.1f  %6.0f\n", N, ch, ts, clk / n_mma, macs / clk,
             r[1] / n_mma, 1e3 * clk / (double)r[1]);
    }
  return 0;
}
