// tc_mma_rates.cu -- microbenchmark: throughput of straight-line tcgen05.mma kind::f16 (bf16 in,
// fp32 accumulate, M=128, K=16 per instruction) on one SM, by N and by A source (shared memory
// descriptor vs tensor memory).  One CTA, thread 0 issues 16 fully unrolled MMAs per iteration
// into one accumulator; the clock covers first issue to the commit's mbarrier arrival.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -o tc_mma_rates tc_mma_rates.cu
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cuda_runtime.h>
#include "../common.cuh"
#include "../tc_ptx.cuh"
using namespace fp8mla;
using namespace fp8mla::tc;

constexpr int kBlk = 16384;  // one 128-row x 128-byte swizzled block
struct __align__(1024) Smem {
  uint8_t buf[12 * kBlk];    // A: blocks 0-3; B: from block 4, up to 256 rows per block step
  uint64_t bar;
  uint32_t tmem;
};

template <int N, bool TS>
__global__ void __launch_bounds__(128, 1) mma_rate(int iters, long long* out) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const uint32_t base = smem_u32(sm);
  Smem& s = *reinterpret_cast<Smem*>(sm + (((base + 1023u) & ~1023u) - base));
  for (int i = threadIdx.x; i < (int)sizeof(s.buf) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(s.buf)[i] = make_uint4(0x3C003C00u, 0, 0x3C003C00u, 0);
  const uint32_t bar = smem_u32(&s.bar);
  if (threadIdx.x == 0) { mbar_init(bar, 1); mbar_init_fence(); }
  if (threadIdx.x < 32) { tmem_alloc(smem_u32(&s.tmem), 512); tmem_relinquish(); }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = idesc_bf16(128, N, false);
    const uint32_t sa = smem_u32(s.buf);
    const uint64_t a0 = sdesc_sw128(sa, 16, 1024), b0 = sdesc_sw128(sa + 4 * kBlk, 16, 1024);
    const uint32_t tA = tmem + 448;  // A operand columns of the TMEM-A form (8 per k-step)
    long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint64_t bd = b0 + (uint64_t)((((k >> 2) * kBlk) + (k & 3) * 32) >> 4);
        if (TS)
          mma_ts(tmem, tA + 8 * (k & 7), bd, idesc, 1u);
        else
          mma_ss(tmem, a0 + (uint64_t)((((k >> 2) * kBlk) + (k & 3) * 32) >> 4), bd, idesc, 1u);
      }
    }
    mma_commit(bar);
    const bool ok = thread_wait(bar, 0, 1);
    out[0] = ok ? clock64() - t0 : -1;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) { tc_fence_after(); tmem_dealloc(tmem, 512); }
}

template <int N, bool TS>
void run(long long* d) {
  const int smem = sizeof(Smem) + 1024, iters = 64;
  cudaFuncSetAttribute(mma_rate<N, TS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  mma_rate<N, TS><<<1, 128, smem>>>(2, d);
  mma_rate<N, TS><<<1, 128, smem>>>(iters, d);
  cudaError_t e = cudaDeviceSynchronize();
  long long clk = 0;
  cudaMemcpy(&clk, d, sizeof(clk), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); exit(1); }
  const double n = 16.0 * iters;
  printf("N=%3d A=%s | %6.1f cycles/MMA  %6.0f MACs/cycle/SM\n", N, TS ? "tmem" : "smem", clk / n,
         n * 128.0 * N * 16 / clk);
}

int main() {
  long long* d;
  cudaMalloc(&d, sizeof(long long));
  run<32, false>(d);  run<32, true>(d);
  run<64, false>(d);  run<64, true>(d);
  run<128, false>(d); run<128, true>(d);
  run<256, false>(d); run<256, true>(d);
  return 0;
}
