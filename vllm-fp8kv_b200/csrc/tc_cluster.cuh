// tc_cluster.cuh -- 2-CTA cluster plumbing for the paired tcgen05 decode:
// cta_group::2 tensor-memory allocation, MMAs and commits, remote mbarrier
// arrivals, cluster-scope waits and the cluster barrier.  Nothing here loads
// with cluster multicast; the only multicast is the commit's arrival on both
// CTAs' barriers.
#pragma once
#include "tc_ptx.cuh"

namespace fp8mla {
namespace tc {

// Waits and remote arrivals use the default (CTA-scope) acquire / release,
// the forms CUTLASS's 2-SM kernels use between the CTAs of a pair.  A release
// at cluster scope first waits for every load the thread has in flight (about
// 4.5 K cycles with a tile of row loads outstanding, 320 with none, measured);
// the data it would order lives in the arriving CTA's own shared memory and
// is read by that SM's tensor core, after the writer's proxy fence.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.b32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool warp_wait_cluster(uint32_t bar, uint32_t parity, uint32_t where) {
  uint32_t ok = 0;
  if ((threadIdx.x & 31) == 0) {
    for (uint32_t it = 0; it < kMaxWaitIters; ++it) {
      if (mbar_try_wait_cluster(bar, parity)) {
        ok = 1;
        break;
      }
    }
    if (!ok) atomicOr(&g_device_status, kStatusWaitTimeout | (where << 8));
  }
  ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
  __syncwarp();
  return ok != 0;
}

__device__ __forceinline__ bool thread_wait_cluster(uint32_t bar, uint32_t parity,
                                                    uint32_t where) {
  for (uint32_t it = 0; it < kMaxWaitIters; ++it)
    if (mbar_try_wait_cluster(bar, parity)) return true;
  atomicOr(&g_device_status, kStatusWaitTimeout | (where << 8));
  return false;
}

// shared::cluster address of `local` (a shared::cta address) in CTA `rank`
__device__ __forceinline__ uint32_t mapa(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// arrive on a barrier in another CTA of the cluster
__device__ __forceinline__ void mbar_arrive_remote(uint32_t raddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];\n" ::"r"(raddr)
               : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" :::
                   "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// Arrive on the barrier at shared::cta offset `bar` of CTA `rank` (this CTA
// included).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar, uint32_t rank) {
  mbar_arrive_remote(mapa(bar, rank));
}

// ---- cta_group::2: one MMA over the tensor cores of both CTAs of the pair.
// Issued by the even CTA; shared-memory descriptors name the same offset in
// both CTAs (each supplies its half of A's rows and of B's N columns) and the
// tensor-memory address the same columns in both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void mma_pair_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_pair_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on the barrier at offset `bar` in both CTAs once every pair MMA this
// thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;\n" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
// Named barrier over `count` threads (id 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

}  // namespace tc
}  // namespace fp8mla
