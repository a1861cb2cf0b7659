// abi_noalloc.cu -- a decode entry point that never allocates device memory.
//
// fp8mla_sparse_decode expects the caller to pass the split-KV workspace.  Some
// callers cannot produce one: an inference engine that sizes its KV cache from
// whatever memory is left after a profiling pass cannot let a library call
// cudaMalloc later (the allocation lands outside its plan and can push it out
// of memory), and a foreign-language host that only holds raw device pointers
// may have no allocator binding at all.  This variant takes its workspace
// from a fixed array in the library's own device memory instead.
//
// The array is a file-scope __device__ object of kNoAllocScratchBytes bytes;
// every GPU that loads this library holds it until the process exits.  Its
// device address is looked up once per device (cudaGetSymbolAddress, with that
// device current) on the first call made on that device; make that first call
// before starting any stream capture.  All calls on a device share the one
// array and it keeps the previous call's contents: calls that may overlap on
// the GPU (different streams, or other threads) race on it and must be
// serialised by the caller.  The split kernels overwrite every workspace entry
// the merge reads, so nothing has to be cleared between calls.
#include <stdio.h>

#include <mutex>

#include "common.cuh"
#include "decode.h"

namespace fp8mla {
namespace {

constexpr int64_t kNoAllocScratchBytes = 32ll << 20;  // 32 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::once_flag g_once[kMaxDevices];
void* g_ptr[kMaxDevices];
cudaError_t g_err[kMaxDevices];

// Device address of the scratch array on the current device (nullptr on failure).
void* scratch_for_current_device(int* dev_out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  *dev_out = dev;
  std::call_once(g_once[dev], [dev] {
    g_err[dev] = cudaGetSymbolAddress(&g_ptr[dev], g_noalloc_scratch);
    if (g_err[dev] != cudaSuccess) g_ptr[dev] = nullptr;
  });
  return g_ptr[dev];
}

}  // namespace
}  // namespace fp8mla

using namespace fp8mla;

extern "C" int fp8mla_sparse_decode_noalloc(
    const void* q, int q_dtype, int64_t T, int64_t H, int64_t q_stride_t, int64_t q_stride_h,
    const uint8_t* kv, int64_t num_slots, const int32_t* indices, int64_t G, int64_t topk,
    int64_t idx_stride_t, int64_t idx_stride_g, float sm_scale, void* out, int64_t out_stride_t,
    int64_t out_stride_h, float* lse, int64_t lse_stride_t, int num_splits, void* stream) {
  int dev = -1;
  void* scratch = scratch_for_current_device(&dev);
  if (scratch == nullptr)
    return set_error(FP8MLA_ERR_CUDA, "fp8mla_sparse_decode_noalloc: scratch lookup failed: %s",
                     dev >= 0 ? cudaGetErrorString(g_err[dev]) : "no current device");
  // The decode sizes the split workspace for the split count it actually
  // runs (after its clamps) and refuses a call that needs more than it is
  // given, before any launch; only the message is specific to this entry.
  const int rc = fp8mla_sparse_decode(q, q_dtype, T, H, q_stride_t, q_stride_h, kv, num_slots,
                                      indices, G, topk, idx_stride_t, idx_stride_g, sm_scale, out,
                                      out_stride_t, out_stride_h, lse, lse_stride_t, num_splits,
                                      scratch, kNoAllocScratchBytes, stream);
  if (rc == FP8MLA_ERR_WORKSPACE) {
    char why[400];
    snprintf(why, sizeof(why), "%s", fp8mla_last_error());
    return set_error(FP8MLA_ERR_WORKSPACE,
                     "fp8mla_sparse_decode_noalloc: the split workspace does not fit the fixed "
                     "%lld-byte scratch (%s); use fewer splits or fp8mla_sparse_decode with a "
                     "caller-provided workspace",
                     (long long)kNoAllocScratchBytes, why);
  }
  return rc;
}
