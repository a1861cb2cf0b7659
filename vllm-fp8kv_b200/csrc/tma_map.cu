// tma_map.cu -- TMA tensor maps over the library's paged formats.  The
// driver's cuTensorMapEncodeTiled is looked up once through the runtime (no
// link-time dependency on libcuda).
#include "common.cuh"
#include "tma_map.h"

namespace fp8mla {
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

int encode_row_map(CUtensorMap* tm, const uint8_t* kv, int64_t num_slots, uint32_t box_u64) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return set_error(FP8MLA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {kRowBytes / 8, (cuuint64_t)num_slots};
  const cuuint64_t strides[1] = {kRowBytes};
  const cuuint32_t box[2] = {box_u64, 1};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(kv), dims, strides,
                         box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FP8MLA_ERR_CUDA, "tensor map encode failed (%d)", (int)r);
  return FP8MLA_OK;
}

int encode_indexer_page_map(CUtensorMap* tm, const uint8_t* k_cache, int64_t num_blocks,
                            int64_t block_size, int64_t head_dim) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return set_error(FP8MLA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  // [num_blocks][block_size][head_dim] bytes, a block `page` bytes apart (its
  // block_size fp32 scales follow the values); one box = one block's values,
  // written into shared memory with the 128-byte swizzle of a K-major operand
  const cuuint64_t page = (cuuint64_t)(block_size * (head_dim + 4));
  const cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)block_size, (cuuint64_t)num_blocks};
  const cuuint64_t strides[2] = {(cuuint64_t)head_dim, page};
  const cuuint32_t box[3] = {(cuuint32_t)head_dim, (cuuint32_t)block_size, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(k_cache), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FP8MLA_ERR_CUDA, "indexer page tensor map encode failed (%d)", (int)r);
  return FP8MLA_OK;
}

}  // namespace fp8mla
