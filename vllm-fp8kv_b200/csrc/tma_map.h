// tma_map.h -- TMA tensor maps over the fp8_ds_mla pool and the indexer's
// paged key cache, and the gather4 copy.
//
// The pool is addressed as [num_slots] rows of 82 uint64 (656 bytes).  A map
// with a one-row box of `box_u64` words lets tile::gather4 fetch the same
// column range of four arbitrary rows in one instruction: the whole row
// (82 words), one 128-byte latent tile (16 words, x = 16 * tile) or the four
// fp32 tile scales (2 words, x = 64).  Row coordinates are int32, so a map
// needs num_slots < 2^31; the byte addressing inside the map is 64-bit.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace fp8mla {

// Encodes `tm` over the pool `kv` (16-byte aligned); returns FP8MLA_OK or an
// error code with the message recorded.
int encode_row_map(CUtensorMap* tm, const uint8_t* kv, int64_t num_slots, uint32_t box_u64);

// Encodes `tm` over the DSA indexer's paged key cache: blocks of block_size
// tokens, each block_size x head_dim e4m3 bytes followed by block_size fp32
// scales.  One box is one block's values (block_size rows of head_dim = 128
// bytes), landing 128-byte swizzled as a K-major tcgen05 operand.
int encode_indexer_page_map(CUtensorMap* tm, const uint8_t* k_cache, int64_t num_blocks,
                            int64_t block_size, int64_t head_dim);

#ifdef __CUDACC__
// Four rows r0..r3 of `tm` at column x (in uint64 words) -> 4 consecutive
// box-wide rows at shared address dst; completion counted on `bar`.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* tm, int32_t x,
                                            int32_t r0, int32_t r1, int32_t r2, int32_t r3,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];\n" ::"r"(dst),
      "l"(tm), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(bar)
      : "memory");
}
#endif

}  // namespace fp8mla
