// decode_tc.cu -- tcgen05/TMEM sparse MLA decode for 128 heads per kv group.
#include "common.cuh"
#include "decode.h"

namespace fp8mla {

bool decode_tc_supported(const DecodeArgs&) { return false; }

int launch_decode_tc(const DecodeArgs&, cudaStream_t) {
  return set_error(FP8MLA_ERR_UNSUPPORTED, "tcgen05 decode not built");
}

}  // namespace fp8mla
