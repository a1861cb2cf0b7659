"""B200-native (sm_100a) fp8_ds_mla sparse-MLA decode, a drop-in for the
reference package of the same name (nickus/vllm-fp8kv).

Modules keep the reference's names and entry points:
  fp8_ds_mla_sparse_decode  -- decode entry point + format constants
  fp8_dequant               -- e4m3fn decode (torch reference + device kernel)
  backend_patch             -- vLLM TRITON_MLA_SPARSE wiring
  cache_writer              -- fp8_ds_mla cache writer (vLLM's concat_and_cache_mla)
  index_convert             -- block-table -> flat slot conversion
All device work runs in libfp8mla.so (hand-written CUDA for sm_100a) through
its C ABI (include/fp8mla.h); there is no Triton and no CPU fallback.
"""
