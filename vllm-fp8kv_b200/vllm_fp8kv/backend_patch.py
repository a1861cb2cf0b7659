"""vLLM TRITON_MLA_SPARSE wiring for fp8_ds_mla KV, served by libfp8mla.

Behaviour matches the reference's backend_patch (vllm_fp8kv/backend_patch.py:50-206):

* ``_forward_fp8_kv``            -- decode over flat global slots; q may be a
                                    (nope, rope) tuple; heads sliced to the layer's count
* ``_forward_fp8_kv_paged``      -- the same decode over request-local top-k
                                    positions: the block-table conversion runs
                                    inside the decode's gather (one launch)
* ``_forward_mqa_fp8_aware``     -- replaces ``forward_mqa``: fp8_ds_mla goes to
                                    the fused sm_100a decode, everything else to
                                    upstream's bf16 path with upstream's converter
* ``_get_kv_cache_shape_fp8_aware`` -- 656-byte rows for fp8_ds_mla
* ``_patch_mla_spec_quant_mode`` -- the MLA KV-cache spec of an fp8_ds_mla pool
                                    declares itself quantized
* ``apply()``                    -- installs all of it into a live vLLM; idempotent
"""

import torch

from vllm_fp8kv.fp8_ds_mla_sparse_decode import (
    ROW_BYTES,
    fp8_ds_mla_sparse_decode,
    fp8_ds_mla_sparse_decode_paged,
)

FP8_DS_MLA = "fp8_ds_mla"
_CLI_FP8_NAMES = ("fp8", "fp8_e4m3")
_MARK = "_vllm_fp8kv_b200"
_CONVERT_BLOCK_N = 128  # entries per program of vLLM's index converter


def _as_single_q(q):
    return torch.cat(q, dim=-1) if isinstance(q, tuple) else q


def _forward_fp8_kv(self, q, kv_c_and_k_pe_cache, topk_indices, attn_metadata):
    """Decode over fp8_ds_mla pages; `topk_indices` are flat global slots (-1 masked)."""
    q = _as_single_q(q)
    n_tok = q.shape[0]
    out = fp8_ds_mla_sparse_decode(
        q, kv_c_and_k_pe_cache, topk_indices.view(n_tok, 1, -1), sm_scale=self.softmax_scale)
    return out[:, : self.num_heads, :]


def _forward_fp8_kv_paged(self, q, kv_c_and_k_pe_cache, topk_indices, attn_metadata):
    """Decode over fp8_ds_mla pages from request-local top-k positions.

    Same result as converting with ``triton_convert_req_index_to_global_index``
    and calling ``_forward_fp8_kv`` (the reference's pair,
    vllm_fp8kv/backend_patch.py:83-89); the conversion happens in the gather.
    """
    q = _as_single_q(q)
    n_tok = q.shape[0]
    md = attn_metadata
    # the converter's contract (vLLM sparse_utils.py, called with
    # NUM_TOPK_TOKENS=attn_metadata.topk_tokens at the reference's
    # backend_patch.py:83-89): the buffer row is exactly topk_tokens wide and
    # topk_tokens is a multiple of its 128-entry block
    width = topk_indices.shape[-1]
    assert width == md.topk_tokens, (
        f"topk_indices_buffer width {width} != attn_metadata.topk_tokens {md.topk_tokens}")
    assert md.topk_tokens % _CONVERT_BLOCK_N == 0, (
        f"NUM_TOPK_TOKENS ({md.topk_tokens}) must be divisible by BLOCK_N ({_CONVERT_BLOCK_N})")
    out = fp8_ds_mla_sparse_decode_paged(
        q, kv_c_and_k_pe_cache, md.req_id_per_token[:n_tok].to(torch.int32).contiguous(),
        md.block_table.to(torch.int32), topk_indices.view(n_tok, 1, -1),
        sm_scale=self.softmax_scale, block_size=md.block_size)
    return out[:, : self.num_heads, :]


def _forward_mqa_fp8_aware(self, q, kv_c_and_k_pe_cache, attn_metadata, layer):
    """Replacement ``forward_mqa`` that accepts fp8_ds_mla KV."""
    q = _as_single_q(q)
    n_tok = q.shape[0]
    assert self.topk_indices_buffer is not None
    topk_indices = self.topk_indices_buffer[:n_tok]
    md = attn_metadata
    if self.kv_cache_dtype == FP8_DS_MLA:
        attn_out = _forward_fp8_kv_paged(self, q, kv_c_and_k_pe_cache, topk_indices, md)
    else:
        from vllm.v1.attention.backends.mla.xpu_mla_sparse import (
            triton_convert_req_index_to_global_index,
        )

        slots = triton_convert_req_index_to_global_index(
            md.req_id_per_token, md.block_table, topk_indices,
            BLOCK_SIZE=md.block_size, NUM_TOPK_TOKENS=md.topk_tokens)
        attn_out = self._forward_bf16_kv(q, kv_c_and_k_pe_cache, slots, md)
    return attn_out, None


def _get_kv_cache_shape_fp8_aware(num_blocks: int, block_size: int, num_kv_heads: int,
                                  head_size: int, cache_dtype_str: str = "auto") -> tuple:
    """fp8_ds_mla pools are (num_blocks, block_size, 656) bytes; others head_size wide."""
    if cache_dtype_str == FP8_DS_MLA:
        return (num_blocks, block_size, ROW_BYTES)
    return (num_blocks, block_size, head_size)


def _patch_mla_spec_quant_mode(mla_mod) -> None:
    """Rebuild the (frozen) MLA KV-cache spec of an fp8_ds_mla layer with its
    quant mode set, so the worker asks the backend for the 656-byte shape that
    matches how the pool was sized."""
    import dataclasses

    from vllm.v1.kv_cache_interface import get_kv_quant_mode

    cls = mla_mod.MLAAttention
    if getattr(cls.get_kv_cache_spec, _MARK, False):
        return
    upstream = cls.get_kv_cache_spec

    def get_kv_cache_spec(self, vllm_config):
        spec = upstream(self, vllm_config)
        dtype = getattr(spec, "cache_dtype_str", None)
        if dtype == FP8_DS_MLA:
            spec = dataclasses.replace(spec, kv_quant_mode=get_kv_quant_mode(dtype))
        return spec

    setattr(get_kv_cache_spec, _MARK, True)
    cls.get_kv_cache_spec = get_kv_cache_spec


def apply() -> None:
    """Install the fp8_ds_mla support into a live vLLM (safe to call twice)."""
    from vllm.model_executor.layers.attention import mla_attention as mla_mod
    from vllm.v1.attention.backends.mla import triton_mla_sparse as tms

    impl, backend = tms.TritonMLASparseImpl, tms.TritonMLASparseBackend
    impl._forward_fp8_kv = _forward_fp8_kv
    impl.forward_mqa = _forward_mqa_fp8_aware
    backend.get_kv_cache_shape = staticmethod(_get_kv_cache_shape_fp8_aware)
    _patch_mla_spec_quant_mode(mla_mod)

    # The backend is selected by the raw --kv-cache-dtype string before it is
    # canonicalized, so the CLI names must be declared as well as the format.
    declared = list(backend.supported_kv_cache_dtypes)
    for name in (FP8_DS_MLA, *_CLI_FP8_NAMES):
        if name not in declared:
            declared.append(name)
    backend.supported_kv_cache_dtypes = declared

    canon = mla_mod._canonicalize_sparse_mla_kv_cache_dtype
    if getattr(canon, _MARK, False):
        return

    def canonicalize(attn_backend, kv_cache_dtype):
        if attn_backend.get_name() == "TRITON_MLA_SPARSE" and kv_cache_dtype in _CLI_FP8_NAMES:
            return FP8_DS_MLA
        return canon(attn_backend, kv_cache_dtype)

    setattr(canonicalize, _MARK, True)
    mla_mod._canonicalize_sparse_mla_kv_cache_dtype = canonicalize
    print(f"[vllm_fp8kv] TRITON_MLA_SPARSE serves {FP8_DS_MLA} on sm_100a "
          f"(kv dtypes: {backend.supported_kv_cache_dtypes})")
