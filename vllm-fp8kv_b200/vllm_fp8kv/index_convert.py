"""Token-relative top-k -> flat global slot indices, on sm_100a.

Same contract as vLLM's ``triton_convert_req_index_to_global_index`` (the
converter the reference's backend calls, vllm_fp8kv/backend_patch.py:83-89;
documented in the installed vllm/v1/attention/backends/mla/sparse_utils.py:85-104):

    out[t, i] = block_table[req_id[t], tok // BLOCK_SIZE] * BLOCK_SIZE + tok % BLOCK_SIZE

with -1 when tok < 0 or the block index falls outside the table row.
"""

from __future__ import annotations

import torch

from vllm_fp8kv import _native as N


def convert_req_index_to_global_index(req_id: torch.Tensor, block_table: torch.Tensor,
                                      token_indices: torch.Tensor, BLOCK_SIZE: int = 64,
                                      NUM_TOPK_TOKENS: int = 2048, BLOCK_N: int = 128,
                                      out: torch.Tensor | None = None) -> torch.Tensor:
    assert req_id.dtype == torch.int32
    assert block_table.dtype == torch.int32
    assert token_indices.dtype == torch.int32
    assert token_indices.shape[1] == NUM_TOPK_TOKENS
    assert NUM_TOPK_TOKENS % BLOCK_N == 0, (
        f"NUM_TOPK_TOKENS ({NUM_TOPK_TOKENS}) must be divisible by BLOCK_N ({BLOCK_N})")
    dev = N.require_cuda(req_id, block_table, token_indices, out)
    req = req_id.contiguous()
    bt = block_table.contiguous()
    ti = token_indices.contiguous()
    T = ti.shape[0]
    if out is None:
        out = torch.empty_like(ti)
    with torch.cuda.device(dev):
        rc = N.lib().fp8mla_convert_req_index(
            req.data_ptr(), bt.data_ptr(), bt.stride(0), bt.shape[1], ti.data_ptr(), ti.stride(0),
            T, NUM_TOPK_TOKENS, BLOCK_SIZE, out.data_ptr(), out.stride(0), N.stream_ptr(dev))
    N.check(rc, "fp8mla_convert_req_index")
    return out
