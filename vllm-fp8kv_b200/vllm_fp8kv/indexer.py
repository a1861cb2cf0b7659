"""DSA indexer read path on sm_100a: fp8 paged MQA logits and per-row top-k.

The sparse-MLA models pick, for every decode token, the top-k context
positions the attention then reads; the indexer that scores them keeps its
own fp8 key cache.  The reference specifies this step and its page format
(PORT_PLAN.md:14, :41 D3, trap 3) but ships no code for it; the entry points
here take the signatures of the vLLM ops a DSA backend calls:

* ``fp8_paged_mqa_logits(q, kv_cache, weights, context_lens, block_tables,
  schedule_metadata, max_model_len)`` (DeepGEMM / vLLM), and
* ``top_k_per_row_decode(logits, next_n, seq_lens, topk_indices, num_rows,
  stride0, stride1, topk_tokens)`` (vLLM's ``torch.ops._C`` op), which fills
  the ``topk_indices_buffer`` that ``backend_patch._forward_mqa_fp8_aware``
  reads (reference backend_patch.py:79-81).

Key cache: ``[num_blocks, 64, 1, 132]`` bytes (or any contiguous view with
8448 bytes per block), per block 64 x 128 e4m3 values then 64 fp32 scales.
Queries ``[B, next_n, 64, 128]`` e4m3 with their scale folded into
``weights [B * next_n, 64]``.
"""

from __future__ import annotations

import torch

from vllm_fp8kv import _native as N

HEADS = 64
DIM = 128
BLOCK = 64
PAGE_BYTES = BLOCK * (DIM + 4)  # 8448


def fp8_paged_mqa_logits(q: torch.Tensor, kv_cache: torch.Tensor, weights: torch.Tensor,
                         context_lens: torch.Tensor, block_tables: torch.Tensor,
                         schedule_metadata=None, max_model_len: int | None = None,
                         logits: torch.Tensor | None = None) -> torch.Tensor:
    """Indexer logits [B * next_n, max_model_len] fp32 (-inf past each row's
    causal limit context_len - next_n + n + 1).  ``schedule_metadata`` is
    accepted for signature compatibility and not needed."""
    assert q.dim() == 4 and q.shape[2] == HEADS and q.shape[3] == DIM, \
        f"q must be [B, next_n, {HEADS}, {DIM}], got {tuple(q.shape)}"
    assert q.dtype in (torch.float8_e4m3fn, torch.uint8), f"q must be e4m3, got {q.dtype}"
    assert q.stride(3) == 1 and q.stride(2) == DIM and q.stride(1) == HEADS * DIM, \
        "a request's query rows must be contiguous"
    B, next_n = q.shape[0], q.shape[1]
    assert next_n in (1, 2), f"next_n must be 1 or 2, got {next_n}"
    assert kv_cache.dtype in (torch.uint8, torch.float8_e4m3fn) and kv_cache.is_contiguous()
    assert kv_cache.numel() % PAGE_BYTES == 0, "the key cache holds 8448-byte blocks"
    kv = kv_cache.view(torch.uint8).reshape(-1, PAGE_BYTES)
    assert weights.dtype == torch.float32 and weights.dim() == 2 and weights.stride(1) == 1
    assert weights.shape[0] == B * next_n and weights.shape[1] == HEADS
    ctx = context_lens.reshape(-1)
    assert ctx.dtype == torch.int32 and ctx.numel() == B and ctx.is_contiguous()
    assert block_tables.dtype == torch.int32 and block_tables.dim() == 2
    assert block_tables.stride(1) == 1 and block_tables.shape[0] == B
    assert max_model_len is not None and max_model_len >= 0
    dev = N.require_cuda(q, kv, weights, ctx, block_tables, logits)
    if logits is None:
        logits = torch.empty((B * next_n, max_model_len), dtype=torch.float32, device=dev)
    assert logits.dtype == torch.float32 and logits.stride(1) == 1
    assert logits.shape[0] == B * next_n and logits.shape[1] >= max_model_len
    qb = q.view(torch.uint8)
    with torch.cuda.device(dev):
        rc = N.lib().fp8mla_indexer_paged_logits(
            qb.data_ptr(), B, next_n, HEADS, DIM, qb.stride(0),
            kv.data_ptr(), kv.shape[0], BLOCK,
            weights.data_ptr(), weights.stride(0),
            ctx.data_ptr(), block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
            logits.data_ptr(), logits.stride(0), max_model_len, N.stream_ptr(dev))
    N.check(rc, "fp8_paged_mqa_logits")
    return logits


def top_k_per_row_decode(logits: torch.Tensor, next_n: int, seq_lens: torch.Tensor,
                         topk_indices: torch.Tensor, num_rows: int, stride0: int, stride1: int,
                         topk_tokens: int) -> None:
    """Write each row's top-k positions into ``topk_indices`` [num_rows, >= topk]:
    ascending kept positions, then -1 (see ``fp8mla_indexer_topk``)."""
    assert logits.dtype == torch.float32 and stride1 == 1, "logits rows must be unit-strided"
    assert topk_indices.dtype == torch.int32 and topk_indices.stride(1) == 1
    assert topk_indices.shape[0] >= num_rows and topk_indices.shape[1] >= topk_tokens
    assert num_rows % next_n == 0, "rows come in groups of next_n per request"
    ctx = seq_lens.reshape(-1)
    assert ctx.dtype == torch.int32 and ctx.is_contiguous() and ctx.numel() * next_n >= num_rows
    dev = N.require_cuda(logits, ctx, topk_indices)
    max_len = logits.shape[1]
    with torch.cuda.device(dev):
        rc = N.lib().fp8mla_indexer_topk(logits.data_ptr(), num_rows, stride0, next_n, ctx.data_ptr(),
                                         topk_indices.data_ptr(), topk_indices.stride(0), topk_tokens,
                                         max_len, N.stream_ptr(dev))
    N.check(rc, "top_k_per_row_decode")


def indexer_topk(logits: torch.Tensor, next_n: int, context_lens: torch.Tensor,
                 topk: int) -> torch.Tensor:
    """[rows, topk] int32 top-k positions of every logits row."""
    out = torch.empty((logits.shape[0], topk), dtype=torch.int32, device=logits.device)
    top_k_per_row_decode(logits, next_n, context_lens, out, logits.shape[0], logits.stride(0),
                         logits.stride(1), topk)
    return out
