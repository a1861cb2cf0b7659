"""Sparse-MLA decode over fp8_ds_mla KV pages on B200 (sm_100a).

Drop-in for the reference entry point of the same name
(vllm_fp8kv/fp8_ds_mla_sparse_decode.py:214-288): same signature, same
asserts, same outputs.  The work runs in libfp8mla.so, which picks the
kernel by head count and q dtype (``decode_kernel_name`` reports the choice):

* 64 or 128 heads per kv group, bf16 q: ``decode_tc3_kernel``, a 2-SM cluster
  whose cta_group::2 tcgen05 MMAs take the heads as the M dimension (QK^T over
  d=576 and PV over d_v=512, accumulators in tensor memory), rows staged by
  TMA gather4;
* any other head count with bf16 q: ``decode_ws_kernel``, persistent and
  warp-specialised, rows staged by TMA gather4;
* fp32 q (the reference's CPU-test dtype): ``decode_mma_kernel``.

Split-KV calls add ``merge_splits_kernel``.  All of them gather 656-byte rows
by flat slot with 64-bit offsets, issue no load for masked slots (index < 0
or >= num_slots), dequantize e4m3 * tile scale to bf16 exactly as the
reference does, and merge top-k splits by LSE with no NaN on fully masked
chunks.

fp8_ds_mla row (656 B/token):
    [  0:512)  512 x fp8e4m3   NoPE latent (kv_lora_rank)
    [512:528)    4 x fp32      per-128-element tile scales (amax / 448)
    [528:656)   64 x bf16      RoPE, stored raw
MLA shares K and V: V is the NoPE half of the same row.  Only the inline tile
scales are applied (the layer's k_scale is not part of this format).
"""

from __future__ import annotations

import torch

from vllm_fp8kv import _native as N

NOPE = 512      # kv_lora_rank
ROPE = 64       # qk_rope_head_dim
TILE = 128      # elements per fp32 scale
ROW_BYTES = NOPE + (NOPE // TILE) * 4 + ROPE * 2   # 656
SCALE_OFF = NOPE                                   # 512
ROPE_OFF = NOPE + (NOPE // TILE) * 4               # 528


def decode_workspace_bytes(T: int, H: int, G: int, topk: int, num_splits: int = 0) -> int:
    """Device workspace one call needs (0 for a single split)."""
    return int(N.lib().fp8mla_decode_workspace_bytes(T, H, G, topk, num_splits))


def choose_num_kv_splits(T: int, H: int, G: int, topk: int, sm_count: int) -> int:
    """Split count the decode picks when num_kv_splits is None / 0."""
    return int(N.lib().fp8mla_choose_num_splits(T, H, G, topk, sm_count))


def decode_kernel_name(T: int, H: int, G: int, topk: int, q_dtype=torch.bfloat16,
                       num_splits: int = 0) -> str:
    """The kernel(s) one call with this shape dispatches to (introspection)."""
    code = N.DTYPE_BF16 if q_dtype == torch.bfloat16 else N.DTYPE_F32
    return N.lib().fp8mla_decode_kernel_name(T, H, G, topk, code, num_splits).decode()


def fp8_ds_mla_sparse_decode(
    q: torch.Tensor,            # [seq_q, h_q, 576]  bf16 (fp32 allowed for tests)
    kv_cache: torch.Tensor,     # [..., 656] uint8 or float8_e4m3fn, contiguous
    indices: torch.Tensor,      # [seq_q, kv_groups, topk] or [seq_q, topk] int32; -1 = masked
    sm_scale: float,
    return_lse: bool = False,
    block_n: int = 16,          # accepted for API compatibility; tiles are fixed per kernel
    block_h: int = 16,
    num_stages: int = 2,
    num_warps: int = 4,
    *,
    num_kv_splits: int | None = None,
    workspace: torch.Tensor | None = None,
):
    """Sparse MLA decode reading fp8_ds_mla pages.

    `indices` are FLAT SLOT indices into the paged cache (block * block_size +
    offset).  Returns `out` [seq_q, h_q, 512] in q.dtype, plus the natural-log
    `lse` [seq_q, h_q] fp32 when `return_lse` (-inf and a zero row for a query
    that selected nothing).  `num_kv_splits`: None/0 = heuristic, 1 = single
    pass, S > 1 = split the top-k axis S ways and merge by LSE.  The tuning
    kwargs of the reference (block_n, block_h, num_stages, num_warps) do not
    change the result and are ignored.
    """
    assert kv_cache.dtype in (torch.uint8, torch.float8_e4m3fn), kv_cache.dtype
    assert kv_cache.is_contiguous(), "kv_cache must be contiguous"
    assert q.stride(-1) == 1 and indices.stride(-1) == 1, "need unit last-dim strides"
    assert q.dtype in (torch.bfloat16, torch.float32), (
        f"rope is stored bf16; q must be bf16 (fp32 allowed for testing), got {q.dtype}"
    )
    kv_u8 = kv_cache.view(torch.uint8).reshape(-1, ROW_BYTES)
    num_slots = kv_u8.shape[0]

    seq_q, h_q, dim_qk = q.shape
    assert dim_qk == NOPE + ROPE, f"expected {NOPE + ROPE}, got {dim_qk}"
    if indices.dim() == 2:
        indices = indices.unsqueeze(1)
    kv_groups, topk = indices.shape[1], indices.shape[2]
    assert h_q % kv_groups == 0, f"h_q={h_q} not divisible by kv_groups={kv_groups}"
    assert indices.dtype == torch.int32, f"indices must be int32, got {indices.dtype}"
    N.require_cuda(q, kv_u8, indices, workspace)

    # the kernels read q in 16-byte vectors; re-lay a misaligned view once
    vec = 8 if q.dtype == torch.bfloat16 else 4
    if q.data_ptr() % 16 or q.stride(0) % vec or q.stride(1) % vec:
        q = q.contiguous()
        if q.data_ptr() % 16:
            q = q.clone()

    out = torch.empty((seq_q, h_q, NOPE), dtype=q.dtype, device=q.device)
    lse = torch.empty((seq_q, h_q), dtype=torch.float32, device=q.device) if return_lse else None

    splits = 0 if num_kv_splits is None else int(num_kv_splits)
    need = decode_workspace_bytes(seq_q, h_q, kv_groups, topk, splits)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if (need and workspace is not None) else None
    ws_bytes = workspace.numel() * workspace.element_size() if (need and workspace is not None) else 0

    with torch.cuda.device(q.device):
        rc = N.lib().fp8mla_sparse_decode(
            q.data_ptr(), N.DTYPE_BF16 if q.dtype == torch.bfloat16 else N.DTYPE_F32,
            seq_q, h_q, q.stride(0), q.stride(1),
            kv_u8.data_ptr(), num_slots,
            indices.data_ptr(), kv_groups, topk, indices.stride(0), indices.stride(1),
            float(sm_scale),
            out.data_ptr(), out.stride(0), out.stride(1),
            lse.data_ptr() if lse is not None else None, lse.stride(0) if lse is not None else 0,
            splits, ws_ptr, ws_bytes, N.stream_ptr(q.device))
    N.check(rc, "fp8_ds_mla_sparse_decode")
    return (out, lse) if return_lse else out


def fp8_ds_mla_sparse_decode_paged(
    q: torch.Tensor,             # [seq_q, h_q, 576]  bf16 (fp32 allowed for tests)
    kv_cache: torch.Tensor,      # [num_blocks, block_size, 656] uint8 / float8_e4m3fn, contiguous
    req_id: torch.Tensor,        # [seq_q] int32: request of each query token
    block_table: torch.Tensor,   # [num_reqs, max_blocks] int32 page ids
    token_indices: torch.Tensor, # [seq_q, kv_groups, topk] or [seq_q, topk] int32; -1 = masked
    sm_scale: float,
    block_size: int = 64,
    return_lse: bool = False,
    *,
    num_kv_splits: int | None = None,
    workspace: torch.Tensor | None = None,
):
    """`fp8_ds_mla_sparse_decode` over request-local token positions.

    Equivalent to converting `token_indices` with vLLM's
    `triton_convert_req_index_to_global_index(req_id, block_table,
    token_indices, BLOCK_SIZE=block_size)` and decoding the flat slots (the
    pair the reference runs per layer, vllm_fp8kv/backend_patch.py:83-89), but
    the conversion happens inside the decode's gather: no slot tensor is
    materialised and there is no separate launch.  Results are bit-identical
    to that pair.
    """
    assert kv_cache.dtype in (torch.uint8, torch.float8_e4m3fn), kv_cache.dtype
    assert kv_cache.is_contiguous(), "kv_cache must be contiguous"
    assert q.stride(-1) == 1 and token_indices.stride(-1) == 1, "need unit last-dim strides"
    assert q.dtype in (torch.bfloat16, torch.float32), (
        f"rope is stored bf16; q must be bf16 (fp32 allowed for testing), got {q.dtype}"
    )
    assert req_id.dtype == torch.int32 and block_table.dtype == torch.int32, "int32 tables"
    assert token_indices.dtype == torch.int32, f"indices must be int32, got {token_indices.dtype}"
    assert block_table.dim() == 2 and block_table.stride(1) == 1, "block_table [reqs, max_blocks]"
    assert req_id.dim() == 1 and req_id.shape[0] == q.shape[0] and req_id.is_contiguous()
    assert block_size > 0
    kv_u8 = kv_cache.view(torch.uint8).reshape(-1, ROW_BYTES)
    num_slots = kv_u8.shape[0]

    seq_q, h_q, dim_qk = q.shape
    assert dim_qk == NOPE + ROPE, f"expected {NOPE + ROPE}, got {dim_qk}"
    if token_indices.dim() == 2:
        token_indices = token_indices.unsqueeze(1)
    kv_groups, topk = token_indices.shape[1], token_indices.shape[2]
    assert h_q % kv_groups == 0, f"h_q={h_q} not divisible by kv_groups={kv_groups}"
    N.require_cuda(q, kv_u8, token_indices, req_id, block_table, workspace)

    vec = 8 if q.dtype == torch.bfloat16 else 4
    if q.data_ptr() % 16 or q.stride(0) % vec or q.stride(1) % vec:
        q = q.contiguous()
        if q.data_ptr() % 16:
            q = q.clone()

    out = torch.empty((seq_q, h_q, NOPE), dtype=q.dtype, device=q.device)
    lse = torch.empty((seq_q, h_q), dtype=torch.float32, device=q.device) if return_lse else None

    splits = 0 if num_kv_splits is None else int(num_kv_splits)
    need = decode_workspace_bytes(seq_q, h_q, kv_groups, topk, splits)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if (need and workspace is not None) else None
    ws_bytes = workspace.numel() * workspace.element_size() if (need and workspace is not None) else 0

    with torch.cuda.device(q.device):
        rc = N.lib().fp8mla_sparse_decode_paged(
            q.data_ptr(), N.DTYPE_BF16 if q.dtype == torch.bfloat16 else N.DTYPE_F32,
            seq_q, h_q, q.stride(0), q.stride(1),
            kv_u8.data_ptr(), num_slots,
            req_id.data_ptr(), block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
            int(block_size),
            token_indices.data_ptr(), kv_groups, topk, token_indices.stride(0),
            token_indices.stride(1),
            float(sm_scale),
            out.data_ptr(), out.stride(0), out.stride(1),
            lse.data_ptr() if lse is not None else None, lse.stride(0) if lse is not None else 0,
            splits, ws_ptr, ws_bytes, N.stream_ptr(q.device))
    N.check(rc, "fp8_ds_mla_sparse_decode_paged")
    return (out, lse) if return_lse else out


def fp8_ds_mla_sparse_decode_shared_topk(
    q: torch.Tensor,          # [batch, next_n, h_q, 576] bf16: next_n query tokens per request
    kv_cache: torch.Tensor,   # [..., 656] uint8 or float8_e4m3fn, contiguous
    indices: torch.Tensor,    # [batch, topk] or [batch, 1, topk] int32 flat slots; -1 = masked
    sm_scale: float,
    return_lse: bool = False,
    *,
    num_kv_splits: int | None = None,
    workspace: torch.Tensor | None = None,
):
    """Decode for requests whose next_n query tokens (multi-token prediction,
    speculative drafts) attend to one shared top-k set.

    Equal to `fp8_ds_mla_sparse_decode` over q.view(batch * next_n, h_q, 576)
    with each request's index row repeated next_n times, because every
    (query token, head) row is computed independently.  Here a request's
    next_n * h_q query heads form one head group of one call: its rows are
    gathered once instead of next_n times, and 64-head models with next_n = 2
    fill the 128-row tile of the paired tensor-core kernel instead of padding
    it.  No reference counterpart (the reference decodes one query token per
    index row).  Returns out [batch, next_n, h_q, 512] (and lse
    [batch, next_n, h_q]).
    """
    assert q.dim() == 4, "q must be [batch, next_n, h_q, 576]"
    B, n, H, D = q.shape
    assert indices.dim() == 2 or (indices.dim() == 3 and indices.shape[1] == 1), \
        "indices must be [batch, topk] (one kv group shared by the next_n tokens)"
    assert indices.shape[0] == B, "one index row per request"
    assert q.stride(1) == H * q.stride(2), "q's next_n and head dims must be mergeable"
    qv = q.view(B, n * H, D)
    res = fp8_ds_mla_sparse_decode(qv, kv_cache, indices, sm_scale, return_lse,
                                   num_kv_splits=num_kv_splits, workspace=workspace)
    if return_lse:
        out, lse = res
        return out.view(B, n, H, out.shape[-1]), lse.view(B, n, H)
    return res.view(B, n, H, res.shape[-1])
