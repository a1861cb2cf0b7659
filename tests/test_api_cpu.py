"""Argument checks of the Python entry points that run before any device work."""

import pytest
import torch

from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode_shared_topk


def _args(B=2, n=2, H=16, topk=64):
    q = torch.zeros(B, n, H, 576, dtype=torch.bfloat16)
    kv = torch.zeros(8, 64, 656, dtype=torch.uint8)
    idx = torch.zeros(B, topk, dtype=torch.int32)
    return q, kv, idx


def test_shared_topk_wants_four_dimensional_q():
    q, kv, idx = _args()
    with pytest.raises(AssertionError):
        fp8_ds_mla_sparse_decode_shared_topk(q[:, 0], kv, idx, 0.1)


def test_shared_topk_wants_one_index_row_per_request():
    q, kv, idx = _args()
    with pytest.raises(AssertionError):
        fp8_ds_mla_sparse_decode_shared_topk(q, kv, idx[:1], 0.1)
    with pytest.raises(AssertionError):
        fp8_ds_mla_sparse_decode_shared_topk(q, kv, idx.view(2, 2, 32), 0.1)


def test_shared_topk_wants_mergeable_token_and_head_dims():
    q, kv, idx = _args()
    with pytest.raises(AssertionError):
        fp8_ds_mla_sparse_decode_shared_topk(q.transpose(1, 2), kv, idx, 0.1)
