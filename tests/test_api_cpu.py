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


def test_host_bitmath_decode_matches_torch_casts_on_all_bytes():
    """The host helper decodes every finite e4m3fn byte exactly as torch's
    cast does (golden dequant.npz, written from torch by the fixture script)
    and gives NaN for 0x7F / 0xFF."""
    import numpy as np

    from tests.conftest import golden
    from vllm_fp8kv.fp8_dequant import dequant_bitmath_torch

    g = golden("dequant.npz")
    b = torch.arange(256, dtype=torch.uint8)
    finite = np.array([(x & 0x7F) != 0x7F for x in range(256)])
    for dt, key in ((torch.float16, "f16_bits"), (torch.bfloat16, "bf16_bits")):
        got = dequant_bitmath_torch(b, dt).view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(got[finite], g[key][finite])
    f32 = dequant_bitmath_torch(b, torch.float32).numpy()
    assert np.array_equal(f32.view(np.uint32)[finite], g["f32_bits"][finite])
    assert np.isnan(f32[~finite]).all()


def test_tensors_on_two_devices_are_rejected():
    """Every tensor of one call must live on q's device (checked on the host)."""
    from vllm_fp8kv import _native as N

    class Fake:
        def __init__(self, dev):
            self.is_cuda, self.device = True, dev

    assert N.require_cuda(Fake("cuda:0"), None, Fake("cuda:0")) == "cuda:0"
    with pytest.raises(AssertionError):
        N.require_cuda(Fake("cuda:0"), Fake("cuda:1"))
