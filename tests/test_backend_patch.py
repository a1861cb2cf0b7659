"""The vLLM wiring (backend_patch) against fakes of vLLM's surface.

Host-only behaviour runs on CPU; the forward paths run the sm_100a decode and
are GPU tests.  Mirrors tests/test_backend_patch.py:27-248 of the reference.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import gpu_util as U
from tests import vllm_fakes
from vllm_fp8kv import backend_patch, synthetic
from vllm_fp8kv.index_convert import convert_req_index_to_global_index
from vllm_fp8kv.fp8_ds_mla_sparse_decode import NOPE, ROPE, ROW_BYTES


@pytest.fixture
def vllm(monkeypatch):
    return vllm_fakes.install(monkeypatch)


def test_apply_declares_format_and_cli_aliases(vllm):
    assert "fp8_ds_mla" not in vllm.backend.supported_kv_cache_dtypes
    backend_patch.apply()
    declared = set(vllm.backend.supported_kv_cache_dtypes)
    assert {"fp8_ds_mla", "fp8", "fp8_e4m3", "auto", "bfloat16"} <= declared


def test_apply_fixes_the_cache_shape(vllm):
    assert vllm.backend.get_kv_cache_shape(8, 64, 1, 576, "fp8_ds_mla")[-1] == 576
    backend_patch.apply()
    assert vllm.backend.get_kv_cache_shape(8, 64, 1, 576, "fp8_ds_mla") == (8, 64, ROW_BYTES)
    assert vllm.backend.get_kv_cache_shape(8, 64, 1, 576, "auto") == (8, 64, 576)


@pytest.mark.parametrize("requested,expect", [("fp8", "fp8_ds_mla"), ("fp8_e4m3", "fp8_ds_mla"),
                                              ("auto", "auto"), ("bfloat16", "bfloat16")])
def test_apply_canonicalizes_cli_dtype(vllm, requested, expect):
    backend_patch.apply()
    assert vllm.mla._canonicalize_sparse_mla_kv_cache_dtype(vllm.backend, requested) == expect


def test_canonicalization_leaves_other_backends_to_upstream(vllm):
    backend_patch.apply()

    class Sm120:
        @staticmethod
        def get_name():
            return "FLASHINFER_MLA_SPARSE_SM120"

    canon = vllm.mla._canonicalize_sparse_mla_kv_cache_dtype
    assert canon(Sm120, "auto") == "fp8_ds_mla"
    assert canon(Sm120, "bfloat16") == "bfloat16"


def test_apply_is_idempotent(vllm):
    backend_patch.apply()
    first = vllm.mla._canonicalize_sparse_mla_kv_cache_dtype
    spec_first = vllm.MLAAttention.get_kv_cache_spec
    backend_patch.apply()
    assert vllm.mla._canonicalize_sparse_mla_kv_cache_dtype is first
    assert vllm.MLAAttention.get_kv_cache_spec is spec_first
    assert vllm.backend.supported_kv_cache_dtypes.count("fp8_ds_mla") == 1


def test_apply_marks_fp8_spec_quantized(vllm):
    backend_patch.apply()
    layer = vllm.MLAAttention("fp8_ds_mla")
    assert layer.get_kv_cache_spec("fp8_ds_mla").kv_quant_mode != "NONE"
    assert layer.get_kv_cache_spec("auto").kv_quant_mode == "NONE"


def test_bf16_path_stays_upstream_on_cpu(vllm):
    """A non-fp8 layer never reaches the library (runs without a GPU)."""
    backend_patch.apply()
    impl = vllm.impl(kv_cache_dtype="auto", softmax_scale=1 / 24.0)
    impl.topk_indices_buffer = torch.tensor([[0, 1, 64, -1] + [-1] * 124], dtype=torch.int32)

    class Md:
        req_id_per_token = torch.zeros(1, dtype=torch.int32)
        block_table = torch.tensor([[3, 1, 0, 2]], dtype=torch.int32)
        block_size = 64
        topk_tokens = 128

    out, extra = impl.forward_mqa(torch.randn(1, 16, 576), torch.zeros(4, 64, 576), Md, None)
    assert extra is None and impl.bf16_calls == 1
    assert impl.bf16_indices[0, :4].tolist() == [192, 193, 64, -1]


# ------------------------------------------------------------------- GPU paths
def _pool(n_slots=512, seed=3):
    rng = np.random.default_rng(seed)
    src = synthetic.bf16_bits((rng.standard_normal((n_slots, 576)) * 0.5).astype(np.float32))
    return U.device_pool(src, check_against_oracle=False)


@pytest.mark.gpu
def test_forward_fp8_kv_runs_the_kernel(vllm, cuda_device):
    backend_patch.apply()
    impl = vllm.impl(kv_cache_dtype="fp8_ds_mla", num_heads=16, softmax_scale=1 / 24.0)
    q = torch.randn(2, 16, NOPE + ROPE, device="cuda").bfloat16()
    idx = torch.randint(0, 512, (2, 128), device="cuda").int()
    pool = _pool()
    out = backend_patch._forward_fp8_kv(impl, q, pool, idx, attn_metadata=None)
    assert out.shape == (2, 16, NOPE) and torch.isfinite(out.float()).all()
    ref, _ = O.sparse_decode(q.float().cpu().numpy(), pool.view(-1, 656).cpu().numpy(),
                             idx.cpu().numpy(), 1 / 24.0)
    U.assert_close(out.float().cpu().numpy(), ref)


@pytest.mark.gpu
def test_forward_fp8_kv_accepts_tuple_q_and_slices_heads(vllm, cuda_device):
    backend_patch.apply()
    impl = vllm.impl(kv_cache_dtype="fp8_ds_mla", num_heads=8, softmax_scale=1 / 24.0)
    qt = (torch.randn(2, 16, NOPE, device="cuda").bfloat16(),
          torch.randn(2, 16, ROPE, device="cuda").bfloat16())
    idx = torch.randint(0, 512, (2, 128), device="cuda").int()
    out = backend_patch._forward_fp8_kv(impl, qt, _pool(), idx, attn_metadata=None)
    assert out.shape == (2, 8, NOPE)


@pytest.mark.gpu
def test_forward_mqa_dispatch_and_fused_index_conversion(vllm, cuda_device):
    """fp8_ds_mla layers decode straight from request-local positions; the
    result equals the reference's pair (convert to flat slots, then decode)."""
    backend_patch.apply()

    class Md:
        req_id_per_token = torch.zeros(1, dtype=torch.int32, device="cuda")
        block_table = torch.tensor([[3, 1, 0, 2, 4, 5, 6, 7]], dtype=torch.int32, device="cuda")
        block_size = 64
        topk_tokens = 128

    impl = vllm.impl(kv_cache_dtype="fp8_ds_mla", softmax_scale=1 / 24.0)
    impl.topk_indices_buffer = torch.tensor([[0, 1, 64, -1] + [-1] * 124], dtype=torch.int32,
                                            device="cuda")
    q = torch.randn(1, 16, NOPE + ROPE, device="cuda").bfloat16()
    pool = _pool(8 * 64)
    out, extra = impl.forward_mqa(q, pool, Md, None)
    assert extra is None and impl.bf16_calls == 0
    assert out.shape == (1, 16, NOPE) and torch.isfinite(out.float()).all()
    slots = convert_req_index_to_global_index(Md.req_id_per_token, Md.block_table,
                                              impl.topk_indices_buffer, BLOCK_SIZE=64,
                                              NUM_TOPK_TOKENS=128)
    assert slots[0, :4].tolist() == [3 * 64, 3 * 64 + 1, 64, -1]
    flat = backend_patch._forward_fp8_kv(impl, q, pool, slots, attn_metadata=None)
    assert torch.equal(out, flat)


@pytest.mark.parametrize("width,topk_tokens", [(256, 128), (128, 256), (192, 192)])
def test_fused_paged_path_keeps_the_converter_contract(vllm, width, topk_tokens):
    """The fp8 path converts inside the decode, so it must refuse what vLLM's
    converter refuses: a top-k buffer whose width is not attn_metadata.topk_tokens,
    and a topk_tokens that is not a multiple of the converter's 128-entry block
    (reference backend_patch.py:83-89).  Checked before any device work."""
    backend_patch.apply()

    class Md:
        req_id_per_token = torch.zeros(1, dtype=torch.int32)
        block_table = torch.zeros((1, 8), dtype=torch.int32)
        block_size = 64

    Md.topk_tokens = topk_tokens
    impl = vllm.impl(kv_cache_dtype="fp8_ds_mla", softmax_scale=1 / 24.0)
    impl.topk_indices_buffer = torch.zeros((1, width), dtype=torch.int32)
    q = torch.zeros(1, 16, NOPE + ROPE, dtype=torch.bfloat16)
    pool = torch.zeros(8, 64, 656, dtype=torch.uint8)
    with pytest.raises(AssertionError):
        impl.forward_mqa(q, pool, Md, None)
