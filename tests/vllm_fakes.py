"""Stand-ins for the slice of vLLM that backend_patch touches.

vLLM's TRITON_MLA_SPARSE backend (PR #47629) is not installed in this image, so
the wiring is driven against small fakes of exactly the surface it patches:
the backend class (supported dtypes, cache shape), the impl (forward_mqa,
_forward_bf16_kv, topk buffer), the MLA attention spec (a frozen dataclass whose
kv_quant_mode defaults to NONE), the dtype canonicalizer and upstream's index
converter.  Same surface as the reference's tests/fakes.py:85-244.
"""

import dataclasses
import sys
import types

import torch

NOPE = 512


def _module(name, **attrs):
    m = types.ModuleType(name)
    m.__dict__.update(attrs)
    return m


def torch_index_converter(req_id_per_token, block_table, token_indices, BLOCK_SIZE,
                          NUM_TOPK_TOKENS):
    """Upstream converter semantics in plain torch (bf16 path of the fakes)."""
    tok = token_indices.long()
    blk = torch.div(tok, BLOCK_SIZE, rounding_mode="floor")
    ok = (tok >= 0) & (blk < block_table.shape[1])
    rows = block_table[req_id_per_token.long()].long()
    base = torch.gather(rows, 1, blk.clamp(0, block_table.shape[1] - 1))
    return torch.where(ok, base * BLOCK_SIZE + tok % BLOCK_SIZE, -1).to(torch.int32)


class Backend:
    supported_kv_cache_dtypes = ["auto", "float16", "bfloat16"]

    @staticmethod
    def get_name():
        return "TRITON_MLA_SPARSE"

    @staticmethod
    def get_kv_cache_shape(num_blocks, block_size, num_kv_heads, head_size, cache_dtype_str="auto"):
        return (num_blocks, block_size, head_size)   # upstream: 576 wide for every dtype


class Impl:
    def __init__(self, kv_cache_dtype="auto", num_heads=16, softmax_scale=1.0):
        self.kv_cache_dtype = kv_cache_dtype
        self.num_heads = num_heads
        self.softmax_scale = softmax_scale
        self.topk_indices_buffer = None
        self.bf16_calls = 0

    def _forward_bf16_kv(self, q, kv_cache, topk_indices, attn_metadata):
        self.bf16_calls += 1
        self.bf16_indices = topk_indices
        return torch.zeros(q.shape[0], self.num_heads, NOPE, dtype=q.dtype, device=q.device)

    def forward_mqa(self, *args, **kwargs):
        return None


@dataclasses.dataclass(frozen=True)
class Spec:
    block_size: int = 64
    num_kv_heads: int = 1
    head_size: int = 576
    cache_dtype_str: str | None = None
    kv_quant_mode: str = "NONE"


class MLAAttention:
    def __init__(self, kv_cache_dtype="auto"):
        self.kv_cache_dtype = kv_cache_dtype

    def get_kv_cache_spec(self, vllm_config):
        return Spec(cache_dtype_str=vllm_config)


def get_kv_quant_mode(kv_cache_dtype):
    return "FP8_PER_TENSOR" if str(kv_cache_dtype).startswith("fp8") else "NONE"


def canonicalize(attn_backend, kv_cache_dtype):
    name = attn_backend.get_name()
    if name == "FLASHMLA_SPARSE" and kv_cache_dtype.startswith("fp8"):
        return "fp8_ds_mla"
    if name == "FLASHINFER_MLA_SPARSE_SM120" and kv_cache_dtype in ("auto", "fp8", "fp8_e4m3"):
        return "fp8_ds_mla"
    return kv_cache_dtype


def install(monkeypatch):
    tms = _module("vllm.v1.attention.backends.mla.triton_mla_sparse",
                  TritonMLASparseBackend=Backend, TritonMLASparseImpl=Impl)
    xpu = _module("vllm.v1.attention.backends.mla.xpu_mla_sparse",
                  triton_convert_req_index_to_global_index=torch_index_converter)
    mla = _module("vllm.model_executor.layers.attention.mla_attention",
                  _canonicalize_sparse_mla_kv_cache_dtype=canonicalize, MLAAttention=MLAAttention)
    iface = _module("vllm.v1.kv_cache_interface", get_kv_quant_mode=get_kv_quant_mode)
    mods = {
        "vllm": _module("vllm"),
        "vllm.model_executor": _module("vllm.model_executor"),
        "vllm.model_executor.layers": _module("vllm.model_executor.layers"),
        "vllm.model_executor.layers.attention": _module("vllm.model_executor.layers.attention",
                                                        mla_attention=mla),
        "vllm.model_executor.layers.attention.mla_attention": mla,
        "vllm.v1": _module("vllm.v1"),
        "vllm.v1.attention": _module("vllm.v1.attention"),
        "vllm.v1.attention.backends": _module("vllm.v1.attention.backends"),
        "vllm.v1.attention.backends.mla": _module("vllm.v1.attention.backends.mla",
                                                  triton_mla_sparse=tms, xpu_mla_sparse=xpu),
        "vllm.v1.attention.backends.mla.triton_mla_sparse": tms,
        "vllm.v1.attention.backends.mla.xpu_mla_sparse": xpu,
        "vllm.v1.kv_cache_interface": iface,
    }
    for name, mod in mods.items():
        monkeypatch.setitem(sys.modules, name, mod)
    monkeypatch.setattr(Backend, "supported_kv_cache_dtypes", ["auto", "float16", "bfloat16"])
    monkeypatch.setattr(Backend, "get_kv_cache_shape", Backend.__dict__["get_kv_cache_shape"])
    monkeypatch.setattr(MLAAttention, "get_kv_cache_spec", MLAAttention.__dict__["get_kv_cache_spec"])
    monkeypatch.setattr(Impl, "forward_mqa", Impl.__dict__["forward_mqa"])
    return types.SimpleNamespace(backend=Backend, impl=Impl, mla=mla, MLAAttention=MLAAttention)
