"""fp8_ds_mla cache writer on sm_100a.

Replaces vLLM's ``ops.concat_and_cache_mla(kv_c, k_pe, kv_cache, slot_mapping,
kv_cache_dtype="fp8_ds_mla", scale)`` (the producer of the format; called at
verify/contract.py:100-103 of the reference).  Per 128-element tile of the
NoPE latent: scale = max(amax / 448, FLT_MIN) stored as fp32 at byte 512 + 4t,
bytes = float8_e4m3fn(x / scale) with round-to-nearest-even; the RoPE half is
copied as raw bf16 at byte 528.  Byte-exact with the reference's mirrors
(tests/fakes.py:28-57, verify/reference.py:68-91).  The layer's k_scale is
not applied: the format carries its scales inline.  Tokens whose slot is
negative (padding) or past the pool are skipped.
"""

from __future__ import annotations

import torch

from vllm_fp8kv import _native as N

ROW_BYTES = 656


def concat_and_cache_ds_mla(kv_c: torch.Tensor, k_pe: torch.Tensor, kv_cache: torch.Tensor,
                            slot_mapping: torch.Tensor) -> None:
    """Quantize kv_c [N, 512] and k_pe [N, 64] (bf16) into kv_cache [..., 656] rows."""
    assert kv_c.dtype == torch.bfloat16 and k_pe.dtype == torch.bfloat16, "bf16 latent/rope"
    assert kv_c.dim() == 2 and kv_c.shape[1] == 512 and kv_c.stride(1) == 1
    assert k_pe.dim() == 2 and k_pe.shape[1] == 64 and k_pe.stride(1) == 1
    assert kv_c.shape[0] == k_pe.shape[0] == slot_mapping.shape[0]
    assert kv_cache.dtype in (torch.uint8, torch.float8_e4m3fn) and kv_cache.is_contiguous()
    assert kv_cache.shape[-1] == ROW_BYTES, "fp8_ds_mla rows are 656 bytes"
    dev = N.require_cuda(kv_c, k_pe, kv_cache, slot_mapping)
    slots = slot_mapping.to(torch.int64).contiguous()
    flat = kv_cache.view(torch.uint8).reshape(-1, ROW_BYTES)
    with torch.cuda.device(dev):
        rc = N.lib().fp8mla_ds_mla_write(
            kv_c.data_ptr(), kv_c.stride(0), k_pe.data_ptr(), k_pe.stride(0),
            slots.data_ptr(), slots.numel(), flat.data_ptr(), flat.shape[0],
            N.stream_ptr(dev))
    N.check(rc, "fp8mla_ds_mla_write")


def concat_and_cache_mla(kv_c: torch.Tensor, k_pe: torch.Tensor, kv_cache: torch.Tensor,
                         slot_mapping: torch.Tensor, kv_cache_dtype: str,
                         scale: torch.Tensor | float | None = None) -> None:
    """vLLM-signature wrapper; only the fp8_ds_mla format is implemented here."""
    if kv_cache_dtype != "fp8_ds_mla":
        raise NotImplementedError(f"only fp8_ds_mla is implemented, got {kv_cache_dtype!r}")
    concat_and_cache_ds_mla(kv_c, k_pe, kv_cache, slot_mapping)
