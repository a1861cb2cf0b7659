"""fp8e4m3fn -> fp16/bf16/fp32 decode.

Same surface as the reference module (vllm_fp8kv/fp8_dequant.py:47-113):

* ``dequant_bitmath_torch`` -- the pure-torch bit-math decode (a host-side
  reference helper; the product kernels never call it);
* ``build_lut`` -- a 256-entry decode table built with torch's own cast;
* ``dequant_device`` -- the sm_100a decode kernel: method 0 is the packed
  hardware conversion (cvt e4m3x2 -> f16x2), method 1 the integer bit-math
  the fused decode uses (byte magnitude placed in fp32 bits [26:20] gives the
  value times 2^-120, rescaled exactly);
* ``dequant_triton_launch`` -- the reference's test driver name, kept for
  callers: returns (bit-math fp16, table-dtype decode) computed on device;
* ``dequant_ds_mla_rows`` -- gather fp8_ds_mla rows by slot and dequantize
  them with the decode kernels' own device code (bf16(e4m3 * tile scale),
  raw rope), the IS_FP8 gather of the reference decode kernel
  (vllm_fp8kv/fp8_ds_mla_sparse_decode.py:136-168) run on its own.

All of them are exact for every finite byte; 0x7F / 0xFF decode to NaN (the
payload differs between torch's CPU and CUDA casts, so compare NaN-ness).
"""

from __future__ import annotations

import torch

from vllm_fp8kv import _native as N

_DT = {torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16, torch.float32: N.DTYPE_F32}


def dequant_bitmath_torch(u8: torch.Tensor, dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """Decode e4m3fn bytes from the format's definition, in integer/fp32 torch ops.

    A byte is sign (bit 7), exponent e (bits 6..3, bias 7) and mantissa m
    (bits 2..0): value = (-1)^s * 2^(e-7) * (1 + m/8) for e > 0, the subnormal
    (-1)^s * 2^-6 * m/8 for e == 0, and NaN for e == 15, m == 7 (the format
    has no infinities).  Every finite value is exact in fp16, bf16 and fp32,
    so this equals torch's float8_e4m3fn cast (NaN payloads aside).
    Same result as the reference's helper (vllm_fp8kv/fp8_dequant.py:47-58).
    """
    assert u8.dtype == torch.uint8
    b = u8.to(torch.int32)
    e = (b >> 3) & 0xF
    m = (b & 0x7).to(torch.float32)
    mag = torch.where(e == 0, m * 2.0 ** -9, torch.ldexp(1.0 + m / 8.0, e - 7))
    val = torch.where((b & 0x80) != 0, -mag, mag)
    val = torch.where((b & 0x7F) == 0x7F, torch.full_like(val, float("nan")), val)
    return val.to(dtype)


def build_lut(dtype: torch.dtype = torch.float16, device="cuda") -> torch.Tensor:
    """256-entry table lut[b] = float8_e4m3fn(b) as `dtype` (torch's own cast)."""
    return (torch.arange(256, dtype=torch.uint8, device=device)
            .view(torch.float8_e4m3fn).to(dtype).contiguous())


def dequant_device(u8: torch.Tensor, dtype: torch.dtype = torch.float16,
                   method: int = 0) -> torch.Tensor:
    """Decode a uint8 CUDA tensor of e4m3fn bytes with the sm_100a kernel."""
    assert u8.dtype == torch.uint8
    assert dtype in _DT, dtype
    dev = N.require_cuda(u8)
    src = u8.contiguous().reshape(-1)
    out = torch.empty(src.shape, dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        rc = N.lib().fp8mla_dequant_e4m3(src.data_ptr(), src.numel(), out.data_ptr(), _DT[dtype],
                                         method, N.stream_ptr(dev))
    N.check(rc, "fp8mla_dequant_e4m3")
    return out.reshape(u8.shape)


def dequant_triton_launch(u8: torch.Tensor, lut: torch.Tensor):
    """Reference-compatible driver: (bit-math decode as fp16, decode in lut.dtype)."""
    return dequant_device(u8, torch.float16, method=1), dequant_device(u8, lut.dtype, method=0)


def dequant_ds_mla_rows(kv_cache: torch.Tensor, slots: torch.Tensor, method: int = 1) -> torch.Tensor:
    """bf16 [n, 576] rows: bf16(float(e4m3) * fp32 tile scale) | raw rope.

    ``kv_cache`` is any uint8 / float8 view of the [num_slots, 656] fp8_ds_mla
    pool (paged shapes are flattened); ``slots`` int32 [n], entries < 0 or
    >= num_slots give zero rows.  method 1 runs the packed-multiply dequant
    both decode kernels use, 0 the same arithmetic unpacked; both must equal
    torch's ``float8_e4m3fn -> float32 * scale -> bfloat16``.
    """
    assert method in (0, 1)
    assert slots.dtype == torch.int32 and slots.dim() == 1
    dev = N.require_cuda(kv_cache, slots)
    kv = kv_cache.view(torch.uint8) if kv_cache.dtype != torch.uint8 else kv_cache
    assert kv.is_contiguous() and kv.numel() % 656 == 0, "fp8_ds_mla pool must be contiguous"
    num_slots = kv.numel() // 656
    sl = slots.contiguous()
    out = torch.empty((sl.numel(), 576), dtype=torch.bfloat16, device=kv.device)
    with torch.cuda.device(dev):
        rc = N.lib().fp8mla_ds_mla_dequant_rows(kv.data_ptr(), num_slots, sl.data_ptr(), sl.numel(),
                                                out.data_ptr(), 576, method, N.stream_ptr(dev))
    N.check(rc, "fp8mla_ds_mla_dequant_rows")
    return out
