"""ctypes binding of libfp8mla.so (the C ABI in include/fp8mla.h).

The library is loaded on first use.  There is no fallback: if the shared
library is missing or the device is not sm_100, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FP8MLA_LIB", os.path.join(_HERE, "libfp8mla.so"))

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_WORKSPACE = -4

DTYPE_BF16, DTYPE_F32, DTYPE_F16 = 0, 1, 2

# exported symbol -> (restype, argtypes); must list every function of include/fp8mla.h
_P, _I64, _I32, _F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
SIGNATURES = {
    "fp8mla_last_error": (ctypes.c_char_p, []),
    "fp8mla_abi_version": (_I32, []),
    "fp8mla_device_status": (_I32, [ctypes.POINTER(ctypes.c_uint), _I32, _P]),
    "fp8mla_selftest_wait_timeout": (_I32, [ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint64), _P]),
    "fp8mla_wait_limit": (ctypes.c_uint32, []),
    "fp8mla_selftest_set_wait_limit": (_I32, [ctypes.c_uint32]),
    "fp8mla_choose_num_splits": (_I32, [_I64, _I64, _I64, _I64, _I32]),
    "fp8mla_decode_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64, _I32]),
    "fp8mla_decode_kernel_name": (ctypes.c_char_p, [_I64, _I64, _I64, _I64, _I32, _I32]),
    "fp8mla_sparse_decode": (_I32, [
        _P, _I32, _I64, _I64, _I64, _I64,      # q, q_dtype, T, H, q strides
        _P, _I64,                              # kv, num_slots
        _P, _I64, _I64, _I64, _I64,            # indices, G, topk, idx strides
        _F32,                                  # sm_scale
        _P, _I64, _I64,                        # out, out strides
        _P, _I64,                              # lse, lse stride
        _I32, _P, _I64, _P]),                  # num_splits, workspace, bytes, stream
    "fp8mla_sparse_decode_paged": (_I32, [
        _P, _I32, _I64, _I64, _I64, _I64,      # q, q_dtype, T, H, q strides
        _P, _I64,                              # kv, num_slots
        _P, _P, _I64, _I64, _I64,              # req_id, block_table, bt stride, max_blocks, block_size
        _P, _I64, _I64, _I64, _I64,            # token_idx, G, topk, token_idx strides
        _F32,                                  # sm_scale
        _P, _I64, _I64, _P, _I64,              # out, out strides, lse, lse stride
        _I32, _P, _I64, _P]),                  # num_splits, workspace, bytes, stream
    "fp8mla_sparse_decode_noalloc": (_I32, [
        _P, _I32, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _F32,
        _P, _I64, _I64, _P, _I64, _I32, _P]),
    "fp8mla_ds_mla_write": (_I32, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P]),
    "fp8mla_dequant_e4m3": (_I32, [_P, _I64, _P, _I32, _I32, _P]),
    "fp8mla_ds_mla_dequant_rows": (_I32, [_P, _I64, _P, _I64, _P, _I64, _I32, _P]),
    "fp8mla_convert_req_index": (_I32, [_P, _P, _I64, _I64, _P, _I64, _I64, _I64, _I64,
                                        _P, _I64, _P]),
    "fp8mla_indexer_paged_logits": (_I32, [
        _P, _I64, _I64, _I64, _I64, _I64,      # q, B, next_n, H, head_dim, q_stride_b
        _P, _I64, _I64,                        # k_cache, num_blocks, block_size
        _P, _I64,                              # weights, w_stride
        _P, _P, _I64, _I64,                    # context_lens, block_table, bt_stride, max_blocks
        _P, _I64, _I64, _P]),                  # logits, logits_stride, max_model_len, stream
    "fp8mla_indexer_topk": (_I32, [_P, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _P]),
}

_lib = None
_lock = threading.Lock()


class Fp8MlaError(RuntimeError):
    """A libfp8mla call failed (CUDA error, unsupported device, workspace)."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise Fp8MlaError(
                        f"libfp8mla.so not found at {LIB_PATH}; build it with "
                        f"`python vllm-fp8kv_b200/build.py` (there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    msg = lib().fp8mla_last_error().decode(errors="replace")
    if rc == ERR_INVALID_ARGUMENT:
        raise AssertionError(f"{what}: {msg}")
    raise Fp8MlaError(f"{what} failed ({rc}): {msg}")


def device_status(reset: bool = True, device=None) -> int:
    """Device status word (0 = no bounded on-chip wait timed out); synchronises."""
    v = ctypes.c_uint(0)
    check(lib().fp8mla_device_status(ctypes.byref(v), int(reset), stream_ptr(device)),
          "fp8mla_device_status")
    return v.value


def stream_ptr(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors):
    """Check that every tensor is a CUDA tensor on one device; return that device.

    The library reads the SM count, the per-device set-up and the launch
    device from the CUDA current device, so callers run it under
    ``torch.cuda.device(<this device>)`` with the stream of this device."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise Fp8MlaError("libfp8mla kernels need CUDA tensors (sm_100); there is no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise AssertionError(f"all tensors must be on one device: {dev} and {t.device}")
    return dev
