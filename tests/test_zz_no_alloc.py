"""fp8mla_sparse_decode_noalloc: the decode entry point that allocates nothing.

Some callers cannot hand the library a workspace or let it call cudaMalloc:
an inference engine that carves its KV cache out of the memory left after a
profiling pass has no room for a later, unplanned allocation, and a
foreign-language host that only holds raw device pointers may have no
allocator binding.  This entry point takes its split-KV scratch from a fixed
32 MiB array inside the library.  These tests call it through the C ABI and
check it against fp8mla_sparse_decode with a caller-provided workspace, on two
calls in a row (the shared array keeps the previous call's contents, which
must not leak into the next result).  The file name makes pytest collect it
last; it also passes when run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import gpu_util as U
from vllm_fp8kv import _native as N
from vllm_fp8kv import synthetic
from vllm_fp8kv.fp8_ds_mla_sparse_decode import decode_workspace_bytes

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20


def _case(H, topk, B, seed):
    s = synthetic.Shape("na", B=B, H=H, topk=topk, ctx=4096, pool_slots=max(16384, B * 4096),
                        mask_frac=0.1)
    w = synthetic.make_host(s, seed=seed)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    return w, pool.view(-1, 656), q, idx


def _call(fn_name, q, kv, idx, sm, splits, ws=None):
    T, H, _ = q.shape
    out = torch.empty((T, H, 512), dtype=q.dtype, device=q.device)
    lse = torch.empty((T, H), dtype=torch.float32, device=q.device)
    stream = torch.cuda.current_stream().cuda_stream
    common = [q.data_ptr(), N.DTYPE_BF16, T, H, q.stride(0), q.stride(1), kv.data_ptr(), kv.shape[0],
              idx.data_ptr(), 1, idx.shape[1], idx.stride(0), idx.shape[1], float(sm),
              out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0), splits]
    L = N.lib()
    if fn_name == "noalloc":
        rc = L.fp8mla_sparse_decode_noalloc(*common, stream)
    else:
        rc = L.fp8mla_sparse_decode(*common, ws.data_ptr() if ws is not None else None,
                                    ws.numel() if ws is not None else 0, stream)
    N.check(rc, fn_name)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("H,topk,B,splits", [(16, 256, 4, 0), (16, 512, 3, 8), (128, 512, 2, 4)])
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, H, topk, B, splits):
    for seed in (1, 2):   # two calls in a row through the shared scratch
        w, kv, q, idx = _case(H, topk, B, seed + H + topk)
        need = decode_workspace_bytes(B, H, 1, topk, splits)
        assert 0 < need <= SCRATCH_BYTES, "the case must exercise the split scratch"
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        got, got_lse = _call("noalloc", q, kv, idx, w.sm_scale, splits)
        want, want_lse = _call("workspace", q, kv, idx, w.sm_scale, splits, ws)
        U.assert_close(got, want)
        U.assert_lse_close(got_lse, want_lse)
        ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits), kv.cpu().numpy(), w.slots,
                                       w.sm_scale)
        U.assert_close(got, ref)
        U.assert_lse_close(got_lse, ref_lse)


def test_noalloc_rejects_shapes_beyond_the_scratch(cuda_device):
    T, H, topk, splits = 1024, 128, 2048, 16
    assert decode_workspace_bytes(T, H, 1, topk, splits) > SCRATCH_BYTES
    rc = N.lib().fp8mla_sparse_decode_noalloc(
        None, N.DTYPE_BF16, T, H, H * 576, 576, None, 0, None, 1, topk, topk, topk, 0.1,
        None, H * 512, 512, None, H, splits, None)
    assert rc == N.ERR_WORKSPACE
    assert b"fixed" in N.lib().fp8mla_last_error()
