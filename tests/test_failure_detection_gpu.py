"""Failure detection of the decode kernels' on-chip waits, without a GPU fault.

Every mbarrier wait in the decode kernels is bounded: after a fixed number of
try_wait calls it gives up, records "wait timed out" and which wait in a
device status word, and the kernel returns instead of hanging.  These tests
drive that path with fp8mla_selftest_wait_timeout (a wait on a barrier that
nothing arrives on), check the word through fp8mla_device_status, and check
that the context still runs a correct decode afterwards.
"""

import ctypes

import pytest
import torch

from oracle import oracle as O
from tests import gpu_util as U
from vllm_fp8kv import _native as N
from vllm_fp8kv import synthetic
from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode

pytestmark = pytest.mark.gpu

SELFTEST_WHERE = 63


def _selftest(iters):
    ns = ctypes.c_uint64(0)
    N.check(N.lib().fp8mla_selftest_wait_timeout(iters, ctypes.byref(ns), N.stream_ptr(None)),
            "fp8mla_selftest_wait_timeout")
    return ns.value


def test_timed_out_wait_is_reported_and_the_context_survives(cuda_device):
    N.device_status(reset=True)
    # the decode kernels' own limit: a broken hand-off ends within bounded time
    # (about 0.4 s on B200)
    ns = _selftest(N.lib().fp8mla_wait_limit())
    print(f"a timed-out wait gave up after {ns * 1e-9:.3f} s")
    assert 0 < ns < 10e9
    assert N.device_status(reset=True) == 1 | (SELFTEST_WHERE << 8)
    assert N.device_status(reset=True) == 0

    s = synthetic.Shape("fd", B=2, H=16, topk=256, ctx=1024, pool_slots=4096, mask_frac=0.1)
    w = synthetic.make_host(s, seed=5)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    out, lse = fp8_ds_mla_sparse_decode(U.bf16_tensor(w.q_bits), pool,
                                        torch.from_numpy(w.slots).cuda(), w.sm_scale,
                                        return_lse=True)
    ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits), pool.view(-1, 656).cpu().numpy(),
                                   w.slots, w.sm_scale)
    U.assert_close(out.float().cpu().numpy(), ref)
    U.assert_lse_close(lse.cpu().numpy(), ref_lse)
    assert N.device_status(reset=True) == 0


def test_selftest_rejects_iteration_counts_outside_the_limit(cuda_device):
    ns = ctypes.c_uint64(0)
    L = N.lib()
    assert L.fp8mla_selftest_wait_timeout(0, ctypes.byref(ns), None) == N.ERR_INVALID_ARGUMENT
    assert L.fp8mla_selftest_wait_timeout(L.fp8mla_wait_limit() + 1, ctypes.byref(ns),
                                          None) == N.ERR_INVALID_ARGUMENT


def test_small_head_decode_timeout_path_returns_and_reports(cuda_device):
    """Drive decode_ws_kernel's own error path: with a hand-off limit of two
    try_wait calls its waits give up while rows are still arriving.  The
    producers then stop issuing copies, wait for the ones they issued, and every
    warp returns: the call completes, the status word carries the timeout bit
    with the small-head kernel's wait codes (20-27, OR-ed together when several
    waits gave up, so within [16, 32)), and after restoring the limit the same
    context decodes correctly."""
    L = N.lib()
    s = synthetic.Shape("fdws", B=16, H=16, topk=1024, ctx=4096, pool_slots=16 * 4096,
                        mask_frac=0.1)
    w = synthetic.make_host(s, seed=21)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    N.device_status(reset=True)
    assert L.fp8mla_selftest_set_wait_limit(L.fp8mla_wait_limit() + 1) == N.ERR_INVALID_ARGUMENT
    N.check(L.fp8mla_selftest_set_wait_limit(2), "set wait limit")
    try:
        fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, num_kv_splits=2)
        torch.cuda.synchronize()
        st = N.device_status(reset=True)
    finally:
        N.check(L.fp8mla_selftest_set_wait_limit(0), "restore wait limit")
    assert st & 1, f"no timeout recorded (status {st:#x})"
    assert 16 <= (st >> 8) < 32, f"unexpected wait code in status {st:#x}"
    out, lse = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, return_lse=True, num_kv_splits=2)
    ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits), pool.view(-1, 656).cpu().numpy(),
                                   w.slots, w.sm_scale)
    U.assert_close(out.float().cpu().numpy(), ref)
    U.assert_lse_close(lse.cpu().numpy(), ref_lse)
    assert N.device_status(reset=True) == 0
