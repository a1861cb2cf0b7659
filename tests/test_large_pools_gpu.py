"""GPU parity at the benchmark pools' full sizes: 64-bit row offsets on every
decode kernel, and the c3 / c4 / c5 shapes checked on request subsets.

A slot's byte offset passes 2^31 above slot 3,273,603 (656-byte rows).  The
reference guards this with its 3.5 M-slot section (verify/run_all.py:155-185;
the int64 row offset of fp8_ds_mla_sparse_decode.py:142-144).  Here every
decode kernel runs on pools of 4,194,304 (c4) and 8,388,608 (c5) slots with
selected slots placed past that boundary, up to num_slots - 1, and the
results are compared with the oracle on the gathered rows.  Full-size
batches are checked on a few requests against the oracle and on the rest by
batch invariance (a request decoded alone gives the same bits).
"""

import dataclasses

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import gpu_util as U
from vllm_fp8kv import synthetic
from vllm_fp8kv.fp8_ds_mla_sparse_decode import (
    decode_kernel_name,
    fp8_ds_mla_sparse_decode,
    fp8_ds_mla_sparse_decode_paged,
)

pytestmark = pytest.mark.gpu

BOUNDARY_SLOT = 3_273_603  # last slot whose byte offset fits below 2^31
C4_SLOTS = 4_194_304


def _release():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _rows_of(kv, slots_row):
    """Host copy of the rows one request selects, and local indices into them."""
    flat = kv.view(-1, 656)
    n = flat.shape[0]
    sl = slots_row.long()
    ok = (sl >= 0) & (sl < n)
    rows = flat[sl.clamp(0, n - 1)].cpu().numpy()
    local = np.where(ok.cpu().numpy(), np.arange(sl.numel()), -1).astype(np.int32)
    return rows, local


def _check_requests(out, lse, q, kv, slots, sm, reqs, **tol):
    """Requests `reqs` of a decode against the oracle on their gathered rows."""
    for b in reqs:
        rows, local = _rows_of(kv, slots[b])
        ref, ref_lse = O.sparse_decode(q[b:b + 1].float().cpu().numpy(), rows, local[None], sm)
        U.assert_close(out[b:b + 1].float().cpu().numpy(), ref, **tol)
        U.assert_lse_close(lse[b:b + 1].cpu().numpy(), ref_lse)


def _place_past_boundary(slots, num_slots, rng):
    """Rewrite request 0 (and 1) so that they select the pool's top rows and
    rows around the 2^31-byte boundary; returns the modified slot tensor."""
    s = slots.clone()
    top = torch.arange(num_slots - 1, num_slots - 1 - 256, -1, dtype=torch.int32)
    edge = torch.arange(BOUNDARY_SLOT - 64, BOUNDARY_SLOT + 192, dtype=torch.int32)
    s[0, :256] = top.to(s.device)
    s[0, 256:512] = edge.to(s.device)
    if s.shape[0] > 1:
        far = rng.integers(BOUNDARY_SLOT + 1, num_slots, size=s.shape[1]).astype(np.int32)
        s[1] = torch.from_numpy(far).to(s.device)
    return s


@pytest.fixture(scope="module")
def c4_pool(cuda_device):
    """The c4 pool (4,194,304 slots, 2.75 GB) with ~N(0,1) latents."""
    shape = dataclasses.replace(synthetic.SHAPES["c4"], amax_spread=False)
    w = synthetic.make_device(shape, seed=31)
    yield w
    del w
    _release()


@pytest.mark.parametrize("H", [128, 64])
def test_pair_kernel_offsets_past_2_31_flat_and_paged(c4_pool, H):
    """decode_tc3_kernel (64 and 128 heads) on the c4 pool: rows at
    num_slots - 1, around slot 3,273,603 and spread above it; the paged entry
    point over a block table whose pages sit at the top of the pool gives the
    same bits as the flat one."""
    w = c4_pool
    n = w.kv.view(-1, 656).shape[0]
    assert n == C4_SLOTS
    rng = np.random.default_rng(H)
    B = 4
    slots = _place_past_boundary(w.slots[:B], n, rng)
    q = torch.randn((B, H, 576), generator=torch.Generator().manual_seed(H)).bfloat16().cuda()
    assert decode_kernel_name(B, H, 1, 2048).startswith("decode_tc3_kernel")
    out, lse = fp8_ds_mla_sparse_decode(q, w.kv, slots, w.sm_scale, return_lse=True)
    _check_requests(out, lse, q, w.kv, slots, w.sm_scale, range(B))

    # paged: request r's block table points at the last pages of the pool
    n_pages = n // 64
    pages_per_req = 64
    bt = torch.arange(n_pages - 1, n_pages - 1 - B * pages_per_req, -1, dtype=torch.int32)
    bt = bt.view(B, pages_per_req).cuda()
    tok = torch.stack([torch.randperm(pages_per_req * 64, generator=torch.Generator().manual_seed(r))
                       [:2048] for r in range(B)]).to(torch.int32).cuda()
    tok[:, ::17] = -1
    req = torch.arange(B, dtype=torch.int32, device="cuda")
    fused, fused_lse = fp8_ds_mla_sparse_decode_paged(q, w.kv, req, bt, tok, w.sm_scale,
                                                      block_size=64, return_lse=True)
    valid = tok >= 0
    flat_slots = torch.where(valid, bt.gather(1, (tok.clamp(min=0) // 64).long()) * 64 + tok % 64,
                             torch.full_like(tok, -1)).to(torch.int32)
    assert int(flat_slots[flat_slots >= 0].min()) > BOUNDARY_SLOT
    flat, flat_lse = fp8_ds_mla_sparse_decode(q, w.kv, flat_slots, w.sm_scale, return_lse=True)
    torch.cuda.synchronize()
    assert torch.equal(fused, flat) and torch.equal(fused_lse, flat_lse)
    _check_requests(fused, fused_lse, q, w.kv, flat_slots, w.sm_scale, (0, B - 1))


@pytest.mark.parametrize("H", [128, 16])
def test_fp32_q_kernel_offsets_past_2_31(c4_pool, H):
    """decode_mma_kernel (fp32 q) reads the same high rows correctly."""
    w = c4_pool
    n = w.kv.view(-1, 656).shape[0]
    rng = np.random.default_rng(100 + H)
    B = 2
    slots = _place_past_boundary(w.slots[:B], n, rng)
    q = torch.randn((B, H, 576), generator=torch.Generator().manual_seed(7 + H)).cuda()
    assert decode_kernel_name(B, H, 1, 2048, torch.float32).startswith("decode_mma_kernel")
    out, lse = fp8_ds_mla_sparse_decode(q, w.kv, slots, w.sm_scale, return_lse=True)
    _check_requests(out, lse, q, w.kv, slots, w.sm_scale, range(B))


def test_small_head_kernel_offsets_past_2_31_on_c4_pool(c4_pool):
    """decode_ws_kernel (TMA gather4 rows) on the same top rows."""
    w = c4_pool
    n = w.kv.view(-1, 656).shape[0]
    slots = _place_past_boundary(w.slots[:3], n, np.random.default_rng(5))
    q = torch.randn((3, 16, 576), generator=torch.Generator().manual_seed(5)).bfloat16().cuda()
    assert decode_kernel_name(3, 16, 1, 2048, torch.bfloat16, 4).startswith("decode_ws_kernel")
    out, lse = fp8_ds_mla_sparse_decode(q, w.kv, slots, w.sm_scale, return_lse=True, num_kv_splits=4)
    _check_requests(out, lse, q, w.kv, slots, w.sm_scale, range(3))


def test_c4_full_shape_edges_a_b_at_the_golden_path_tolerance(c4_pool):
    """c4 at full size (B=32, H=64, top-k 2048, 4,194,304 slots) with edges
    (a) the leading 512 indices of 8 requests masked and (b) offsets past 2^31
    (a random permutation of the pool's pages: about a fifth of all selected
    slots are above 3,273,603), on ~N(0,1) latents: max-abs <= 2e-2 and cosine
    >= 0.9999 against the fp32 golden path on a subset, batch invariance on
    the rest."""
    w = c4_pool
    n = w.kv.view(-1, 656).shape[0]
    B = w.slots.shape[0]
    assert B == 32 and (w.slots[:8, :512] == -1).all()
    high = (w.slots > BOUNDARY_SLOT).float().mean().item()
    assert high > 0.1, high
    # two splits: the count the library picks for 32 pairs of this shape
    assert decode_kernel_name(B, 64, 1, 2048) == "decode_tc3_kernel+merge_splits_kernel"
    out, lse = fp8_ds_mla_sparse_decode(w.q, w.kv, w.slots, w.sm_scale, return_lse=True,
                                        num_kv_splits=2)
    _check_requests(out, lse, w.q, w.kv, w.slots, w.sm_scale, (0, 7, 8, 19, 31))
    for b in (3, 12, 27):
        one = fp8_ds_mla_sparse_decode(w.q[b:b + 1], w.kv, w.slots[b:b + 1], w.sm_scale,
                                       num_kv_splits=2)
        assert torch.equal(one, out[b:b + 1]), b
    assert n == C4_SLOTS


def test_c4_full_shape_amax_spread_edge_c(cuda_device):
    """c4 edge (c): tile amax log-uniform in [1e-4, 1e4] plus zero tiles, at
    the full pool.  Scores reach ~1e4, so the softmax is argmax-like and bf16
    keys (the reference kernel's own operand precision,
    fp8_ds_mla_sparse_decode.py:164) move the result by up to ~1e4 against the
    fp32 golden path; the bar is the oracle with that operand rounding, within
    2e-2 of the output scale, and no further from the golden than that
    rounding itself is."""
    w = synthetic.make_device("c4", seed=32)
    try:
        out, lse = fp8_ds_mla_sparse_decode(w.q, w.kv, w.slots, w.sm_scale, return_lse=True)
        torch.cuda.synchronize()
        report = []
        for b in (0, 9, 30):
            rows, local = _rows_of(w.kv, w.slots[b])
            qf = w.q[b:b + 1].float().cpu().numpy()
            gold, gold_lse = O.sparse_decode(qf, rows, local[None], w.sm_scale, acc_dtype=np.float64)
            kr, kr_lse = O.sparse_decode(qf, rows, local[None], w.sm_scale, acc_dtype=np.float64,
                                         kernel_rounding=True)
            got = out[b:b + 1].float().cpu().numpy()
            scale = max(1.0, float(np.abs(gold).max()))
            U.assert_close(got, kr, max_abs=2e-2 * scale)
            lscale = max(1.0, float(np.abs(gold_lse[np.isfinite(gold_lse)]).max()))
            U.assert_lse_close(lse[b:b + 1].cpu().numpy(), kr_lse, max_abs=2e-2 * lscale)
            assert O.max_abs(got, gold) <= O.max_abs(kr, gold) + 2e-2 * scale
            assert O.cosine(got, gold) >= O.cosine(kr, gold) - 1e-4
            report.append((b, O.max_abs(got, kr), O.cosine(got, kr), O.max_abs(got, gold),
                           O.cosine(got, gold), O.max_abs(kr, gold), O.cosine(kr, gold), scale))
        for r in report:
            print("c4 edge (c) request %d: vs rounded oracle max-abs %.3e cos %.7f; vs golden "
                  "max-abs %.3e cos %.7f; rounded oracle vs golden max-abs %.3e cos %.7f; "
                  "output scale %.3e" % r)
        assert torch.isfinite(out.float()).all()
    finally:
        del w
        _release()


def test_c3_full_pool_eight_splits_subset(cuda_device):
    """c3 at its real size: B=256, H=16, top-k 2048, 3,500,032-slot pool,
    S=8; four requests against the oracle, one by batch invariance."""
    w = synthetic.make_device("c3", seed=33)
    try:
        assert w.kv.view(-1, 656).shape[0] == 3_500_032
        out, lse = fp8_ds_mla_sparse_decode(w.q, w.kv, w.slots, w.sm_scale, return_lse=True,
                                            num_kv_splits=8)
        _check_requests(out, lse, w.q, w.kv, w.slots, w.sm_scale, (0, 77, 128, 255))
        one = fp8_ds_mla_sparse_decode(w.q[200:201], w.kv, w.slots[200:201], w.sm_scale,
                                       num_kv_splits=8)
        assert torch.equal(one, out[200:201])
    finally:
        del w
        _release()


def test_c5_full_pool_subset(cuda_device):
    """c5's per-GPU shape: B=128, H=128, top-k 2048 over 128 disjoint
    65536-token contexts = 8,388,608 slots (5.5 GB; byte offsets up to
    5.5e9): four requests against the oracle, two by batch invariance."""
    w = synthetic.make_device("c5", seed=34)
    try:
        n = w.kv.view(-1, 656).shape[0]
        assert n == 8_388_608
        assert int(w.slots.max()) > 2 * BOUNDARY_SLOT
        assert decode_kernel_name(128, 128, 1, 2048) == "decode_tc3_kernel"
        out, lse = fp8_ds_mla_sparse_decode(w.q, w.kv, w.slots, w.sm_scale, return_lse=True)
        _check_requests(out, lse, w.q, w.kv, w.slots, w.sm_scale, (0, 45, 90, 127))
        for b in (17, 101):
            one = fp8_ds_mla_sparse_decode(w.q[b:b + 1], w.kv, w.slots[b:b + 1], w.sm_scale,
                                           num_kv_splits=1)
            assert torch.equal(one, out[b:b + 1]), b
        assert torch.isfinite(out.float()).all()
    finally:
        del w
        _release()
