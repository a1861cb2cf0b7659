"""GPU parity of the sm_100a decode against the oracle and the reference's golden vectors.

Mirrors the reference's decode tests (tests/test_sparse_decode.py:44-194) and
harness sections (verify/run_all.py:78-185), with the decode's stated tolerance:
max-abs <= 2e-2 and cosine >= 0.9999 against the fp32 golden path.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import gpu_util as U
from tests.conftest import golden
from vllm_fp8kv import synthetic
from vllm_fp8kv.fp8_ds_mla_sparse_decode import NOPE, ROW_BYTES, fp8_ds_mla_sparse_decode

pytestmark = pytest.mark.gpu


def _run(q, pool, idx, sm, **kw):
    out, lse = fp8_ds_mla_sparse_decode(q, pool, idx, sm, return_lse=True, **kw)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


# ------------------------------------------------------------ golden fixtures
@pytest.mark.parametrize("splits", [None, 1, 2, 4])
def test_c1_matches_reference_golden(cuda_device, splits):
    g = golden("decode_c1.npz")
    w = synthetic.make_host("c1", seed=0)
    pool = U.device_pool(w.kv_src_bits)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    out, lse = _run(q, pool, idx, float(g["sm_scale"]), num_kv_splits=splits)
    U.assert_close(out, g["ref_out"])
    U.assert_lse_close(lse, g["ref_lse"])
    # tighter: the oracle with the tensor-core operand rounding
    ko, _ = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits), pool.view(-1, 656).cpu().numpy(),
                            w.slots, float(g["sm_scale"]), kernel_rounding=True)
    U.assert_close(out, ko, max_abs=U.MAX_ABS_KERNEL_ROUNDING)


TRAPS = ["masked", "leading_one", "leading_48", "empty_row", "out_of_range",
         "groups2_h32", "heads8", "matrix_q4"]


@pytest.mark.parametrize("case", TRAPS)
@pytest.mark.parametrize("qdtype", [torch.float32, torch.bfloat16])
def test_trap_cases_match_reference(cuda_device, case, qdtype):
    g = golden("traps.npz")
    q = torch.from_numpy(g[f"{case}__q"]).cuda().to(qdtype)
    pool = torch.from_numpy(g[str(g[f"{case}__pool"])]).cuda()
    idx = torch.from_numpy(g[f"{case}__idx"]).cuda()
    out, lse = _run(q, pool, idx, float(g["sm_scale"]))
    assert out.dtype == np.float32
    ref_q = q.float().cpu().numpy()
    ref, ref_lse = O.sparse_decode(ref_q, g[str(g[f"{case}__pool"])], g[f"{case}__idx"],
                                   float(g["sm_scale"]))
    U.assert_close(out, ref)
    U.assert_lse_close(lse, ref_lse)
    if qdtype == torch.float32:   # same inputs as the reference's own kernel run
        U.assert_close(out, g[f"{case}__ref_out"])


def test_empty_row_is_zero_with_minus_inf_lse(cuda_device):
    g = golden("traps.npz")
    q = torch.from_numpy(g["empty_row__q"]).cuda().bfloat16()
    pool = torch.from_numpy(g[str(g["empty_row__pool"])]).cuda()
    idx = torch.from_numpy(g["empty_row__idx"]).cuda()
    for splits in (1, 2, 8):
        out, lse = _run(q, pool, idx, float(g["sm_scale"]), num_kv_splits=splits)
        assert not out[1].any() and np.isneginf(lse[1]).all()
        assert out[0].any() and np.isfinite(lse[0]).all()


def test_leading_fully_masked_splits_do_not_poison(cuda_device):
    """Fully masked leading chunks AND whole leading splits: no NaN, the rest
    of the row unchanged."""
    w = synthetic.make_host("c1", seed=3)
    pool = U.device_pool(w.kv_src_bits)
    slots = w.slots.copy()
    slots[:, :192] = -1                       # 3 of 4 splits of 64 fully masked
    q = U.bf16_tensor(w.q_bits)
    ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits), pool.view(-1, 656).cpu().numpy(),
                                   slots, w.sm_scale)
    for splits in (1, 2, 4, 8):
        out, lse = _run(q, pool, torch.from_numpy(slots).cuda(), w.sm_scale, num_kv_splits=splits)
        U.assert_close(out, ref)
        U.assert_lse_close(lse, ref_lse)


def test_2d_and_3d_indices_and_fp8_view_and_paged_shape_agree(cuda_device):
    w = synthetic.make_host("c1", seed=4)
    pool = U.device_pool(w.kv_src_bits)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    a = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale)
    b = fp8_ds_mla_sparse_decode(q, pool.view(-1, ROW_BYTES), idx.unsqueeze(1), w.sm_scale)
    c = fp8_ds_mla_sparse_decode(q, pool.view(torch.float8_e4m3fn), idx, w.sm_scale)
    assert torch.equal(a, b) and torch.equal(a, c)


def test_tuning_kwargs_do_not_change_the_result(cuda_device):
    w = synthetic.make_host("c1", seed=5)
    pool = U.device_pool(w.kv_src_bits)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    a = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, block_n=16)
    b = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, block_n=32, num_warps=8)
    assert torch.equal(a, b)


def test_out_of_range_indices_issue_no_load(cuda_device):
    """Indices >= num_slots and < 0 behave as masked (the pool's last row is
    the boundary; nothing past it is read)."""
    w = synthetic.make_host("c1", seed=6)
    pool = U.device_pool(w.kv_src_bits)
    slots = w.slots.copy()
    slots[:, ::4] = 4096 + np.arange(slots[:, ::4].size).reshape(slots[:, ::4].shape)
    slots[:, 1::9] = np.iinfo(np.int32).max
    slots[:, 2::11] = np.iinfo(np.int32).min
    q = U.bf16_tensor(w.q_bits)
    out, lse = _run(q, pool, torch.from_numpy(slots).cuda(), w.sm_scale)
    ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits), pool.view(-1, 656).cpu().numpy(),
                                   slots, w.sm_scale)
    U.assert_close(out, ref)
    U.assert_lse_close(lse, ref_lse)


# ------------------------------------------------------------ benchmark shapes
def _shape_case(name, B, pool_slots, splits=None, seed=0):
    w = synthetic.make_host(name, seed=seed, B=B, pool_slots=pool_slots)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    out, lse = _run(q, pool, torch.from_numpy(w.slots).cuda(), w.sm_scale, num_kv_splits=splits)
    host_pool = pool.view(-1, 656).cpu().numpy()
    qf = synthetic.bf16_to_f32(w.q_bits)
    ref, ref_lse = O.sparse_decode(qf, host_pool, w.slots, w.sm_scale)
    U.assert_close(out, ref)
    U.assert_lse_close(lse, ref_lse)
    ko, _ = O.sparse_decode(qf, host_pool, w.slots, w.sm_scale, kernel_rounding=True)
    U.assert_close_rounded(out, ko)


def test_c2_shape_h128_topk2048(cuda_device):
    _shape_case("c2", B=4, pool_slots=4 * 32768)


def test_c3_shape_h16_eight_splits(cuda_device):
    _shape_case("c3", B=8, pool_slots=1 << 18, splits=8)


def test_c3_shape_large_grid_and_chunk_sizes_agree(cuda_device):
    """A grid of at least two CTAs per SM takes the 32-token-chunk general
    kernel (two CTAs share an SM); a small grid takes 64-token chunks.  Both
    match the oracle, and the same requests decoded either way agree."""
    w = synthetic.make_host("c3", seed=3, B=64, pool_slots=1 << 18)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    big, big_lse = _run(q, pool, idx, w.sm_scale, num_kv_splits=8)      # 512 CTAs
    host_pool = pool.view(-1, 656).cpu().numpy()
    qf = synthetic.bf16_to_f32(w.q_bits)
    ref, ref_lse = O.sparse_decode(qf, host_pool, w.slots, w.sm_scale)
    U.assert_close(big, ref)
    U.assert_lse_close(big_lse, ref_lse)
    small, small_lse = _run(q[:4], pool, idx[:4], w.sm_scale, num_kv_splits=8)  # 32 CTAs
    U.assert_close(small, big[:4], max_abs=U.MAX_ABS_KERNEL_ROUNDING)
    U.assert_lse_close(small_lse, big_lse[:4], max_abs=U.MAX_ABS_KERNEL_ROUNDING)


def test_c4_shape_h64_edge_cases(cuda_device):
    """c4: tile amax log-uniform in [1e-4, 1e4] + zero tiles, leading 512
    indices of 8 requests masked.  Latents up to 1e4 make the scores ~1e4, so
    the softmax is argmax-like and bf16 keys (the reference kernel's own
    operand precision, fp8_ds_mla_sparse_decode.py:164) can flip near-ties
    against the fp32 golden.  The bar: match the oracle with the reference
    kernel's operand rounding to 2e-2 of the output scale and cosine 0.9999,
    and be no further from the fp32 golden than that rounding itself is."""
    w = synthetic.make_host("c4", seed=0, B=10, pool_slots=10 * 131072)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    out, lse = _run(q, pool, torch.from_numpy(w.slots).cuda(), w.sm_scale)
    host_pool = pool.view(-1, 656).cpu().numpy()
    qf = synthetic.bf16_to_f32(w.q_bits)
    gold, gold_lse = O.sparse_decode(qf, host_pool, w.slots, w.sm_scale, acc_dtype=np.float64)
    kr, kr_lse = O.sparse_decode(qf, host_pool, w.slots, w.sm_scale, acc_dtype=np.float64,
                                 kernel_rounding=True)
    scale = max(1.0, float(np.abs(gold).max()))
    U.assert_close(out, kr, max_abs=2e-2 * scale)
    lscale = max(1.0, float(np.abs(gold_lse[np.isfinite(gold_lse)]).max()))
    U.assert_lse_close(lse, kr_lse, max_abs=2e-2 * lscale)
    assert O.max_abs(out, gold) <= O.max_abs(kr, gold) + 2e-2 * scale
    assert O.cosine(out, gold) >= O.cosine(kr, gold) - 1e-4
    # the masked-prefix requests stay finite and equal the unmasked suffix result
    assert np.isfinite(out[:8]).all()


@pytest.mark.parametrize("H", [1, 2, 8, 24, 48, 64, 96, 128, 256])
def test_head_counts(cuda_device, H):
    s = synthetic.Shape("h", B=2, H=H, topk=320, ctx=1024, pool_slots=4096, mask_frac=0.1)
    w = synthetic.make_host(s, seed=H)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    out, lse = _run(q, pool, torch.from_numpy(w.slots).cuda(), w.sm_scale)
    ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits),
                                   pool.view(-1, 656).cpu().numpy(), w.slots, w.sm_scale)
    U.assert_close(out, ref)
    U.assert_lse_close(lse, ref_lse)


@pytest.mark.parametrize("topk", [1, 16, 63, 64, 65, 200, 2048])
def test_ragged_topk(cuda_device, topk):
    s = synthetic.Shape("k", B=3, H=16, topk=topk, ctx=4096, pool_slots=16384)
    w = synthetic.make_host(s, seed=topk)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    for splits in (1, 3):
        out, lse = _run(q, pool, torch.from_numpy(w.slots).cuda(), w.sm_scale, num_kv_splits=splits)
        ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits),
                                       pool.view(-1, 656).cpu().numpy(), w.slots, w.sm_scale)
        U.assert_close(out, ref)
        U.assert_lse_close(lse, ref_lse)


def test_many_units_per_cta_with_padded_head_blocks_and_empty_splits(cuda_device):
    """The small-head kernel is persistent: with 800 units (100 tokens x head
    blocks of 16 and 8 heads x 4 splits, the last split empty) each CTA walks
    several units, so rows, Q and state cross unit boundaries."""
    from vllm_fp8kv import _native as N

    s = synthetic.Shape("u", B=100, H=24, topk=3, ctx=128, pool_slots=100 * 128, mask_frac=0.2)
    w = synthetic.make_host(s, seed=11)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    out, lse = _run(q, pool, torch.from_numpy(w.slots).cuda(), w.sm_scale, num_kv_splits=4)
    ref, ref_lse = O.sparse_decode(synthetic.bf16_to_f32(w.q_bits),
                                   pool.view(-1, 656).cpu().numpy(), w.slots, w.sm_scale)
    U.assert_close(out, ref)
    U.assert_lse_close(lse, ref_lse)
    assert N.device_status(reset=True) == 0


def test_topk_zero_gives_zeros(cuda_device):
    q = torch.randn(2, 16, 576, device="cuda").bfloat16()
    pool = torch.zeros(64, 656, dtype=torch.uint8, device="cuda")
    out, lse = fp8_ds_mla_sparse_decode(q, pool, torch.zeros(2, 0, dtype=torch.int32, device="cuda"),
                                        0.1, return_lse=True)
    assert not out.any() and torch.isneginf(lse).all()


def test_int64_offsets_past_2_31(cuda_device):
    """verify/run_all.py:155-185: slot * 656 > 2^31 in a 3.5M-slot pool."""
    n = 3_500_000
    kv = torch.zeros(n, 656, dtype=torch.uint8, device="cuda")
    rng = np.random.default_rng(7)
    src = synthetic.bf16_bits(rng.standard_normal((2, 576)).astype(np.float32) * 0.5)
    rows = O.quantize_rows(src)
    kv[0] = torch.from_numpy(rows[0]).cuda()
    kv[n - 1] = torch.from_numpy(rows[1]).cuda()
    q = U.bf16_tensor(synthetic.bf16_bits(rng.standard_normal((1, 16, 576)).astype(np.float32) * 0.5))
    idx = torch.tensor([[0, n - 1]], dtype=torch.int32, device="cuda")
    out, lse = _run(q, kv, idx, 576 ** -0.5)
    host = np.stack([rows[0], rows[1]])
    ref, ref_lse = O.sparse_decode(q.float().cpu().numpy(), host, np.array([[0, 1]], np.int32),
                                   576 ** -0.5)
    del kv
    torch.cuda.empty_cache()
    U.assert_close(out, ref)
    U.assert_lse_close(lse, ref_lse)


def test_full_c2_subset_against_oracle(cuda_device):
    """Full-size c2 (B=64, 2M-slot pool) built on the GPU; 4 requests checked
    against the oracle, the rest by batch invariance (each request alone gives
    the same bits as inside the batch)."""
    w = synthetic.make_device("c2", seed=1)
    out, lse = fp8_ds_mla_sparse_decode(w.q, w.kv, w.slots, w.sm_scale, return_lse=True)
    flat = w.kv.view(-1, 656)
    for b in (0, 17, 40, 63):
        sl = w.slots[b].long()
        ok = sl >= 0
        rows = flat[sl.clamp(min=0)].cpu().numpy()
        local = np.where(ok.cpu().numpy(), np.arange(sl.numel()), -1).astype(np.int32)
        ref, ref_lse = O.sparse_decode(w.q[b:b + 1].float().cpu().numpy(), rows, local[None],
                                       w.sm_scale)
        U.assert_close(out[b:b + 1].float().cpu().numpy(), ref)
        U.assert_lse_close(lse[b:b + 1].cpu().numpy(), ref_lse)
    # batch invariance at a fixed split count (the heuristic itself depends on T)
    one = fp8_ds_mla_sparse_decode(w.q[5:6], w.kv, w.slots[5:6], w.sm_scale, num_kv_splits=1)
    assert torch.equal(one, out[5:6])
    assert torch.isfinite(out.float()).all()
    del w
    torch.cuda.empty_cache()


def test_output_is_written_on_the_current_stream(cuda_device):
    w = synthetic.make_host("c1", seed=8)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    ref = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        got = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale)
    s.synchronize()
    assert torch.equal(ref, got)


def test_cuda_graph_capture_replays_identically(cuda_device):
    w = synthetic.make_host("c1", seed=9)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    ws = torch.empty(1 << 22, dtype=torch.uint8, device="cuda")
    eager = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, num_kv_splits=4, workspace=ws)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, num_kv_splits=4, workspace=ws)
        with torch.cuda.graph(g, stream=s):
            out = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, num_kv_splits=4, workspace=ws)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    del g


def test_no_on_chip_wait_timed_out(cuda_device):
    """Runs after the decode tests in this file: no bounded wait gave up."""
    from vllm_fp8kv import _native as N

    w = synthetic.make_host(synthetic.Shape("s", B=3, H=128, topk=200, ctx=2048, pool_slots=8192),
                            seed=11)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    fp8_ds_mla_sparse_decode(U.bf16_tensor(w.q_bits), pool, torch.from_numpy(w.slots).cuda(),
                             w.sm_scale)
    assert N.device_status(reset=True) == 0


def test_dispatch_by_heads_and_dtype(cuda_device):
    from vllm_fp8kv.fp8_ds_mla_sparse_decode import decode_kernel_name

    assert decode_kernel_name(64, 128, 1, 2048) == "decode_tc3_kernel"
    assert decode_kernel_name(64, 256, 2, 2048) == "decode_tc3_kernel"
    # 64 heads per group run on the pair kernel too (the odd CTA's rows are
    # padding); 32 tokens x 1 group would fill 32 of 74 SM pairs, so the
    # automatic split count doubles to 2
    assert decode_kernel_name(32, 64, 1, 2048) == "decode_tc3_kernel+merge_splits_kernel"
    assert decode_kernel_name(64, 128, 1, 2048, torch.float32) == "decode_mma_kernel"
    # small head counts with bf16 q: the persistent TMA-gather warp-MMA kernel
    assert decode_kernel_name(256, 16, 1, 2048, torch.bfloat16, 8) == \
        "decode_ws_kernel+merge_splits_kernel"
    assert decode_kernel_name(4, 8, 2, 256, torch.bfloat16, 1) == "decode_ws_kernel"
    assert decode_kernel_name(4, 16, 1, 256, torch.float32, 1) == "decode_mma_kernel"


# ------------------------------------------------------------ fused block-table conversion
@pytest.mark.parametrize("H,splits", [(128, 1), (128, 2), (16, 8), (16, None), (64, None)])
def test_paged_decode_equals_convert_then_decode(cuda_device, H, splits):
    """fp8mla_sparse_decode_paged == vLLM's converter followed by the flat
    decode, bit for bit: tokens of one request share a block table, positions
    past the table and masked positions decode as masked, and the table is a
    strided view."""
    from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode_paged
    from vllm_fp8kv.index_convert import convert_req_index_to_global_index

    shape = synthetic.Shape("paged", B=5, H=H, topk=256, ctx=4096, pool_slots=5 * 4096,
                            mask_frac=0.1)
    w = synthetic.make_host(shape, seed=H)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    T = 7
    rng = np.random.default_rng(H + 1)
    req = rng.integers(0, shape.B, size=T).astype(np.int32)          # several tokens per request
    tok = w.token_idx[req].copy()
    tok[:, 5::37] = shape.ctx + 64 * np.arange(tok[:, 5::37].shape[1])  # blocks past the table
    wide = np.full((shape.B, w.block_table.shape[1] + 3), 7, dtype=np.int32)
    wide[:, : w.block_table.shape[1]] = w.block_table
    bt = torch.from_numpy(wide).cuda()[:, : w.block_table.shape[1]]   # strided view
    req_t, tok_t = torch.from_numpy(req).cuda(), torch.from_numpy(tok).cuda()
    q = torch.randn((T, H, 576), generator=torch.Generator().manual_seed(H)).bfloat16().cuda()

    slots = convert_req_index_to_global_index(req_t, bt, tok_t, BLOCK_SIZE=64, NUM_TOPK_TOKENS=256)
    flat, flat_lse = fp8_ds_mla_sparse_decode(q, pool, slots, w.sm_scale, return_lse=True,
                                              num_kv_splits=splits)
    fused, fused_lse = fp8_ds_mla_sparse_decode_paged(q, pool, req_t, bt, tok_t, w.sm_scale,
                                                      block_size=64, return_lse=True,
                                                      num_kv_splits=splits)
    torch.cuda.synchronize()
    assert torch.equal(fused, flat) and torch.equal(fused_lse, flat_lse)

    ref_slots = O.convert_req_index(req, wide[:, : w.block_table.shape[1]], tok, 64)
    assert np.array_equal(slots.cpu().numpy(), ref_slots)
    ref, ref_lse = O.sparse_decode(q.float().cpu().numpy(), pool.view(-1, 656).cpu().numpy(),
                                   ref_slots, w.sm_scale)
    U.assert_close(fused.float().cpu().numpy(), ref)
    U.assert_lse_close(fused_lse.cpu().numpy(), ref_lse)


@pytest.mark.parametrize("H", [128, 16])
def test_paged_decode_with_non_power_of_two_pages(cuda_device, H):
    """Pages of 48 slots take the division path of the position -> block step
    (powers of two take a shift): still bit-identical to convert-then-decode."""
    from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode_paged
    from vllm_fp8kv.index_convert import convert_req_index_to_global_index

    bs, B, T, topk, max_blocks = 48, 3, 6, 256, 40
    shape = synthetic.Shape("paged48", B=B, H=H, topk=topk, ctx=1024, pool_slots=8192, mask_frac=0.1)
    w = synthetic.make_host(shape, seed=3)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    rng = np.random.default_rng(4)
    n_blocks = 8192 // bs
    bt = rng.integers(0, n_blocks, size=(B, max_blocks)).astype(np.int32)
    req = rng.integers(0, B, size=T).astype(np.int32)
    tok = np.stack([rng.choice(max_blocks * bs + 96, size=topk, replace=False) for _ in range(T)])
    tok = tok.astype(np.int32)
    tok[:, ::29] = -1
    q = torch.randn((T, H, 576), generator=torch.Generator().manual_seed(H)).bfloat16().cuda()
    req_t, bt_t, tok_t = (torch.from_numpy(x).cuda() for x in (req, bt, tok))
    slots = convert_req_index_to_global_index(req_t, bt_t, tok_t, BLOCK_SIZE=bs, NUM_TOPK_TOKENS=topk)
    assert np.array_equal(slots.cpu().numpy(), O.convert_req_index(req, bt, tok, bs))
    flat, flat_lse = fp8_ds_mla_sparse_decode(q, pool, slots, w.sm_scale, return_lse=True)
    fused, fused_lse = fp8_ds_mla_sparse_decode_paged(q, pool, req_t, bt_t, tok_t, w.sm_scale,
                                                      block_size=bs, return_lse=True)
    torch.cuda.synchronize()
    assert torch.equal(fused, flat) and torch.equal(fused_lse, flat_lse)


@pytest.mark.parametrize("next_n,H", [(2, 64), (3, 16)])
def test_shared_topk_equals_per_token_decode(cuda_device, next_n, H):
    """next_n query tokens of a request sharing one top-k row, decoded as one
    head group, give the per-token decode's result (each index row repeated)."""
    from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode_shared_topk

    B, topk = 4, 512
    s = synthetic.Shape("mtp", B=B, H=H, topk=topk, ctx=2048, pool_slots=B * 2048, mask_frac=0.1)
    w = synthetic.make_host(s, seed=next_n + H)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = torch.randn((B, next_n, H, 576), generator=torch.Generator().manual_seed(H)).bfloat16().cuda()
    idx = torch.from_numpy(w.slots).cuda()
    out, lse = fp8_ds_mla_sparse_decode_shared_topk(q, pool, idx, w.sm_scale, return_lse=True,
                                                    num_kv_splits=1)
    per_tok, per_lse = fp8_ds_mla_sparse_decode(q.view(B * next_n, H, 576), pool,
                                                idx.repeat_interleave(next_n, dim=0), w.sm_scale,
                                                return_lse=True, num_kv_splits=1)
    torch.cuda.synchronize()
    U.assert_close(out.float().cpu().numpy().reshape(B * next_n, H, 512),
                   per_tok.float().cpu().numpy())
    U.assert_lse_close(lse.cpu().numpy().reshape(B * next_n, H), per_lse.cpu().numpy())
    ref, ref_lse = O.sparse_decode(q.float().cpu().numpy().reshape(B * next_n, H, 576),
                                   pool.view(-1, 656).cpu().numpy(),
                                   np.repeat(w.slots, next_n, axis=0), w.sm_scale)
    U.assert_close(out.float().cpu().numpy().reshape(B * next_n, H, 512), ref)


def test_paged_decode_rejects_bad_tables(cuda_device):
    from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode_paged

    q = torch.zeros((1, 16, 576), dtype=torch.bfloat16, device="cuda")
    pool = torch.zeros((4, 64, ROW_BYTES), dtype=torch.uint8, device="cuda")
    req = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok = torch.zeros((1, 128), dtype=torch.int32, device="cuda")
    bt = torch.zeros((1, 4), dtype=torch.int32, device="cuda")
    with pytest.raises(AssertionError):
        fp8_ds_mla_sparse_decode_paged(q, pool, req, bt, tok, 0.1, block_size=0)
    with pytest.raises(AssertionError):
        fp8_ds_mla_sparse_decode_paged(q, pool, req.long(), bt, tok, 0.1)
