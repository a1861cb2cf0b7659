"""GPU parity of the DSA indexer read path (fp8 paged MQA logits, per-row
top-k) against the oracle and the golden vectors from vLLM's torch
restatement of DeepGEMM's reference (tests/golden/make_indexer_golden.py).

Logits: the e4m3 x e4m3 products are exact and the tensor cores sum 128 of
them in fp32, so the kernel differs from the fp64 oracle by accumulation
rounding only: max-abs <= 1e-3 of the row's largest |logit|.  Top-k: the
kernel's selection over its own logits equals the oracle's selection over the
same logits exactly (ascending positions, ties to the lower position), and
overlaps the selection over the oracle's logits by >= 99%.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import gpu_util as U
from tests.conftest import golden
from vllm_fp8kv import synthetic
from vllm_fp8kv.indexer import fp8_paged_mqa_logits, indexer_topk

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _run(q_u8, pages, w, ctx, bt, max_len, topk):
    q = torch.from_numpy(np.ascontiguousarray(q_u8)).cuda().view(torch.float8_e4m3fn)
    kv = torch.from_numpy(np.ascontiguousarray(pages)).cuda().view(-1, 64, 1, 132)
    wt = torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda()
    ct = torch.from_numpy(np.ascontiguousarray(ctx, np.int32)).cuda()
    btt = torch.from_numpy(np.ascontiguousarray(bt, np.int32)).cuda()
    logits = fp8_paged_mqa_logits(q, kv, wt, ct, btt, None, max_len)
    top = indexer_topk(logits, q_u8.shape[1], ct, topk)
    torch.cuda.synchronize()
    return logits.cpu().numpy(), top.cpu().numpy()


def _check_logits(got, want):
    assert np.array_equal(np.isneginf(got), np.isneginf(want)), "masked positions differ"
    for r in range(got.shape[0]):
        fin = np.isfinite(want[r])
        if fin.any():
            scale = max(1e-30, float(np.abs(want[r][fin]).max()))
            err = float(np.abs(got[r][fin] - want[r][fin]).max())
            assert err <= REL_TOL * scale, (r, err, scale)


def _check_topk(top, logits_gpu, logits_ref, next_n, ctx, topk):
    own = O.indexer_topk(logits_gpu, next_n, ctx, topk)
    assert np.array_equal(top, own), "selection over the same logits differs"
    ref = O.indexer_topk(logits_ref, next_n, ctx, topk)
    a = top[top >= 0].size
    inter = sum(len(set(top[r][top[r] >= 0]) & set(ref[r][ref[r] >= 0])) for r in range(top.shape[0]))
    assert a == ref[ref >= 0].size
    assert inter >= 0.99 * max(a, 1), (inter, a)


@pytest.mark.parametrize("name", ["n1", "n2"])
def test_indexer_matches_vllm_reference_golden(cuda_device, name):
    g = golden("indexer.npz")
    c = {k.split("__", 1)[1]: g[k] for k in g.files if k.startswith(name + "__")}
    nn, k, L = int(c["next_n"]), int(c["k"]), int(c["max_len"])
    logits, top = _run(c["q"], c["pages"], c["w"], c["ctx"], c["bt"], L, k)
    _check_logits(logits, c["logits"])
    ora = O.indexer_logits(c["q"], c["pages"], c["w"], c["ctx"], c["bt"], L)
    _check_logits(logits, ora)
    _check_topk(top, logits, ora, nn, c["ctx"], k)
    for r in range(top.shape[0]):  # same sets as torch.topk over the golden logits
        assert set(top[r][top[r] >= 0]) == set(c["topk"][r][c["topk"][r] >= 0]), r


def _random_case(seed, B, next_n, ctx, num_blocks, max_len, bad_block=False):
    rng = np.random.default_rng(seed)
    keys = rng.standard_normal((num_blocks * 64, 128)).astype(np.float32)
    pages = O.indexer_quantize(keys, 64)
    q = O.f32_to_e4m3(rng.standard_normal((B, next_n, 64, 128)).astype(np.float32))
    q = q.reshape(B, next_n, 64, 128)
    w = (rng.standard_normal((B * next_n, 64)) / 8).astype(np.float32)
    maxb = -(-max_len // 64)
    bt = np.stack([rng.permutation(num_blocks)[:maxb] for _ in range(B)]).astype(np.int32)
    ctx = np.asarray(ctx, np.int32)
    for b in range(B):  # entries past the context are junk the kernel must not read
        bt[b, -(-int(ctx[b]) // 64):] = -7
    if bad_block:
        bt[0, 1] = num_blocks + 5  # an id outside the cache inside the context: scores -inf
    return q, pages, w, ctx, bt


@pytest.mark.parametrize("next_n", [1, 2])
def test_indexer_long_contexts_against_oracle(cuda_device, next_n):
    """Contexts up to 20000 tokens, ragged ends, several CTAs per request."""
    ctx = [20000, 4097, 64, 1, 12345, 128, 0, 9999][: 8]
    q, pages, w, c, bt = _random_case(11 + next_n, 8, next_n, ctx, 2048, 20480)
    logits, top = _run(q, pages, w, c, bt, 20480, 2048)
    ora = O.indexer_logits(q, pages, w, c, bt, 20480)
    _check_logits(logits, ora)
    _check_topk(top, logits, ora, next_n, c, 2048)
    # short rows: every position ascending, then -1; empty context: all -1
    assert top[2 * next_n + next_n - 1][:64].tolist() == list(range(64))
    assert (top[2 * next_n + next_n - 1][64:] == -1).all()
    assert (top[6 * next_n: 7 * next_n] == -1).all()
    assert np.isneginf(logits[6 * next_n: 7 * next_n]).all()


def test_indexer_block_ids_outside_the_cache_score_minus_inf(cuda_device):
    q, pages, w, c, bt = _random_case(5, 2, 1, [300, 200], 64, 384, bad_block=True)
    logits, _ = _run(q, pages, w, c, bt, 384, 128)
    assert np.isneginf(logits[0, 64:128]).all()  # block 1 of request 0 is outside the cache
    assert np.isfinite(logits[0, :64]).all() and np.isfinite(logits[0, 128:300]).all()
    bt_ok = bt.copy()
    bt_ok[0, 1] = 0
    ora = O.indexer_logits(q, pages, w, c, bt_ok, 384)
    ora[0, 64:128] = -np.inf
    _check_logits(logits, ora)


def test_indexer_topk_ties_keep_the_lower_positions(cuda_device):
    rng = np.random.default_rng(9)
    L = 5000
    lg = rng.integers(0, 16, size=(3, L)).astype(np.float32)  # heavy ties
    lg[1, 4000:] = -np.inf
    ctx = np.array([5000, 4000, 5000], np.int32)
    t = torch.from_numpy(lg).cuda()
    top = indexer_topk(t, 1, torch.from_numpy(ctx).cuda(), 1000).cpu().numpy()
    assert np.array_equal(top, O.indexer_topk(lg, 1, ctx, 1000))


def test_indexer_topk_feeds_the_paged_decode(cuda_device):
    """The chain a DSA layer runs: indexer logits -> top-k positions ->
    paged fp8 decode over the same requests' block tables.  The decode of the
    kernel's positions equals the decode of the oracle's positions when the two
    sets agree, and is finite."""
    from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode_paged

    B, ctx_len, topk = 4, 4096, 512
    q, pages, w, c, bt = _random_case(21, B, 1, [ctx_len] * B, 512, ctx_len)
    logits, top = _run(q, pages, w, c, bt, ctx_len, topk)
    s = synthetic.Shape("dsa", B=B, H=128, topk=topk, ctx=ctx_len, pool_slots=B * ctx_len)
    wk = synthetic.make_host(s, seed=22)
    pool = U.device_pool(wk.kv_src_bits, check_against_oracle=False)
    qd = U.bf16_tensor(wk.q_bits)
    req = torch.arange(B, dtype=torch.int32, device="cuda")
    btd = torch.from_numpy(wk.block_table).cuda()
    out = fp8_ds_mla_sparse_decode_paged(qd, pool, req, btd, torch.from_numpy(top).cuda(), wk.sm_scale)
    slots = O.convert_req_index(np.arange(B, dtype=np.int32), wk.block_table, top, 64)
    ref, _ = O.sparse_decode(synthetic.bf16_to_f32(wk.q_bits), pool.view(-1, 656).cpu().numpy(),
                             slots, wk.sm_scale)
    U.assert_close(out.float().cpu().numpy(), ref)


def test_indexer_topk_rows_longer_than_the_resident_limit(cuda_device):
    """Rows above 48 K positions take two write rounds in each CTA of the
    pair: same result as the oracle, ties included."""
    rng = np.random.default_rng(10)
    L = 70000
    lg = rng.standard_normal((2, L)).astype(np.float32)
    lg[0, ::3] = 0.5  # a large tie class near the threshold
    ctx = np.array([L, 65000], np.int32)
    top = indexer_topk(torch.from_numpy(lg).cuda(), 1, torch.from_numpy(ctx).cuda(), 2048).cpu().numpy()
    assert np.array_equal(top, O.indexer_topk(lg, 1, ctx, 2048))


def test_indexer_topk_rows_at_the_pair_limit(cuda_device):
    """Rows of exactly 92,160 positions, the longest the CTA pair keeps in
    shared memory (46 K keys per CTA), and one position more (the single-CTA
    kernel), in one call each: both equal the oracle, ties included."""
    rng = np.random.default_rng(16)
    for L in (92160, 92161):
        lg = rng.standard_normal((2, L)).astype(np.float32)
        lg[1, ::5] = 0.75  # a tie class near the threshold
        ctx = np.array([L, L - 1], np.int32)
        top = indexer_topk(torch.from_numpy(lg).cuda(), 1, torch.from_numpy(ctx).cuda(), 2048).cpu().numpy()
        assert np.array_equal(top, O.indexer_topk(lg, 1, ctx, 2048)), L


def test_indexer_topk_row_in_one_first_pass_bin(cuda_device):
    """Every logit in [1, 1.25) shares the first pass's 11-bit bin, more keys
    than the compacted candidate list holds: the refining passes then scan the
    whole row.  Ties (values on a 1/4096 grid) resolve to the lower positions."""
    rng = np.random.default_rng(12)
    L = 32768
    lg = (1.0 + rng.integers(0, 1024, size=(3, L)) / 4096.0).astype(np.float32)
    lg[2, :5000] = 1.0  # a tie class at the bottom
    ctx = np.array([L, 30000, L], np.int32)
    top = indexer_topk(torch.from_numpy(lg).cuda(), 1, torch.from_numpy(ctx).cuda(), 2048).cpu().numpy()
    assert np.array_equal(top, O.indexer_topk(lg, 1, ctx, 2048))


def test_indexer_topk_rows_above_the_pair_limit(cuda_device):
    """Rows of more than 92,160 positions take the single-CTA kernel that
    re-reads the row per pass; a short row in the same call leaves early."""
    rng = np.random.default_rng(14)
    L = 100000
    lg = rng.standard_normal((2, L)).astype(np.float32)
    lg[0, ::7] = 0.25  # a tie class
    ctx = np.array([L, 1500], np.int32)
    top = indexer_topk(torch.from_numpy(lg).cuda(), 1, torch.from_numpy(ctx).cuda(), 2048).cpu().numpy()
    assert np.array_equal(top, O.indexer_topk(lg, 1, ctx, 2048))
