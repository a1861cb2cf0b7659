"""CPU oracle for the fp8_ds_mla sparse-MLA decode path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by ``bench.py``'s CPU-baseline leg, as the checker.  The product
(``vllm_fp8kv`` + ``libfp8mla.so``) never imports it.

Two halves:

* byte/integer work (e4m3 <-> fp32, fp32 -> bf16, the 656-byte row parser,
  the cache writer, the block-table index converter) is restated in plain C
  (``fp8mla_oracle.c``) and called through ctypes;
* the fp32 golden decode (``sparse_decode``) is restated in numpy, following
  ``verify/reference.py:36-65`` (``ref_sparse_mla_decode``) plus the natural-log
  LSE of ``verify/run_all.py:145-151``.

Parity of this oracle with the reference itself is pinned by
``tests/test_oracle_golden.py`` against vectors the reference produced
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

NOPE, ROPE, TILE = 512, 64, 128
N_TILES = NOPE // TILE
ROW_BYTES = 656
SCALE_OFF = 512
ROPE_OFF = 528

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libfp8mla_oracle.so")
_lib = None


def build() -> str:
    """Compile the C half (``make -C oracle``); returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        L.oracle_e4m3_to_f32_n.argtypes = [P, I64, P]
        L.oracle_f32_to_e4m3_n.argtypes = [P, I64, P]
        L.oracle_f32_to_bf16_n.argtypes = [P, I64, P]
        L.oracle_dequant_rows.argtypes = [P, I64, P]
        L.oracle_ds_mla_write.argtypes = [P, I64, P, I64, P, I64, P, I64]
        L.oracle_convert_req_index.argtypes = [P, P, I64, I64, P, I64, I64, I64, I64, P, I64]
        for f in (L.oracle_e4m3_to_f32_n, L.oracle_f32_to_e4m3_n, L.oracle_f32_to_bf16_n,
                  L.oracle_dequant_rows, L.oracle_ds_mla_write, L.oracle_convert_req_index):
            f.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


# --------------------------------------------------------------- conversions
def e4m3_to_f32(u8: np.ndarray) -> np.ndarray:
    """float8_e4m3fn bytes -> fp32 (exact; 0x7F/0xFF -> NaN)."""
    u8 = np.ascontiguousarray(u8, dtype=np.uint8)
    out = np.empty(u8.shape, np.float32)
    lib().oracle_e4m3_to_f32_n(_ptr(u8), u8.size, _ptr(out))
    return out


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn bytes, RNE, non-saturating (torch's cast)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().oracle_f32_to_e4m3_n(_ptr(x), x.size, _ptr(out))
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), RNE, NaN -> 0x7FC0."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_f32_to_bf16_n(_ptr(x), x.size, _ptr(out))
    return out


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (returned as fp32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# --------------------------------------------------------------- row format
def dequant_rows(rows_u8: np.ndarray) -> np.ndarray:
    """(..., 656) uint8 -> (..., 576) fp32; verify/reference.py:22-33."""
    flat = np.ascontiguousarray(rows_u8, dtype=np.uint8).reshape(-1, ROW_BYTES)
    out = np.empty((flat.shape[0], NOPE + ROPE), np.float32)
    lib().oracle_dequant_rows(_ptr(flat), flat.shape[0], _ptr(out))
    return out.reshape(*rows_u8.shape[:-1], NOPE + ROPE)


def ds_mla_write(kv_c_bits: np.ndarray, k_pe_bits: np.ndarray, slot_mapping: np.ndarray,
                 cache: np.ndarray) -> None:
    """Quantize bf16 latent/rope into ``cache`` rows in place (tests/fakes.py:28-57)."""
    kv_c_bits = np.ascontiguousarray(kv_c_bits, dtype=np.uint16)
    k_pe_bits = np.ascontiguousarray(k_pe_bits, dtype=np.uint16)
    slots = np.ascontiguousarray(slot_mapping, dtype=np.int64)
    assert cache.dtype == np.uint8 and cache.flags["C_CONTIGUOUS"]
    flat = cache.reshape(-1, ROW_BYTES)
    n = kv_c_bits.shape[0]
    lib().oracle_ds_mla_write(_ptr(kv_c_bits), kv_c_bits.shape[1], _ptr(k_pe_bits),
                              k_pe_bits.shape[1], _ptr(slots), n, _ptr(flat), flat.shape[0])


def quantize_rows(kv_bits: np.ndarray) -> np.ndarray:
    """bf16 (n, 576) bit patterns -> packed (n, 656) rows (verify/reference.py:68-91)."""
    n = kv_bits.shape[0]
    cache = np.zeros((n, ROW_BYTES), np.uint8)
    ds_mla_write(kv_bits[:, :NOPE], kv_bits[:, NOPE:], np.arange(n, dtype=np.int64), cache)
    return cache


def convert_req_index(req_id, block_table, token_idx, block_size: int) -> np.ndarray:
    """Token-relative -> flat slot (vLLM sparse_utils.py:85-104; tests/fakes.py:70-82)."""
    req_id = np.ascontiguousarray(req_id, dtype=np.int32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    ti = np.ascontiguousarray(token_idx, dtype=np.int32)
    T, topk = ti.shape
    out = np.empty((T, topk), np.int32)
    lib().oracle_convert_req_index(_ptr(req_id), _ptr(bt), bt.shape[1], bt.shape[1],
                                   _ptr(ti), topk, T, topk, block_size, _ptr(out), topk)
    return out


# --------------------------------------------------------------- decode
def sparse_decode(q: np.ndarray, kv_u8: np.ndarray, indices: np.ndarray, sm_scale: float,
                  *, acc_dtype=np.float32, kernel_rounding: bool = False):
    """fp32 golden sparse-MLA decode + natural-log LSE.

    Restates ``ref_sparse_mla_decode`` (verify/reference.py:36-65): for each
    query token, keep the indices in [0, num_slots), gather then dequantize
    those rows, softmax(q . k^T * sm_scale) over them, and attend over the NoPE
    half (V = the first 512 dims of the same rows).  A row that selects nothing
    yields zeros.  LSE = logsumexp(q . k^T * sm_scale) as in
    verify/run_all.py:145-151, and -inf for an empty row (the kernel contract
    of vllm_fp8kv/fp8_ds_mla_sparse_decode.py:209-211).

    ``indices`` is [T, topk] or [T, G, topk]; head h reads group h // (H // G)
    (fp8_ds_mla_sparse_decode.py:115).  ``q`` is fp32 values (bf16 queries are
    passed widened).  ``kernel_rounding`` additionally rounds q and the
    dequantized keys to bf16, the operand precision of the tensor-core path
    (fp8_ds_mla_sparse_decode.py:164, :171).
    """
    q = np.asarray(q, dtype=np.float32)
    T, H, D = q.shape
    assert D == NOPE + ROPE
    idx = np.asarray(indices)
    if idx.ndim == 2:
        idx = idx[:, None, :]
    G = idx.shape[1]
    assert H % G == 0
    hpg = H // G
    rows = kv_u8.reshape(-1, ROW_BYTES)
    n_slots = rows.shape[0]
    out = np.zeros((T, H, NOPE), np.float32)
    lse = np.full((T, H), -np.inf, np.float32)
    qq = round_bf16(q) if kernel_rounding else q
    for t in range(T):
        for g in range(G):
            sel = idx[t, g]
            sel = sel[(sel >= 0) & (sel < n_slots)].astype(np.int64)
            if sel.size == 0:
                continue
            k = dequant_rows(rows[sel])
            if kernel_rounding:
                k = round_bf16(k)
            qh = qq[t, g * hpg:(g + 1) * hpg].astype(acc_dtype)
            kk = k.astype(acc_dtype)
            s = (qh @ kk.T) * acc_dtype(sm_scale)
            m = s.max(axis=-1, keepdims=True)
            e = np.exp(s - m)
            z = e.sum(axis=-1, keepdims=True)
            w = e / z
            out[t, g * hpg:(g + 1) * hpg] = (w @ kk[:, :NOPE]).astype(np.float32)
            lse[t, g * hpg:(g + 1) * hpg] = (m + np.log(z))[:, 0].astype(np.float32)
    return out, lse


def choose_num_splits(T: int, H: int, G: int, topk: int, sm_count: int) -> int:
    """Split-count heuristic of tests/fixtures/triton_mla_sparse_kernel_pr47629.py:406-423."""
    head_blocks = G * -(-(H // G) // min(16, H // G))
    baseline = T * head_blocks
    if baseline == 0 or baseline * 4 >= sm_count:
        return 1
    ideal = 1
    while ideal < max(1, topk // 128):
        ideal *= 2
    max_splits = max(1, sm_count // baseline)
    max_splits = 1 << (max_splits.bit_length() - 1)
    n = min(ideal, max_splits)
    while n > 1 and topk % n != 0:
        n //= 2
    return max(1, n)


# --------------------------------------------------------------- metrics
def max_abs(a, b) -> float:
    """verify/metrics.py:8-9."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max()) if a.size else 0.0


def cosine(a, b) -> float:
    """verify/metrics.py:12-16 (torch cosine_similarity clamps the norms at 1e-8)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if a.size == 0:
        return 1.0
    na = max(np.linalg.norm(a), 1e-8)
    nb = max(np.linalg.norm(b), 1e-8)
    return float(a @ b / (na * nb))


# --------------------------------------------------------------- DSA indexer
# The indexer of the sparse-MLA models scores every context token for each
# query token and keeps the top-k positions that the decode then reads.  Its
# key cache is a paged fp8 format of its own: per page of `block_size` tokens,
# block_size x 128 e4m3 bytes followed by block_size fp32 scales (structure of
# arrays; 8448 B at block_size 64, reference PORT_PLAN.md:14 and its trap 3).
# The reference repository ships no code for this path; these restatements
# follow vLLM 0.22's torch restatement of DeepGEMM's test reference
# (installed vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:256-354,
# ``fp8_paged_mqa_logits_torch``, and :572-600, ``_topk_indices_torch``),
# against which tests/golden/indexer.npz pins them.
IDX_DIM = 128


def indexer_page_bytes(block_size: int) -> int:
    return block_size * (IDX_DIM + 4)


def indexer_limit(context_len: int, next_n: int, n: int) -> int:
    """Positions [0, limit) that query token n of next_n may score: the draft
    tokens of a request sit at the end of its context, so token n sees up to
    position context_len - next_n + n."""
    return int(context_len) - next_n + n + 1


def indexer_logits(q_u8: np.ndarray, kv_pages: np.ndarray, weights: np.ndarray,
                   context_lens: np.ndarray, block_table: np.ndarray,
                   max_model_len: int) -> np.ndarray:
    """fp8 paged MQA logits.

    q_u8      [B, next_n, H, 128] e4m3 bytes
    kv_pages  [num_blocks, block_size * 132] uint8 pages (SoA as above)
    weights   [B * next_n, H] fp32 (the query scale folded in by the caller)
    -> logits [B * next_n, max_model_len] fp32:
       sum_h relu(q[b, n, h] . k_s) * weights[b*next_n + n, h] * scale_s for
       s < indexer_limit(context_len_b, next_n, n), -inf elsewhere.
    Accumulated in fp64 (the reference's fp32 sums differ by rounding only).
    """
    q_u8 = np.asarray(q_u8, np.uint8)
    B, nn, H, D = q_u8.shape
    assert D == IDX_DIM
    pages = np.asarray(kv_pages, np.uint8).reshape(kv_pages.shape[0], -1)
    bs = pages.shape[1] // (D + 4)
    q = e4m3_to_f32(q_u8).astype(np.float64).reshape(B, nn * H, D)
    w = np.asarray(weights, np.float64).reshape(B, nn, H)
    out = np.full((B * nn, max_model_len), -np.inf, np.float32)
    for b in range(B):
        ctx = int(context_lens[b])
        if ctx <= 0:
            continue
        npg = -(-ctx // bs)
        pg = pages[np.asarray(block_table[b, :npg], np.int64)]
        k = e4m3_to_f32(pg[:, : bs * D]).astype(np.float64).reshape(npg * bs, D)
        scale = np.ascontiguousarray(pg[:, bs * D:]).view(np.float32).reshape(npg * bs)
        s = np.maximum(k @ q[b].T, 0.0).reshape(npg * bs, nn, H)
        lg = (s * w[b][None]).sum(-1) * scale.astype(np.float64)[:, None]
        for n in range(nn):
            lim = min(indexer_limit(ctx, nn, n), max_model_len)
            if lim > 0:
                out[b * nn + n, :lim] = lg[:lim, n].astype(np.float32)
    return out


def _sortable_keys(v: np.ndarray) -> np.ndarray:
    """fp32 -> uint32 keys whose unsigned order is the float order (NaN with
    the sign bit clear sorts above +inf, as torch.topk ranks NaN highest)."""
    u = np.ascontiguousarray(v, np.float32).view(np.uint32)
    return np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)


def indexer_topk(logits: np.ndarray, next_n: int, context_lens: np.ndarray,
                 topk: int) -> np.ndarray:
    """Top-k positions per logits row -> [rows, topk] int32.

    Row r = b * next_n + n keeps positions [0, limit) (indexer_limit).  With
    limit <= topk every position is kept; otherwise the topk largest logits,
    ties at the threshold broken by the lower position.  The kept positions are
    written in ascending order, then -1 (the decode's masked entry) pads the
    row.  The set equals torch.topk's on untied values; the order is not part
    of the contract (the decode treats indices as a set).
    """
    logits = np.asarray(logits, np.float32)
    rows, L = logits.shape
    out = np.full((rows, topk), -1, np.int32)
    for r in range(rows):
        b, n = divmod(r, next_n)
        lim = min(L, indexer_limit(int(context_lens[b]), next_n, n))
        if lim <= 0:
            continue
        if lim <= topk:
            out[r, :lim] = np.arange(lim, dtype=np.int32)
            continue
        key = _sortable_keys(logits[r, :lim]).astype(np.int64)
        order = np.lexsort((np.arange(lim), -key))
        out[r] = np.sort(order[:topk]).astype(np.int32)
    return out


def indexer_quantize(k_f32: np.ndarray, block_size: int = 64) -> np.ndarray:
    """Pack [N, 128] fp32 keys into SoA pages: per token scale = amax / 448
    (1 for an all-zero row), bytes = e4m3(k / scale).  Test data only: the
    indexer's own cache writer is not part of this library."""
    k = np.asarray(k_f32, np.float32)
    N, D = k.shape
    assert D == IDX_DIM and N % block_size == 0
    amax = np.abs(k).max(axis=1)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    q8 = f32_to_e4m3((k / scale[:, None]).astype(np.float32))
    nb = N // block_size
    pages = np.empty((nb, block_size * (D + 4)), np.uint8)
    pages[:, : block_size * D] = q8.reshape(nb, block_size * D)
    pages[:, block_size * D:] = scale.reshape(nb, block_size).view(np.uint8).reshape(nb, block_size * 4)
    return pages
