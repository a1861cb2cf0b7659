"""Helpers shared by the GPU parity tests (host workload -> device tensors)."""

import numpy as np
import torch

from oracle import oracle as O
from vllm_fp8kv import synthetic

# North-star tolerance for output and LSE vs the reference's fp32 golden path.
MAX_ABS = 2e-2
MIN_COS = 0.9999
# Against the oracle with bf16 operand rounding (the tensor-core operand
# precision) the only remaining differences are P's bf16 rounding and
# accumulation order.
MAX_ABS_KERNEL_ROUNDING = 5e-3
# Split-KV partials are stored as bf16 before the merge: one more rounding of a
# value of the output's size, at most one bf16 ulp (2^-8 relative).
BF16_ULP = 2.0 ** -8


def bf16_tensor(bits: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def device_pool(kv_src_bits: np.ndarray, device="cuda", check_against_oracle=True) -> torch.Tensor:
    """Quantize a bf16 [n, 576] source into an [n/64, 64, 656] pool with the
    library's writer; optionally assert byte equality with the oracle writer."""
    from vllm_fp8kv.cache_writer import concat_and_cache_ds_mla

    n = kv_src_bits.shape[0]
    src = bf16_tensor(kv_src_bits, device)
    pool = torch.zeros((n + 63) // 64, 64, 656, dtype=torch.uint8, device=device)
    concat_and_cache_ds_mla(src[:, :512].contiguous(), src[:, 512:].contiguous(),
                            pool.view(-1, 656), torch.arange(n, device=device))
    if check_against_oracle:
        want = O.quantize_rows(kv_src_bits)
        got = pool.view(-1, 656)[:n].cpu().numpy()
        assert np.array_equal(got, want), "GPU writer differs from the oracle writer"
    return pool


def assert_close(out, ref, max_abs=MAX_ABS, min_cos=MIN_COS, what="out"):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(out).all(), f"{what}: non-finite values"
    m, c = O.max_abs(out, ref), O.cosine(out, ref)
    assert m <= max_abs and c >= min_cos, f"{what}: max_abs={m:.3e} cosine={c:.6f}"
    return m, c


def assert_close_rounded(out, ko, what="out"):
    """Kernel output vs the oracle with tensor-core operand rounding: within
    MAX_ABS_KERNEL_ROUNDING plus one bf16 rounding of each value (the split
    partial's), cosine >= MIN_COS."""
    out = np.asarray(out, np.float64)
    ko = np.asarray(ko, np.float64)
    assert np.isfinite(out).all(), f"{what}: non-finite values"
    err = np.abs(out - ko)
    bound = MAX_ABS_KERNEL_ROUNDING + BF16_ULP * np.abs(ko)
    i = np.unravel_index(int(np.argmax(err - bound)), err.shape)
    c = O.cosine(out, ko)
    assert (err <= bound).all() and c >= MIN_COS, \
        f"{what}: |err| {err[i]:.3e} > {bound[i]:.3e} at {i} (|ref| {abs(ko[i]):.3f}), cosine={c:.6f}"
    return float(err.max()), c


def assert_lse_close(lse, ref, max_abs=MAX_ABS):
    lse = np.asarray(lse, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.array_equal(np.isneginf(lse), np.isneginf(ref)), "-inf pattern of LSE differs"
    fin = np.isfinite(ref)
    assert np.isfinite(lse[fin]).all()
    if fin.any():
        m = O.max_abs(lse[fin], ref[fin])
        assert m <= max_abs, f"lse max_abs={m:.3e}"


def host_workload(name, seed=0, **kw):
    return synthetic.make_host(name, seed=seed, **kw)
