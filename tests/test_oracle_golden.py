"""Pin the CPU oracle against vectors the reference itself produced.

Every fixture under tests/golden/ was written by tests/golden/make_golden.py
from the reference's own code (torch casts, the writer mirrors, vLLM's index
converter, the golden decode and the reference's Triton kernel run under the
interpreter).  If the oracle disagrees with one of them, every GPU parity test
that trusts the oracle is void, so these run on CPU in every round.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import golden
from vllm_fp8kv import synthetic


def _nan_aware_equal(got_bits, want_bits, got_f, want_f):
    assert np.array_equal(np.isnan(got_f), np.isnan(want_f)), "NaN positions differ"
    ok = np.isnan(want_f) | (got_bits == want_bits)
    assert ok.all(), f"{(~ok).sum()} mismatches, first at {np.argwhere(~ok)[0]}"


def test_e4m3_to_f32_all_256_bytes():
    g = golden("dequant.npz")
    got = O.e4m3_to_f32(np.arange(256, dtype=np.uint8))
    want = g["f32_bits"].view(np.float32)
    _nan_aware_equal(got.view(np.uint32), g["f32_bits"], got, want)
    # NaN only for 0x7F / 0xFF (tests/test_fp8_dequant.py:19-37)
    assert set(np.flatnonzero(np.isnan(got)).tolist()) == {0x7F, 0xFF}


def test_e4m3_values_are_exact_in_bf16_and_fp16():
    g = golden("dequant.npz")
    f = O.e4m3_to_f32(np.arange(256, dtype=np.uint8))
    bf = O.f32_to_bf16_bits(f)
    _nan_aware_equal(bf, g["bf16_bits"], f, f)
    f16 = f.astype(np.float16).view(np.uint16)
    _nan_aware_equal(f16, g["f16_bits"], f, f)
    # the reference's own bit-math decode agrees with torch's cast
    _nan_aware_equal(g["ref_bitmath_f16_bits"], g["f16_bits"], f, f)


def test_f32_to_e4m3_matches_torch_cast_bytes():
    g = golden("casts.npz")
    got = O.f32_to_e4m3(g["e4m3_in"])
    bad = np.flatnonzero(got != g["e4m3_out"])
    assert bad.size == 0, (
        f"{bad.size} mismatches; first x={g['e4m3_in'][bad[0]]!r} "
        f"got=0x{got[bad[0]]:02X} want=0x{g['e4m3_out'][bad[0]]:02X}")


def test_f32_to_bf16_matches_torch_cast():
    g = golden("casts.npz")
    x = g["bf16_in"]
    got = O.f32_to_bf16_bits(x)
    want = g["bf16_out"]
    _nan_aware_equal(got, want, O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(want))


def test_writer_is_byte_exact_with_the_reference_mirrors():
    g = golden("writer.npz")
    cache = np.zeros_like(g["cache"])
    O.ds_mla_write(g["kv_c_bits"], g["k_pe_bits"], g["slots"], cache)
    diff = np.argwhere(cache != g["cache"])
    assert diff.size == 0, f"{len(diff)} bytes differ, first at {diff[0]}"


def test_row_parser_matches_reference_parser():
    g = golden("writer.npz")
    got = O.dequant_rows(g["cache"])
    want = g["dequant"]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)) or \
        np.array_equal(got, want, equal_nan=True)


def test_writer_skips_padding_slots():
    g = golden("writer.npz")
    cache = np.zeros_like(g["cache"])
    slots = g["slots"].copy()
    slots[::3] = -1
    slots[1::5] = 10 ** 9
    O.ds_mla_write(g["kv_c_bits"], g["k_pe_bits"], slots, cache)
    keep = (slots >= 0) & (slots < cache.shape[0])
    assert np.array_equal(cache[slots[keep]], g["cache"][slots[keep]])
    untouched = np.setdiff1d(np.arange(cache.shape[0]), slots[keep])
    assert not cache[untouched].any()


@pytest.mark.parametrize("which", ["in_range", "oob"])
def test_index_conversion_matches_vllm_converter(which):
    g = golden("index.npz")
    ti = g["token_idx"] if which == "in_range" else g["token_idx_oob"]
    want = g["out"] if which == "in_range" else g["out_oob"]
    got = O.convert_req_index(g["req_id"], g["block_table"], ti, int(g["block_size"]))
    assert np.array_equal(got, want)


def _c1_inputs():
    g = golden("decode_c1.npz")
    w = synthetic.make_host("c1", seed=0)
    import hashlib

    h = hashlib.sha256()
    for a in (w.q_bits, w.kv_src_bits, w.slots):
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.hexdigest() == str(g["inputs_sha"]), "synthetic generator drifted from the fixture"
    pool = O.quantize_rows(w.kv_src_bits)
    h = hashlib.sha256(pool.tobytes())
    assert h.hexdigest() == str(g["pool_sha"]), "oracle writer != reference writer on c1"
    return g, w, pool


def test_c1_decode_oracle_matches_reference_golden_path():
    g, w, pool = _c1_inputs()
    q = synthetic.bf16_to_f32(w.q_bits)
    out, lse = O.sparse_decode(q, pool, w.slots, float(g["sm_scale"]))
    assert O.max_abs(out, g["ref_out"]) < 1e-5
    assert O.max_abs(lse, g["ref_lse"]) < 1e-4
    # and against the reference's Triton kernel (fp32 q, interpreter)
    assert O.max_abs(out, g["kernel_out"]) < 1e-4
    assert O.max_abs(lse, g["kernel_lse"]) < 1e-4


def test_c1_decode_oracle_fp64_accumulation_agrees():
    g, w, pool = _c1_inputs()
    q = synthetic.bf16_to_f32(w.q_bits)
    out, lse = O.sparse_decode(q, pool, w.slots, float(g["sm_scale"]), acc_dtype=np.float64)
    assert O.max_abs(out, g["ref_out"]) < 1e-5
    assert O.max_abs(lse, g["ref_lse"]) < 1e-4


TRAPS = ["masked", "leading_one", "leading_48", "empty_row", "out_of_range",
         "groups2_h32", "heads8", "matrix_q4"]


@pytest.mark.parametrize("case", TRAPS)
def test_trap_cases_oracle_vs_reference(case):
    g = golden("traps.npz")
    q = g[f"{case}__q"]
    pool = g[str(g[f"{case}__pool"])]
    idx = g[f"{case}__idx"]
    out, lse = O.sparse_decode(q, pool, idx, float(g["sm_scale"]))
    assert np.isfinite(out).all()
    assert O.max_abs(out, g[f"{case}__ref_out"]) < 1e-5
    assert O.max_abs(out, g[f"{case}__kernel_out"]) < 1e-4
    klse = g[f"{case}__kernel_lse"]
    assert np.array_equal(np.isinf(lse), np.isinf(klse))
    fin = np.isfinite(klse)
    assert O.max_abs(lse[fin], klse[fin]) < 1e-4


def test_empty_row_gives_zeros_and_minus_inf_lse():
    g = golden("traps.npz")
    out, lse = O.sparse_decode(g["empty_row__q"], g[str(g["empty_row__pool"])],
                               g["empty_row__idx"], float(g["sm_scale"]))
    assert not out[1].any()
    assert np.isneginf(lse[1]).all()


def test_split_heuristic_matches_upstream():
    g = golden("splits.npz")
    for T, groups, topk, sms, want in g["table"]:
        got = O.choose_num_splits(int(T), 16 * int(groups), 1, int(topk), int(sms))
        assert got == want, (T, groups, topk, sms, got, want)


def test_metrics_match_reference_semantics():
    a = np.array([1.0, 2.0, 3.0])
    assert O.cosine(a, 5 * a) == pytest.approx(1.0)
    assert O.max_abs(a, 5 * a) == pytest.approx(12.0)
    assert O.cosine(np.zeros(0), np.zeros(0)) == 1.0
