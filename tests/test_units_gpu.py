"""GPU parity of the unit kernels: e4m3 decode (all 256 bytes, both methods),
the fp8_ds_mla cache writer (byte-exact) and the index converter (bit-exact).
Mirrors tests/test_fp8_dequant.py, tests/test_dequant_triton_cpu.py,
tests/test_reference_and_metrics.py:26-53 and tests/test_backend_patch.py:184-214
of the reference."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import gpu_util as U
from tests.conftest import golden
from vllm_fp8kv import synthetic
from vllm_fp8kv.cache_writer import concat_and_cache_ds_mla, concat_and_cache_mla
from vllm_fp8kv.fp8_dequant import (build_lut, dequant_device, dequant_ds_mla_rows,
                                     dequant_triton_launch)
from vllm_fp8kv.index_convert import convert_req_index_to_global_index

pytestmark = pytest.mark.gpu

ALL = torch.arange(256, dtype=torch.uint8)


def _bits(t):
    t = t.cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.element_size() == 2 else \
        t.view(torch.int32).numpy().view(np.uint32)


def _assert_bit_exact(got: torch.Tensor, want_bits: np.ndarray, want_f: np.ndarray):
    g = got.cpu().float().numpy()
    assert np.array_equal(np.isnan(g), np.isnan(want_f)), "NaN positions differ"
    ok = np.isnan(want_f) | (_bits(got) == want_bits)
    assert ok.all(), f"{(~ok).sum()} mismatches at bytes {np.flatnonzero(~ok)[:8]}"


@pytest.mark.parametrize("method", [0, 1])
@pytest.mark.parametrize("dtype,key", [(torch.float16, "f16_bits"), (torch.bfloat16, "bf16_bits"),
                                       (torch.float32, "f32_bits")])
def test_dequant_all_256_bytes_bit_exact(cuda_device, method, dtype, key):
    g = golden("dequant.npz")
    got = dequant_device(ALL.cuda(), dtype, method)
    _assert_bit_exact(got, g[key], g["f32_bits"].view(np.float32))


def test_dequant_denormals_and_signed_zero(cuda_device):
    b = torch.tensor([0x01, 0x02, 0x07, 0x80, 0x81, 0x87], dtype=torch.uint8, device="cuda")
    for method in (0, 1):
        out = dequant_device(b, torch.float16, method)
        ref = b.view(torch.float8_e4m3fn).to(torch.float16)
        assert torch.equal(out, ref)
        assert torch.signbit(out[3]), "-0.0 lost its sign"


def _rows_with_all_bytes_and_scales(scales):
    """One fp8_ds_mla row per scale: latent = all 256 bytes twice, the same
    scale in all four tiles, rope random bf16 bits."""
    n = len(scales)
    rows = np.zeros((n, 656), dtype=np.uint8)
    rows[:, :512] = np.concatenate([np.arange(256), np.arange(256)[::-1]]).astype(np.uint8)
    rows[:, 512:528] = np.repeat(np.asarray(scales, dtype=np.float32)[:, None], 4, 1).view(np.uint8)
    rng = np.random.default_rng(7)
    rope = rng.standard_normal((n, 64)).astype(np.float32)
    rows[:, 528:] = torch.from_numpy(rope).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint8)
    return rows


@pytest.mark.parametrize("method", [0, 1])
def test_decode_row_dequant_bit_exact_all_bytes_and_scales(cuda_device, method):
    # scales: typical amax/448, the extreme tiles of the edge-case workload
    # (amax 1e-4 .. 1e4), exact zero, a power of two, products that land in
    # bf16's subnormal range and ones that overflow to inf
    scales = [1.0, 2.0 ** -7, 2.3 / 448, 1e-4 / 448, 1e4 / 448, 0.0, 3.1e-38, 1e-30, 7.7e35,
              1.7e38, 0.1234567]
    rows = _rows_with_all_bytes_and_scales(scales)
    kv = torch.from_numpy(rows).cuda()
    n = len(scales)
    slots = torch.tensor(list(range(n)) + [-1, n, 2 ** 31 - 1], dtype=torch.int32, device="cuda")
    got = dequant_ds_mla_rows(kv, slots, method)
    torch.cuda.synchronize()
    lat = torch.from_numpy(rows[:, :512].copy()).view(torch.float8_e4m3fn).float()
    sc = torch.from_numpy(rows[:, 512:528].copy()).view(torch.float32)       # [n, 4]
    want = (lat.view(n, 4, 128) * sc[:, :, None]).view(n, 512).to(torch.bfloat16)
    g = got[:n, :512].cpu()
    assert torch.equal(torch.isnan(g), torch.isnan(want)), "NaN positions differ"
    fin = ~torch.isnan(want)
    assert torch.equal(g.view(torch.int16)[fin], want.view(torch.int16)[fin])
    assert np.array_equal(got[:n, 512:].cpu().view(torch.uint8).numpy().reshape(n, 128),
                          rows[:, 528:])
    assert not got[n:].any(), "masked / out-of-range slots must give zero rows"


def test_decode_row_dequant_methods_agree_on_synthetic_pool(cuda_device):
    # the edge-case workload's value distribution: tile amax 1e-4 .. 1e4 and zero tiles
    w = synthetic.make_device("c4", seed=3, device="cuda", B=1, pool_slots=1 << 17)
    n = w.kv.numel() // 656
    slots = torch.arange(-1, n + 1, dtype=torch.int32, device="cuda")
    a = dequant_ds_mla_rows(w.kv, slots, 0)
    b = dequant_ds_mla_rows(w.kv, slots, 1)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("n", [300, 1 << 20])
def test_dequant_ragged_and_large_random(cuda_device, n):
    g = torch.Generator().manual_seed(n)
    u8 = torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8).cuda()
    lut = build_lut(torch.float16, device="cuda")
    bm, lt = dequant_triton_launch(u8, lut)
    ref = u8.view(torch.float8_e4m3fn).to(torch.float16)
    for got in (bm, lt):
        assert got.shape == (n,)
        assert torch.equal(got.isnan(), ref.isnan())
        keep = ~ref.isnan()
        assert torch.equal(got[keep].view(torch.int16), ref[keep].view(torch.int16))


def test_writer_byte_exact_with_reference_golden(cuda_device):
    g = golden("writer.npz")
    kv_c = U.bf16_tensor(g["kv_c_bits"])
    k_pe = U.bf16_tensor(g["k_pe_bits"])
    cache = torch.zeros(64, 656, dtype=torch.uint8, device="cuda")
    concat_and_cache_ds_mla(kv_c, k_pe, cache, torch.from_numpy(g["slots"]).cuda())
    got = cache.cpu().numpy()
    diff = np.argwhere(got != g["cache"])
    assert diff.size == 0, f"{len(diff)} bytes differ, first at {diff[0]}"


def test_writer_byte_exact_on_amax_spread_and_zero_tiles(cuda_device):
    """c4 edge (c): tile amax log-uniform in [1e-4, 1e4] plus exact-zero tiles."""
    s = synthetic.Shape("spread", B=1, H=16, topk=128, ctx=8192, pool_slots=8192,
                        amax_spread=True)
    w = synthetic.make_host(s, seed=2)
    U.device_pool(w.kv_src_bits, check_against_oracle=True)


def test_writer_skips_padding_and_ignores_k_scale(cuda_device):
    g = golden("writer.npz")
    kv_c = U.bf16_tensor(g["kv_c_bits"])
    k_pe = U.bf16_tensor(g["k_pe_bits"])
    slots = g["slots"].copy()
    slots[::3] = -1
    cache = torch.zeros(64, 656, dtype=torch.uint8, device="cuda")
    concat_and_cache_mla(kv_c, k_pe, cache, torch.from_numpy(slots).cuda(), "fp8_ds_mla",
                         torch.tensor(2.0))
    want = np.zeros_like(g["cache"])
    O.ds_mla_write(g["kv_c_bits"], g["k_pe_bits"], slots, want)
    assert np.array_equal(cache.cpu().numpy(), want)


def test_writer_strided_inputs(cuda_device):
    rng = np.random.default_rng(3)
    src = synthetic.bf16_bits(rng.standard_normal((100, 700)).astype(np.float32))
    t = U.bf16_tensor(src)
    kv_c, k_pe = t[:, :512], t[:, 600:664]
    cache = torch.zeros(2, 64, 656, dtype=torch.uint8, device="cuda")
    slots = torch.from_numpy(rng.permutation(128)[:100].astype(np.int64)).cuda()
    concat_and_cache_ds_mla(kv_c, k_pe, cache, slots)
    want = np.zeros((128, 656), np.uint8)
    O.ds_mla_write(src[:, :512], src[:, 600:664], slots.cpu().numpy(), want)
    assert np.array_equal(cache.view(-1, 656).cpu().numpy(), want)


def test_writer_byte_exact_on_special_values_and_large_random(cuda_device):
    """Tiles holding +-inf, +-NaN, values near the bf16 maximum, subnormals and
    signed zeros, then 16,384 tokens of mixed magnitudes: every byte equals the
    oracle writer, which follows torch's cast, except the sign of a NaN code
    (0x7F / 0xFF).  inf/inf and NaN propagation give a negative NaN on the
    host and the canonical positive one on the GPU, so, as the reference's
    tests do (tests/test_fp8_dequant.py:19-27), NaN codes are compared for
    NaN-ness only."""
    rng = np.random.default_rng(4)
    n = 16384
    x = rng.standard_normal((n, 576)).astype(np.float32)
    tile_scale = np.exp(rng.uniform(-20, 20, size=(n, 4))).astype(np.float32)
    x[:, :512] *= np.repeat(tile_scale, 128, axis=1)
    specials = [np.inf, -np.inf, np.nan, -np.nan, 3.3e38, -3.3e38, 1e-40, -1e-40, 0.0, -0.0, 1e-38]
    for r, v in enumerate(specials):
        x[r, 5 + 128 * (r % 4)] = v
    x[20, 0:128] = 0.0
    x[21, 128:256] = -0.0
    x[22, 256:384] = 1e-39  # a tile whose scale clamps to FLT_MIN
    src = synthetic.bf16_bits(x)
    t = U.bf16_tensor(src)
    cache = torch.zeros(n // 64, 64, 656, dtype=torch.uint8, device="cuda")
    slots = rng.permutation(n).astype(np.int64)
    concat_and_cache_ds_mla(t[:, :512].contiguous(), t[:, 512:].contiguous(), cache,
                            torch.from_numpy(slots).cuda())
    want = np.zeros((n, 656), np.uint8)
    O.ds_mla_write(src[:, :512], src[:, 512:], slots, want)
    got = cache.view(-1, 656).cpu().numpy()
    latent = np.zeros((656,), bool)
    latent[:512] = True  # e4m3 codes; scales and rope compare byte for byte
    nan_code = lambda b: (b & 0x7F) == 0x7F
    same = (got == want) | (latent & nan_code(want) & nan_code(got))
    diff = np.argwhere(~same)
    assert diff.size == 0, f"{len(diff)} bytes differ, first at {diff[:4].tolist()}"
    assert np.array_equal(nan_code(got) & latent, nan_code(want) & latent)


@pytest.mark.parametrize("which", ["in_range", "oob"])
def test_index_converter_matches_vllm(cuda_device, which):
    g = golden("index.npz")
    ti = g["token_idx"] if which == "in_range" else g["token_idx_oob"]
    want = g["out"] if which == "in_range" else g["out_oob"]
    got = convert_req_index_to_global_index(
        torch.from_numpy(g["req_id"]).cuda(), torch.from_numpy(g["block_table"]).cuda(),
        torch.from_numpy(ti).cuda(), BLOCK_SIZE=int(g["block_size"]), NUM_TOPK_TOKENS=ti.shape[1])
    assert np.array_equal(got.cpu().numpy(), want)


def test_index_converter_large_random_vs_oracle(cuda_device):
    rng = np.random.default_rng(4)
    T, R, nb, topk = 512, 64, 512, 2048
    req = rng.integers(0, R, T).astype(np.int32)
    bt = rng.integers(0, 1 << 16, (R, nb)).astype(np.int32)
    ti = rng.integers(-1, nb * 64 + 100, (T, topk)).astype(np.int32)
    got = convert_req_index_to_global_index(torch.from_numpy(req).cuda(), torch.from_numpy(bt).cuda(),
                                            torch.from_numpy(ti).cuda(), 64, topk)
    assert np.array_equal(got.cpu().numpy(), O.convert_req_index(req, bt, ti, 64))
