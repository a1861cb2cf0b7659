"""The C-ABI library loads without a GPU, exports every entry point that
include/fp8mla.h declares, and its host-only logic (split heuristic, workspace
sizing, argument validation) behaves as the reference's."""

import ctypes
import os
import re

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import REPO, golden
from vllm_fp8kv import _native as N

HEADER = os.path.join(REPO, "include", "fp8mla.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:FP8MLA_API\s+)?(?:const\s+char\s*\*|int64_t|uint32_t|int)\s+(fp8mla_\w+)\s*\(",
                                 text, flags=re.M)))


def test_library_is_built_in_tree():
    assert os.path.exists(N.LIB_PATH), "run `python vllm-fp8kv_b200/build.py` (or __graft_entry__.build())"
    assert os.path.realpath(N.LIB_PATH).startswith(os.path.realpath(REPO))


def test_every_declared_symbol_is_exported_and_bound():
    syms = declared_symbols()
    assert len(syms) >= 8, syms
    L = ctypes.CDLL(N.LIB_PATH)
    for s in syms:
        assert hasattr(L, s), f"{s} declared in fp8mla.h but not exported"
    assert set(syms) == set(N.SIGNATURES), "ctypes binding and header disagree"


def test_abi_version_and_empty_error():
    assert N.lib().fp8mla_abi_version() == 1
    assert isinstance(N.lib().fp8mla_last_error(), bytes)


def test_split_heuristic_matches_upstream_table():
    g = golden("splits.npz")
    for T, groups, topk, sms, want in g["table"]:
        got = N.lib().fp8mla_choose_num_splits(int(T), 16 * int(groups), 1, int(topk), int(sms))
        assert got == want, (T, groups, topk, sms, got, want)


@pytest.mark.parametrize("T,H,G,topk,sms", [(1, 16, 1, 2048, 148), (4, 16, 1, 256, 148),
                                            (2, 8, 1, 512, 148), (1, 32, 2, 1024, 148),
                                            (64, 128, 1, 2048, 148), (256, 16, 1, 2048, 148)])
def test_split_heuristic_matches_oracle_for_grouped_heads(T, H, G, topk, sms):
    assert N.lib().fp8mla_choose_num_splits(T, H, G, topk, sms) == \
        O.choose_num_splits(T, H, G, topk, sms)


def test_workspace_bytes():
    L = N.lib()
    assert L.fp8mla_decode_workspace_bytes(4, 16, 1, 256, 1) == 0
    T, H, S = 4, 16, 8
    want = ((T * H * S * 512 * 4 + 255) // 256) * 256 + T * H * S * 4
    assert L.fp8mla_decode_workspace_bytes(T, H, 1, 256, S) == want


def _decode(**over):
    args = dict(q=None, q_dtype=0, T=1, H=16, q_st=16 * 576, q_sh=576, kv=None, num_slots=0,
                idx=None, G=1, topk=32, idx_st=32, idx_sg=32, sm=0.1, out=None, out_st=16 * 512,
                out_sh=512, lse=None, lse_st=16, splits=1, ws=None, ws_bytes=0, stream=None)
    args.update(over)
    return N.lib().fp8mla_sparse_decode(*args.values())


@pytest.mark.parametrize("over,needle", [
    (dict(q_dtype=2), b"q must be bf16"),
    (dict(H=16, G=3), b"not divisible"),
    (dict(T=-1), b"bad sizes"),
    (dict(q=8), b"16-byte aligned"),
])
def test_invalid_arguments_are_rejected_before_touching_the_device(over, needle):
    rc = _decode(**over)
    assert rc == N.ERR_INVALID_ARGUMENT
    assert needle in N.lib().fp8mla_last_error()


def test_zero_tokens_is_a_no_op():
    assert _decode(T=0) == N.OK


def test_writer_and_converter_validate_arguments():
    L = N.lib()
    assert L.fp8mla_ds_mla_write(None, 100, None, 64, None, 4, None, 0, None) == N.ERR_INVALID_ARGUMENT
    assert L.fp8mla_ds_mla_write(None, 512, None, 64, None, 0, None, 0, None) == N.OK
    rc = L.fp8mla_convert_req_index(None, None, 1, 1, None, 100, 1, 100, 64, None, 100, None)
    assert rc == N.ERR_INVALID_ARGUMENT and b"divisible by BLOCK_N" in L.fp8mla_last_error()
    assert L.fp8mla_dequant_e4m3(None, 4, None, 7, 0, None) == N.ERR_INVALID_ARGUMENT


def test_check_maps_invalid_argument_to_assertion_error():
    _decode(q_dtype=2)
    with pytest.raises(AssertionError):
        N.check(N.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(N.Fp8MlaError):
        N.check(N.ERR_CUDA, "x")


def test_guard_assertions_fire_before_any_device_work():
    """tests/test_sparse_decode.py:159-183 of the reference: argument errors are
    AssertionError, raised on the host (so they hold on a CPU-only box too)."""
    import torch

    from vllm_fp8kv.fp8_ds_mla_sparse_decode import ROW_BYTES, fp8_ds_mla_sparse_decode

    packed = torch.zeros(64, ROW_BYTES, dtype=torch.uint8)
    q = torch.zeros(2, 16, 576)
    idx = torch.zeros(2, 32, dtype=torch.int32)
    cases = [
        (q.to(torch.float16), packed),               # fp16 q: rope bitcast would be garbage
        (q, packed.to(torch.int8)),                  # cache dtype
        (q, packed.t()),                             # non-contiguous pool
        (q[..., :512].contiguous(), packed),         # wrong head dim
    ]
    for qq, cache in cases:
        with pytest.raises(AssertionError):
            fp8_ds_mla_sparse_decode(qq, cache, idx, 0.1)
    with pytest.raises(AssertionError):
        fp8_ds_mla_sparse_decode(q, packed, torch.zeros(2, 3, 32, dtype=torch.int32), 0.1)


def test_cpu_tensors_fail_loudly_no_fallback():
    import torch

    from vllm_fp8kv.fp8_ds_mla_sparse_decode import fp8_ds_mla_sparse_decode

    with pytest.raises(N.Fp8MlaError, match="no CPU path"):
        fp8_ds_mla_sparse_decode(torch.zeros(1, 16, 576), torch.zeros(64, 656, dtype=torch.uint8),
                                 torch.zeros(1, 32, dtype=torch.int32), 0.1)


def test_oracle_is_not_imported_by_the_product():
    """The product package must not reach into oracle/."""
    pkg = os.path.join(REPO, "vllm-fp8kv_b200", "vllm_fp8kv")
    for f in os.listdir(pkg):
        if f.endswith(".py"):
            src = open(os.path.join(pkg, f)).read()
            assert "oracle" not in re.sub(r"#.*|\"\"\"[\s\S]*?\"\"\"", "", src), f


def test_header_constants_match_python_module():
    from vllm_fp8kv import fp8_ds_mla_sparse_decode as D

    text = open(HEADER).read()
    for name, val in [("NOPE", D.NOPE), ("ROPE", D.ROPE), ("TILE", D.TILE),
                      ("ROW_BYTES", D.ROW_BYTES), ("SCALE_OFF", D.SCALE_OFF),
                      ("ROPE_OFF", D.ROPE_OFF)]:
        m = re.search(rf"#define FP8MLA_{name} (\d+)", text)
        assert m and int(m.group(1)) == val, name
    assert np.int64(D.ROW_BYTES) == 656
