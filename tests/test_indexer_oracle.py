"""The DSA indexer oracle against golden vectors from vLLM's torch restatement
of DeepGEMM's reference (tests/golden/make_indexer_golden.py): logits of the
fp8 paged MQA scoring and the per-row top-k sets, next_n = 1 and 2."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import golden


@pytest.mark.parametrize("name", ["n1", "n2"])
def test_indexer_logits_match_vllm_reference(name):
    g = golden("indexer.npz")
    c = {k.split("__", 1)[1]: g[k] for k in g.files if k.startswith(name + "__")}
    got = O.indexer_logits(c["q"], c["pages"], c["w"], c["ctx"], c["bt"], int(c["max_len"]))
    want = c["logits"]
    assert np.array_equal(np.isneginf(got), np.isneginf(want)), "masked positions differ"
    fin = np.isfinite(want)
    scale = np.abs(want[fin]).max()
    assert np.abs(got[fin] - want[fin]).max() <= 1e-5 * scale


@pytest.mark.parametrize("name", ["n1", "n2"])
def test_indexer_topk_sets_match_vllm_reference(name):
    g = golden("indexer.npz")
    c = {k.split("__", 1)[1]: g[k] for k in g.files if k.startswith(name + "__")}
    nn, k = int(c["next_n"]), int(c["k"])
    got = O.indexer_topk(c["logits"], nn, c["ctx"], k)
    want = c["topk"]
    for r in range(got.shape[0]):
        a = set(got[r][got[r] >= 0].tolist())
        b = set(want[r][want[r] >= 0].tolist())
        assert a == b, r
        assert (np.diff(got[r][got[r] >= 0]) > 0).all(), "kept positions ascend"


def test_indexer_topk_ties_keep_lower_positions_and_short_rows_pad():
    lg = np.full((2, 10), -np.inf, np.float32)
    lg[0, :10] = [1, 5, 5, 5, 0, 5, 2, 9, 5, 5]
    lg[1, :3] = [3, 2, 1]
    got = O.indexer_topk(lg, 1, np.array([10, 3]), 4)
    assert got[0].tolist() == [1, 2, 3, 7]          # 9, then the three lowest of the tied 5s
    assert got[1].tolist() == [0, 1, 2, -1]         # fewer valid positions than k


def test_indexer_page_layout_is_structure_of_arrays():
    rng = np.random.default_rng(3)
    k = rng.standard_normal((128, 128)).astype(np.float32)
    pages = O.indexer_quantize(k, 64)
    assert pages.shape == (2, 64 * 132) and O.indexer_page_bytes(64) == 8448
    scale = pages[1, 64 * 128:].copy().view(np.float32)
    np.testing.assert_allclose(scale, np.abs(k[64:]).max(1) / 448, rtol=1e-6)
    deq = O.e4m3_to_f32(pages[1, :64 * 128]).reshape(64, 128) * scale[:, None]
    np.testing.assert_allclose(deq, k[64:], rtol=0.07, atol=1e-6)
