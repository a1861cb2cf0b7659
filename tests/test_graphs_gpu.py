"""CUDA-graph capture of the library's kernels (vLLM runs its decode step as a
captured graph): the paired tcgen05 decode, the indexer's logits and top-k,
and the cache writer each replay bit-identically to their eager call.

Every kernel launches with programmatic dependent launch; inside a graph the
launches become programmatic edges, so a replay keeps the same ordering.
"""

import numpy as np
import pytest
import torch

from tests import gpu_util as U
from tests.conftest import golden
from vllm_fp8kv import synthetic
from vllm_fp8kv.cache_writer import concat_and_cache_ds_mla
from vllm_fp8kv.fp8_ds_mla_sparse_decode import decode_kernel_name, fp8_ds_mla_sparse_decode
from vllm_fp8kv.indexer import fp8_paged_mqa_logits, top_k_per_row_decode

pytestmark = pytest.mark.gpu


def _capture(fn):
    """Run fn once eagerly on a side stream, capture it, replay once."""
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    return g


def test_pair_decode_graph_replays_identically(cuda_device):
    w = synthetic.make_host(synthetic.Shape("s", B=3, H=128, topk=512, ctx=4096, pool_slots=16384),
                            seed=21)
    pool = U.device_pool(w.kv_src_bits, check_against_oracle=False)
    q = U.bf16_tensor(w.q_bits)
    idx = torch.from_numpy(w.slots).cuda()
    assert decode_kernel_name(3, 128, 1, 512, torch.bfloat16, 1).startswith("decode_tc3_kernel")
    eager, eager_lse = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, return_lse=True, num_kv_splits=1)
    out = torch.empty_like(eager)
    lse = torch.empty_like(eager_lse)

    def step():
        o, l = fp8_ds_mla_sparse_decode(q, pool, idx, w.sm_scale, return_lse=True, num_kv_splits=1)
        out.copy_(o)
        lse.copy_(l)

    g = _capture(step)
    assert torch.equal(out, eager) and torch.equal(lse, eager_lse)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_indexer_graph_replays_identically(cuda_device):
    gd = golden("indexer.npz")
    name = sorted({k.split("__", 1)[0] for k in gd.files})[0]
    c = {k.split("__", 1)[1]: gd[k] for k in gd.files if k.startswith(name + "__")}
    nn, k, L = int(c["next_n"]), int(c["k"]), int(c["max_len"])
    q = torch.from_numpy(np.ascontiguousarray(c["q"])).cuda().view(torch.float8_e4m3fn)
    kv = torch.from_numpy(np.ascontiguousarray(c["pages"])).cuda().view(-1, 64, 1, 132)
    wt = torch.from_numpy(np.ascontiguousarray(c["w"], np.float32)).cuda()
    ct = torch.from_numpy(np.ascontiguousarray(c["ctx"], np.int32)).cuda()
    bt = torch.from_numpy(np.ascontiguousarray(c["bt"], np.int32)).cuda()
    rows = q.shape[0] * nn
    logits = torch.empty((rows, L), dtype=torch.float32, device="cuda")
    top = torch.empty((rows, k), dtype=torch.int32, device="cuda")

    def step():
        fp8_paged_mqa_logits(q, kv, wt, ct, bt, None, L, logits=logits)
        top_k_per_row_decode(logits, nn, ct, top, rows, logits.stride(0), 1, k)

    step()
    torch.cuda.synchronize()
    eager_logits, eager_top = logits.clone(), top.clone()
    logits.zero_()
    top.zero_()
    _capture(step)
    assert torch.equal(logits, eager_logits) and torch.equal(top, eager_top)


def test_writer_graph_replays_identically(cuda_device):
    gd = golden("writer.npz")
    kv_c = U.bf16_tensor(gd["kv_c_bits"])
    k_pe = U.bf16_tensor(gd["k_pe_bits"])
    slots = torch.from_numpy(gd["slots"]).cuda()
    cache = torch.zeros(64, 656, dtype=torch.uint8, device="cuda")
    _capture(lambda: concat_and_cache_ds_mla(kv_c, k_pe, cache, slots))
    assert np.array_equal(cache.cpu().numpy(), gd["cache"])
