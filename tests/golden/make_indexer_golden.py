"""Generate tests/golden/indexer.npz: golden vectors for the DSA indexer read
path (fp8 paged MQA logits + per-row top-k), computed by vLLM's own torch
restatement of DeepGEMM's test reference.

    python tests/golden/make_indexer_golden.py      (needs vLLM importable)

The reference repository (nickus/vllm-fp8kv) has no code for this path, only
its specification (PORT_PLAN.md:14, :41, trap 3: SoA pages of block_size x 128
e4m3 bytes then block_size fp32 scales).  vLLM 0.22 ships
``fp8_paged_mqa_logits_torch`` and ``_topk_indices_torch``
(vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:256-354, :572-600).  Its
next_n == 1 branch reads the SoA page; its next_n > 1 branch reads each token
as 132 contiguous bytes, so for next_n = 2 the same pages are handed to it
re-laid token by token (identical values; only the byte order differs).
Inputs are generated from fixed seeds and stored with the outputs.
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402  (only to pack pages and fp8 bytes)
from vllm.v1.attention.ops.rocm_aiter_mla_sparse import (  # noqa: E402
    _topk_indices_torch,
    fp8_paged_mqa_logits_torch,
)

BS, D, H = 64, 128, 64


def case(seed, ctx, next_n, num_blocks, max_model_len, topk):
    rng = np.random.default_rng(seed)
    B = len(ctx)
    pages = O.indexer_quantize(rng.standard_normal((num_blocks * BS, D)).astype(np.float32), BS)
    q_u8 = O.f32_to_e4m3(rng.standard_normal((B, next_n, H, D)).astype(np.float32))
    q_u8 = q_u8.reshape(B, next_n, H, D)
    w = (rng.standard_normal((B * next_n, H)) / 8).astype(np.float32)
    need = max(-(-c // BS) for c in ctx)
    bt = np.stack([rng.permutation(num_blocks)[:need] for _ in range(B)]).astype(np.int32)
    ctx = np.asarray(ctx, np.int32)
    q_t = torch.from_numpy(q_u8).view(torch.float8_e4m3fn)
    if next_n == 1:
        kv = torch.from_numpy(pages).view(num_blocks, BS, 1, D + 4)
    else:  # token-major copy of the same pages for the next_n > 1 branch
        vals = pages[:, : BS * D].reshape(num_blocks, BS, D)
        scl = pages[:, BS * D:].reshape(num_blocks, BS, 4)
        kv = torch.from_numpy(np.concatenate([vals, scl], axis=2)).view(num_blocks, BS, 1, D + 4)
    logits = fp8_paged_mqa_logits_torch(q_t, kv, torch.from_numpy(w), torch.from_numpy(ctx),
                                        torch.from_numpy(bt), max_model_len)
    top = _topk_indices_torch(logits, topk)
    return dict(q=q_u8, pages=pages, w=w, ctx=ctx, bt=bt, logits=logits.numpy(),
                topk=top.numpy(), next_n=np.int32(next_n), max_len=np.int32(max_model_len),
                k=np.int32(topk))


def main():
    cases = {
        "n1": case(1, [1, 100, 300, 512], 1, 16, 576, 128),
        "n2": case(2, [130, 257, 2], 2, 16, 320, 96),
    }
    flat = {f"{name}__{k}": v for name, c in cases.items() for k, v in c.items()}
    np.savez_compressed(os.path.join(HERE, "indexer.npz"), **flat)
    print("wrote", os.path.join(HERE, "indexer.npz"))


if __name__ == "__main__":
    main()
