"""Seeded synthetic decode workloads in the fp8_ds_mla shapes.

The reference measures on random tensors (verify/rebench.py:50-57,
verify/run_all.py:30-33); these generators produce the same kind of inputs at
the five benchmark shapes:

  c1  B=4,   H=16,  top-k=256,  1024-token contexts, 4096-slot pool, 10% -1
  c2  B=64,  H=128, top-k=2048, 32768-token contexts (2,097,152 slots)
  c3  B=256, H=16,  top-k=2048, 131072-token contexts over a shared
      3,500,032-slot pool, 8 splits
  c4  B=32,  H=64,  top-k=2048, 4,194,304-slot pool; leading 512 indices of 8
      requests masked; latent tile amax log-uniform in [1e-4, 1e4] + zero tiles
  c5  B=128, H=128, top-k=2048 per GPU, 65536-token contexts (8,388,608 slots)

Values: q ~ N(0,1) bf16, latent ~ N(0,1) quantized per 128-tile with scale
amax/448, rope ~ N(0,1) bf16, softmax scale 192**-0.5, page size 64, block
tables random permutations of pages, top-k drawn uniformly without
replacement from each request's context, then converted to flat slots.

Two generators share the recipe:
* ``make_host`` (numpy PCG64, bit-reproducible; small shapes, fixtures);
* ``make_device`` (torch CUDA generator; full-size pools built on the GPU
  with the library's own cache writer).
"""

from __future__ import annotations

import dataclasses

import numpy as np

NOPE, ROPE = 512, 64
PAGE = 64
SM_SCALE = 192 ** -0.5


@dataclasses.dataclass(frozen=True)
class Shape:
    name: str
    B: int
    H: int
    topk: int
    ctx: int               # tokens of context per request
    pool_slots: int        # slots in the KV pool
    shared_pool: bool = False   # block tables drawn from a shared pool
    mask_frac: float = 0.0      # fraction of top-k entries set to -1
    lead_masked_reqs: int = 0   # requests whose first `lead_masked` entries are -1
    lead_masked: int = 0
    amax_spread: bool = False   # per-tile amax log-uniform in [1e-4, 1e4] + zero tiles
    num_splits: int = 0         # 0 = library heuristic


SHAPES = {
    "c1": Shape("c1", 4, 16, 256, 1024, 4096, mask_frac=0.10),
    "c2": Shape("c2", 64, 128, 2048, 32768, 64 * 32768),
    "c3": Shape("c3", 256, 16, 2048, 131072, 3_500_032, shared_pool=True, num_splits=8),
    "c4": Shape("c4", 32, 64, 2048, 131072, 4_194_304, lead_masked_reqs=8,
                lead_masked=512, amax_spread=True),
    "c5": Shape("c5", 128, 128, 2048, 65536, 128 * 65536),
}


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _spread_tiles(rng, latent: np.ndarray, zero_frac: float = 0.05) -> np.ndarray:
    n = latent.shape[0]
    tiles = latent.reshape(n, NOPE // 128, 128)
    amax = np.abs(tiles).max(axis=-1, keepdims=True)
    target = 10.0 ** rng.uniform(-4.0, 4.0, size=(n, NOPE // 128, 1))
    tiles = tiles * (target / amax)
    zero = rng.random((n, NOPE // 128)) < zero_frac
    tiles[zero] = 0.0
    return tiles.reshape(n, NOPE).astype(np.float32)


@dataclasses.dataclass
class HostWorkload:
    shape: Shape
    q_bits: np.ndarray          # [B, H, 576] uint16 (bf16)
    kv_src_bits: np.ndarray     # [pool_slots, 576] uint16 (bf16 latent | rope)
    block_table: np.ndarray     # [B, ctx // 64] int32
    token_idx: np.ndarray       # [B, topk] int32, token-relative, -1 masked
    slots: np.ndarray           # [B, topk] int32 flat slots, -1 masked
    sm_scale: float = SM_SCALE


def make_host(shape: Shape | str, seed: int = 0, *, B: int | None = None,
              pool_slots: int | None = None) -> HostWorkload:
    """numpy-generated workload (deterministic for a given seed)."""
    s = SHAPES[shape] if isinstance(shape, str) else shape
    if B is not None or pool_slots is not None:
        s = dataclasses.replace(s, B=B or s.B, pool_slots=pool_slots or s.pool_slots)
    rng = np.random.default_rng(seed)
    n_pages = s.pool_slots // PAGE
    pages_per_req = s.ctx // PAGE
    if s.shared_pool:
        block_table = rng.integers(0, n_pages, size=(s.B, pages_per_req), dtype=np.int64)
    else:
        assert s.B * pages_per_req <= n_pages, "pool too small for disjoint contexts"
        block_table = rng.permutation(n_pages)[: s.B * pages_per_req].reshape(s.B, pages_per_req)
    block_table = block_table.astype(np.int32)

    latent = rng.standard_normal((s.pool_slots, NOPE), dtype=np.float32)
    if s.amax_spread:
        latent = _spread_tiles(rng, latent)
    rope = rng.standard_normal((s.pool_slots, ROPE), dtype=np.float32)
    kv_src_bits = np.concatenate([bf16_bits(latent), bf16_bits(rope)], axis=1)
    q_bits = bf16_bits(rng.standard_normal((s.B, s.H, NOPE + ROPE), dtype=np.float32))

    token_idx = np.empty((s.B, s.topk), np.int32)
    for b in range(s.B):
        token_idx[b] = rng.choice(s.ctx, size=s.topk, replace=False)
    if s.mask_frac > 0:
        n_mask = int(round(s.mask_frac * s.topk))
        for b in range(s.B):
            token_idx[b, rng.choice(s.topk, size=n_mask, replace=False)] = -1
    for b in range(min(s.lead_masked_reqs, s.B)):
        token_idx[b, : s.lead_masked] = -1

    valid = token_idx >= 0
    tok = np.where(valid, token_idx, 0)
    page = np.take_along_axis(block_table, tok // PAGE, axis=1)
    slots = np.where(valid, page * PAGE + tok % PAGE, -1).astype(np.int32)
    return HostWorkload(s, q_bits, kv_src_bits, block_table, token_idx, slots)


@dataclasses.dataclass
class DeviceWorkload:
    shape: Shape
    q: "object"            # torch.Tensor [B, H, 576] bf16 (cuda)
    kv: "object"           # torch.Tensor [pool_slots // 64, 64, 656] uint8 (cuda)
    slots: "object"        # torch.Tensor [B, topk] int32 (cuda)
    block_table: "object"  # torch.Tensor [B, ctx // 64] int32 (cuda)
    token_idx: "object"    # torch.Tensor [B, topk] int32 (cuda)
    sm_scale: float = SM_SCALE


def make_device(shape: Shape | str, seed: int = 0, device="cuda", *, B: int | None = None,
                pool_slots: int | None = None, write_chunk: int = 1 << 20) -> DeviceWorkload:
    """Full-size workload generated on the GPU; the pool is quantized by the
    library's own fp8_ds_mla writer (byte-exact with the reference writer)."""
    import torch

    from vllm_fp8kv.cache_writer import concat_and_cache_ds_mla

    s = SHAPES[shape] if isinstance(shape, str) else shape
    if B is not None or pool_slots is not None:
        s = dataclasses.replace(s, B=B or s.B, pool_slots=pool_slots or s.pool_slots)
    g = torch.Generator(device=device).manual_seed(seed)
    n_pages = s.pool_slots // PAGE
    pages_per_req = s.ctx // PAGE
    if s.shared_pool:
        block_table = torch.randint(0, n_pages, (s.B, pages_per_req), generator=g,
                                    device=device, dtype=torch.int64)
    else:
        assert s.B * pages_per_req <= n_pages
        block_table = torch.randperm(n_pages, generator=g, device=device)[: s.B * pages_per_req]
        block_table = block_table.view(s.B, pages_per_req)
    block_table = block_table.to(torch.int32)

    kv = torch.empty((n_pages, PAGE, 656), dtype=torch.uint8, device=device)
    flat = kv.view(-1, 656)
    for start in range(0, s.pool_slots, write_chunk):
        n = min(write_chunk, s.pool_slots - start)
        latent = torch.randn((n, NOPE), generator=g, device=device, dtype=torch.float32)
        if s.amax_spread:
            t = latent.view(n, NOPE // 128, 128)
            amax = t.abs().amax(-1, keepdim=True)
            target = 10.0 ** (torch.rand((n, NOPE // 128, 1), generator=g, device=device) * 8 - 4)
            t = t * (target / amax)
            zero = torch.rand((n, NOPE // 128), generator=g, device=device) < 0.05
            t[zero] = 0.0
            latent = t.view(n, NOPE)
        rope = torch.randn((n, ROPE), generator=g, device=device, dtype=torch.float32)
        slot_map = torch.arange(start, start + n, device=device, dtype=torch.int64)
        concat_and_cache_ds_mla(latent.to(torch.bfloat16), rope.to(torch.bfloat16), flat, slot_map)
    q = torch.randn((s.B, s.H, NOPE + ROPE), generator=g, device=device).to(torch.bfloat16)

    token_idx = torch.rand((s.B, s.ctx), generator=g, device=device).argsort(dim=1)[:, : s.topk]
    token_idx = token_idx.to(torch.int32).contiguous()
    if s.mask_frac > 0:
        n_mask = int(round(s.mask_frac * s.topk))
        pos = torch.rand((s.B, s.topk), generator=g, device=device).argsort(dim=1)[:, :n_mask]
        token_idx.scatter_(1, pos, -1)
    if s.lead_masked_reqs:
        token_idx[: s.lead_masked_reqs, : s.lead_masked] = -1
    valid = token_idx >= 0
    tok = torch.where(valid, token_idx, torch.zeros_like(token_idx)).long()
    page = torch.gather(block_table.long(), 1, tok // PAGE)
    slots = torch.where(valid, page * PAGE + tok % PAGE, torch.full_like(page, -1)).to(torch.int32)
    return DeviceWorkload(s, q, kv, slots.contiguous(), block_table, token_idx)


def kv_bytes(B: int, topk: int) -> int:
    """Algorithmic KV bytes one decode call reads: every top-k row, 656 B."""
    return B * topk * 656


def algorithmic_bytes(B: int, H: int, topk: int) -> int:
    """KV rows + indices + q + out + LSE (all top-k counted)."""
    return B * topk * 656 + B * topk * 4 + B * H * 576 * 2 + B * H * 512 * 2 + B * H * 4


def algorithmic_flops(B: int, H: int, topk: int) -> int:
    """2 * B * H * topk * (576 + 512): QK^T over d=576 and PV over d_v=512."""
    return 2 * B * H * topk * (576 + 512)
