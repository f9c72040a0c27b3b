"""Seeded synthetic workloads for the paged attention path (tests and bench).

A case is a shared paged pool [num_blocks][num_layers][Hkv][16][hd] (bf16 bits
~N(0,1)), one block table row per sequence holding a shuffled slice of the
pool, per-sequence context lengths and query rows. Table padding is -1, so an
out-of-range read would show up in the kernels' status word.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

import oracle.oracle as O

BLOCK = 16

# BASELINE configs (shapes only; inputs are synthetic and seeded).
CONFIGS = {
    "c1_0p5b_single": dict(batch=1, hq=14, hkv=2, hd=64, layers=24, ctx=("fixed", 1024)),
    "c2_0p5b_ragged": dict(batch=64, hq=14, hkv=2, hd=64, layers=24, ctx=("uniform", 256, 4096)),
    "c3_7b_batched": dict(batch=32, hq=28, hkv=4, hd=128, layers=28, ctx=("fixed", 8192)),
    "c4_1p5b_prefill": dict(batch=4, hq=12, hkv=2, hd=128, layers=28, ctx=("fixed", 4096)),
    "c5_72b_wide": dict(batch=128, hq=64, hkv=8, hd=128, layers=80, ctx=("uniform", 1024, 32768)),
}


def context_lengths(spec, batch: int, rng: np.random.Generator) -> np.ndarray:
    if spec[0] == "fixed":
        return np.full(batch, spec[1], np.int32)
    lo, hi = spec[1], spec[2]
    return rng.integers(lo, hi + 1, size=batch, dtype=np.int64).astype(np.int32)


def randn_bf16(rng: np.random.Generator, shape) -> np.ndarray:
    return O.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32))


@dataclass
class PagedCase:
    batch: int
    hq: int
    hkv: int
    hd: int
    num_layers: int
    layer: int
    ctx: np.ndarray            # [B] int32 cached tokens per sequence
    tables: np.ndarray         # [B, table_stride] int32, -1 padded
    num_blocks: int
    k_pool: np.ndarray = field(repr=False, default=None)  # uint16 [nb, L, Hkv, 16, hd]
    v_pool: np.ndarray = field(repr=False, default=None)
    q: np.ndarray = field(repr=False, default=None)       # uint16 [B, Hq*hd]

    @property
    def max_ctx(self) -> int:
        return int(self.ctx.max()) if self.batch else 0


def make_tables(ctx_pages: np.ndarray, rng: np.random.Generator, spare_blocks: int = 3,
                table_stride: int | None = None):
    """Shuffled shared pool: sequence b gets ctx_pages[b] distinct random blocks."""
    total = int(ctx_pages.sum())
    num_blocks = total + spare_blocks
    perm = rng.permutation(num_blocks).astype(np.int32)
    stride = table_stride or max(1, int(ctx_pages.max()) if len(ctx_pages) else 1)
    tables = np.full((len(ctx_pages), stride), -1, np.int32)
    off = 0
    for b, n in enumerate(ctx_pages):
        tables[b, :n] = perm[off:off + n]
        off += n
    return tables, num_blocks


def make_case(batch, hq, hkv, hd, ctx, num_layers=2, layer=1, seed=0, extra_pages=0,
              spare_blocks=3, table_stride=None, with_data=True) -> PagedCase:
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, np.int32)
    pages = (ctx + BLOCK - 1) // BLOCK + extra_pages
    tables, nb = make_tables(pages, rng, spare_blocks, table_stride)
    case = PagedCase(batch, hq, hkv, hd, num_layers, layer, ctx, tables, nb)
    if with_data:
        shape = (nb, num_layers, hkv, BLOCK, hd)
        case.k_pool = randn_bf16(rng, shape)
        case.v_pool = randn_bf16(rng, shape)
        case.q = randn_bf16(rng, (batch, hq * hd))
    return case


def to_device(a: np.ndarray, device="cuda"):
    """numpy (uint16 bf16 bits / int32 / float32) -> torch tensor on device."""
    import torch
    if a.dtype == np.uint16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def from_device(t) -> np.ndarray:
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()
