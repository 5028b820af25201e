"""Seeded small paged-cache cases for the oracle and golden fixtures (test infrastructure).

Deterministic across machines (numpy default_rng), so the golden fixtures only
store seeds, shapes and the reference's outputs.  Rows of a sequence beyond
its seq_len, and pages its block-table row references beyond
ceil(seq_len/page), are POISONED with NaN: an implementation that reads them
produces NaN and fails parity.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .bf16 import round_bf16


@dataclass
class PagedCase:
    q: np.ndarray          # [B, Hq, D] float32 holding bf16 values
    kv: np.ndarray         # [num_blocks, 2, P, Hkv, D] float32 holding bf16 values (NaN poison)
    block_table: np.ndarray  # [B, max_pages] int32
    seq_lens: np.ndarray   # [B] int32
    page: int
    scale: float


def paged_case(seed: int, seq_lens, *, num_q_heads: int = 8, num_kv_heads: int = 2, head_dim: int = 128,
               page: int = 16, spare_pages: int = 3, extra_cols: int = 2, scale: float | None = None,
               poison: bool = True) -> PagedCase:
    rng = np.random.default_rng(seed)
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    B = len(seq_lens)
    pages = (seq_lens.astype(np.int64) + page - 1) // page
    # page 0 is the never-allocated null block (vLLM's BlockPool reserves it);
    # it stays finite so that the reference's masked gathers of page 0 are harmless.
    total = 1 + int(pages.sum()) + spare_pages
    perm = (1 + rng.permutation(total - 1)).astype(np.int32)
    maxp = int(pages.max()) + extra_cols
    maxp = max(maxp, 1)
    bt = np.zeros((B, maxp), dtype=np.int32)
    off = 0
    used = np.zeros(total, dtype=bool)
    for b in range(B):
        n = int(pages[b])
        bt[b, :n] = perm[off:off + n]
        used[perm[off:off + n]] = True
        off += n
    spare = perm[off:]
    kv = round_bf16(rng.standard_normal((total, 2, page, num_kv_heads, head_dim)).astype(np.float32))
    kv[0] = 0.0
    q = round_bf16(rng.standard_normal((B, num_q_heads, head_dim)).astype(np.float32))
    if poison:
        # unused table columns point at poisoned spare pages (or page 0 if none)
        for b in range(B):
            n = int(pages[b])
            for j in range(n, maxp):
                bt[b, j] = spare[(b + j) % len(spare)] if len(spare) else 0
        if len(spare):
            kv[spare] = np.nan
        for b in range(B):
            s = int(seq_lens[b])
            if s % page:
                kv[bt[b, s // page], :, s % page:] = np.nan
    if scale is None:
        scale = 1.0 / np.sqrt(head_dim)
    return PagedCase(q=q, kv=kv, block_table=bt, seq_lens=seq_lens, page=page, scale=float(scale))
