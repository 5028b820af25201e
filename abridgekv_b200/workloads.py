"""Synthetic, seeded workloads shaped like the reference's Qwen3-4B serving caches.

No public dataset is involved: K/V/Q are N(0,1) bf16 drawn from seeded
generators, page ids are a random permutation of each pool (non-contiguous
pages), and sequence layouts follow the reference's compressed-cache geometry:

  rows kept by layer l for a sequence = raw prompt
                                      + (completed blocks) x quota_l code rows
                                      + live tail of the current block

(third_party/vllm_overlay/vllm/v1/core/compresslm/processor.py:537-556 removes
a finished block's response content and its code slots >= quota_l; the
schedule below is results/schedules/sched_trunc_perlayer_mean128.json of the
reference, one quota per layer).

Layers that share a quota share one block table and one seq_lens vector (one
KV-cache group per quota, vllm/v1/kv_cache_interface.py:162-178); every layer
owns its cache tensor [num_blocks, 2, page, Hkv, D].
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

# Qwen3-4B attention geometry.
QWEN3_4B = dict(num_layers=36, num_q_heads=32, num_kv_heads=8, head_dim=128)

# Per-layer code quotas of results/schedules/sched_trunc_perlayer_mean128.json
# (6 layers x 256, 18 x 128, 12 x 64).
SCHEDULE_PERLAYER_MEAN128 = (
    256, 64, 64, 64, 64, 64, 64, 128, 64, 128, 64, 128, 128, 128, 128, 256, 128, 128,
    256, 128, 256, 256, 128, 128, 256, 128, 128, 128, 128, 128, 64, 64, 64, 128, 128, 64,
)

BLOCK_C = 512  # content tokens per compressed block
PAGE = 16      # vLLM / FlashInfer page size


@dataclass
class DecodeWorkload:
    name: str
    quotas: tuple[int, ...]
    num_seqs: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    page: int
    rows: np.ndarray                  # [L, B] cache rows each layer keeps per sequence
    queries: list[torch.Tensor]       # per layer [B, Hq, D] bf16
    kv_caches: list[torch.Tensor]     # per layer [num_blocks, 2, page, Hkv, D] bf16
    block_tables: list[torch.Tensor]  # per layer [B, max_pages] int32 (shared within a quota group)
    seq_lens: list[torch.Tensor]      # per layer [B] int32 (shared within a quota group)
    meta: dict = field(default_factory=dict)

    @property
    def num_layers(self) -> int:
        return len(self.quotas)

    @property
    def kv_bytes(self) -> int:
        """Algorithmic K+V bytes one decode step must read (each kept row once)."""
        return int(self.rows.sum()) * self.num_kv_heads * self.head_dim * 2 * 2

    @property
    def qo_bytes(self) -> int:
        return self.num_layers * self.num_seqs * self.num_q_heads * self.head_dim * 2 * 2

    @property
    def max_pages(self) -> int:
        return max(int(bt.shape[1]) for bt in self.block_tables)


def compressed_rows(quota: int, prompt: int, blocks: int, tail: np.ndarray) -> np.ndarray:
    return prompt + blocks * quota + tail


def build_decode_workload(
    name: str,
    quotas: tuple[int, ...],
    rows_per_quota: dict[int, np.ndarray],
    *,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    page: int = PAGE,
    device: torch.device | str = "cuda",
    seed: int = 0,
    spare_pages: int = 0,
    meta: dict | None = None,
) -> DecodeWorkload:
    """Materialise caches for the given per-quota row counts ([B] arrays)."""
    device = torch.device(device)
    gen_dev = torch.Generator(device=device).manual_seed(seed)
    rng = np.random.default_rng(seed)
    B = len(next(iter(rows_per_quota.values())))
    tables: dict[int, torch.Tensor] = {}
    lens: dict[int, torch.Tensor] = {}
    nblocks: dict[int, int] = {}
    for q, rows in rows_per_quota.items():
        pages = (rows + page - 1) // page
        total = int(pages.sum()) + spare_pages
        perm = rng.permutation(total).astype(np.int32)
        maxp = max(int(pages.max()), 1)
        bt = np.zeros((B, maxp), dtype=np.int32)
        off = 0
        for b in range(B):
            n = int(pages[b])
            bt[b, :n] = perm[off:off + n]
            off += n
        tables[q] = torch.from_numpy(bt).to(device)
        lens[q] = torch.from_numpy(rows.astype(np.int32)).to(device)
        nblocks[q] = max(total, 1)
    queries, caches, bts, sls = [], [], [], []
    all_rows = []
    for l, q in enumerate(quotas):
        kv = torch.randn((nblocks[q], 2, page, num_kv_heads, head_dim), generator=gen_dev,
                         device=device, dtype=torch.float32).to(torch.bfloat16) \
            if device.type == "cpu" else \
            torch.randn((nblocks[q], 2, page, num_kv_heads, head_dim), generator=gen_dev,
                        device=device, dtype=torch.bfloat16)
        caches.append(kv)
        queries.append(torch.randn((B, num_q_heads, head_dim), generator=gen_dev, device=device,
                                   dtype=torch.float32).to(torch.bfloat16))
        bts.append(tables[q])
        sls.append(lens[q])
        all_rows.append(rows_per_quota[q])
    return DecodeWorkload(
        name=name, quotas=tuple(quotas), num_seqs=B, num_q_heads=num_q_heads,
        num_kv_heads=num_kv_heads, head_dim=head_dim, page=page,
        rows=np.stack(all_rows).astype(np.int64), queries=queries, kv_caches=caches,
        block_tables=bts, seq_lens=sls, meta=dict(meta or {}),
    )


def config2_rows(num_seqs: int = 64, seed: int = 0, quotas=SCHEDULE_PERLAYER_MEAN128,
                 prompt: int = 256, blocks: int = 31) -> dict[int, np.ndarray]:
    """256-token prompt + 16K generated tokens = 31 compressed
    blocks + a live tail ~ U[0, 511] drawn per sequence (shared by all layers)."""
    rng = np.random.default_rng(seed + 1)
    tail = rng.integers(0, BLOCK_C, size=num_seqs)
    return {q: compressed_rows(q, prompt, blocks, tail) for q in sorted(set(quotas))}


def config3_rows(num_seqs: int = 512, seed: int = 0, quotas=SCHEDULE_PERLAYER_MEAN128,
                 prompt: int = 256) -> dict[int, np.ndarray]:
    """generated length log-uniform in [2K, 32K]; blocks =
    (prompt + g) // 512, tail = (prompt + g) % 512."""
    rng = np.random.default_rng(seed + 3)
    g = np.exp(rng.uniform(math.log(2048), math.log(32768), size=num_seqs)).astype(np.int64)
    total = prompt + g
    blocks, tail = total // BLOCK_C, total % BLOCK_C
    return {q: prompt + blocks * q + tail for q in sorted(set(quotas))}


def config5_rows(num_seqs: int = 256, seed: int = 0, prompt: int = 256, blocks: int = 63
                 ) -> dict[int, np.ndarray]:
    """uniform 128 rows per block, 32K generated (63 blocks) + tail."""
    rng = np.random.default_rng(seed + 5)
    tail = rng.integers(0, BLOCK_C, size=num_seqs)
    return {128: compressed_rows(128, prompt, blocks, tail)}


def qwen3_decode_workload(config: int = 2, *, num_seqs: int | None = None, device="cuda", seed: int = 0,
                          seq_slice: slice | np.ndarray | None = None, kv_heads: slice | None = None
                          ) -> DecodeWorkload:
    """Config 2 / 3 / 5 decode workloads at Qwen3-4B shape.

    seq_slice picks this rank's sequences (sequence sharding: a slice or an index array);
    kv_heads picks this rank's KV heads (KV-head sharding)."""
    geo = dict(QWEN3_4B)
    if config == 2:
        rows = config2_rows(num_seqs or 64, seed)
        quotas = SCHEDULE_PERLAYER_MEAN128
    elif config == 3:
        rows = config3_rows(num_seqs or 512, seed)
        quotas = SCHEDULE_PERLAYER_MEAN128
    elif config == 5:
        rows = config5_rows(num_seqs or 256, seed)
        quotas = (128,) * 36
    else:
        raise ValueError(f"no decode workload for config {config}")
    if seq_slice is not None:
        rows = {q: r[seq_slice] for q, r in rows.items()}
    hkv = geo["num_kv_heads"]
    hq = geo["num_q_heads"]
    if kv_heads is not None:
        n = len(range(*kv_heads.indices(hkv)))
        hq = hq // hkv * n
        hkv = n
    return build_decode_workload(
        f"config{config}", quotas, rows, num_q_heads=hq, num_kv_heads=hkv,
        head_dim=geo["head_dim"], device=device, seed=seed,
        meta={"config": config, "kv_heads": str(kv_heads),
              "seqs": str(seq_slice) if not isinstance(seq_slice, np.ndarray) else f"{len(seq_slice)} indexed"},
    )
