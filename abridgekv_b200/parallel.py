"""Multi-GPU layouts of the compressed-cache decode (one process per GPU).

* Sequence sharding (default): decode and compaction are independent per
  sequence, so each rank owns whole sequences -- their pages, block tables and
  compaction plans -- and runs the same kernels with no collective on the data
  path.  ``shard_sequences`` gives a rank's contiguous share of equal count;
  ``shard_by_bytes`` balances the K/V bytes of sequences of unequal length.
* KV-head sharding (optional): each rank holds KV heads
  [r*Hkv/W, (r+1)*Hkv/W) of every sequence and computes the matching query
  heads; after each layer's attention one all-gather (NCCL over NVLink /
  NVSwitch on GPUs, gloo on CPU) assembles the [B, Hq, D] head outputs.
  Compaction is per rank with identical page tables everywhere.

The reference serves on one GPU; its vLLM TP groups are compatible by design
because every head of a layer has the same quota
(scripts/compresslm_schedules.py:17-25).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def shard_sequences(num_seqs: int, world: int, rank: int) -> slice:
    """Contiguous, balanced share of `num_seqs` sequences for `rank`."""
    base, extra = divmod(num_seqs, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def shard_by_bytes(seq_bytes, world: int, rank: int) -> np.ndarray:
    """Sequences of ``rank`` when whole sequences are spread so that every rank reads about the same
    K/V bytes per decode step (strong scaling of a fixed batch of unequal sequences).

    Greedy longest-first: sequences in decreasing byte order (ties by index) go one by one to the
    rank with the fewest bytes so far (ties to the lowest rank).  Every rank computes the same
    assignment from the same byte counts, so no exchange is needed.  Returns the rank's sequence
    indices in increasing order."""
    w = np.asarray(seq_bytes, dtype=np.float64)
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    order = np.lexsort((np.arange(len(w)), -w))
    load = np.zeros(world)
    owner = np.empty(len(w), dtype=np.int64)
    for i in order:
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += w[i]
    return np.nonzero(owner == rank)[0]


def kv_head_shard(num_kv_heads: int, world: int, rank: int) -> slice:
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} ranks")
    per = num_kv_heads // world
    return slice(rank * per, (rank + 1) * per)


def gather_head_outputs(local: torch.Tensor, group=None) -> torch.Tensor:
    """[B, Hq/W, D] per rank -> [B, Hq, D] on every rank (heads in rank order)."""
    world = dist.get_world_size(group)
    B, hl, D = local.shape
    out = torch.empty((world * B, hl, D), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out.view(world, B, hl, D).permute(1, 0, 2, 3).reshape(B, world * hl, D)
