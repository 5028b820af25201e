"""KV compaction executor (host side) over libabkv's sm_100a copy kernels.

* ``execute_kv_copy_operations(kv_copy_operations, kv_caches_by_group)``
  mirrors ``GPUModelRunner._execute_kv_copy_operations``
  (third_party/vllm_overlay/vllm/v1/worker/gpu_model_runner.py:1147-1176): for
  each KV-cache group, the b-th batch of every request is merged and the
  batches are applied in order, each with gather-all-then-scatter semantics,
  to every layer tensor of the group.  One ``abkv_compact`` call per group.
* ``execute_kv_copy_group(all_ops, layer_caches)`` mirrors
  ``_execute_kv_copy_group`` (:1194-1220): one batch.
* ``evict_columns(K, V, keep_cols)`` mirrors ``KVStore.evict``
  (abridgekv/gen_compress.py:72-77) for all layers in one launch.

Both paged layouts are accepted, detected like the reference: a leading dim of
2 is the FlashAttention layout ``[2, num_blocks, page, Hkv, D]``, otherwise
FlashInfer ``[num_blocks, 2, page, Hkv, D]``.  The copy is byte-exact for any
2-byte or wider element type.
"""
from __future__ import annotations

import itertools
from collections.abc import Sequence as _SequenceABC
from typing import Hashable, Sequence

import numpy as np
import torch

from . import _lib
from .workspace import Workspace, default_workspace


class CopyOps(_SequenceABC):
    """One ordered batch of ``(src_block, src_off, dst_block, dst_off)`` copy operations held as
    an int32 array ``[n, 4]``.  It behaves like the reference's list of tuples (length, indexing,
    iteration, equality with a list), so callers of ``take_pending`` see the reference structure,
    while the executor hands the array to the kernel without a round trip through Python ints."""

    __slots__ = ("array",)

    def __init__(self, array) -> None:
        self.array = np.ascontiguousarray(np.asarray(array, dtype=np.int32).reshape(-1, 4))

    @classmethod
    def wrap(cls, array: np.ndarray) -> "CopyOps":
        """A batch over ``array`` as it is: a C-contiguous int32 ``[n, 4]`` array (no conversion)."""
        obj = object.__new__(cls)
        obj.array = array
        return obj

    def __len__(self) -> int:
        return int(self.array.shape[0])

    def __getitem__(self, i):
        if isinstance(i, slice):
            return CopyOps(self.array[i])
        return tuple(int(v) for v in self.array[i])

    def __iter__(self):
        return iter(map(tuple, self.array.tolist()))

    def __eq__(self, other) -> bool:
        if isinstance(other, CopyOps):
            return bool(np.array_equal(self.array, other.array))
        try:
            return list(self) == [tuple(op) for op in other]
        except TypeError:
            return NotImplemented

    def __repr__(self) -> str:
        return f"CopyOps({list(self)!r})"


def _flatten(batches) -> tuple[np.ndarray, list[int]]:
    """Concatenated [4 x ops] int32 and per-batch counts of a list of batches."""
    counts = [len(b) for b in batches]
    if batches and all(isinstance(b, CopyOps) for b in batches):
        return np.concatenate([b.array for b in batches]).reshape(-1), counts
    flat = np.fromiter(itertools.chain.from_iterable(itertools.chain.from_iterable(batches)), dtype=np.int32,
                       count=4 * sum(counts))
    return flat, counts


def _layout_of(kv: torch.Tensor) -> tuple[int, int, int, int, int]:
    if kv.dim() != 5:
        raise ValueError(f"unsupported KV cache shape {tuple(kv.shape)}")
    if kv.shape[0] == 2:
        _, nb, page, hkv, d = kv.shape
        return 1, nb, page, hkv, d
    nb, two, page, hkv, d = kv.shape
    if two != 2:
        raise ValueError(f"unsupported KV cache shape {tuple(kv.shape)}")
    return 0, nb, page, hkv, d


def _compact(layer_caches: Sequence[torch.Tensor], batches: Sequence[Sequence[Sequence[int]]],
             workspace: Workspace | None, stream: torch.cuda.Stream | None) -> None:
    if not layer_caches:
        return
    kv0 = layer_caches[0]
    layout, nb, page, hkv, d = _layout_of(kv0)
    for kv in layer_caches:
        if not kv.is_cuda or not kv.is_contiguous():
            raise TypeError("KV caches must be contiguous CUDA tensors (libabkv has no CPU path)")
        if kv.shape != kv0.shape or kv.dtype != kv0.dtype:
            raise ValueError("every layer tensor of a group must share shape and dtype")
    elem = kv0.element_size()
    # the kernel moves rows as bytes: express the row as 2-byte units
    units = hkv * d * elem // 2
    n_batches = len(batches)
    if sum(len(b) for b in batches) == 0:
        return
    flat, counts = _flatten(batches)
    offsets = np.zeros(n_batches + 1, dtype=np.int64)
    np.cumsum(counts, out=offsets[1:])
    max_ops = max(counts)
    lib = _lib.lib()
    need = lib.abkv_compact_workspace_size(len(layer_caches), page, 1, units, max_ops)
    ws = (workspace or default_workspace(kv0.device)).ensure(need)
    s = torch.cuda.current_stream(kv0.device) if stream is None else stream
    ops_arr = flat.ctypes.data_as(_lib.c_i32p)
    off_arr = offsets.ctypes.data_as(_lib.c_i64p)
    with torch.cuda.device(kv0.device):
        st = lib.abkv_compact(_lib.ptr_array([kv.data_ptr() for kv in layer_caches]), len(layer_caches),
                              layout, nb, page, 1, units, ops_arr, off_arr, n_batches, ws.ptr(), ws.nbytes,
                              s.cuda_stream)
    _lib.check("abkv_compact", st)


def execute_kv_copy_group(all_ops: Sequence[Sequence[int]], layer_caches: Sequence[torch.Tensor],
                          workspace: Workspace | None = None, stream=None) -> None:
    """One batch of (src_block, src_off, dst_block, dst_off) over every layer tensor."""
    _compact(layer_caches, [list(all_ops)], workspace, stream)


def _group_batches(kv_copy_operations, g: int) -> list:
    """Group g's ordered batches: batch b of every request concatenated (the reference's order)."""
    per_req = [ops[g] for ops in kv_copy_operations.values() if g < len(ops)]
    nb = max((len(b) for b in per_req), default=0)
    batches = []
    for b in range(nb):
        parts = [req_batches[b] for req_batches in per_req if b < len(req_batches)]
        if parts and all(isinstance(x, CopyOps) for x in parts):
            merged = CopyOps(np.concatenate([x.array for x in parts]))
        else:
            merged = [tuple(op) for x in parts for op in x]
        if len(merged):
            batches.append(merged)
    return batches


def _blocks_of(batches) -> np.ndarray:
    """Every block id (source or destination) the batches touch, with repeats."""
    if not batches:
        return np.zeros(0, dtype=np.int64)
    flat, _ = _flatten(batches)
    ops = flat.reshape(-1, 4)
    return np.concatenate([ops[:, 0], ops[:, 2]])


def _disjoint(block_sets: Sequence[np.ndarray], num_blocks: int) -> bool:
    """No block id in two of the sets: each set marks its blocks once in a flag array and the
    counts add up (ids outside [0, num_blocks) all land in one extra slot, so two sets holding such
    ids count as overlapping)."""
    count = np.zeros(num_blocks + 1, dtype=np.uint16)
    for ids in block_sets:
        seen = np.zeros(num_blocks + 1, dtype=bool)
        seen[np.clip(ids, -1, num_blocks)] = True  # -1 indexes the extra slot, as num_blocks does
        count += seen
    return len(block_sets) < 2 or int(count.max()) <= 1


def execute_kv_copy_operations(kv_copy_operations: dict[Hashable, list[list[list[tuple[int, int, int, int]]]]],
                               kv_caches_by_group: Sequence[Sequence[torch.Tensor]],
                               workspace: Workspace | None = None, stream=None) -> None:
    """request -> per group -> ordered batches, applied group by group.

    When every group names the same layer tensors (the hybrid layout, where the groups share
    physical tensors and own disjoint blocks of one pool) and no block is touched by two groups,
    batch b of every group goes into one call: the groups then move disjoint rows, so applying them
    together equals applying them one after another, with one launch per batch instead of one per
    group and batch."""
    per_group = [_group_batches(kv_copy_operations, g) for g in range(len(kv_caches_by_group))]
    busy = [g for g, batches in enumerate(per_group) if batches]
    if len(busy) > 1:
        first = kv_caches_by_group[busy[0]]
        same = all(len(kv_caches_by_group[g]) == len(first) and
                   all(a is b or (a.data_ptr() == b.data_ptr() and a.shape == b.shape and a.dtype == b.dtype)
                       for a, b in zip(kv_caches_by_group[g], first)) for g in busy)
        if same:
            if _disjoint([_blocks_of(per_group[g]) for g in busy], _layout_of(first[0])[1]):
                n = max(len(per_group[g]) for g in busy)
                merged = []
                for b in range(n):
                    parts = [per_group[g][b] for g in busy if b < len(per_group[g])]
                    if all(isinstance(x, CopyOps) for x in parts):
                        merged.append(CopyOps(np.concatenate([x.array for x in parts])))
                    else:
                        merged.append([tuple(op) for x in parts for op in x])
                _compact(first, merged, workspace, stream)
                return
    for g, layer_caches in enumerate(kv_caches_by_group):
        if per_group[g]:
            _compact(layer_caches, per_group[g], workspace, stream)


def evict_columns(K: Sequence[torch.Tensor], V: Sequence[torch.Tensor], keep_cols: torch.Tensor,
                  workspace: Workspace | None = None, stream=None) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
    """KVStore.evict: K[l][:, :, keep_cols, :] and V[l][...] for every layer, one launch.

    K[l], V[l]: contiguous CUDA [B, Hkv, T, D]; keep_cols: 1-D integer tensor.
    Returns new contiguous tensors [B, Hkv, len(keep_cols), D]."""
    tensors = list(K) + list(V)
    if not tensors:
        return [], []
    t0 = tensors[0]
    for t in tensors:
        if not t.is_cuda or not t.is_contiguous() or t.shape != t0.shape or t.dtype != t0.dtype:
            raise ValueError("evict_columns needs contiguous CUDA tensors of one shape and dtype")
    b, h, T, d = t0.shape
    keep = keep_cols.to(device=t0.device, dtype=torch.int64).contiguous()
    n = keep.numel()
    outs = [torch.empty((b, h, n, d), dtype=t0.dtype, device=t0.device) for _ in tensors]
    ws = workspace or default_workspace(t0.device)
    s = torch.cuda.current_stream(t0.device) if stream is None else stream
    with torch.cuda.device(t0.device):
        st = _lib.lib().abkv_gather_rows(
            _lib.ptr_array([t.data_ptr() for t in tensors]), _lib.ptr_array([o.data_ptr() for o in outs]),
            len(tensors), b * h, T, n, d * t0.element_size(), keep.data_ptr(), ws.ptr(), ws.nbytes,
            s.cuda_stream)
    _lib.check("abkv_gather_rows", st)
    L = len(K)
    return outs[:L], outs[L:]
