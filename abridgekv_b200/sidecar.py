"""Packed per-head-quota sidecar: layout, page pool and decode (host side).

Mirrors the reference's packed KV storage for per-head code quotas
(third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py):

* ``PackedKVLayout`` (:13-155): ``K[layer, kv_head]`` quotas of one compressed
  block; ``pack_layer`` turns the dense ``[2, K_max, H_kv, D]`` code rows of a
  block into one packed page ``[2, sum_h q_h, D]`` in which KV head h owns
  slots ``[offsets[h], offsets[h] + q_h)``; ``unpack_layer`` is the inverse.
* ``SidecarPool`` holds the packed pages of one layer for many requests in one
  device tensor ``[num_pages, 2, slots, D]`` with a page table
  ``[num_requests, max_pages]`` and per-request page counts -- the device form
  of the reference's ``PackedKVSidecar.pages[request][layer]`` lists that
  ``capture`` (:290-320) appends to.
* ``attend_decode_batched_packed`` is ``PackedKVSidecar._attend_decode_batched``
  with sidecar pages (:526-616): for KV head h of a request the keys are head
  h's slots of each of its sidecar pages, then its main rows from the paged
  cache.  It runs ``abkv_decode_packed`` (libabkv.so); quotas must be multiples
  of 16.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

from . import _lib
from .decode import _validate
from .workspace import Workspace, default_workspace


@dataclass(frozen=True)
class PackedKVLayout:
    """Static ``K[layer, kv_head]`` quotas of one compressed block (the reference dataclass's fields and
    error messages): KV head h of layer l owns ``quotas[l][h]`` slots of each packed page, at slot
    offset ``offsets[l][h]``.  Checked on construction; the geometry is read from one int array."""

    quotas: tuple[tuple[int, ...], ...]
    k_max: int

    def __post_init__(self) -> None:
        if self.k_max <= 0:
            raise ValueError("packed KV k_max must be positive")
        widths = [len(row) for row in self.quotas]
        if not widths or widths[0] == 0:
            raise ValueError("packed KV quotas must be a non-empty 2D schedule")
        uneven = next((l for l, w in enumerate(widths) if w != widths[0]), None)
        if uneven is not None:
            raise ValueError("packed KV quota rows must have equal length; "
                             f"layer 0 has {widths[0]}, layer {uneven} has {widths[uneven]}")
        q = self._array()
        bad = np.argwhere((q <= 0) | (q > self.k_max))  # row-major: the first layer, then its first head
        if len(bad):
            layer, head = (int(x) for x in bad[0])
            raise ValueError(f"packed KV quota[{layer}][{head}]={int(q[layer, head])} must be in [1, {self.k_max}]")

    def _array(self) -> np.ndarray:
        return np.asarray(self.quotas, dtype=np.int64).reshape(len(self.quotas), -1)

    @classmethod
    def from_schedule(cls, schedule: Sequence[Sequence[int]] | None, *, num_layers: int, num_kv_heads: int,
                      k_max: int) -> "PackedKVLayout":
        """Layout of a quota schedule ([layer][KV head]); without one, every head keeps all k_max slots."""
        if num_layers <= 0 or num_kv_heads <= 0:
            raise ValueError("packed KV model dimensions must be positive")
        rows = [tuple(map(int, r)) for r in schedule] if schedule else [(int(k_max),) * num_kv_heads] * num_layers
        if len(rows) != num_layers:
            raise ValueError(f"packed KV schedule has {len(rows)} layers; model has {num_layers}")
        widths = sorted({len(r) for r in rows})
        if widths != [num_kv_heads]:
            raise ValueError(f"packed KV schedule row widths {widths} do not match model num_kv_heads={num_kv_heads}")
        return cls(quotas=tuple(rows), k_max=int(k_max))

    @property
    def num_layers(self) -> int:
        return len(self.quotas)

    @property
    def num_kv_heads(self) -> int:
        return len(self.quotas[0])

    @property
    def offsets(self) -> tuple[tuple[int, ...], ...]:
        """Per layer, the first slot of every head and the end: [0, q_0, q_0 + q_1, ..., sum q]."""
        q = self._array()
        edges = np.concatenate([np.zeros((q.shape[0], 1), dtype=np.int64), np.cumsum(q, axis=1)], axis=1)
        return tuple(tuple(row) for row in edges.tolist())

    @property
    def packed_slots_per_layer(self) -> tuple[int, ...]:
        return tuple(self._array().sum(axis=1).tolist())

    def _index(self, layer: int, device) -> torch.Tensor:
        """Dense (slot, head) pairs of the packed slots, head-major: [slots, 2]."""
        pairs = [(s, h) for h, q in enumerate(self.quotas[layer]) for s in range(q)]
        return torch.tensor(pairs, dtype=torch.long, device=device)

    def pack_layer(self, layer: int, dense: torch.Tensor) -> torch.Tensor:
        """Pack ``[2, K_max, H_kv, D]`` into ``[2, sum_h K_lh, D]`` (one gather)."""
        expected = (2, self.k_max, self.num_kv_heads)
        if dense.ndim != 4 or tuple(dense.shape[:3]) != expected:
            raise ValueError(f"dense layer KV must start with shape {expected}; got {tuple(dense.shape)}")
        idx = self._index(layer, dense.device)
        return dense[:, idx[:, 0], idx[:, 1], :].contiguous()

    def unpack_layer(self, layer: int, packed: torch.Tensor, *, fill_value: float = 0.0) -> torch.Tensor:
        """Expand a packed layer page to ``[2, K_max, H_kv, D]`` (one scatter)."""
        expected_slots = self.packed_slots_per_layer[layer]
        if packed.ndim != 3 or packed.shape[0] != 2:
            raise ValueError("packed layer KV must have shape [2, packed_slots, head_size]")
        if packed.shape[1] != expected_slots:
            raise ValueError(f"packed layer {layer} has {packed.shape[1]} slots; expected {expected_slots}")
        dense = packed.new_full((2, self.k_max, self.num_kv_heads, packed.shape[-1]), fill_value)
        idx = self._index(layer, packed.device)
        dense[:, idx[:, 0], idx[:, 1], :] = packed
        return dense


class SidecarPool:
    """Packed pages of one layer for ``num_requests`` request slots: ``pages`` [capacity, 2,
    slots, D] bf16, ``page_table`` [num_requests, max_pages] int32, ``page_count``
    [num_requests] int32 (device).  ``append`` stores one packed page for a request (the
    reference's ``capture``); ``free`` drops a request's pages (they are reused)."""

    def __init__(self, layout: PackedKVLayout, layer: int, *, capacity: int, num_requests: int, max_pages: int,
                 head_dim: int, device: torch.device | str = "cuda"):
        self.layout, self.layer = layout, layer
        self.quotas = layout.quotas[layer]
        if any(q % 16 for q in self.quotas):
            raise ValueError("the sm_100a sidecar decode needs quotas that are multiples of 16")
        self.slots = layout.packed_slots_per_layer[layer]
        self.pages = torch.zeros((capacity, 2, self.slots, head_dim), dtype=torch.bfloat16, device=device)
        self.page_table = torch.zeros((num_requests, max_pages), dtype=torch.int32, device=device)
        self.page_count = torch.zeros((num_requests,), dtype=torch.int32, device=device)
        self._free = list(range(capacity - 1, -1, -1))
        self._owned: dict[int, list[int]] = {}

    def append(self, request: int, packed_page: torch.Tensor) -> int:
        owned = self._owned.setdefault(request, [])
        if len(owned) >= self.page_table.shape[1]:
            raise RuntimeError(f"request slot {request} already holds {len(owned)} sidecar pages")
        if not self._free:
            raise RuntimeError("sidecar pool is full")
        pid = self._free.pop()
        self.pages[pid].copy_(packed_page)
        self.page_table[request, len(owned)] = pid
        owned.append(pid)
        self.page_count[request] = len(owned)
        return pid

    def free(self, request: int) -> None:
        for pid in self._owned.pop(request, []):
            self._free.append(pid)
        self.page_count[request] = 0

    def descriptor(self) -> _lib.SidecarT:
        d = _lib.SidecarT()
        d.pages, d.page_table, d.page_count = self.pages.data_ptr(), self.page_table.data_ptr(), \
            self.page_count.data_ptr()
        d.page_table_stride, d.num_pages, d.slots = self.page_table.stride(0), self.pages.shape[0], self.slots
        for h, q in enumerate(self.quotas):
            d.quotas[h] = q
        return d


def packed_decode(queries: Sequence[torch.Tensor], kv_caches: Sequence[torch.Tensor],
                  block_tables: Sequence[torch.Tensor], seq_lens: Sequence[torch.Tensor],
                  sidecars: Sequence[SidecarPool | None], *, scale: float | None = None,
                  outputs: Sequence[torch.Tensor] | None = None, chunk_tokens: int = 0,
                  workspace: Workspace | None = None, stream: torch.cuda.Stream | None = None) -> list[torch.Tensor]:
    """``paged_decode`` with a packed sidecar per layer (None = none): one launch for all layers."""
    L = len(queries)
    if len(sidecars) != L:
        raise ValueError("one sidecar entry per layer")
    B, Hq, Hkv, D, page, outs = _validate(queries, kv_caches, block_tables, seq_lens, outputs)
    if Hkv > 8:
        raise ValueError("at most 8 KV heads")
    descs = (_lib.SidecarT * L)()
    max_side_rows = 0
    for l, sc in enumerate(sidecars):
        if sc is None:
            continue
        if len(sc.quotas) != Hkv or sc.pages.shape[-1] != D or sc.page_table.shape[0] < B:
            raise ValueError(f"layer {l}: sidecar does not match the cache geometry")
        descs[l] = sc.descriptor()
        max_side_rows = max(max_side_rows, sc.page_table.stride(0) * sc.slots)
    max_pages = max(int(bt.shape[1]) for bt in block_tables)
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    lib = _lib.lib()
    need = lib.abkv_decode_packed_workspace_size(L, B, Hq, D, page, max_pages, chunk_tokens, max_side_rows)
    if need == 0:
        raise _lib.AbkvError("abkv_decode_packed_workspace_size", 3, f"unsupported shape (B={B}, Hq={Hq}, D={D})")
    device = queries[0].device
    ws = (workspace or default_workspace(device)).ensure(need)
    s = torch.cuda.current_stream(device) if stream is None else stream
    with torch.cuda.device(device):
        st = lib.abkv_decode_packed(
            _lib.ptr_array([q.data_ptr() for q in queries]), _lib.ptr_array([kv.data_ptr() for kv in kv_caches]),
            _lib.ptr_array([bt.data_ptr() for bt in block_tables]),
            _lib.i64_array([bt.stride(0) for bt in block_tables]),
            _lib.ptr_array([sl.data_ptr() for sl in seq_lens]), _lib.i64_array([kv.shape[0] for kv in kv_caches]),
            _lib.ptr_array([o.data_ptr() for o in outs]), L, B, Hq, Hkv, D, page, max_pages, scale, chunk_tokens,
            C.cast(descs, C.c_void_p), ws.ptr(), ws.nbytes, s.cuda_stream)
    _lib.check("abkv_decode_packed", st)
    return outs


def attend_decode_batched_packed(*, query: torch.Tensor, kv_cache: torch.Tensor, output: torch.Tensor,
                                 seq_lens: torch.Tensor, block_table: torch.Tensor, num_kv_heads: int, groups: int,
                                 scale: float, sidecar: SidecarPool | None, num_requests: int | None = None,
                                 workspace: Workspace | None = None) -> None:
    """Drop-in for ``PackedKVSidecar._attend_decode_batched`` with sidecar pages: request i of
    the active batch is request slot i of ``sidecar``; writes ``output[:n]`` in place."""
    n = int(num_requests if num_requests is not None else block_table.shape[0])
    D = kv_cache.shape[-1]
    Hq = num_kv_heads * groups
    q = query[:n].reshape(n, Hq, D).contiguous()
    sl = seq_lens[:n].to(device=kv_cache.device, dtype=torch.int32).contiguous()
    bt = block_table[:n].to(torch.int32).contiguous()
    out_view = output[:n].reshape(n, Hq, D)
    direct = out_view.is_contiguous() and out_view.dtype == torch.bfloat16
    o = out_view if direct else torch.empty((n, Hq, D), dtype=torch.bfloat16, device=kv_cache.device)
    packed_decode([q], [kv_cache], [bt], [sl], [sidecar], scale=scale, outputs=[o], workspace=workspace)
    if not direct:
        out_view.copy_(o)
