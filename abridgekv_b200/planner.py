"""Compaction planner (host side) over libabkv's C++ planner.

Mirrors the scheduler-side interfaces of the reference's vLLM overlay:

* ``mask_token_span(request_id, start, end, groups=None) -> SpanRemovalResult``
  is ``Scheduler.mask_token_span`` (vllm/v1/core/sched/scheduler.py:2060-2204):
  same validation order, same messages, nothing applied when a span is rejected.
* ``take_pending()`` returns the worker-bound structure of
  ``Scheduler.pending_kv_copy_operations``: request -> per KV-cache group ->
  ORDERED list of batches -> list of ``(src_block, src_off, dst_block, dst_off)``
  (each batch a ``compaction.CopyOps``: it reads like the reference's list of
  tuples and carries the int32 array the executor passes to the kernel)
  (consumed by ``GPUModelRunner._execute_kv_copy_operations``,
  vllm/v1/worker/gpu_model_runner.py:1147-1176).
* ``finish_block`` is the physical-quota branch of
  ``CompressLMProcessor._compact_response_content``
  (vllm/v1/core/compresslm/processor.py:467-557); like ``_mask_or_raise`` it
  raises ``RuntimeError`` when a removal is rejected.
* ``allocate_slots`` / ``free`` follow ``KVCacheManager.allocate_slots`` (per-group
  compacted-token deduction, kv_cache_manager.py:281-330) and
  ``SingleTypeKVCacheManager.free``.

Request ids may be any hashable; they are mapped to int64 keys.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Hashable, Iterable, Sequence

import numpy as np

from . import _lib
from .compaction import CopyOps


@dataclass
class SpanRemovalResult:
    """Same fields as vllm.v1.engine.SpanRemovalResult (engine/__init__.py:203-213)."""

    success: bool
    tokens_removed: int = 0
    blocks_freed: int = 0
    error_message: str | None = None


class _SpanResultC(C.Structure):
    _fields_ = [("success", C.c_int32), ("tokens_removed", C.c_int32), ("blocks_freed", C.c_int32),
                ("error_message", C.c_char * 160)]


class BlockPlanner:
    def __init__(self, num_blocks: int, block_size: int, num_groups: int = 1):
        self._lib = _lib.lib()
        self._h = self._lib.abkv_planner_create(num_blocks, block_size, num_groups)
        if not self._h:
            raise ValueError("invalid planner geometry")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_groups = num_groups
        self._ids: dict[Hashable, int] = {}
        self._names: dict[int, Hashable] = {}
        self._next_key = 1 << 62

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.abkv_planner_destroy(h)
            self._h = None

    # -- request bookkeeping -------------------------------------------------
    def _key(self, request_id: Hashable) -> int:
        k = self._ids.get(request_id)
        if k is None:
            raise KeyError(f"unknown request {request_id!r}")
        return k

    def add_request(self, request_id: Hashable) -> None:
        if request_id in self._ids:
            raise ValueError(f"request {request_id!r} already present")
        if (isinstance(request_id, int) and not isinstance(request_id, bool)
                and 0 <= request_id < (1 << 62) and request_id not in self._names):
            k = request_id
        else:
            k = self._next_key
            self._next_key += 1
        _lib.check("abkv_planner_add_request", self._lib.abkv_planner_add_request(self._h, k))
        self._ids[request_id] = k
        self._names[k] = request_id

    def set_num_computed_tokens(self, request_id: Hashable, n: int) -> None:
        _lib.check("abkv_planner_set_num_computed",
                   self._lib.abkv_planner_set_num_computed(self._h, self._key(request_id), n))

    def allocate_slots(self, request_id: Hashable, num_tokens: int) -> bool:
        """Give the request slots for `num_tokens` logical tokens in every group
        (minus that group's compacted tokens).  False when the pool is short."""
        st = self._lib.abkv_planner_allocate_slots(self._h, self._key(request_id), num_tokens)
        if st == 8:  # ABKV_ERR_NO_BLOCKS
            return False
        _lib.check("abkv_planner_allocate_slots", st)
        return True

    def free(self, request_id: Hashable) -> None:
        k = self._key(request_id)
        _lib.check("abkv_planner_free_request", self._lib.abkv_planner_free_request(self._h, k))
        del self._ids[request_id]
        del self._names[k]

    # -- compaction ------------------------------------------------------------
    def mask_token_span(self, request_id: Hashable, start_position: int, end_position: int,
                        groups: Iterable[int] | None = None) -> SpanRemovalResult:
        k = self._ids.get(request_id)
        res = _SpanResultC()
        if k is None:
            return SpanRemovalResult(False, 0, 0, f"Request {request_id} not found")
        if groups is None:
            st = self._lib.abkv_planner_mask_token_span(self._h, k, start_position, end_position, None, 0,
                                                         C.byref(res))
        else:
            g = list(groups)
            arr = _lib.i32_array(g if g else [0])
            st = self._lib.abkv_planner_mask_token_span(self._h, k, start_position, end_position,
                                                         arr, len(g), C.byref(res))
        _lib.check("abkv_planner_mask_token_span", st)
        if res.success:
            return SpanRemovalResult(True, res.tokens_removed, res.blocks_freed, None)
        return SpanRemovalResult(False, 0, 0, res.error_message.decode())

    def finish_block(self, request_id: Hashable, response_span: tuple[int, int] | None,
                     code_span: tuple[int, int], group_quotas: Sequence[int], num_code_tokens: int) -> None:
        res = _SpanResultC()
        rs, re_ = response_span if response_span else (0, 0)
        q = _lib.i32_array(group_quotas)
        st = self._lib.abkv_planner_finish_block(self._h, self._key(request_id), rs, re_, code_span[0],
                                                 code_span[1], q, len(group_quotas), num_code_tokens,
                                                 C.byref(res))
        if st == 7:  # ABKV_ERR_SPAN: _mask_or_raise semantics
            raise RuntimeError(f"CompressLM KV compaction failed: {res.error_message.decode()}")
        _lib.check("abkv_planner_finish_block", st)

    # -- state readers ---------------------------------------------------------
    def block_table(self, request_id: Hashable, group: int = 0) -> list[int]:
        k = self._ids.get(request_id)
        if k is None:
            return []
        n = C.c_int(0)
        self._lib.abkv_planner_block_table(self._h, k, group, None, 0, C.byref(n))
        buf = (C.c_int32 * max(n.value, 1))()
        _lib.check("abkv_planner_block_table",
                   self._lib.abkv_planner_block_table(self._h, k, group, buf, n.value, C.byref(n)))
        return list(buf[:n.value])

    def free_queue(self) -> list[int]:
        n = C.c_int(0)
        buf = (C.c_int32 * self.num_blocks)()
        _lib.check("abkv_planner_free_queue",
                   self._lib.abkv_planner_free_queue(self._h, buf, self.num_blocks, C.byref(n)))
        return list(buf[:n.value])

    def num_free_blocks(self) -> int:
        return int(self._lib.abkv_planner_num_free(self._h))

    def compacted_spans(self, request_id: Hashable, group: int = 0) -> list[tuple[int, int]]:
        k = self._key(request_id)
        n = C.c_int(0)
        self._lib.abkv_planner_compacted_spans(self._h, k, group, None, 0, C.byref(n))
        buf = (C.c_int64 * max(2 * n.value, 2))()
        _lib.check("abkv_planner_compacted_spans",
                   self._lib.abkv_planner_compacted_spans(self._h, k, group, buf, n.value, C.byref(n)))
        return [(buf[2 * i], buf[2 * i + 1]) for i in range(n.value)]

    def logical_to_physical(self, request_id: Hashable, position: int, group: int = 0) -> int:
        out = C.c_int64(0)
        _lib.check("abkv_planner_span_map",
                   self._lib.abkv_planner_span_map(self._h, self._key(request_id), group, position, 1,
                                                   C.byref(out)))
        return int(out.value)

    def physical_to_logical(self, request_id: Hashable, position: int, group: int = 0) -> int:
        out = C.c_int64(0)
        _lib.check("abkv_planner_span_map",
                   self._lib.abkv_planner_span_map(self._h, self._key(request_id), group, position, 0,
                                                   C.byref(out)))
        return int(out.value)

    def get_compacted_token_count(self, request_id: Hashable, group: int = 0) -> int:
        return sum(e - s for s, e in self.compacted_spans(request_id, group))

    def take_pending(self) -> tuple[dict, dict]:
        """Worker-bound output of the removals since the last call, then clear it:

        ops: request -> per KV-cache group -> ORDERED batches -> [(src_block,
        src_off, dst_block, dst_off)] (Scheduler.pending_kv_copy_operations);
        truncations: request -> per-group block count after compaction
        (Scheduler.pending_block_table_truncations)."""
        G = self.num_groups
        nr, nb, no = C.c_int(0), C.c_int(0), C.c_int(0)
        _lib.check("abkv_planner_pending_export",
                   self._lib.abkv_planner_pending_export(self._h, None, None, None, None, 0, 0, 0, C.byref(nr),
                                                         C.byref(nb), C.byref(no)))
        req_ids = np.zeros(max(nr.value, 1), dtype=np.int64)
        group_batches = np.zeros(max(nr.value * G, 1), dtype=np.int32)
        batch_ops = np.zeros(max(nb.value, 1), dtype=np.int32)
        flat = np.zeros(max(4 * no.value, 4), dtype=np.int32)
        _lib.check("abkv_planner_pending_export",
                   self._lib.abkv_planner_pending_export(
                       self._h, req_ids.ctypes.data_as(_lib.c_i64p), group_batches.ctypes.data_as(_lib.c_i32p),
                       batch_ops.ctypes.data_as(_lib.c_i32p), flat.ctypes.data_as(_lib.c_i32p), nr.value, nb.value,
                       no.value, C.byref(nr), C.byref(nb), C.byref(no)))
        # each batch is a row slice of this call's own array (C-contiguous, never reused)
        ops_arr = flat[:4 * no.value].reshape(-1, 4)
        n_batches = group_batches[:nr.value * G].tolist()
        counts = batch_ops[:nb.value].tolist()
        ops: dict = {}
        bi = oi = 0
        for r, k in enumerate(req_ids[:nr.value].tolist()):
            per_group = []
            for g in range(G):
                batches = []
                for _ in range(n_batches[r * G + g]):
                    cnt = counts[bi]
                    batches.append(CopyOps.wrap(ops_arr[oi:oi + cnt]))
                    bi += 1
                    oi += cnt
                per_group.append(batches)
            ops[self._names.get(k, k)] = per_group
        nt = C.c_int(0)
        _lib.check("abkv_planner_pending_trunc_export",
                   self._lib.abkv_planner_pending_trunc_export(self._h, None, None, 0, C.byref(nt)))
        t_ids = np.zeros(max(nt.value, 1), dtype=np.int64)
        t_counts = np.zeros(max(nt.value * G, 1), dtype=np.int32)
        _lib.check("abkv_planner_pending_trunc_export",
                   self._lib.abkv_planner_pending_trunc_export(
                       self._h, t_ids.ctypes.data_as(_lib.c_i64p), t_counts.ctypes.data_as(_lib.c_i32p), nt.value,
                       C.byref(nt)))
        by_id = dict(zip(t_ids[:nt.value].tolist(), map(tuple, t_counts[:nt.value * G].reshape(-1, G).tolist())))
        trunc = {rid: by_id[k] for rid, k in self._ids.items() if k in by_id}
        self.clear_pending()
        return ops, trunc

    def clear_pending(self) -> None:
        _lib.check("abkv_planner_clear_pending", self._lib.abkv_planner_clear_pending(self._h))
