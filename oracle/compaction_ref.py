"""Compaction oracle (test infrastructure): plain-Python/numpy restatements of
the reference's planner and executor.

Planner (host, integer work):
  * FreeQueue/BlockPool: vLLM FreeKVCacheBlockQueue order (pinned dependency
    vllm==0.13.0; the overlay's BlockPool, vllm/v1/core/block_pool.py:148-175
    pops the null block 0 at start; get_new_blocks :295-325 pops from the head;
    free_blocks :385-399 appends blocks whose ref count reaches zero, in order).
  * GroupManager.compact_span / truncate: single_type_kv_cache_manager.py:358-420
    with BlockPool.copy_kv_slots (block_pool.py:488-550).
  * SpanIndex: vllm/v1/compacted_spans.py:8-68.
  * Planner.mask_token_span: core/sched/scheduler.py:2060-2204.
  * Planner.finish_block: core/compresslm/processor.py:467-557 (physical quotas).
Executor (bytes):
  * execute_kv_copy_group: vllm/v1/worker/gpu_model_runner.py:1194-1220
    (gather every source, then scatter), both paged layouts.
  * execute_kv_copy_operations: gpu_model_runner.py:1147-1176 (per group, the
    b-th batches of all requests merged, batches in order).
"""
from __future__ import annotations

import bisect
from collections import defaultdict

import numpy as np


# ---------------------------------------------------------------- planner
class FreeQueue:
    def __init__(self, n: int):
        self.order = list(range(n))  # head at index 0

    def popleft_n(self, k: int) -> list[int]:
        out, self.order = self.order[:k], self.order[k:]
        return out

    def append_n(self, blocks: list[int]) -> None:
        self.order.extend(blocks)


class BlockPool:
    def __init__(self, n: int):
        self.q = FreeQueue(n)
        self.null = self.q.popleft_n(1)[0]
        self.ref = [0] * n

    def num_free(self) -> int:
        return len(self.q.order)

    def get_new_blocks(self, k: int) -> list[int]:
        if k > self.num_free():
            raise ValueError(f"Cannot get {k} free blocks from the pool")
        out = self.q.popleft_n(k)
        for b in out:
            self.ref[b] += 1
        return out

    def free_blocks(self, ordered: list[int]) -> None:
        for b in ordered:
            self.ref[b] -= 1
        self.q.append_n([b for b in ordered if self.ref[b] == 0 and b != self.null])


class SpanIndex:
    def __init__(self, spans: list[tuple[int, int]]):
        self.spans = list(spans)
        self.starts = [s for s, _ in self.spans]
        self.cum, self.gap_p, self.gap_l = [], [0], [0]
        tot = 0
        for s, e in self.spans:
            tot += e - s
            self.cum.append(tot)
            self.gap_p.append(e - tot)
            self.gap_l.append(e)
        self.total_removed = tot

    def logical_to_physical(self, pos: int) -> int:
        i = bisect.bisect_right(self.starts, pos) - 1
        if i < 0:
            return pos
        if pos >= self.spans[i][1]:
            return pos - self.cum[i]
        prev = self.cum[i - 1] if i > 0 else 0
        return pos - prev - (pos - self.starts[i])

    def physical_to_logical(self, phys: int) -> int:
        i = bisect.bisect_right(self.gap_p, phys) - 1
        return self.gap_l[i] + (phys - self.gap_p[i])


def merge_spans(spans):
    if not spans:
        return []
    out = [sorted(spans)[0]]
    for s, e in sorted(spans)[1:]:
        if s <= out[-1][1]:
            out[-1] = (out[-1][0], max(out[-1][1], e))
        else:
            out.append((s, e))
    return out


class Planner:
    def __init__(self, num_blocks: int, block_size: int, num_groups: int):
        self.pool = BlockPool(num_blocks)
        self.bs = block_size
        self.G = num_groups
        self.blocks = [defaultdict(list) for _ in range(num_groups)]
        self.computed: dict = {}
        self.spans: dict = {}
        self.pending_ops: dict = {}
        self.pending_trunc: dict = {}

    def add_request(self, r):
        self.computed[r] = 0
        self.spans[r] = [SpanIndex([]) for _ in range(self.G)]

    def allocate_slots(self, r, num_tokens: int) -> bool:
        per = [num_tokens - self.spans[r][g].total_removed for g in range(self.G)]
        need = sum(-(-per[g] // self.bs) - len(self.blocks[g][r]) for g in range(self.G))
        if need > self.pool.num_free():
            return False
        for g in range(self.G):
            k = -(-per[g] // self.bs) - len(self.blocks[g][r])
            if k > 0:
                self.blocks[g][r].extend(self.pool.get_new_blocks(k))
        return True

    def free(self, r):
        for g in range(self.G):
            self.pool.free_blocks(list(reversed(self.blocks[g].pop(r, []))))
        self.computed.pop(r, None)
        self.spans.pop(r, None)

    def _truncate(self, blocks: list[int], n_active: int) -> int:
        need = -(-n_active // self.bs)
        to_free = []
        for i in range(need, len(blocks)):
            if blocks[i] != self.pool.null:
                to_free.append(blocks[i])
                blocks[i] = self.pool.null
        del blocks[need:]
        if to_free:
            self.pool.free_blocks(list(reversed(to_free)))
        return len(to_free)

    def compact_span(self, g, r, start, end, n_active):
        blocks = self.blocks[g].get(r)
        if not blocks:
            return 0, []
        removed = end - start
        ops = []
        for s in range(end, n_active):
            d = s - removed
            ops.append((blocks[s // self.bs], s % self.bs, blocks[d // self.bs], d % self.bs))
        return self._truncate(blocks, n_active - removed), ops

    def mask_token_span(self, r, start, end, groups=None):
        def fail(msg):
            return (False, 0, 0, msg)

        if r not in self.computed:
            return fail(f"Request {r} not found")
        if start < 0 or end <= start:
            return fail("Invalid span: must have 0 <= start < end")
        if end > self.computed[r]:
            return fail(f"end_position ({end}) exceeds computed tokens ({self.computed[r]})")
        tokens = end - start
        target = list(range(self.G)) if groups is None else sorted(set(groups))
        plans = []
        for g in target:
            if not 0 <= g < self.G:
                return fail(f"KV cache group {g} out of range")
            si = self.spans[r][g]
            if any(start < e and end > s for s, e in si.spans):
                return fail(f"Cannot compact an already-removed token span (group {g})")
            ps, pe = si.logical_to_physical(start), si.logical_to_physical(end)
            if pe - ps != tokens:
                return fail(f"Logical span does not map to one active physical span (group {g})")
            n_active = self.computed[r] - si.total_removed
            if n_active == tokens:
                return fail("Cannot compact: all tokens would be removed")
            plans.append((g, ps, pe, n_active))
        freed = 0
        for g, ps, pe, n_active in plans:
            f, ops = self.compact_span(g, r, ps, pe, n_active)
            freed += f
            if ops:
                self.pending_ops.setdefault(r, [[] for _ in range(self.G)])[g].append(ops)
            self.spans[r][g] = SpanIndex(merge_spans(self.spans[r][g].spans + [(start, end)]))
        self.pending_trunc[r] = tuple(len(self.blocks[g].get(r) or []) for g in range(self.G))
        return (True, tokens, freed, None)

    def finish_block(self, r, resp, code, quotas, K):
        if resp:
            res = self.mask_token_span(r, resp[0], resp[1])
            if not res[0]:
                raise RuntimeError(res[3])
        for q in sorted(set(quotas)):
            if q >= K:
                continue
            res = self.mask_token_span(r, code[0] + q, code[1], [g for g, x in enumerate(quotas) if x == q])
            if not res[0]:
                raise RuntimeError(res[3])

    def take_pending(self):
        ops, trunc = self.pending_ops, self.pending_trunc
        self.pending_ops, self.pending_trunc = {}, {}
        return ops, trunc


# ---------------------------------------------------------------- executor
def labelled_cache(layout: int, num_blocks: int, page: int, tensor_index: int, heads: int = 1,
                   dim: int = 4) -> np.ndarray:
    """int32 cache whose every element is unique (labels), in layout 0
    ([num_blocks, 2, page, H, D]) or layout 1 ([2, num_blocks, page, H, D])."""
    shape = (num_blocks, 2, page, heads, dim)
    n = int(np.prod(shape))
    lab = (np.arange(n, dtype=np.int64).reshape(shape) + tensor_index * n) % (1 << 31)
    t = lab.astype(np.int32)
    if layout == 1:
        t = np.ascontiguousarray(t.transpose(1, 0, 2, 3, 4))
    return t


def execute_kv_copy_group(all_ops, layer_caches: list[np.ndarray]) -> None:
    """Gather every source row, then scatter (in place, numpy)."""
    if not all_ops:
        return
    o = np.asarray(all_ops, dtype=np.int64)
    sb, so, db, do = o[:, 0], o[:, 1], o[:, 2], o[:, 3]
    for kv in layer_caches:
        if kv.shape[0] == 2:
            src = kv[:, sb, so].copy()
            kv[:, db, do] = src
        else:
            src = kv[sb, :, so].copy()
            kv[db, :, do] = src


def execute_kv_copy_operations(ops_by_request: dict, caches_by_group: list[list[np.ndarray]]) -> None:
    for g, layer_caches in enumerate(caches_by_group):
        batches = [ops[g] for ops in ops_by_request.values() if g < len(ops)]
        nb = max((len(b) for b in batches), default=0)
        for b in range(nb):
            merged = []
            for req_batches in batches:
                if b < len(req_batches):
                    merged.extend(req_batches[b])
            if merged:
                execute_kv_copy_group(merged, layer_caches)
