"""Decode attention over device-resident caches with queries and outputs in pinned host memory.

``HostDecode.run`` is ``paged_decode`` for a caller that holds the step's queries, block
tables and seq_lens on the host and wants the outputs back on the host.  The layers are cut
into launch groups: the upload of group g+1 and the download of group g-1 run on their own
streams (one copy engine each way) while group g decodes, so a step costs the decode plus
the upload of the first group and the download of the last one, instead of the decode plus
all copies.  Each call starts only after everything queued on the caller's stream before it,
including the previous call's downloads, so one call is one self-contained step; nothing of
a step overlaps the next one.

There is no CPU path: the decode itself is ``abkv_decode`` (libabkv.so), and host buffers
must be pinned so the copies are asynchronous.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import decode
from .workspace import Workspace, default_workspace


def split_layers(num_layers: int, max_group: int = 16, edge: int = 2) -> list[range]:
    """Launch groups for ``num_layers`` layers: ``edge`` layers first and last (their copies are
    the only ones not hidden behind a decode), the rest in near-equal groups of at most
    ``max_group`` layers (each group is one persistent launch, so fewer groups means fewer
    launch tails)."""
    if num_layers <= 0:
        raise ValueError("num_layers must be positive")
    if max_group <= 0 or edge < 0:
        raise ValueError("max_group must be positive and edge non-negative")
    e = min(edge, num_layers // 2)
    lo, hi = e, num_layers - e
    groups: list[range] = [range(0, e)] if e else []
    mid = hi - lo
    if mid > 0:
        n = -(-mid // max_group)
        base, extra = divmod(mid, n)
        for i in range(n):
            size = base + (1 if i < extra else 0)
            groups.append(range(lo, lo + size))
            lo += size
    if e:
        groups.append(range(hi, num_layers))
    return groups


class HostDecode:
    """Decode ``len(kv_caches)`` layers per call with host-resident inputs and outputs.

    kv_caches[l]: device [num_blocks, 2, page, Hkv, D] bf16 (stay resident);
    ``run`` takes pinned host queries [B, Hq, D] bf16, block tables [B, max_pages] int32 and
    seq_lens [B] int32 per layer (a tensor shared by several layers is uploaded once) and
    fills pinned host outputs [B, Hq, D] bf16.
    """

    def __init__(self, kv_caches: Sequence[torch.Tensor], *, groups: Sequence[range] | None = None,
                 max_pages_per_seq: int | None = None, chunk_tokens: int = 0,
                 workspace: Workspace | None = None):
        if not kv_caches:
            raise ValueError("at least one layer")
        self.kv_caches = list(kv_caches)
        self.device = self.kv_caches[0].device
        if self.device.type != "cuda":
            raise TypeError("kv caches must be CUDA tensors (libabkv has no CPU path)")
        L = len(self.kv_caches)
        self.groups = list(groups) if groups is not None else split_layers(L)
        covered = [l for g in self.groups for l in g]
        if covered != list(range(L)):
            raise ValueError("groups must cover layers 0..L-1 in order, each once")
        self.max_pages_per_seq = max_pages_per_seq
        self.chunk_tokens = chunk_tokens
        self.workspace = workspace or default_workspace(self.device)
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self._q: list[torch.Tensor] = []
        self._out: list[torch.Tensor] = []
        self._tables: dict[int, torch.Tensor] = {}

    def _device_buffers(self, q_host, tables_host) -> None:
        shapes_ok = len(self._q) == len(q_host) and all(
            d.shape == h.shape for d, h in zip(self._q, q_host))
        if not shapes_ok:
            self._q = [torch.empty(h.shape, dtype=h.dtype, device=self.device) for h in q_host]
            self._out = [torch.empty(h.shape, dtype=h.dtype, device=self.device) for h in q_host]
        for key, h in tables_host.items():
            d = self._tables.get(key)
            if d is None or d.shape != h.shape or d.dtype != h.dtype:
                self._tables[key] = torch.empty(h.shape, dtype=h.dtype, device=self.device)
        for key in [k for k in self._tables if k not in tables_host]:
            del self._tables[key]

    def run(self, queries: Sequence[torch.Tensor], block_tables: Sequence[torch.Tensor],
            seq_lens: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor], *, scale: float | None = None,
            stream: torch.cuda.Stream | None = None) -> Sequence[torch.Tensor]:
        L = len(self.kv_caches)
        if not (len(queries) == len(block_tables) == len(seq_lens) == len(outputs) == L):
            raise ValueError(f"one query, block table, seq_lens and output per layer ({L})")
        host = list(queries) + list(block_tables) + list(seq_lens) + list(outputs)
        for t in host:
            if not isinstance(t, torch.Tensor) or t.is_cuda or not t.is_pinned() or not t.is_contiguous():
                raise ValueError("HostDecode.run takes contiguous pinned host tensors")
        for q, o in zip(queries, outputs):
            if o.shape != q.shape or o.dtype != q.dtype:
                raise ValueError("every output must match its query's shape and dtype")
        tables_host = {id(t): t for t in list(block_tables) + list(seq_lens)}
        self._device_buffers(queries, tables_host)
        bt_dev = [self._tables[id(t)] for t in block_tables]
        sl_dev = [self._tables[id(t)] for t in seq_lens]

        cs = torch.cuda.current_stream(self.device) if stream is None else stream
        begin = torch.cuda.Event()
        begin.record(cs)
        # uploads: tables, then the queries group after group, back to back on one engine
        self.h2d.wait_event(begin)
        up = []
        with torch.cuda.stream(self.h2d):
            for key, h in tables_host.items():
                self._tables[key].copy_(h, non_blocking=True)
            for g in self.groups:
                for l in g:
                    self._q[l].copy_(queries[l], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.h2d)
                up.append(ev)
        # group g decodes once its queries are in; its outputs go down while g+1 decodes
        for g, ev in zip(self.groups, up):
            cs.wait_event(ev)
            ls = list(g)
            decode.paged_decode([self._q[l] for l in ls], [self.kv_caches[l] for l in ls],
                                [bt_dev[l] for l in ls], [sl_dev[l] for l in ls], scale=scale,
                                outputs=[self._out[l] for l in ls], max_pages_per_seq=self.max_pages_per_seq,
                                chunk_tokens=self.chunk_tokens, workspace=self.workspace, stream=cs)
            done = torch.cuda.Event()
            done.record(cs)
            self.d2h.wait_event(done)
            with torch.cuda.stream(self.d2h):
                for l in ls:
                    outputs[l].copy_(self._out[l], non_blocking=True)
        end = torch.cuda.Event()
        end.record(self.d2h)
        cs.wait_event(end)  # the caller's stream sees the outputs on the host
        return outputs
