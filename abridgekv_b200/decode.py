"""Paged decode attention over per-quota-group page tables (host side).

Mirrors the reference's decode entry points:

* ``attend_decode_batched`` takes the arguments of
  ``PackedKVSidecar._attend_decode_batched``
  (third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:564-616):
  one query row per active request, the layer's paged ``kv_cache``
  ``[num_blocks, 2, page, H_kv, D]``, the KV-cache group's ``block_table``
  ``[R, max_pages]`` and physical ``seq_lens`` ``[R]``; it writes
  ``output[:n]`` in place.
* ``paged_decode`` runs many layers in one launch: layer ``l`` brings its own
  query, cache tensor, block table and seq_lens (its quota group's physical
  layout, gpu_model_runner.py:1672-1681, 2184-2204).

Both go through ``abkv_decode`` in libabkv.so.  There is no fallback: a
missing library or a non-CUDA tensor raises.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch

from . import _lib
from .workspace import Workspace, default_workspace

def _check_cuda(name: str, t: torch.Tensor, dtype: torch.dtype | None = None) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor (libabkv has no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")


def _validate(queries, kv_caches, block_tables, seq_lens, outputs, out_shape=None, alloc=True):
    """Check the per-layer arguments; -> (B, Hq, Hkv, D, page, outputs) (no outputs
    are allocated when `outputs` is None and `alloc` is False)."""
    L = len(queries)
    if not (L == len(kv_caches) == len(block_tables) == len(seq_lens)) or L == 0:
        raise ValueError("per-layer argument lists must be non-empty and of equal length")
    q0, kv0 = queries[0], kv_caches[0]
    B, Hq, D = q0.shape
    _, two, page, Hkv, D2 = kv0.shape
    if two != 2 or D2 != D:
        raise ValueError(f"kv cache must be [num_blocks, 2, page, Hkv, {D}], got {tuple(kv0.shape)}")
    device = q0.device
    out_shape = (B, Hq, D) if out_shape is None else tuple(out_shape)
    outs = []
    for l in range(L):
        q, kv, bt, sl = queries[l], kv_caches[l], block_tables[l], seq_lens[l]
        _check_cuda("query", q, torch.bfloat16)
        _check_cuda("kv_cache", kv, torch.bfloat16)
        _check_cuda("block_table", bt, torch.int32)
        _check_cuda("seq_lens", sl, torch.int32)
        if tuple(q.shape) != (B, Hq, D) or not q.is_contiguous():
            raise ValueError("every query must be a contiguous [B, Hq, D] tensor")
        if tuple(kv.shape[1:]) != (2, page, Hkv, D) or not kv.is_contiguous():
            raise ValueError("every kv cache must be a contiguous [num_blocks, 2, page, Hkv, D] tensor")
        if bt.dim() != 2 or bt.shape[0] < B or not bt.is_contiguous():
            raise ValueError("block_table must be a contiguous [>=B, max_pages] tensor")
        if sl.dim() != 1 or sl.shape[0] < B or not sl.is_contiguous():
            raise ValueError("seq_lens must be a contiguous [>=B] tensor")
        if outputs is not None:
            o = outputs[l]
            _check_cuda("output", o, torch.bfloat16)
            if tuple(o.shape) != out_shape or not o.is_contiguous():
                raise ValueError(f"every output must be a contiguous {list(out_shape)} tensor")
        elif alloc:
            o = torch.empty(out_shape, dtype=torch.bfloat16, device=device)
        else:
            continue
        outs.append(o)
    return B, Hq, Hkv, D, page, outs


def paged_decode(
    queries: Sequence[torch.Tensor],
    kv_caches: Sequence[torch.Tensor],
    block_tables: Sequence[torch.Tensor],
    seq_lens: Sequence[torch.Tensor],
    *,
    scale: float | None = None,
    outputs: Sequence[torch.Tensor] | None = None,
    max_pages_per_seq: int | None = None,
    chunk_tokens: int = 0,
    workspace: Workspace | None = None,
    stream: torch.cuda.Stream | None = None,
) -> list[torch.Tensor]:
    """Decode attention for ``len(queries)`` layers in one launch.

    queries[l]: [B, Hq, D] bf16; kv_caches[l]: [num_blocks, 2, page, Hkv, D] bf16;
    block_tables[l]: [B, max_pages_l] int32; seq_lens[l]: [B] int32.
    Returns outputs[l]: [B, Hq, D] bf16.
    """
    L = len(queries)
    B, Hq, Hkv, D, page, outs = _validate(queries, kv_caches, block_tables, seq_lens, outputs)
    device = queries[0].device
    if max_pages_per_seq is None:
        max_pages_per_seq = max(int(bt.shape[1]) for bt in block_tables)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lib = _lib.lib()
    need = lib.abkv_decode_workspace_size(L, B, Hq, D, page, max_pages_per_seq, chunk_tokens)
    if need == 0:
        raise _lib.AbkvError("abkv_decode_workspace_size", 3,
                             f"unsupported shape (B={B}, Hq={Hq}, D={D}, page={page})")
    ws = (workspace or default_workspace(device)).ensure(need)
    s = torch.cuda.current_stream(device) if stream is None else stream
    with torch.cuda.device(device):
        st = _call_decode(lib, queries, kv_caches, block_tables, seq_lens, outs, L, B, Hq, Hkv, D, page,
                          max_pages_per_seq, scale, chunk_tokens, ws, s)
    _lib.check("abkv_decode", st)
    return outs


def _call_decode(lib, queries, kv_caches, block_tables, seq_lens, outs, L, B, Hq, Hkv, D, page,
                 max_pages_per_seq, scale, chunk_tokens, ws, s):
    return lib.abkv_decode(
        _lib.ptr_array([q.data_ptr() for q in queries]),
        _lib.ptr_array([kv.data_ptr() for kv in kv_caches]),
        _lib.ptr_array([bt.data_ptr() for bt in block_tables]),
        _lib.i64_array([bt.stride(0) for bt in block_tables]),
        _lib.ptr_array([sl.data_ptr() for sl in seq_lens]),
        _lib.i64_array([kv.shape[0] for kv in kv_caches]),
        _lib.ptr_array([o.data_ptr() for o in outs]),
        L, B, Hq, Hkv, D, page, max_pages_per_seq, float(scale), chunk_tokens,
        ws.ptr(), ws.nbytes, s.cuda_stream,
    )


def attend_decode_batched(
    *,
    query: torch.Tensor,
    kv_cache: torch.Tensor,
    output: torch.Tensor,
    seq_lens: torch.Tensor,
    block_table: torch.Tensor,
    num_kv_heads: int,
    groups: int,
    scale: float,
    num_requests: int | None = None,
    workspace: Workspace | None = None,
) -> None:
    """Drop-in for ``PackedKVSidecar._attend_decode_batched`` (no sidecar pages).

    query: [>=n, Hq, D] (or [>=n, Hq*D]); output: same shape, written for the
    first n rows in place.  ``seq_lens`` may live on the host (vLLM's
    ``_seq_lens_cpu``); it is copied to the device when needed.
    """
    n = int(num_requests if num_requests is not None else block_table.shape[0])
    D = kv_cache.shape[-1]
    Hq = num_kv_heads * groups
    q = query[:n].reshape(n, Hq, D)
    if not q.is_contiguous():
        q = q.contiguous()
    sl = seq_lens[:n]
    if not sl.is_cuda:
        sl = sl.to(kv_cache.device, non_blocking=True)
    sl = sl.to(torch.int32).contiguous()
    bt = block_table[:n]
    if bt.dtype != torch.int32 or not bt.is_contiguous():
        bt = bt.to(torch.int32).contiguous()
    out_view = output[:n].reshape(n, Hq, D)
    direct = out_view.is_contiguous() and out_view.dtype == torch.bfloat16
    o = out_view if direct else torch.empty((n, Hq, D), dtype=torch.bfloat16, device=kv_cache.device)
    paged_decode([q], [kv_cache], [bt], [sl], scale=scale, outputs=[o], workspace=workspace)
    if not direct:
        out_view.copy_(o)


def forward_decode(
    query: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float,
    output: torch.Tensor | None = None,
    workspace: Workspace | None = None,
) -> torch.Tensor:
    """vLLM ``AttentionImpl.forward``-shaped decode for one layer:
    query [T, Hq, D] (T = one decode row per request), output [T, Hq*D]."""
    T, Hq, D = query.shape
    if output is None:
        output = torch.empty((T, Hq * D), dtype=query.dtype, device=query.device)
    Hkv = kv_cache.shape[3]
    attend_decode_batched(query=query, kv_cache=kv_cache, output=output, seq_lens=seq_lens,
                          block_table=block_table, num_kv_heads=Hkv, groups=Hq // Hkv,
                          scale=scale, num_requests=T, workspace=workspace)
    return output
