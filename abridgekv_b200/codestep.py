"""Code step over the paged cache (host side).

The code step runs the K code queries of every active request in one forward
pass: they attend, non-causally, to the request's rows [0, seq_len) in the
paged KV cache, where a KV head with quota q sees only the first q of the
request's own K code slots (the last K rows), and an optional per-request
"tail exclusion" range of rows is hidden as well.  This is the noncausal branch
of PackedKVSidecar._attend_request_vectorized
(third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:648-741),
driven per request from override_attention (:329-420) with
query_start_loc / seq_lens / block_table from the common attention metadata
and ranges from set_code_excluded_ranges (:244-260).

``code_step_attention`` runs all requests, all heads in one launch of
``abkv_code_step_attention`` (tcgen05 tensor cores; libabkv.so).  There is no
CPU path: a missing library or a non-CUDA tensor raises.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Mapping, Sequence

import numpy as np
import torch

from . import _lib
from .workspace import Workspace, default_workspace


def _layout_of(kv: torch.Tensor, num_kv_heads: int) -> tuple[int, int, int]:
    """-> (kv_layout, num_blocks, page) for a contiguous paged cache."""
    if kv.dim() != 5 or not kv.is_contiguous():
        raise ValueError("kv_cache must be a contiguous 5-D paged cache")
    if kv.shape[1] == 2 and kv.shape[3] == num_kv_heads:
        return 0, kv.shape[0], kv.shape[2]           # FlashInfer [nb, 2, page, Hkv, D]
    if kv.shape[0] == 2 and kv.shape[3] == num_kv_heads:
        return 1, kv.shape[1], kv.shape[2]           # FlashAttention [2, nb, page, Hkv, D]
    raise ValueError(f"unrecognised paged KV layout {tuple(kv.shape)}")


def _prepare(query, kv_cache, block_table, seq_lens, query_start_loc, quota_per_kv_head, scale, excluded,
             num_requests, out, num_kv_heads=None):
    """Checks the code-step (or, with quota_per_kv_head None, the causal prefill) arguments ->
    (leading arguments of the C call, out, R, num_blocks, page, T, scale)."""
    for name, t in (("query", query), ("kv_cache", kv_cache)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be a bf16 CUDA tensor (libabkv has no CPU path)")
    if query.dim() != 3 or query.stride(2) != 1:
        raise ValueError("query must be [T, Hq, D] with a contiguous last dimension")
    T, Hq, D = query.shape
    Hkv = len(quota_per_kv_head) if quota_per_kv_head is not None else int(num_kv_heads)
    if Hkv <= 0 or Hq % Hkv:
        raise ValueError("the KV heads (one quota per KV head) must divide the query heads")
    layout, nb, page = _layout_of(kv_cache, Hkv)
    R = block_table.shape[0] if num_requests is None else int(num_requests)
    dev = query.device

    def i32(name, t, shape_ok):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.int32:
            raise TypeError(f"{name} must be an int32 CUDA tensor")
        if not shape_ok(t):
            raise ValueError(f"{name} has shape {tuple(t.shape)}")
        return t.contiguous()

    bt = i32("block_table", block_table, lambda t: t.dim() == 2 and t.shape[0] >= R)
    if bt.stride(1) != 1:
        raise ValueError("block_table rows must be contiguous")
    sl = i32("seq_lens", seq_lens, lambda t: t.dim() == 1 and t.shape[0] >= R)
    need_qs = R if quota_per_kv_head is not None else R + 1  # the causal mode reads query_start_loc[r + 1]
    qs = i32("query_start_loc", query_start_loc, lambda t: t.dim() == 1 and t.shape[0] >= need_qs)
    ex = None
    if excluded is not None:
        ex = i32("excluded", excluded, lambda t: t.dim() == 2 and t.shape[0] >= R and t.shape[1] == 2)
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=dev)
    if tuple(out.shape) != (T, Hq, D) or out.dtype != torch.bfloat16 or out.stride(2) != 1:
        raise ValueError("out must be a bf16 [T, Hq, D] tensor with a contiguous last dimension")
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    if quota_per_kv_head is None:  # abkv_paged_prefill's leading arguments
        head = (query.data_ptr(), query.stride(0), query.stride(1), out.data_ptr(), out.stride(0), out.stride(1),
                qs.data_ptr(), kv_cache.data_ptr(), layout, nb, page, bt.data_ptr(), bt.stride(0), sl.data_ptr(),
                R, Hq, Hkv, D)
        return head, out, R, nb, page, T, scale
    head = (query.data_ptr(), query.stride(0), query.stride(1), out.data_ptr(), out.stride(0), out.stride(1),
            qs.data_ptr(), kv_cache.data_ptr(), layout, nb, page, bt.data_ptr(), bt.stride(0), sl.data_ptr(),
            ex.data_ptr() if ex is not None else None, _lib.i32_array(quota_per_kv_head), R, Hq, Hkv, D)
    return head, out, R, nb, page, T, scale


def _sidecar(sidecar, Hkv: int, D: int, R: int):
    """abkv_sidecar_t of a SidecarPool (its request slot i = request i of the launch)."""
    if len(sidecar.quotas) != Hkv or sidecar.pages.shape[-1] != D or sidecar.page_table.shape[0] < R:
        raise ValueError("the sidecar pool does not match the cache geometry or the number of requests")
    return sidecar.descriptor()


def code_step_attention(query: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                        seq_lens: torch.Tensor, query_start_loc: torch.Tensor, *,
                        quota_per_kv_head: Sequence[int], k_max: int, scale: float | None = None,
                        excluded: torch.Tensor | None = None, num_requests: int | None = None,
                        out: torch.Tensor | None = None, workspace: Workspace | None = None,
                        stream: torch.cuda.Stream | None = None, sidecar=None) -> torch.Tensor:
    """query [T, Hq, D] bf16 (last dim contiguous); kv_cache paged bf16 (either layout);
    block_table [R, max_pages] int32; seq_lens [R] int32 (each >= k_max); query_start_loc
    [>= R] int32 (request r's code queries are rows query_start_loc[r] .. + k_max - 1);
    quota_per_kv_head: this layer's quotas (each in [0, k_max]); excluded: optional [R, 2]
    int32 hidden row ranges (start == end = none); sidecar: an optional ``sidecar.SidecarPool`` of this
    layer whose request slot i holds request i's packed pages -- KV head h then first attends to its
    slots of those pages (``abkv_code_step_attention_packed``).  Writes and returns out [T, Hq, D]."""
    head, out, R, nb, page, T, scale = _prepare(query, kv_cache, block_table, seq_lens, query_start_loc,
                                                quota_per_kv_head, scale, excluded, num_requests, out)
    dev = query.device
    ws = workspace or default_workspace(dev)
    s = torch.cuda.current_stream(dev) if stream is None else stream
    lib = _lib.lib()
    with torch.cuda.device(dev):
        if sidecar is None:
            st = lib.abkv_code_step_attention(*head, int(k_max), T, scale, ws.ptr(), ws.nbytes, s.cuda_stream)
        else:
            desc = _sidecar(sidecar, len(quota_per_kv_head), query.shape[2], R)
            st = lib.abkv_code_step_attention_packed(*head, int(k_max), T, scale, C.addressof(desc), ws.ptr(),
                                                     ws.nbytes, s.cuda_stream)
    _lib.check("abkv_code_step_attention" + ("_packed" if sidecar is not None else ""), st)
    return out


def paged_prefill(query: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                  query_start_loc: torch.Tensor, *, max_query_len: int, num_kv_heads: int,
                  scale: float | None = None, num_requests: int | None = None, out: torch.Tensor | None = None,
                  workspace: Workspace | None = None, stream: torch.cuda.Stream | None = None,
                  sidecar=None) -> torch.Tensor:
    """Causal attention of ragged query rows over the paged cache (prompt prefill, chunked prefill and
    mixed prefill/decode batches): request r's rows are ``query_start_loc[r] .. query_start_loc[r + 1] - 1``
    (qlen rows, their keys already written at cache rows [seq_len - qlen, seq_len)), and row i attends
    to cache rows ``[0, seq_len - qlen + i + 1)``.  This is the causal branch of
    PackedKVSidecar._attend_request_vectorized (compresslm_packed_kv.py:700-707) without sidecar
    pages, and the paged causal prefill the stock backend runs for a CompressLM KV-cache group.

    query [T, Hq, D] bf16 (last dim contiguous), D = 128; kv_cache paged bf16 (either layout);
    block_table [R, max_pages] int32; seq_lens [R] int32 (each >= its qlen); query_start_loc
    [>= R + 1] int32; max_query_len >= every qlen (vLLM's ``max_query_len``); sidecar: an optional
    ``sidecar.SidecarPool`` (request slot i = request i): KV head h first attends to its slots of the
    request's packed pages, from every query row (``abkv_paged_prefill_packed``).  Writes and returns
    out [T, Hq, D] (rows of no request are left untouched)."""
    head, out, R, nb, page, T, scale = _prepare(query, kv_cache, block_table, seq_lens, query_start_loc, None,
                                                scale, None, num_requests, out, num_kv_heads=num_kv_heads)
    if int(max_query_len) <= 0 or int(max_query_len) > T:
        raise ValueError(f"max_query_len must be in [1, T={T}]")
    dev = query.device
    ws = workspace or default_workspace(dev)
    s = torch.cuda.current_stream(dev) if stream is None else stream
    lib = _lib.lib()
    with torch.cuda.device(dev):
        if sidecar is None:
            st = lib.abkv_paged_prefill(*head, int(max_query_len), T, scale, ws.ptr(), ws.nbytes, s.cuda_stream)
        else:
            desc = _sidecar(sidecar, int(num_kv_heads), query.shape[2], R)
            st = lib.abkv_paged_prefill_packed(*head, int(max_query_len), T, scale, C.addressof(desc), ws.ptr(),
                                               ws.nbytes, s.cuda_stream)
    _lib.check("abkv_paged_prefill" + ("_packed" if sidecar is not None else ""), st)
    return out


def check_op_ownership(ops: np.ndarray, op_offsets: np.ndarray, block_table_host, seq_lens_host,
                       page: int) -> None:
    """Raise ValueError unless request r's copy ops read and write only pages of its own live
    block-table row (the first ceil(seq_len / page) entries) and no other request's live row holds
    a page that r writes.  Shared (prefix-cached) pages fail the check: their copies would race
    with the other request's loads inside the fused launch."""
    bt = np.asarray(block_table_host)
    sl = np.asarray(seq_lens_host).astype(np.int64)
    R = len(op_offsets) - 1
    if bt.ndim != 2 or bt.shape[0] < R or sl.shape[0] < R:
        raise ValueError("block_table_host / seq_lens_host must cover every request of the launch")
    live = [bt[r, :(int(sl[r]) + page - 1) // page].astype(np.int64) for r in range(R)]
    owners: dict[int, set[int]] = {}
    for r, row in enumerate(live):
        for pg in np.unique(row).tolist():
            owners.setdefault(pg, set()).add(r)
    for r in range(R):
        mine = ops[op_offsets[r]:op_offsets[r + 1]]
        if not len(mine):
            continue
        own = set(live[r].tolist())
        for pg in np.unique(np.concatenate([mine[:, 0], mine[:, 2]])).tolist():
            if pg not in own:
                raise ValueError(f"request {r}: copy op touches page {pg} outside its own block-table row")
        for pg in np.unique(mine[:, 2]).tolist():
            if owners.get(pg, {r}) != {r}:
                raise ValueError(f"request {r}: copy op writes page {pg}, which other requests of the launch "
                                 "also read (shared pages): use code_step_attention + the executor")


def code_step_attention_compact(query: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                                seq_lens: torch.Tensor, query_start_loc: torch.Tensor, *, ops,
                                op_offsets: Sequence[int], quota_per_kv_head: Sequence[int], k_max: int,
                                replay_tail: int, block_table_host=None, seq_lens_host=None,
                                scale: float | None = None, excluded: torch.Tensor | None = None,
                                num_requests: int | None = None, out: torch.Tensor | None = None,
                                workspace: Workspace | None = None,
                                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """``code_step_attention`` followed, in the same launch, by the compaction of this layer's cache:
    request r's (src_block, src_off, dst_block, dst_off) row copies ``ops[op_offsets[r] ..
    op_offsets[r + 1])`` are applied once every CTA of request r has read the cache.  Same result as
    ``code_step_attention`` then ``compaction.execute_kv_copy_group(ops, [kv_cache])``; a batch whose
    destinations repeat or overlap its sources is rejected (use the separate executor for it).

    Ordering: the reference finishes a block (and plans its compaction) right after the code step
    only when the configuration has no replay tail -- ``CompressLMProcessor.update_after_step``
    calls ``_finish_block`` at the end of the code role only when the block has no replay positions
    (third_party/vllm_overlay/vllm/v1/core/compresslm/processor.py:236-255); with a replay tail the
    block finishes after the replay step, whose queries still read the uncompacted rows.  So the
    caller states ``replay_tail`` (``CompressLMConfig.replay_tail``) and any value but 0 is refused;
    the ops are those the planner's ``finish_block`` produced for the block, planned before this
    launch.  Ownership: each request's ops must stay in its own pages; pass ``block_table_host`` and
    ``seq_lens_host`` (host copies of the launch's tables) to have that checked."""
    if int(replay_tail) != 0:
        raise ValueError(f"code_step_attention_compact needs replay_tail == 0 (got {replay_tail}): with a replay "
                         "tail the block finishes after its replay step, so its compaction cannot ride in the "
                         "code step; use code_step_attention and apply the ops after the replay step")
    head, out, R, nb, page, T, scale = _prepare(query, kv_cache, block_table, seq_lens, query_start_loc,
                                                quota_per_kv_head, scale, excluded, num_requests, out)
    arr = np.ascontiguousarray(getattr(ops, "array", ops), dtype=np.int32).reshape(-1, 4)
    off = np.ascontiguousarray(op_offsets, dtype=np.int64)
    if off.shape != (R + 1,):
        raise ValueError(f"op_offsets must hold R + 1 = {R + 1} entries")
    if block_table_host is not None or seq_lens_host is not None:
        if block_table_host is None or seq_lens_host is None:
            raise ValueError("the ownership check needs both block_table_host and seq_lens_host")
        check_op_ownership(arr, off, block_table_host, seq_lens_host, page)
    dev = query.device
    lib = _lib.lib()
    need = lib.abkv_code_step_compact_workspace_size(R, len(arr))
    if need == 0:
        raise ValueError("too many copy ops")
    ws = (workspace or default_workspace(dev)).ensure(need)
    s = torch.cuda.current_stream(dev) if stream is None else stream
    with torch.cuda.device(dev):
        st = lib.abkv_code_step_attention_compact(*head, int(k_max), T, scale, arr.ctypes.data_as(_lib.c_i32p),
                                                  off.ctypes.data_as(_lib.c_i64p), len(arr), ws.ptr(), ws.nbytes,
                                                  s.cuda_stream)
    _lib.check("abkv_code_step_attention_compact", st)
    return out


def excluded_tensor(request_ids: Sequence[str], ranges: Mapping[str, tuple[int, int]] | None,
                    device: torch.device | str) -> torch.Tensor | None:
    """[R, 2] int32 exclusion ranges in active-request order from the mapping the reference's
    set_code_excluded_ranges takes (compresslm_packed_kv.py:244-260): None when there is none.
    A request missing from a non-empty mapping raises, as _code_excluded_range does."""
    if not ranges:
        return None
    rows = []
    for rid in request_ids:
        if rid not in ranges:
            raise RuntimeError(f"packed KV code step: request {rid} has no tail exclusion range")
        rows.append(tuple(int(x) for x in ranges[rid]))
    return torch.tensor(rows, dtype=torch.int32, device=device).reshape(len(rows), 2)
