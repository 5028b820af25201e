"""vLLM-shaped attention boundary of the compressed cache (host side).

The reference serves CompressLM through vLLM 0.13.0 with an overlay.  Its
attention meets the cache at two places, both reproduced here over libabkv:

* The stock backend of each KV-cache group.  Per-layer quotas are served as one
  KV-cache group per quota, each with its own compacted block table and
  physical ``seq_lens`` (gpu_model_runner.py:1872-1886, 2184-2266).  The
  backend's ``AttentionImpl.forward(layer, query, key, value, kv_cache,
  attn_metadata, output)`` first writes the step's K/V rows into the cache
  (vLLM's reshape_and_cache_flash) and then attends.  Decode steps are causal
  with one query row per request.  Prompt, chunked-prefill and replay steps are
  causal with ragged query rows.  The code step is noncausal: the K code
  queries of each request see every row except the block's own code slots at
  or past the group's quota and an optional static-tail range.  The reference
  passes that visibility as a FlashInfer custom mask built by
  ``build_layer_quota_masks`` (compresslm_masks.py:165-239).
  ``AbkvAttentionBackend`` / ``AbkvMetadataBuilder`` / ``AbkvAttentionImpl``
  take the same calls.  ``build_layer_quota_masks`` here has the reference's
  signature but returns a ``CodeStepMask`` descriptor (quota + excluded ranges)
  instead of a boolean matrix, which the code-step kernel evaluates on the fly.
* The packed per-head-quota hook ``maybe_override_attention(layer, query,
  kv_cache, attn_metadata, output)`` (compresslm_packed_kv.py:744-761,
  installed into vLLM's ``Attention.forward`` by patch_stock_attention.py:
  20-42), which calls the layer's sidecar ``override_attention``
  (:329-420).  ``CompressedKVSidecar`` keeps the reference sidecar's state
  (active request ids, common metadata, code exclusion ranges, packed pages)
  and dispatches in the same way:
  causal with one row per request -> decode over sidecar pages + the paged cache;
  causal with ragged rows -> causal paged prefill; noncausal -> the code step
  with the layer's per-KV-head quotas.

Every attention call runs a libabkv kernel (abkv_decode, abkv_decode_packed,
abkv_paged_prefill[_packed], abkv_code_step_attention[_packed], abkv_store_kv).
There is no CPU path and no fallback.  Masked (non-physical) per-layer quotas,
which the kernels do not serve, raise ``NotImplementedError``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np
import torch

from . import _lib, codestep, decode
from .sidecar import PackedKVLayout, SidecarPool, packed_decode
from .workspace import Workspace, default_workspace


# ---------------------------------------------------------------------------
# code-step visibility (build_layer_quota_masks)
@dataclass
class CodeStepMask:
    """Visibility of one quota group's code step, as the kernel takes it.

    For every request of the step, the code queries see cache rows
    ``[0, seq_len - (num_code_tokens - quota))``: the block's own code slots at or past ``quota``
    (the last ``num_code_tokens - quota`` rows) are hidden.  A request's optional ``excluded`` range
    ``[start, end)`` is hidden as well (start == end: none).  ``quota >= num_code_tokens`` hides
    no code slot (exclusion only).  This is what the reference's boolean mask holds for a code
    step of a physical quota group (compresslm_masks.py:165-239 with causal=False and one resident
    span per request, the block's own codes)."""

    quota: int
    num_code_tokens: int
    excluded: np.ndarray | None = None  # [R, 2] int32 or None
    _dev: dict = field(default_factory=dict, repr=False, compare=False)

    def excluded_device(self, device: torch.device) -> torch.Tensor | None:
        if self.excluded is None:
            return None
        key = str(device)
        if key not in self._dev:
            self._dev[key] = torch.as_tensor(self.excluded, dtype=torch.int32).to(device)
        return self._dev[key]


def build_layer_quota_masks(
    requests: list[tuple[int, int, list[tuple[int, int]], tuple[int, int] | None]],
    quotas: list[int],
    num_code_tokens: int,
    causal: bool,
    device: torch.device | str | None = None,
) -> dict[int, CodeStepMask]:
    """Drop-in for the reference's ``build_layer_quota_masks`` (compresslm_masks.py:165-239).

    ``requests`` holds one ``(query_len, seq_len, code_spans, excluded_range)`` per request in
    batch order, as the reference's model runner builds it (gpu_model_runner.py:2064-2107).
    Returns ``{quota: CodeStepMask}``.  The reference fills
    ``compresslm_custom_mask`` with the same dictionary's values, and ``AbkvMetadataBuilder``
    reads them from there.  Only the code step of physical quota groups is served:
    ``causal=True`` (the masked layer-quota mode, where one shared cache keeps every code row and
    each layer masks them) raises ``NotImplementedError``.  A code span that hides rows must be the
    request's own code rows, the last ``num_code_tokens`` rows of the request, with every query
    row a code query."""
    if not requests:
        return {}
    qlens = [int(q) for q, _, _, _ in requests]
    slens = [int(s) for _, s, _, _ in requests]
    if any(q <= 0 for q in qlens) or any(q > s for q, s in zip(qlens, slens)):
        raise ValueError("invalid query_len/seq_len in layer-quota mask build")
    if causal:
        raise NotImplementedError(
            "masked per-layer code quotas (one shared cache holding every code row) are not served by "
            "libabkv: use physical_layer_quotas (one KV-cache group per quota)")
    K = int(num_code_tokens)
    excl = np.zeros((len(requests), 2), dtype=np.int32)
    any_excl = False
    for r, (_, _, _, ex) in enumerate(requests):
        if ex is not None:
            excl[r] = (int(ex[0]), int(ex[1]))
            any_excl = any_excl or ex[1] > ex[0]
    out: dict[int, CodeStepMask] = {}
    for q in quotas:
        q = int(q)
        if q < K:
            for r, (qlen, s_len, spans, _) in enumerate(requests):
                hides = [(int(a), int(b)) for a, b in spans if int(a) + q < int(b)]
                if not hides:
                    raise NotImplementedError(
                        f"request {r}: no resident code span to hide for quota {q}; the code-step kernel "
                        "hides the block's own code slots of every request")
                if hides != [(s_len - K, s_len)] or qlen != K:
                    raise NotImplementedError(
                        f"request {r}: code spans {hides} are not the step's own {K} code rows "
                        f"[{s_len - K}, {s_len}) with {K} code queries")
        out[q] = CodeStepMask(quota=min(q, K), num_code_tokens=K, excluded=excl.copy() if any_excl else None)
    return out


# ---------------------------------------------------------------------------
# the stock backend of a KV-cache group
@dataclass
class AbkvAttentionMetadata:
    """Per-step metadata of one KV-cache group (the fields of vLLM's CommonAttentionMetadata this
    backend reads, gpu_model_runner.py:1872-1886, plus the derived dispatch facts)."""

    num_actual_tokens: int
    num_reqs: int
    max_query_len: int
    query_start_loc: torch.Tensor       # device int32 [R + 1]
    query_start_loc_cpu: torch.Tensor   # host   int32 [R + 1]
    seq_lens: torch.Tensor              # device int32 [R] (the group's physical lengths)
    seq_lens_cpu: torch.Tensor          # host   int32 [R]
    block_table: torch.Tensor           # device int32 [R, max_pages]
    slot_mapping: torch.Tensor          # device int64 [T]
    causal: bool
    code_mask: CodeStepMask | None
    decode_only: bool                   # every request has exactly one query row


class AbkvMetadataBuilder:
    """vLLM's ``AttentionMetadataBuilder`` shape: ``build(common_prefix_len, common_attn_metadata)``
    -> ``AbkvAttentionMetadata``.  Reads ``query_start_loc(_cpu)``, ``seq_lens`` /
    ``_seq_lens_cpu``, ``block_table_tensor``, ``slot_mapping``, ``num_reqs``,
    ``num_actual_tokens``, ``max_query_len``, ``causal`` and ``compresslm_custom_mask`` (a
    ``CodeStepMask`` from this module's ``build_layer_quota_masks``).  Prefix cascades are not used
    (the reference disables them under CompressLM masks)."""

    def __init__(self, kv_cache_spec: Any = None, layer_names: Sequence[str] | None = None,
                 vllm_config: Any = None, device: torch.device | str | None = None):
        self.kv_cache_spec = kv_cache_spec
        self.layer_names = list(layer_names or [])
        self.vllm_config = vllm_config
        self.device = device

    def build(self, common_prefix_len: int, common_attn_metadata: Any, fast_build: bool = False
              ) -> AbkvAttentionMetadata:
        cm = common_attn_metadata
        R = int(cm.num_reqs)
        T = int(cm.num_actual_tokens)
        qsl_cpu = torch.as_tensor(cm.query_start_loc_cpu[:R + 1], dtype=torch.int32)
        seq_cpu = getattr(cm, "_seq_lens_cpu", None)
        if seq_cpu is None:
            seq_cpu = getattr(cm, "seq_lens_cpu")
        seq_cpu = torch.as_tensor(seq_cpu[:R], dtype=torch.int32)
        qlens = (qsl_cpu[1:] - qsl_cpu[:-1]).tolist()
        mask = getattr(cm, "compresslm_custom_mask", None)
        if mask is not None and not isinstance(mask, CodeStepMask):
            raise TypeError("compresslm_custom_mask must come from abridgekv_b200.attention.build_layer_quota_masks "
                            "(a CodeStepMask), not a dense boolean mask")
        bt = cm.block_table_tensor[:R]
        if bt.dtype != torch.int32 or not bt.is_contiguous():
            bt = bt.to(torch.int32).contiguous()
        qsl = cm.query_start_loc[:R + 1]
        sl = cm.seq_lens[:R]
        return AbkvAttentionMetadata(
            num_actual_tokens=T, num_reqs=R, max_query_len=int(max(qlens) if qlens else 0),
            query_start_loc=qsl if qsl.dtype == torch.int32 else qsl.to(torch.int32),
            query_start_loc_cpu=qsl_cpu,
            seq_lens=sl if sl.dtype == torch.int32 else sl.to(torch.int32),
            seq_lens_cpu=seq_cpu, block_table=bt, slot_mapping=cm.slot_mapping[:T],
            causal=bool(cm.causal), code_mask=mask, decode_only=bool(qlens) and all(q == 1 for q in qlens))


class AbkvAttentionImpl:
    """vLLM's ``AttentionImpl`` shape for a CompressLM KV-cache group, on libabkv kernels.

    ``forward(layer, query, key, value, kv_cache, attn_metadata, output)``: query ``[T, Hq, D]``
    (or ``[T, Hq*D]``), key / value ``[T, Hkv, D]`` (the step's new rows; None to skip the cache
    write), kv_cache ``[num_blocks, 2, page, Hkv, D]`` bf16, output ``[T, Hq*D]`` (written in place
    for the step's ``num_actual_tokens`` rows and returned)."""

    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int | None = None,
                 alibi_slopes: Any = None, sliding_window: int | None = None, kv_cache_dtype: str = "auto",
                 logits_soft_cap: float | None = None, attn_type: str = "decoder",
                 kv_sharing_target_layer_name: str | None = None, workspace: Workspace | None = None):
        if alibi_slopes is not None or sliding_window not in (None, -1) or logits_soft_cap:
            raise NotImplementedError("alibi, sliding windows and logit soft-capping are not part of the "
                                      "compressed-cache attention path")
        if kv_cache_dtype not in ("auto", "bfloat16"):
            raise NotImplementedError(f"kv_cache_dtype {kv_cache_dtype!r}: the kernels read bf16 caches")
        self.num_heads = int(num_heads)
        self.head_size = int(head_size)
        self.scale = float(scale)
        self.num_kv_heads = int(num_kv_heads or num_heads)
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        self.workspace = workspace

    def _ws(self, device) -> Workspace:
        return self.workspace or default_workspace(device)

    def forward(self, layer: Any, query: torch.Tensor, key: torch.Tensor | None, value: torch.Tensor | None,
                kv_cache: torch.Tensor, attn_metadata: AbkvAttentionMetadata | None,
                output: torch.Tensor | None = None, output_scale: Any = None,
                output_block_scale: Any = None) -> torch.Tensor:
        Hq, Hkv, D = self.num_heads, self.num_kv_heads, self.head_size
        if output is None:
            output = torch.empty((query.shape[0], Hq * D), dtype=torch.bfloat16, device=query.device)
        if attn_metadata is None:  # vLLM's profiling run
            return output.fill_(0)
        md = attn_metadata
        T = md.num_actual_tokens
        ws = self._ws(query.device)
        if key is not None and value is not None and self.kv_sharing_target_layer_name is None:
            store_kv(key[:T].view(T, Hkv, D), value[:T].view(T, Hkv, D), kv_cache, md.slot_mapping[:T],
                     workspace=ws)
        q = query[:T].view(T, Hq, D)
        out = output[:T].view(T, Hq, D)
        attend(q, kv_cache, md, out, num_kv_heads=Hkv, scale=self.scale, workspace=ws)
        return output


def attend(q: torch.Tensor, kv_cache: torch.Tensor, md: AbkvAttentionMetadata, out: torch.Tensor, *,
           num_kv_heads: int, scale: float, workspace: Workspace | None = None,
           k_max: int | None = None, quota_per_kv_head: Sequence[int] | None = None,
           excluded: torch.Tensor | None = None, sidecar: SidecarPool | None = None) -> None:
    """Attention of one layer's step over its KV-cache group (the dispatch of AbkvAttentionImpl and of
    the sidecar hook): decode, causal paged prefill, or the code step; with a sidecar pool, the causal
    prefill and the code step read the requests' packed pages first.  q / out ``[T, Hq, D]``."""
    R = md.num_reqs
    if R == 0 or md.num_actual_tokens == 0:
        return
    if md.causal:
        if md.decode_only and sidecar is None:
            qc = q if q.is_contiguous() else q.contiguous()
            direct = out.is_contiguous()
            o = out if direct else torch.empty_like(qc)
            decode.paged_decode([qc[:R]], [kv_cache], [md.block_table], [md.seq_lens], scale=scale,
                                outputs=[o[:R]], workspace=workspace)
            if not direct:
                out.copy_(o)
            return
        codestep.paged_prefill(q, kv_cache, md.block_table, md.seq_lens, md.query_start_loc,
                               max_query_len=md.max_query_len, num_kv_heads=num_kv_heads, scale=scale,
                               num_requests=R, out=out, workspace=workspace, sidecar=sidecar)
        return
    # noncausal: the code step (every request's query rows are its code queries)
    qlens = (md.query_start_loc_cpu[1:] - md.query_start_loc_cpu[:-1]).tolist()
    mask = md.code_mask
    if k_max is None:
        k_max = mask.num_code_tokens if mask is not None else qlens[0]
    if any(n != k_max for n in qlens):
        raise NotImplementedError(f"a code step needs every request to bring its {k_max} code queries; got "
                                  f"query lengths {sorted(set(qlens))}")
    if quota_per_kv_head is None:
        quota_per_kv_head = [mask.quota if mask is not None else k_max] * num_kv_heads
    if excluded is None and mask is not None:
        excluded = mask.excluded_device(q.device)
    codestep.code_step_attention(q, kv_cache, md.block_table, md.seq_lens, md.query_start_loc,
                                 quota_per_kv_head=list(quota_per_kv_head), k_max=k_max, scale=scale,
                                 excluded=excluded, num_requests=R, out=out, workspace=workspace, sidecar=sidecar)


class AbkvAttentionBackend:
    """vLLM's ``AttentionBackend`` shape: names the impl / builder / metadata classes and the paged
    cache shape (FlashInfer's NHD layout, gpu_model_runner.py:1216-1217)."""

    accept_output_buffer = True

    @staticmethod
    def get_name() -> str:
        return "ABKV_SM100"

    @staticmethod
    def get_impl_cls():
        return AbkvAttentionImpl

    @staticmethod
    def get_builder_cls():
        return AbkvMetadataBuilder

    @staticmethod
    def get_metadata_cls():
        return AbkvAttentionMetadata

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        return (num_blocks, 2, block_size, num_kv_heads, head_size)

    @staticmethod
    def get_supported_head_sizes() -> list[int]:
        return [128]


def store_kv(key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor, slot_mapping: torch.Tensor, *,
             workspace: Workspace | None = None, stream: torch.cuda.Stream | None = None) -> None:
    """The step's new rows into the paged cache (``abkv_store_kv``): key / value ``[T, Hkv, D]`` bf16
    (each head's D contiguous), slot_mapping ``[T]`` int64 (negative = padding, skipped)."""
    for name, t in (("key", key), ("value", value), ("kv_cache", kv_cache)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be a bf16 CUDA tensor (libabkv has no CPU path)")
    if key.dim() != 3 or key.shape != value.shape or key.stride(2) != 1 or value.stride(2) != 1:
        raise ValueError("key and value must be [T, Hkv, D] with a contiguous last dimension")
    T, Hkv, D = key.shape
    layout, nb, page = codestep._layout_of(kv_cache, Hkv)
    sm = slot_mapping
    if not isinstance(sm, torch.Tensor) or not sm.is_cuda:
        raise TypeError("slot_mapping must be a CUDA tensor")
    if sm.dtype != torch.int64 or not sm.is_contiguous():
        sm = sm.to(torch.int64).contiguous()
    if sm.shape[0] < T:
        raise ValueError("slot_mapping must hold one slot per token")
    dev = key.device
    ws = workspace or default_workspace(dev)
    s = torch.cuda.current_stream(dev) if stream is None else stream
    with torch.cuda.device(dev):
        st = _lib.lib().abkv_store_kv(key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
                                      value.stride(0), value.stride(1), kv_cache.data_ptr(), layout, nb, page, Hkv,
                                      D, sm.data_ptr(), T, ws.ptr(), ws.nbytes, s.cuda_stream)
    _lib.check("abkv_store_kv", st)


# ---------------------------------------------------------------------------
# the packed per-head-quota hook (maybe_override_attention)
class CompressedKVSidecar:
    """Worker-side state of the packed per-head-quota mode, in the reference sidecar's shape
    (PackedKVSidecar, compresslm_packed_kv.py:212-420): one ``SidecarPool`` per layer holds every
    active request's packed pages on the device; ``capture`` appends a finished block's code rows,
    ``free`` drops a request; ``override_attention`` runs the layer's attention on libabkv.

    Request slots: request ``active_request_ids[i]`` is row i of the step's block table and row i of
    every pool's page table (``set_active_request_ids`` re-seats the pools when the batch changes)."""

    def __init__(self, layout: PackedKVLayout, attention_layers: Sequence[object], *, block_size: int,
                 max_requests: int = 256, max_pages_per_request: int = 128, pages_per_layer: int | None = None,
                 head_dim: int = 128, device: torch.device | str = "cuda", workspace: Workspace | None = None):
        if len(attention_layers) != layout.num_layers:
            raise ValueError(f"received {len(attention_layers)} attention layers for "
                             f"{layout.num_layers}-layer packed layout")
        self.layout = layout
        self.attention_layers = tuple(attention_layers)
        self.block_size = int(block_size)
        cap = pages_per_layer or max_requests * max_pages_per_request
        self.pools = [SidecarPool(layout, l, capacity=cap, num_requests=max_requests,
                                  max_pages=max_pages_per_request, head_dim=head_dim, device=device)
                      for l in range(layout.num_layers)]
        self.pages: dict[str, list[list[torch.Tensor]]] = {}  # request -> per layer packed pages (dense copies)
        self.active_request_ids: tuple[str, ...] = ()
        self.common_attn_metadata: object | None = None
        self.code_excluded_ranges: dict[str, tuple[int, int]] | None = None
        self.workspace = workspace
        self._seated: tuple[str, ...] = ()

    # -- state (same calls as the reference sidecar) --------------------------------------
    def set_active_request_ids(self, request_ids: Sequence[str]) -> None:
        self.active_request_ids = tuple(request_ids)

    def set_code_excluded_ranges(self, ranges: dict[str, tuple[int, int]] | None) -> None:
        self.code_excluded_ranges = dict(ranges) if ranges else None

    def set_common_attn_metadata(self, metadata: object) -> None:
        self.common_attn_metadata = metadata

    def free(self, request_id: str) -> None:
        self.pages.pop(request_id, None)

    def capture(self, request_id: str, *, physical_start: int, physical_end: int, block_ids: Sequence[int]) -> None:
        """Pack the finished block's code rows ``[physical_start, physical_end)`` (exactly ``k_max``
        rows, through ``block_ids``) of every layer's cache (compresslm_packed_kv.py:290-320)."""
        if physical_end - physical_start != self.layout.k_max:
            raise ValueError("packed KV capture must contain exactly k_max code rows; "
                             f"got {physical_end - physical_start}, expected {self.layout.k_max}")
        per_layer = self.pages.setdefault(request_id, [[] for _ in range(self.layout.num_layers)])
        for l, attention in enumerate(self.attention_layers):
            kv = attention.kv_cache[0]
            pos = torch.arange(physical_start, physical_end, device=kv.device)
            blocks = torch.as_tensor(list(block_ids), dtype=torch.long, device=kv.device)[pos // self.block_size]
            dense = kv[blocks, :, pos % self.block_size].permute(1, 0, 2, 3)  # [2, K, Hkv, D]
            per_layer[l].append(self.layout.pack_layer(l, dense))
        self._seated = ()  # re-seat the pools at the next step

    def _seat(self) -> None:
        """Make pool slot i hold the pages of active request i (only when the batch changed)."""
        if self._seated == self.active_request_ids:
            return
        for l, pool in enumerate(self.pools):
            for slot in range(pool.page_table.shape[0]):
                pool.free(slot)
            for i, rid in enumerate(self.active_request_ids):
                for page in self.pages.get(rid, [[]] * self.layout.num_layers)[l]:
                    pool.append(i, page)
        self._seated = self.active_request_ids

    # -- attention -------------------------------------------------------------------------
    def override_attention(self, *, layer_index: int, layer: object, query: torch.Tensor, kv_cache: torch.Tensor,
                           attn_metadata: object, output: torch.Tensor) -> None:
        if not self.active_request_ids:
            return
        if query.dtype != torch.bfloat16:
            raise RuntimeError(f"packed KV attention on libabkv needs bf16 queries, got {query.dtype}")
        common = self.common_attn_metadata
        if common is None:
            raise RuntimeError("packed KV common attention metadata is absent")
        n = len(self.active_request_ids)
        Hq, Hkv = int(layer.num_heads), int(layer.num_kv_heads)
        scale = float(layer.impl.scale)
        D = kv_cache.shape[-1]
        md = AbkvMetadataBuilder().build(0, _SidecarView(common, n))
        ws = self.workspace or default_workspace(query.device)
        T = md.num_actual_tokens
        q = query[:T].view(T, Hq, D)
        out = output[:T].view(T, Hq, D)
        self._seat()
        has_pages = any(self.pages.get(rid) and self.pages[rid][layer_index] for rid in self.active_request_ids)
        if md.causal and md.decode_only:
            pool = self.pools[layer_index] if has_pages else None
            qc = q[:n].contiguous()
            o = torch.empty_like(qc)
            packed_decode([qc], [kv_cache], [md.block_table], [md.seq_lens], [pool], scale=scale, outputs=[o],
                          workspace=ws)
            out[:n].copy_(o)
            return
        excluded = None
        if not md.causal:
            excluded = codestep.excluded_tensor(self.active_request_ids, self.code_excluded_ranges, query.device)
        attend(q, kv_cache, md, out, num_kv_heads=Hkv, scale=scale, workspace=ws, k_max=self.layout.k_max,
               quota_per_kv_head=self.layout.quotas[layer_index], excluded=excluded,
               sidecar=self.pools[layer_index] if has_pages else None)


class _SidecarView:
    """The reference sidecar's reading of the common metadata (query_start_loc_cpu, _seq_lens_cpu,
    block_table_tensor, causal for the first n active requests) as a CommonAttentionMetadata."""

    def __init__(self, common: Any, n: int):
        self._c = common
        self.num_reqs = n
        qsl = torch.as_tensor(common.query_start_loc_cpu[:n + 1], dtype=torch.int32)
        self.query_start_loc_cpu = qsl
        self.num_actual_tokens = int(qsl[-1])
        dev = common.block_table_tensor.device
        qdev = getattr(common, "query_start_loc", None)
        self.query_start_loc = qdev[:n + 1] if qdev is not None else qsl.to(dev)
        self._seq_lens_cpu = torch.as_tensor(common._seq_lens_cpu[:n], dtype=torch.int32)
        sdev = getattr(common, "seq_lens", None)
        self.seq_lens = sdev[:n] if sdev is not None else self._seq_lens_cpu.to(dev)
        self.block_table_tensor = common.block_table_tensor[:n]
        self.slot_mapping = getattr(common, "slot_mapping", torch.empty(0, dtype=torch.int64, device=dev))
        self.causal = bool(common.causal)
        self.compresslm_custom_mask = None


def maybe_override_attention(layer: object, query: torch.Tensor, kv_cache: torch.Tensor, attn_metadata: object,
                             output: torch.Tensor) -> None:
    """Drop-in for the overlay's ``maybe_override_attention`` (compresslm_packed_kv.py:744-761):
    when the layer carries a sidecar (``install_sidecar``), run its attention in place."""
    sidecar = getattr(layer, "_compresslm_packed_sidecar", None)
    if sidecar is None or attn_metadata is None:
        return
    sidecar.override_attention(layer_index=layer._compresslm_packed_layer_index, layer=layer, query=query,
                               kv_cache=kv_cache, attn_metadata=attn_metadata, output=output)


def install_sidecar(attention_layers: Sequence[object], sidecar: CompressedKVSidecar) -> None:
    """Attach the sidecar to each attention layer under the attribute names the overlay's
    Attention.forward patch looks for (patch_stock_attention.py:20-42)."""
    for i, layer in enumerate(attention_layers):
        layer._compresslm_packed_sidecar = sidecar
        layer._compresslm_packed_layer_index = i
