"""Pause-token prefill attention with the compressed-cache mask (host side).

``prefill_masked`` runs ``abkv_prefill_masked`` (tcgen05 tensor cores) on
q [B, H, S, D], k/v [B, Hkv, S, D] bf16 CUDA tensors (last dim contiguous,
other strides free), evaluating CompressLM._arith_mask_mod
(abridgekv/compress_forward.py:695-727) arithmetically per tile from
(C, K_layout, per-query-head quotas, per-sequence raw-prompt lengths) instead of
materialising a BlockMask.

``abkv_attention_forward`` has the signature of transformers'
``flex_attention_forward`` (the attention function CompressLM forces with
``_attn_implementation = "flex_attention"``, compress_forward.py:248) and is
registered under the name ``"abkv_sm100"``.  It expects ``attention_mask`` to
be a :class:`CompressMask` descriptor: CompressLM's per-layer dispatch hook
(compress_forward.py:557-564) can hand each layer its own descriptor exactly as
it hands each layer its own BlockMask today.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _lib
from .workspace import Workspace, default_workspace

TILE = 128


@dataclass(frozen=True)
class CompressMask:
    """The arithmetic mask of one layer: block layout [C content | K_layout codes],
    per-query-head code quotas (None = all K_layout slots) and optional raw
    prompt lengths [B] (int32 CUDA tensor)."""

    C: int
    K_layout: int
    quota_per_head: tuple[int, ...] | None = None
    prompt_len: torch.Tensor | None = None


def _check(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be a bf16 CUDA tensor (libabkv has no CPU path)")
    if t.dim() != 4 or t.stride(3) != 1:
        raise ValueError(f"{name} must be 4-D with a contiguous last dimension")


def prefill_masked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, C: int, K_layout: int,
                   quota_per_head: Sequence[int] | None = None, prompt_len: torch.Tensor | None = None,
                   scale: float | None = None, out: torch.Tensor | None = None, return_lse: bool = False,
                   workspace: Workspace | None = None, stream: torch.cuda.Stream | None = None):
    _check("query", q)
    _check("key", k)
    _check("value", v)
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    if tuple(k.shape) != (B, Hkv, S, D) or tuple(v.shape) != (B, Hkv, S, D):
        raise ValueError("key/value must be [B, Hkv, S, D] matching the query")
    if out is None:
        out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=q.device).transpose(1, 2)
    _check("out", out)
    if tuple(out.shape) != (B, H, S, D):
        raise ValueError("out must be [B, H, S, D] (any strides, last dim contiguous)")
    lse = torch.empty((B, H, S), dtype=torch.float32, device=q.device) if return_lse else None
    pl = None
    if prompt_len is not None:
        pl = prompt_len.to(device=q.device, dtype=torch.int32).contiguous()
        if pl.numel() != B:
            raise ValueError("prompt_len must hold one length per sequence")
    if quota_per_head is not None and len(quota_per_head) != H:
        raise ValueError("quota_per_head must hold one quota per query head")
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    ws = workspace or default_workspace(q.device)
    s = torch.cuda.current_stream(q.device) if stream is None else stream
    strides = lambda t: _lib.i64_array([t.stride(0), t.stride(1), t.stride(2)])  # noqa: E731
    quota = _lib.i32_array(quota_per_head) if quota_per_head is not None else None
    with torch.cuda.device(q.device):
        st = _lib.lib().abkv_prefill_masked(
            q.data_ptr(), strides(q), k.data_ptr(), strides(k), v.data_ptr(), strides(v), out.data_ptr(),
            strides(out), lse.data_ptr() if lse is not None else None, quota,
            pl.data_ptr() if pl is not None else None, B, H, Hkv, S, D, C, K_layout, scale, ws.ptr(),
            ws.nbytes, s.cuda_stream)
    _lib.check("abkv_prefill_masked", st)
    return (out, lse) if return_lse else out


def prefill_masked_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                            dout: torch.Tensor, lse: torch.Tensor, *, C: int, K_layout: int,
                            quota_per_head: Sequence[int] | None = None, prompt_len: torch.Tensor | None = None,
                            scale: float | None = None, workspace: Workspace | None = None,
                            stream: torch.cuda.Stream | None = None):
    """Gradients (dq, dk, dv) of ``prefill_masked`` for the upstream gradient ``dout``, from the
    forward's output and log-sum-exp (abkv_prefill_masked_backward)."""
    for name, t in (("query", q), ("key", k), ("value", v), ("out", out), ("dout", dout)):
        _check(name, t)
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    if tuple(out.shape) != (B, H, S, D) or tuple(dout.shape) != (B, H, S, D):
        raise ValueError("out and dout must be [B, H, S, D] like the query")
    if lse.dtype != torch.float32 or tuple(lse.shape) != (B, H, S) or not lse.is_contiguous():
        raise ValueError("lse must be the forward's contiguous float32 [B, H, S] log-sum-exp")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    for name, t in (("query", q), ("key", k), ("value", v), ("out", out), ("dout", dout), ("dq", dq), ("dk", dk),
                    ("dv", dv)):
        if t.data_ptr() % 16:
            raise ValueError(f"{name} must start on a 16-byte boundary")
    for name, t in (("out", out), ("dout", dout), ("dq", dq), ("dk", dk), ("dv", dv)):
        if any(t.stride(i) % 8 for i in range(3)):
            raise ValueError(f"{name} strides must be multiples of 8 elements, got {tuple(t.stride())}")
    pl = None
    if prompt_len is not None:
        pl = prompt_len.to(device=q.device, dtype=torch.int32).contiguous()
    if quota_per_head is not None and len(quota_per_head) != H:
        raise ValueError("quota_per_head must hold one quota per query head")
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    lib = _lib.lib()
    need = lib.abkv_prefill_masked_backward_workspace_size(B, H, S, D)
    if need == 0:
        raise _lib.AbkvError("abkv_prefill_masked_backward_workspace_size", 3, f"unsupported shape D={D}")
    ws = (workspace or default_workspace(q.device)).ensure(need)
    s = torch.cuda.current_stream(q.device) if stream is None else stream
    strides = lambda t: _lib.i64_array([t.stride(0), t.stride(1), t.stride(2)])  # noqa: E731
    quota = _lib.i32_array(quota_per_head) if quota_per_head is not None else None
    with torch.cuda.device(q.device):
        st = lib.abkv_prefill_masked_backward(
            q.data_ptr(), strides(q), k.data_ptr(), strides(k), v.data_ptr(), strides(v), out.data_ptr(),
            strides(out), dout.data_ptr(), strides(dout), lse.data_ptr(), dq.data_ptr(), strides(dq), dk.data_ptr(),
            strides(dk), dv.data_ptr(), strides(dv), quota, pl.data_ptr() if pl is not None else None, B, H, Hkv,
            S, D, C, K_layout, scale, ws.ptr(), ws.nbytes, s.cuda_stream)
    _lib.check("abkv_prefill_masked_backward", st,
               f"B={B} H={H} Hkv={Hkv} S={S} D={D} C={C} K_layout={K_layout} scale={scale} "
               f"quota={None if quota_per_head is None else list(quota_per_head)} "
               f"strides q{tuple(q.stride())} k{tuple(k.stride())} out{tuple(out.stride())} "
               f"dout{tuple(dout.stride())} dq{tuple(dq.stride())} dk{tuple(dk.stride())}")
    return dq, dk, dv


class PrefillMaskedAttention(torch.autograd.Function):
    """prefill_masked with its backward: the forward keeps its output and log-sum-exp."""

    @staticmethod
    def forward(ctx, q, k, v, C, K_layout, quota_per_head, prompt_len, scale):
        out, lse = prefill_masked(q, k, v, C=C, K_layout=K_layout, quota_per_head=quota_per_head,
                                  prompt_len=prompt_len, scale=scale, return_lse=True)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.args = (C, K_layout, quota_per_head, prompt_len, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        C, K_layout, quota, pl, scale = ctx.args
        if dout.stride(-1) != 1:
            dout = dout.contiguous()
        dq, dk, dv = prefill_masked_backward(q, k, v, out, dout, lse, C=C, K_layout=K_layout, quota_per_head=quota,
                                             prompt_len=pl, scale=scale)
        return dq, dk, dv, None, None, None, None, None


def prefill_masked_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, C: int, K_layout: int,
                             quota_per_head: Sequence[int] | None = None, prompt_len: torch.Tensor | None = None,
                             scale: float | None = None) -> torch.Tensor:
    """Differentiable ``prefill_masked`` (forward and backward on the tcgen05 kernels)."""
    return PrefillMaskedAttention.apply(q, k, v, C, K_layout, quota_per_head, prompt_len, scale)


def abkv_attention_forward(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                           attention_mask, scaling: float | None = None, dropout: float = 0.0,
                           softcap: float | None = None, s_aux=None, **kwargs):
    """transformers AttentionInterface function: (attn_output [B, S, H, D], None)."""
    if not isinstance(attention_mask, CompressMask):
        raise TypeError("abkv_sm100 attention needs a CompressMask descriptor as attention_mask")
    if dropout != 0.0 or softcap is not None or s_aux is not None:
        raise ValueError("abkv_sm100 attention supports no dropout, softcap or attention sinks")
    kw = dict(C=attention_mask.C, K_layout=attention_mask.K_layout,
              quota_per_head=attention_mask.quota_per_head, prompt_len=attention_mask.prompt_len, scale=scaling)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (query, key, value)):
        out = prefill_masked_attention(query, key, value, **kw)  # training: gradients through the backward kernel
    else:
        out = prefill_masked(query, key, value, **kw)
    return out.transpose(1, 2), None


def register(name: str = "abkv_sm100") -> str:
    """Register abkv_attention_forward with transformers' AttentionInterface."""
    from transformers import AttentionInterface

    AttentionInterface.register(name, abkv_attention_forward)
    return name
