"""Prefill-mask oracle (test infrastructure).

* ``arith_mask`` restates CompressLM._arith_mask_mod
  (abridgekv/compress_forward.py:695-727) as a dense boolean array
  [B, H, S0, S0] (per = C + K; content keys visible within the own block
  causally, earlier blocks' code rows always, the raw prompt to everyone,
  code rows of the own block bidirectionally among codes, per-head quota on
  code slots).
* ``bitrev_code_offsets`` restates _bitrev_code_offsets (:46-60).
* ``masked_attention`` is dense masked softmax attention in float64 (GQA:
  query head h reads KV head h // (H // Hkv)), the math FlexAttention computes
  for this mask (compress_forward.py:1229 via transformers' flex path).
"""
from __future__ import annotations

import numpy as np


def arith_mask(S0: int, C: int, K: int, quota_per_head=None, prompt_len=None, num_heads: int = 1,
               batch: int = 1) -> np.ndarray:
    per = C + K
    q = np.arange(S0)[:, None]
    kv = np.arange(S0)[None, :]
    qb, qw = q // per, q % per
    kb, kw = kv // per, kv % per
    kc = kw < C
    same = kb == qb
    base = (kc & same) | (~kc & (kb < qb))
    H = num_heads if quota_per_head is None else len(quota_per_head)
    out = np.zeros((batch, H, S0, S0), dtype=bool)
    for b in range(batch):
        vis = base.copy()
        if prompt_len is not None:
            vis |= kc & (kb * C + kw < int(prompt_len[b]))
        vis &= kv <= q
        vis |= (qw >= C) & ~kc & same
        for h in range(H):
            if quota_per_head is None:
                out[b, h] = vis
            else:
                out[b, h] = vis & (kc | ((kw - C) < int(quota_per_head[h])))
    return out


def bitrev_code_offsets(K: int, C: int, span: int | None = None) -> np.ndarray:
    span = C if span is None else int(span)
    bits = K.bit_length() - 1
    k = np.arange(K)
    rev = np.zeros_like(k)
    for b in range(bits):
        rev |= ((k >> b) & 1) << (bits - 1 - b)
    return (rev * span) // K


def masked_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray, scale: float):
    """q [B,H,S,D], k/v [B,Hkv,S,D], mask [B,H,S,S] -> (out [B,H,S,D] float64, lse [B,H,S] natural log)."""
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    out = np.zeros((B, H, S, D))
    lse = np.full((B, H, S), -np.inf)
    for b in range(B):
        for h in range(H):
            s = (q[b, h].astype(np.float64) @ k[b, h // G].astype(np.float64).T) * scale
            s = np.where(mask[b, h], s, -np.inf)
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            e = np.exp(s - m)
            l = e.sum(axis=1, keepdims=True)
            out[b, h] = (e / np.where(l > 0, l, 1.0)) @ v[b, h // G].astype(np.float64)
            lse[b, h] = np.where(l[:, 0] > 0, m[:, 0] + np.log(np.where(l[:, 0] > 0, l[:, 0], 1.0)), -np.inf)
    return out, lse


def masked_attention_grad(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray, scale: float,
                          dout: np.ndarray):
    """Gradients of masked_attention for the upstream gradient dout [B,H,S,D], float64:
    P = softmax(scale q k^T + mask), O = P v;  dV = sum over the KV head's query heads of P^T dO;
    dP = dO v^T;  dS = P * (dP - rowsum(dO * O));  dQ = scale dS k;  dK = scale sum dS^T q.
    -> (dq [B,H,S,D], dk [B,Hkv,S,D], dv [B,Hkv,S,D])."""
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    dq = np.zeros((B, H, S, D))
    dk = np.zeros((B, Hkv, S, D))
    dv = np.zeros((B, Hkv, S, D))
    for b in range(B):
        for h in range(H):
            kh, vh = k[b, h // G].astype(np.float64), v[b, h // G].astype(np.float64)
            qh, do = q[b, h].astype(np.float64), dout[b, h].astype(np.float64)
            s = np.where(mask[b, h], (qh @ kh.T) * scale, -np.inf)
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            e = np.exp(s - m)
            l = e.sum(axis=1, keepdims=True)
            p = e / np.where(l > 0, l, 1.0)
            o = p @ vh
            dv[b, h // G] += p.T @ do
            dp = do @ vh.T
            ds = p * (dp - (do * o).sum(axis=1, keepdims=True))
            dq[b, h] = scale * (ds @ kh)
            dk[b, h // G] += scale * (ds.T @ qh)
    return dq, dk, dv
