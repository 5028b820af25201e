"""Decode-attention oracle (test infrastructure).

Restates PackedKVSidecar._attend_decode_batched
(third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:564-616) for
the physical per-quota cache (no sidecar pages):

  * rows 0..seq_len-1 of a request are gathered through its block-table row
    (page = table[r // P], offset = r % P; _batched_main_index :501-524);
  * scores = (q . K) * scale, computed in bf16 (two roundings: the einsum's
    bf16 result, then the scaled bf16 product) (:610);
  * rows >= seq_len are masked to -inf (:611);
  * softmax in fp32, weights rounded to bf16 (:612);
  * out = sum_t w_t V_t with fp32 accumulation, rounded to bf16 (:613-616).

Two numpy forms: ``decode_reference`` reproduces those roundings,
``decode_exact`` is float64 ground truth on the same bf16 inputs.
``sidecar_decode_torch`` is the same computation as torch CPU ops (used to
time the reference's CPU path in bench.py).  ``codestep_exact`` (float64) and
``sidecar_codestep_torch`` (torch CPU, the reference's op sequence) restate the
noncausal code step of _attend_request_vectorized (:648-741); ``paged_causal_exact``
(float64) its causal branch for ragged query rows (:700-707).
"""
from __future__ import annotations

import numpy as np

from .bf16 import round_bf16


def _gather(kv: np.ndarray, bt_row: np.ndarray, seq_len: int, page: int) -> tuple[np.ndarray, np.ndarray]:
    r = np.arange(seq_len)
    pages = bt_row[r // page]
    offs = r % page
    k = kv[pages, 0, offs]  # [T, Hkv, D]
    v = kv[pages, 1, offs]
    return k, v


def decode_reference(q, kv, block_table, seq_lens, scale, page) -> np.ndarray:
    """Reference-rounding decode. q [B,Hq,D] (bf16 values in float32) -> [B,Hq,D] float32 (bf16 values)."""
    B, Hq, D = q.shape
    Hkv = kv.shape[3]
    G = Hq // Hkv
    out = np.zeros((B, Hq, D), dtype=np.float32)
    for b in range(B):
        s_len = int(seq_lens[b])
        if s_len == 0:
            continue
        k, v = _gather(kv, block_table[b], s_len, page)
        for h in range(Hq):
            kh = k[:, h // G, :].astype(np.float32)
            vh = v[:, h // G, :].astype(np.float32)
            s = round_bf16(kh @ q[b, h].astype(np.float32))
            s = round_bf16(s * np.float32(scale))
            m = s.max()
            e = np.exp((s - m).astype(np.float32))
            w = round_bf16((e / e.sum()).astype(np.float32))
            out[b, h] = round_bf16((w.astype(np.float64) @ vh.astype(np.float64)).astype(np.float32))
    return out


def decode_exact(q, kv, block_table, seq_lens, scale, page) -> np.ndarray:
    """float64 ground truth on the same inputs (no intermediate rounding)."""
    B, Hq, D = q.shape
    Hkv = kv.shape[3]
    G = Hq // Hkv
    out = np.zeros((B, Hq, D), dtype=np.float64)
    for b in range(B):
        s_len = int(seq_lens[b])
        if s_len == 0:
            continue
        k, v = _gather(kv, block_table[b], s_len, page)
        for h in range(Hq):
            kh = k[:, h // G, :].astype(np.float64)
            vh = v[:, h // G, :].astype(np.float64)
            s = (kh @ q[b, h].astype(np.float64)) * scale
            e = np.exp(s - s.max())
            out[b, h] = (e / e.sum()) @ vh
    return out


def sidecar_decode_torch(query, kv_cache, seq_lens, block_table, num_kv_heads: int, groups: int,
                         scale: float, page: int):
    """torch (CPU) form of the reference's batched decode for one layer.

    query [n, Hq, D] bf16, kv_cache [nb, 2, P, Hkv, D] bf16, seq_lens [n] int,
    block_table [n, maxp] int -> [n, Hq, D] bf16.  Same op sequence as
    compresslm_packed_kv.py:579-616 (gather, bf16 einsum, -inf mask, fp32
    softmax, bf16 weights, bf16 einsum)."""
    import torch

    n = query.shape[0]
    lens = seq_lens[:n].to(torch.long)
    s_max = int(lens.max())
    pos = torch.arange(s_max)
    hidden = pos.unsqueeze(0) >= lens.unsqueeze(1)
    bidx = torch.clamp(pos // page, max=block_table.shape[1] - 1)
    blocks = block_table[:n].to(torch.long)[:, bidx].masked_fill(hidden, 0)
    offs = (pos % page).unsqueeze(0).expand(n, -1).masked_fill(hidden, 0)
    rows = kv_cache[blocks, :, offs]                  # [n, S, 2, Hkv, D]
    key = rows[:, :, 0].permute(0, 2, 1, 3)           # [n, Hkv, S, D]
    value = rows[:, :, 1].permute(0, 2, 1, 3)
    D = query.shape[-1]
    q = query[:n].reshape(n, num_kv_heads, groups, D)
    scores = torch.einsum("rhgd,rhtd->rhgt", q, key) * scale
    scores.masked_fill_(hidden.view(n, 1, 1, s_max), -torch.inf)
    weights = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    att = torch.einsum("rhgt,rhtd->rhgd", weights, value)
    return att.reshape(n, num_kv_heads * groups, D)


def codestep_exact(qrows, kv, block_table, seq_lens, K, quota_per_kv_head, scale, page, excluded=None):
    """Code-step attention in float64 (compresslm_packed_kv.py:708-733 noncausal branch, no
    sidecar pages): the K code queries of request r (rows r*K .. r*K+K-1 of qrows, [T, Hq, D])
    attend to physical rows [0, seq_len) of its block-table row, own code slots >= the head's
    quota hidden (rows >= seq_len - K + quota), and rows [excluded[r][0], excluded[r][1])
    hidden when ``excluded`` is given (:721-726, _code_excluded_range :249-260).
    Returns [T, Hq, D]."""
    T, Hq, D = qrows.shape
    Hkv = kv.shape[3]
    G = Hq // Hkv
    out = np.zeros((T, Hq, D))
    for r, s_len in enumerate(seq_lens):
        s_len = int(s_len)
        k, v = _gather(kv, block_table[r], s_len, page)
        prefix = s_len - K
        for h in range(Hq):
            limit = prefix + int(quota_per_kv_head[h // G])
            keep = np.arange(limit)
            if excluded is not None and excluded[r][1] > excluded[r][0]:
                keep = keep[(keep < excluded[r][0]) | (keep >= excluded[r][1])]
            kh = k[keep, h // G, :].astype(np.float64)
            vh = v[keep, h // G, :].astype(np.float64)
            s = (qrows[r * K:(r + 1) * K, h].astype(np.float64) @ kh.T) * scale
            e = np.exp(s - s.max(axis=1, keepdims=True))
            out[r * K:(r + 1) * K, h] = (e / e.sum(axis=1, keepdims=True)) @ vh
    return out


def paged_causal_exact(qrows, kv, block_table, seq_lens, query_start, scale, page) -> np.ndarray:
    """Causal attention of ragged query rows over the paged cache in float64: the causal branch of
    PackedKVSidecar._attend_request_vectorized without sidecar pages (compresslm_packed_kv.py:
    700-707, per request from override_attention :371-399).  Request r's queries are rows
    query_start[r] .. query_start[r + 1] - 1 of qrows ([T, Hq, D]); with qlen of them and
    prefix = seq_len - qlen, query i sees cache rows [0, prefix + i + 1).  Rows of qrows outside
    every request stay zero.  Returns [T, Hq, D]."""
    T, Hq, D = qrows.shape
    Hkv = kv.shape[3]
    G = Hq // Hkv
    out = np.zeros((T, Hq, D))
    for r, s_len in enumerate(seq_lens):
        s_len = int(s_len)
        q0, q1 = int(query_start[r]), int(query_start[r + 1])
        qlen = q1 - q0
        if qlen <= 0:
            continue
        k, v = _gather(kv, block_table[r], s_len, page)
        prefix = s_len - qlen
        hidden = np.arange(s_len)[None, :] >= (prefix + np.arange(1, qlen + 1))[:, None]   # [qlen, S]
        for h in range(Hq):
            kh = k[:, h // G, :].astype(np.float64)
            vh = v[:, h // G, :].astype(np.float64)
            sc = (qrows[q0:q1, h].astype(np.float64) @ kh.T) * scale
            sc[hidden] = -np.inf
            e = np.exp(sc - sc.max(axis=1, keepdims=True))
            out[q0:q1, h] = (e / e.sum(axis=1, keepdims=True)) @ vh
    return out


def sidecar_codestep_torch(query, kv_cache, seq_len: int, block_row, quotas_per_kv_head, k_max: int,
                           num_kv_heads: int, groups: int, scale: float, page: int, excluded=None):
    """torch (CPU) form of one request's noncausal code step,
    PackedKVSidecar._attend_request_vectorized(causal=False) without sidecar pages
    (compresslm_packed_kv.py:648-741): gather rows [0, seq_len) through the block-table row
    (_gather_cache_span_indexed), bf16 score einsum, hide rows >= prefix + quota per KV head and
    the optional exclusion range, fp32 softmax, bf16 weights, bf16 value einsum.
    query [k_max, Hq, D] bf16 -> [k_max, Hq, D] bf16."""
    import torch

    pos = torch.arange(seq_len)
    blocks = block_row.to(torch.long)[pos // page]
    rows = kv_cache[blocks, :, pos % page]                    # [S, 2, Hkv, D]
    key = rows[:, 0].permute(1, 0, 2)                         # [Hkv, S, D]
    value = rows[:, 1].permute(1, 0, 2)
    D = query.shape[-1]
    q = query.reshape(k_max, num_kv_heads, groups, D)
    scores = torch.einsum("qhgd,htd->qhgt", q, key) * scale
    prefix = seq_len - k_max
    quotas = torch.as_tensor(list(quotas_per_kv_head))
    hidden = pos.unsqueeze(0) >= (prefix + quotas).unsqueeze(1)   # [Hkv, S]
    hidden = hidden.unsqueeze(0).expand(k_max, -1, -1).clone()
    if excluded is not None and excluded[1] > excluded[0]:
        hidden[:, :, int(excluded[0]):int(excluded[1])] = True
    scores.masked_fill_(hidden.unsqueeze(2), -torch.inf)
    weights = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    att = torch.einsum("qhgt,htd->qhgd", weights, value)
    return att.reshape(k_max, num_kv_heads * groups, D)


def packed_offsets(quotas):
    """Slot offset of each KV head inside a packed page (PackedKVLayout.offsets,
    compresslm_packed_kv.py:76-84): head h owns slots [off[h], off[h] + quotas[h])."""
    off = [0]
    for q in quotas:
        off.append(off[-1] + int(q))
    return off


def packed_decode_exact(q, kv, block_table, seq_lens, side_pages, counts, quotas, scale, page):
    """Decode over packed sidecar pages + the paged main cache in float64
    (PackedKVSidecar._attend_decode_batched with pages, compresslm_packed_kv.py:526-616):
    for KV head h of request r the keys are, in order, slots [off_h, off_h + q_h) of each of
    the request's sidecar pages (side_pages[first_r + i], [2, slots, D]), then main rows
    [0, seq_len).  side_pages holds every request's pages, request after request."""
    B, Hq, D = q.shape
    Hkv = kv.shape[3]
    G = Hq // Hkv
    off = packed_offsets(quotas)
    out = np.zeros((B, Hq, D))
    first = 0
    for b in range(B):
        cnt = int(counts[b])
        pages = side_pages[first:first + cnt]
        first += cnt
        s_len = int(seq_lens[b])
        k_main, v_main = _gather(kv, block_table[b], s_len, page)
        for h in range(Hq):
            kh = h // G
            ks = [pages[i, 0, off[kh]:off[kh + 1]] for i in range(cnt)] + [k_main[:, kh]]
            vs = [pages[i, 1, off[kh]:off[kh + 1]] for i in range(cnt)] + [v_main[:, kh]]
            keys = np.concatenate(ks).astype(np.float64)
            vals = np.concatenate(vs).astype(np.float64)
            if len(keys) == 0:
                continue
            s = (keys @ q[b, h].astype(np.float64)) * scale
            e = np.exp(s - s.max())
            out[b, h] = (e / e.sum()) @ vals
    return out


def packed_step_exact(qrows, kv, block_table, seq_lens, query_start, side_pages, counts, quotas, causal, scale,
                      page, excluded=None) -> np.ndarray:
    """The code step (causal=False) or causal rows of requests holding packed sidecar pages, in float64:
    PackedKVSidecar._attend_request_vectorized with layer_pages (compresslm_packed_kv.py:648-741).
    For KV head h of request r the keys are head h's slots [off_h, off_h + quotas[h]) of each of its
    counts[r] pages (side_pages[first_r + i], [2, slots, D]; every query row sees them), then its main
    rows [0, seq_len): noncausal, rows < prefix + quotas[h] minus the optional excluded[r] range
    (:711-726); causal, rows < prefix + i + 1 for query i (:700-707), prefix = seq_len - query_len.
    Returns [T, Hq, D]."""
    T, Hq, D = qrows.shape
    Hkv = kv.shape[3]
    G = Hq // Hkv
    off = packed_offsets(quotas)
    out = np.zeros((T, Hq, D))
    first = 0
    for r, s_len in enumerate(seq_lens):
        s_len = int(s_len)
        q0, q1 = int(query_start[r]), int(query_start[r + 1])
        qlen = q1 - q0
        pages = side_pages[first:first + int(counts[r])]
        first += int(counts[r])
        if qlen <= 0:
            continue
        k_main, v_main = _gather(kv, block_table[r], s_len, page)
        prefix = s_len - qlen
        pos = np.arange(s_len)
        for h in range(Hq):
            kh = h // G
            ks = np.concatenate([pg[0, off[kh]:off[kh + 1]] for pg in pages] + [k_main[:, kh]]).astype(np.float64)
            vs = np.concatenate([pg[1, off[kh]:off[kh + 1]] for pg in pages] + [v_main[:, kh]]).astype(np.float64)
            n_side = ks.shape[0] - s_len
            if causal:
                hidden_main = pos[None, :] >= (prefix + np.arange(1, qlen + 1))[:, None]
            else:
                hidden_main = np.broadcast_to(pos >= prefix + int(quotas[kh]), (qlen, s_len)).copy()
                if excluded is not None and excluded[r][1] > excluded[r][0]:
                    hidden_main[:, int(excluded[r][0]):int(excluded[r][1])] = True
            hidden = np.concatenate([np.zeros((qlen, n_side), bool), hidden_main], axis=1)
            sc = (qrows[q0:q1, h].astype(np.float64) @ ks.T) * scale
            sc[hidden] = -np.inf
            e = np.exp(sc - sc.max(axis=1, keepdims=True))
            out[q0:q1, h] = (e / e.sum(axis=1, keepdims=True)) @ vs
    return out
