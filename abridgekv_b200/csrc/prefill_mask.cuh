// The pause-token mask of CompressLM._arith_mask_mod
// (abridgekv/compress_forward.py:695-727) at tile granularity (128 x 128 by default), shared
// by the forward (prefill.cu) and backward (prefill_bwd.cu) kernels.  With
// per = C + K, qb = q / per, kb = kv / per, qw = q % per, kw = kv % per:
//   vis = (kw < C & kb == qb) | (kw >= C & kb < qb)
//   vis |= kw < C & (kb*C + kw < prompt_len[b]);  vis &= kv <= q
//   vis |= qw >= C & kw >= C & kb == qb;           vis &= kw < C | kw - C < quota[h]
// C and K are multiples of 128, so no tile straddles a block or the content /
// code boundary.  P is any parameter struct with fields per, C and quota[].
#pragma once

namespace abkv {
namespace mask {

constexpr int kTile = 128;

// 0 = empty, 1 = full, 2 = partial, for query tile qt (kQT rows) / key tile kt
// (kKT keys) of head h; kQT and kKT divide 128.
template <int kQT, int kKT, class P>
__device__ __forceinline__ int tile_class_t(const P& p, int h, int qt, int kt, int pl) {
  const int q0 = qt * kQT, q1 = q0 + kQT - 1;
  const int k0 = kt * kKT, k1 = k0 + kKT - 1;
  const int qb = q0 / p.per, kb = k0 / p.per;
  if (kb > qb) return 0;
  const int qw0 = q0 - qb * p.per;
  const int kw0 = k0 - kb * p.per, kw1 = k1 - kb * p.per;
  const bool q_code = qw0 >= p.C;
  if (kw0 < p.C) {  // content keys
    if (kb == qb) {  // own block: causal (the raw-prompt term adds nothing here)
      if (q_code || k1 <= q0) return 1;
      if (k0 > q1) return 0;
      return 2;
    }
    // earlier block: visible only as raw prompt (kb*C + kw < prompt_len)
    const int a0 = kb * p.C + kw0, a1 = kb * p.C + kw1;
    if (a1 < pl) return 1;
    if (a0 >= pl) return 0;
    return 2;
  }
  // code keys: quota on the slot; own block only for code queries
  const int s0 = kw0 - p.C, s1 = kw1 - p.C;
  const int qq = p.quota[h];
  const int qc = (s1 < qq) ? 1 : (s0 >= qq ? 0 : 2);
  if (kb < qb) return qc;
  return q_code ? qc : 0;
}
template <class P>
__device__ __forceinline__ int tile_class(const P& p, int h, int qt, int kt, int pl) {
  return tile_class_t<kTile, kTile>(p, h, qt, kt, pl);
}

// Inside any tile the visible keys of one query row are a PREFIX of the tile's
// columns: the causal diagonal of the own block (kv <= q), the raw-prompt
// boundary of an earlier block (kb*C + kw < prompt_len) or the quota boundary
// of a code tile (kw - C < quota).  tile_limit_t returns that prefix length in
// [0, kKT] from precomputed coordinates: the row's block qb and in-block offset
// qw, the tile's block kb and in-block offset kw0 (k0 = key tile start).
template <int kKT, class P>
__device__ __forceinline__ int tile_limit_t(const P& p, int quota, int q, int qb, int qw, int kb, int kw0, int k0,
                                            int pl) {
  int lim;
  if (kw0 < p.C) {
    if (kb == qb) lim = (qw >= p.C) ? kKT : q - k0 + 1;
    else lim = pl - (kb * p.C + kw0);
  } else {
    if (kb == qb && qw < p.C) return 0;
    lim = quota - (kw0 - p.C);
  }
  return lim < 0 ? 0 : (lim > kKT ? kKT : lim);
}
template <class P>
__device__ __forceinline__ int tile_limit_fast(const P& p, int quota, int q, int qb, int qw, int kb, int kw0,
                                               int k0, int pl) {
  return tile_limit_t<kTile>(p, quota, q, qb, qw, kb, kw0, k0, pl);
}

}  // namespace mask
}  // namespace abkv
