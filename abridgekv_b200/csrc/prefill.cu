// Pause-token prefill attention with the in-block-position causal/pause mask,
// on 5th-generation tensor cores (tcgen05 + TMEM) for sm_100a.
//
// Mask: CompressLM._arith_mask_mod (abridgekv/compress_forward.py:695-727),
// equal to _mask_mod / _mask_rawprompt_mod for the simple config (L=1, no
// tails, pause_xattn="full"; :678-688).  With per = C + K, qb = q / per,
// kb = kv / per, qw = q % per, kw = kv % per, k_content = kw < C:
//   vis = (k_content & kb == qb) | (!k_content & kb < qb)
//   vis |= k_content & (kb*C + kw < prompt_len[b])           (raw prompt)
//   vis &= kv <= q                                            (causal)
//   vis |= (qw >= C) & !k_content & kb == qb                  (codes <-> codes)
//   vis &= k_content | (kw - C < quota[h])                    (per-head quota)
// out = softmax(q.k^T * scale + mask) v, fp32 softmax.  The attention math is
// that of torch FlexAttention, which the reference runs for this mask
// (compress_forward.py:248,1229).
//
// Tiling: 128 query rows x 64 keys.  C and K are multiples of 128, so no tile
// straddles a block or the content/code boundary, and every tile is FULL,
// PARTIAL or EMPTY by the analytic classification below (the block structure
// of _fast_layer_blockmasks, :760-789).  EMPTY tiles are never loaded; inside
// a PARTIAL tile the visible keys of a row are a prefix of the tile.
//
// CTA = one 128-row query tile of TWO query heads of the same KV head.  Their
// masks are the same block structure, so both heads share every K/V tile
// (loaded once); 10 warps:
//   warp 0      TMA producer: Q of both heads, then K/V tiles into a 3-stage
//               ring (cp.async.bulk.tensor, 128B swizzle, no multicast)
//   warp 1      TMEM owner (512 columns: per head two S buffers + O); lane 0
//               issues tcgen05.mma in the order
//               S_A(0) S_B(0) S_A(1) S_B(1) | PV_A(j) S_A(j+2) PV_B(j) S_B(j+2) | ...
//                 S  = Q K^T   (A = Q, B = K, both K-major, fp32 in TMEM)
//                 O += P V     (A = P from TMEM, B = V, MN-major)
//               so each head's softmax overlaps the other head's MMAs
//   warps 2..5  softmax of head A, warps 6..9 softmax of head B: thread = one
//               TMEM lane = one query row; S read with tcgen05.ld, masked online
//               softmax in fp32, P (bf16 pairs) stored back into the upper half
//               of its own S buffer with tcgen05.st -- so P is double-buffered
//               with S, and a head's softmax of tile j+1 never waits for its
//               P.V of tile j unless O must be rescaled; epilogue divides by the
//               row sum.  The S MMA of tile j+2 overwrites P(j) after P.V(j) read
//               it: tcgen05.mma operations of one thread run in issue order.
// Every mbarrier wait is bounded and records ABKV_DEVERR_TIMEOUT on expiry.
#include <cuda.h>

#include <cstring>

#include "common.cuh"

namespace abkv {
namespace {

constexpr int kBM = 128, kBN = 64, kD = 128;
constexpr int kThreads = 320;
constexpr int kMaxHeads = 128;
constexpr int kStages = 4;
constexpr uint32_t kTmemCols = 512;  // per head (A at 0, B at 256): S buffers [0,64) [64,128), O [128,256)
constexpr uint32_t kPCol = 32;       // P (64 bf16 = 32 columns) lives in columns [32, 64) of its S buffer

// dynamic shared memory layout (1024-byte aligned pieces for 128B swizzle)
constexpr int kQBytes = kBM * kD * 2;          // 32 KiB: 2 atoms of [128 rows][128 B]
constexpr int kKVHalf = kBN * kD * 2;          // 16 KiB: 2 atoms of [64 rows][128 B]
constexpr int kStageBytes = 2 * kKVHalf;       // K then V
constexpr int kOffQ = 0;                        // Q_A, Q_B
constexpr int kOffKV = 2 * kQBytes;
constexpr int kOffBar = kOffKV + kStages * kStageBytes;
// mbarriers (u64 slots from kOffBar): q_full, kv_full[kStages], kv_empty[kStages],
// s_full[head][S buffer], p_full[head][S buffer], o_done[head], o_full, then the TMEM
// address.  p_full is double-buffered like S: a head's softmax may finish tile j+1
// before the MMA thread has taken tile j's P, and one barrier per buffer keeps the
// two arrivals in different barriers (a parity wait cannot tell phases 2 apart).
constexpr int kBarKvFull = 1, kBarKvEmpty = kBarKvFull + kStages, kBarSFull = kBarKvEmpty + kStages,
              kBarPFull = kBarSFull + 4, kBarODone = kBarPFull + 4, kBarOFull = kBarODone + 2,
              kBarTmem = kBarOFull + 1;
static_assert((kBarTmem + 1) * 8 <= 256, "barrier area");
constexpr int kOffList = kOffBar + 256;         // visited key tiles: (kb << 16) | kw0, per 64-key tile
constexpr int kMaxKeyTiles = 2048;              // keys up to 2048 x 64 = 128K rows
constexpr int kSmemBytes = kOffList + 4 * kMaxKeyTiles + 16 + 1024;  // + slack for 1024-byte alignment
// Lazy rescaling: a row keeps its reference maximum until a tile's maximum
// exceeds it by more than this (log2 units), so P <= 2^8 and O is rescaled
// only on large jumps (O and the row sum always share the reference).
constexpr float kRescaleThreshold = 8.f;

struct alignas(64) PrefillParams {
  CUtensorMap tm_q, tm_k, tm_v;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_ss;
  float* lse;  // [B][H][S] or null
  const int32_t* prompt_len;  // [B] or null
  int32_t* err;
  int quota[kMaxHeads];
  int B, H, Hkv, G, npairs, S, C, KL, per, n_qtiles;
  float scale_log2;
  // code step (paged K/V): request r's K code queries are rows q_start[r] ..
  // q_start[r] + Kc - 1 of q [T][H][D]; its keys are the first seq_lens[r]
  // rows of the paged cache through block-table row r.
  const int32_t* bt;
  const int32_t* seq_lens;
  const int32_t* q_start;
  const int32_t* excl;  // optional [R][2]: rows [start, end) hidden from the code queries
  int64_t bt_stride, num_blocks;
  int page, Kc, T, fa_layout;
};

// 0 = empty, 1 = full, 2 = partial, for query tile qt / key tile kt of head h.
__device__ __forceinline__ int tile_class(const PrefillParams& p, int h, int qt, int kt, int pl) {
  const int q0 = qt * kBM, q1 = q0 + kBM - 1;
  const int k0 = kt * kBN, k1 = k0 + kBN - 1;
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

// Inside any tile the visible keys of one query row are a PREFIX of the tile's
// columns: the causal diagonal of the own block (kv <= q), the raw-prompt
// boundary of an earlier block (kb*C + kw < prompt_len) or the quota boundary
// of a code tile (kw - C < quota).  tile_limit_fast returns that prefix length
// in [0, kBN] from precomputed coordinates: the row's block qb and in-block
// offset qw, the tile's block kb and in-block offset kw0 (k0 = key tile start).
__device__ __forceinline__ int tile_limit_fast(const PrefillParams& p, int quota, int q, int qb, int qw, int kb,
                                               int kw0, int k0, int pl) {
  int lim;
  if (kw0 < p.C) {
    if (kb == qb) lim = (qw >= p.C) ? kBN : q - k0 + 1;
    else lim = pl - (kb * p.C + kw0);
  } else {
    if (kb == qb && qw < p.C) return 0;
    lim = quota - (kw0 - p.C);
  }
  return lim < 0 ? 0 : (lim > kBN ? kBN : lim);
}

// Packed fp32 pairs (sm_100 f32x2 pipes) and a three-input max: fewer issue
// slots per score in the softmax.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n .reg .b64 x, y, z, r;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %4};\n mov.b64 z, {%5, %5};\n"
      " fma.rn.f32x2 r, x, y, z;\n mov.b64 {%0, %1}, r;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1) {
  asm("{\n .reg .b64 x, y, r;\n mov.b64 x, {%0, %1};\n mov.b64 y, {%2, %3};\n"
      " add.rn.f32x2 r, x, y;\n mov.b64 {%0, %1}, r;\n}\n"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// ---- tcgen05 / TMA helpers --------------------------------------------------
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) {
  // K-major, 128B swizzle: rows of 128 B, 8-row atoms 1024 B apart (SBO),
  // LBO unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B).
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t saddr, uint32_t lbo) {
  // MN-major, 128B swizzle: a K row = 64 MN elements (128 B); 8 K rows form a
  // 1024 B atom (SBO = 1024); the next 64 MN elements are `lbo` bytes away.
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptors: D f32, A/B bf16, M = 128.
//   S = Q K^T : N = kBN keys, A and B K-major
//   O += P V  : N = head_dim, A (P) K-major, B (V) MN-major
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 4) << 24);
constexpr uint32_t kIdescQK = kIdescBase | ((uint32_t)(kBN >> 3) << 17);
constexpr uint32_t kIdescPV = kIdescBase | ((uint32_t)(kD >> 3) << 17) | (1u << 16);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// A operand from TMEM (128 lanes x 16 bf16 = 8 columns per K step of 16).
__device__ __forceinline__ void umma_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
// Bounded wait; after the first expiry a thread stops waiting altogether (its
// remaining work is skipped and the error word says why), so a fault in one
// role cannot stall the CTA for long.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, bool& dead, int32_t* err) {
  if (dead) return false;
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < (1u << 20); ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  set_error(err, ABKV_DEVERR_TIMEOUT);
  dead = true;
  return false;
}

__device__ __forceinline__ void mbar_arrive_one(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}


// ---------------------------------------------------------------------------
// Softmax of one head: thread = query row `row` of the tile (TMEM lane).
struct SoftmaxState {
  float m_run, l_run;
};

// Softmax of one (head, key tile) for query row `row` (= TMEM lane):
// reads S, updates the reference maximum / row sum, waits until the previous
// P.V of this head has completed (o_done), rescales O when needed and writes
// P (bf16, 128B-swizzled K-major: 16-byte chunk index ^= row % 8).
// kHole: columns [hs, he) are hidden as well (the code step's tail exclusion).
template <bool kHole>
__device__ __forceinline__ void softmax_tile(const PrefillParams& p, int lim, int hs, int he, int row,
                                             uint32_t tmem_s, uint32_t tmem_o, uint32_t lane_base, int j,
                                             uint64_t* o_done, bool& dead, SoftmaxState& st) {
  const float sl2 = p.scale_log2;  // lim: visible columns of this row are c < lim
  float t0[32], t1[32];
  tmem_ld32(tmem_s + lane_base, t0);
  tmem_ld32(tmem_s + lane_base + 32, t1);
  tmem_wait_ld();
  auto vis = [&](int c) { return c < lim && (!kHole || c < hs || c >= he); };
  const bool full = lim == kBN && (!kHole || he <= 0 || hs >= kBN);
  float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
  if (full) {
#pragma unroll
    for (int i = 0; i < 32; ++i) mxa[i & 3] = fmax3(mxa[i & 3], t0[i], t1[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      mxa[i & 3] = fmax3(mxa[i & 3], vis(i) ? t0[i] : -INFINITY, vis(i + 32) ? t1[i] : -INFINITY);
  }
  const float mx = fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])) * sl2;
  const bool need = mx > st.m_run + kRescaleThreshold || (st.m_run == -INFINITY && mx > -INFINITY);
  const float m_new = need ? mx : st.m_run;
  const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
  const float alpha = need ? fast_exp2(st.m_run - m_use) : 1.f;
  float rsa[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};  // packed pair accumulators
  uint32_t w[8][4];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const float* t = half ? t1 : t0;
#pragma unroll
    for (int e8 = 0; e8 < 4; ++e8) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = half * 32 + e8 * 8 + 2 * e;
        float x0, x1;
        ffma2(x0, x1, t[e8 * 8 + 2 * e], t[e8 * 8 + 2 * e + 1], sl2, -m_use);
        float p0 = fast_exp2(x0);
        float p1 = fast_exp2(x1);
        if (!full) {
          p0 = vis(c) ? p0 : 0.f;
          p1 = vis(c + 1) ? p1 : 0.f;
        }
        fadd2(rsa[e][0], rsa[e][1], p0, p1);
        w[half * 4 + e8][e] = pack_bf16x2(p0, p1);
      }
    }
  }
  fadd2(rsa[0][0], rsa[0][1], rsa[1][0], rsa[1][1]);
  fadd2(rsa[2][0], rsa[2][1], rsa[3][0], rsa[3][1]);
  st.l_run = st.l_run * alpha + ((rsa[0][0] + rsa[0][1]) + (rsa[2][0] + rsa[2][1]));
  st.m_run = m_new;
  // P(j) into the upper half of this tile's S buffer (already read into registers);
  // the buffer's previous P was consumed by P.V(j-2), which completed before S(j)
  // was signalled
  tmem_st32(tmem_s + lane_base + kPCol, reinterpret_cast<const float(&)[32]>(w));
  if (j > 0 && __any_sync(0xffffffffu, need)) {
    // O is touched only after the previous P.V of this head completed
    const bool ok = __all_sync(0xffffffffu, wait_or_abort(o_done, (uint32_t)((j - 1) & 1), dead, p.err));
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        float t[32];
        tmem_ld32(tmem_o + lane_base + c4 * 32, t);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i] *= alpha;
        tmem_st32(tmem_o + lane_base + c4 * 32, t);
      }
    }
  }
  tmem_wait_st();
}

__device__ __forceinline__ bool visit_tile(const PrefillParams& p, int hA, int hB, int qt, int kt, int pl) {
  return tile_class(p, hA, qt, kt, pl) != 0 || (hB >= 0 && tile_class(p, hB, qt, kt, pl) != 0);
}

template <bool kPaged>
__device__ __forceinline__ void attn_body(const PrefillParams& p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + kBarKvFull;    // [kStages]
  uint64_t* kv_empty = bar + kBarKvEmpty;  // [kStages]
  uint64_t* s_full = bar + kBarSFull;      // [head][S buffer]
  uint64_t* p_full = bar + kBarPFull;      // [head][S buffer]
  uint64_t* o_done = bar + kBarODone;      // [head]: one phase per P.V
  uint64_t* o_full = bar + kBarOFull;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar + kBarTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // dense: heaviest query tiles first; paged: query tile of the request's code rows
  const int qt = kPaged ? (int)blockIdx.x : p.n_qtiles - 1 - (int)blockIdx.x;
  const int hk = blockIdx.y / p.npairs, hp = blockIdx.y % p.npairs;
  const int hA = hk * p.G + 2 * hp;
  const int hB = (2 * hp + 1 < p.G) ? hA + 1 : -1;  // odd group size: the last pair has one head
  const int b = blockIdx.z;                         // sequence (dense) or request (paged)
  int pl = 0, kt_end = 0, seq_len = 0, leffA = 0, leffB = 0, hole_s = 0, hole_e = 0;
  if constexpr (kPaged) {
    // every thread reads the same values, so an early return is CTA-uniform and
    // happens before any barrier, TMEM allocation or copy
    const int q0 = __ldg(p.q_start + b);
    if (q0 < 0 || (int64_t)q0 + p.Kc > p.T) {
      if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_RANGE);
      return;
    }
    // trim identity: a head with quota q sees rows [0, seq_len - (Kc - q)) --
    // its own code slots >= q are the last Kc - q rows of the request
    int sl = __ldg(p.seq_lens + b);
    const int64_t cap = min(p.bt_stride * (int64_t)p.page, (int64_t)kMaxKeyTiles * kBN);
    if (sl < p.Kc || (int64_t)sl > cap) {
      if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_SEQ_OOB);
      sl = sl < p.Kc ? p.Kc : (int)cap;
    }
    seq_len = sl;
    if (p.excl) {
      hole_s = __ldg(p.excl + 2 * b);
      hole_e = __ldg(p.excl + 2 * b + 1);
      if (hole_s == hole_e) {
        hole_s = hole_e = 0;  // no exclusion for this request
      } else if (!(0 <= hole_s && hole_s < hole_e && hole_e <= seq_len - p.Kc)) {
        if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_RANGE);
        hole_s = hole_e = 0;
      }
    }
    leffA = min(max(seq_len - (p.Kc - p.quota[hA]), 0), seq_len);
    leffB = hB >= 0 ? min(max(seq_len - (p.Kc - p.quota[hB]), 0), seq_len) : 0;
    kt_end = (max(leffA, leffB) + kBN - 1) / kBN;
  } else {
    pl = p.prompt_len ? __ldg(p.prompt_len + b) : 0;
    const int qb = qt * kBM / p.per;
    kt_end = (qb + 1) * p.per / kBN;  // key tiles beyond the query's block are never visible
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&s_full[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&p_full[i], 128);
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    mbar_init(o_full, 1);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  // the visited key tiles, in order, built once by warp 2 (ballot compaction)
  int32_t* s_list = reinterpret_cast<int32_t*>(smem + kOffList);
  int32_t* s_nlist = s_list + kMaxKeyTiles;
  if (warp == 2) {
    int n = 0;
    for (int base = 0; base < kt_end; base += 32) {
      const int kt = base + lane;
      bool vis;
      if constexpr (kPaged) vis = kt < kt_end && !(kt * kBN >= hole_s && kt * kBN + kBN <= hole_e);
      else vis = kt < kt_end && visit_tile(p, hA, hB, qt, kt, pl);
      const uint32_t m = __ballot_sync(0xffffffffu, vis);
      if (vis) {
        const int k0 = kt * kBN, kb = kPaged ? 0 : k0 / p.per;
        s_list[n + __popc(m & ((1u << lane) - 1u))] = kPaged ? kt : (kb << 16) | (k0 - kb * p.per);
      }
      n += __popc(m);
    }
    if (lane == 0) *s_nlist = n;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_tiles = *s_nlist;
  bool dead = false;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_expect_tx(q_full, (hB >= 0 ? 2 : 1) * kQBytes);
      if constexpr (kPaged) {
        const int qrow = __ldg(p.q_start + b) + qt * kBM;
        tma_load_4d(smem + kOffQ, &p.tm_q, 0, hA, qrow, 0, q_full);
        tma_load_4d(smem + kOffQ + kQBytes / 2, &p.tm_q, 64, hA, qrow, 0, q_full);
        if (hB >= 0) {
          tma_load_4d(smem + kOffQ + kQBytes, &p.tm_q, 0, hB, qrow, 0, q_full);
          tma_load_4d(smem + kOffQ + kQBytes + kQBytes / 2, &p.tm_q, 64, hB, qrow, 0, q_full);
        }
      } else {
        tma_load_4d(smem + kOffQ, &p.tm_q, 0, qt * kBM, hA, b, q_full);
        tma_load_4d(smem + kOffQ + kQBytes / 2, &p.tm_q, 64, qt * kBM, hA, b, q_full);
        if (hB >= 0) {
          tma_load_4d(smem + kOffQ + kQBytes, &p.tm_q, 0, qt * kBM, hB, b, q_full);
          tma_load_4d(smem + kOffQ + kQBytes + kQBytes / 2, &p.tm_q, 64, qt * kBM, hB, b, q_full);
        }
      }
    }
    if constexpr (kPaged) {
      // The whole warp: lane i holds the page id of 16-row slice i % 4 of tile
      // j0 + i / 4, so one coalesced block-table read covers 8 tiles and the
      // next batch's read is in flight while this batch's copies are issued.
      // Slices past seq_len (or with an invalid page id) are not loaded; their
      // V rows are zero-filled by the softmax warps.
      auto slice_page = [&](int j0) -> int {
        const int j = j0 + (lane >> 2);
        if (j >= n_tiles) return -1;
        const int row0 = s_list[j] * kBN + 16 * (lane & 3);
        if (row0 >= seq_len) return -1;
        const int v = __ldg(p.bt + (int64_t)b * p.bt_stride + row0 / p.page);
        if (v < 0 || (int64_t)v >= p.num_blocks) {
          set_error(p.err, ABKV_DEVERR_PAGE_OOB);
          return -1;
        }
        return v;
      };
      int cur = slice_page(0);
      bool stop = false;
      for (int j0 = 0; j0 < n_tiles && !stop; j0 += 8) {
        const int nxt = slice_page(j0 + 8);
        for (int jj = 0; jj < 8 && j0 + jj < n_tiles; ++jj) {
          const int j = j0 + jj, st = j % kStages;
          const int kt = s_list[j];
          const int pg = __shfl_sync(0xffffffffu, cur, 4 * jj + (lane & 3));  // lanes 0..3: slices 0..3
          const uint32_t valid = __ballot_sync(0xffffffffu, pg >= 0) & 0xFu;
          bool ok = true;
          if (lane == 0) {
            ok = wait_or_abort(&kv_empty[st], (uint32_t)(((j / kStages) & 1) ^ 1), dead, p.err);
            if (ok) mbar_expect_tx(&kv_full[st], (uint32_t)__popc(valid) * 4u * 2048u);
          }
          if (!__shfl_sync(0xffffffffu, ok, 0)) {
            stop = true;
            break;
          }
          if (lane < 4 && pg >= 0) {
            uint8_t* kbuf = smem + kOffKV + st * kStageBytes + lane * 2048;
            const int off = (kt * kBN + 16 * lane) % p.page;
            const int pk = p.fa_layout ? pg : 2 * pg;
            const int pv = p.fa_layout ? pg + (int)p.num_blocks : 2 * pg + 1;
            tma_load_4d(kbuf, &p.tm_k, 0, hk, off, pk, &kv_full[st]);
            tma_load_4d(kbuf + kKVHalf / 2, &p.tm_k, 64, hk, off, pk, &kv_full[st]);
            tma_load_4d(kbuf + kKVHalf, &p.tm_k, 0, hk, off, pv, &kv_full[st]);
            tma_load_4d(kbuf + kKVHalf + kKVHalf / 2, &p.tm_k, 64, hk, off, pv, &kv_full[st]);
          }
        }
        cur = nxt;
      }
    } else if (lane == 0) {
      for (int j = 0; j < n_tiles; ++j) {
        const int e = s_list[j];
        const int kt = ((e >> 16) * p.per + (e & 0xFFFF)) / kBN;
        const int st = j % kStages;
        if (!wait_or_abort(&kv_empty[st], (uint32_t)(((j / kStages) & 1) ^ 1), dead, p.err)) break;
        uint8_t* kbuf = smem + kOffKV + st * kStageBytes;
        mbar_expect_tx(&kv_full[st], kStageBytes);
        tma_load_4d(kbuf, &p.tm_k, 0, kt * kBN, hk, b, &kv_full[st]);
        tma_load_4d(kbuf + kKVHalf / 2, &p.tm_k, 64, kt * kBN, hk, b, &kv_full[st]);
        tma_load_4d(kbuf + kKVHalf, &p.tm_v, 0, kt * kBN, hk, b, &kv_full[st]);
        tma_load_4d(kbuf + kKVHalf + kKVHalf / 2, &p.tm_v, 64, kt * kBN, hk, b, &kv_full[st]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const bool two = hB >= 0;
      wait_or_abort(q_full, 0, dead, p.err);
      const uint32_t qa = smem_u32(smem + kOffQ), qbv = qa + kQBytes;
      const uint32_t sA = tmem, oA = tmem + 128, sB = tmem + 256, oB = tmem + 384;
      auto issue_s = [&](uint32_t qaddr, uint32_t sd, int st) {
        const uint32_t kaddr = smem_u32(smem + kOffKV + st * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // over head_dim in steps of 16
          umma(sd, desc_kmajor_sw128(qaddr + (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32),
               desc_kmajor_sw128(kaddr + (kk >> 2) * (kKVHalf / 2) + (kk & 3) * 32), kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](uint32_t ptmem, uint32_t od, int st, bool first) {
        const uint32_t vaddr = smem_u32(smem + kOffKV + st * kStageBytes + kKVHalf);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {  // over the tile's keys in steps of 16 (8 TMEM columns)
          umma_tmem_a(od, ptmem + kk * 8, desc_mnmajor_sw128(vaddr + kk * 2048, kKVHalf / 2), kIdescPV,
                      (!first || kk > 0) ? 1u : 0u);
        }
      };
      // tile sequence; S of tile j goes to S buffer j % 2 of each head
      const int n = n_tiles;
      for (int t = 0; t < 2 && t < n && !dead; ++t) {
        if (!wait_or_abort(&kv_full[t], 0, dead, p.err)) break;
        tc_fence_after();
        issue_s(qa, sA + 64 * t, t);
        umma_commit(&s_full[t]);
        if (two) {
          issue_s(qbv, sB + 64 * t, t);
          umma_commit(&s_full[2 + t]);
        }
      }
      for (int j = 0; j < n && !dead; ++j) {
        const int st = j % kStages, st2 = (j + 2) % kStages;
        const bool more = j + 2 < n;
        // head A: P_A(j) V_j; S_A(j+2) into the S buffer softmax A(j) has released
        if (!wait_or_abort(&p_full[j & 1], (uint32_t)((j >> 1) & 1), dead, p.err)) break;
        tc_fence_after();
        issue_pv(sA + 64 * (j & 1) + kPCol, oA, st, j == 0);
        umma_commit(&o_done[0]);
        if (!two) umma_commit(&kv_empty[st]);
        if (more) {
          if (!wait_or_abort(&kv_full[st2], (uint32_t)(((j + 2) / kStages) & 1), dead, p.err)) break;
          tc_fence_after();
          issue_s(qa, sA + 64 * (j & 1), st2);
          umma_commit(&s_full[j & 1]);
        }
        if (two) {
          // head B: P_B(j) V_j (last use of this K/V stage), then S_B(j+2)
          if (!wait_or_abort(&p_full[2 + (j & 1)], (uint32_t)((j >> 1) & 1), dead, p.err)) break;
          tc_fence_after();
          issue_pv(sB + 64 * (j & 1) + kPCol, oB, st, j == 0);
          umma_commit(&o_done[1]);
          umma_commit(&kv_empty[st]);
          if (more) {
            issue_s(qbv, sB + 64 * (j & 1), st2);
            umma_commit(&s_full[2 + (j & 1)]);
          }
        }
      }
      umma_commit(o_full);
    }
  } else {
    // ---------------- softmax / correction / epilogue ----------------
    const int head_slot = (warp - 2) >> 2;          // 0: head A (warps 2..5), 1: head B (warps 6..9)
    const int h = head_slot ? hB : hA;
    const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;             // query row within the tile
    const int q = qt * kBM + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t tmem_h = tmem + (head_slot ? 256 : 0), tmem_o = tmem_h + 128;
    if (h >= 0) {
      SoftmaxState st{-INFINITY, 0.f};
      const int qbr = kPaged ? 0 : q / p.per, qwr = kPaged ? 0 : q - qbr * p.per, quota = p.quota[h];
      const int leff = head_slot ? leffB : leffA;
      for (int j = 0; j < n_tiles; ++j) {
        const int e = s_list[j];
        int lim;
        if constexpr (kPaged) {
          lim = min(max(leff - e * kBN, 0), kBN);
        } else {
          const int kb = e >> 16, kw0 = e & 0xFFFF;
          lim = tile_limit_fast(p, quota, q, qbr, qwr, kb, kw0, kb * p.per + kw0, pl);
        }
        // warp-uniform decision: tcgen05.ld is a warp-collective
        const bool ok = __all_sync(
            0xffffffffu, wait_or_abort(&s_full[2 * head_slot + (j & 1)], (uint32_t)((j >> 1) & 1), dead, p.err));
        if (!ok) {
          dead = true;
          break;
        }
        tc_fence_after();
        if (kPaged && head_slot == 0 && e * kBN + kBN > seq_len) {
          // V rows at or past seq_len (stale page slots or unloaded slices) become
          // zeros before either head's P.V reads them (P is 0 there, but 0 * NaN
          // would not be)
          const int first = max(seq_len - e * kBN, 0);
          uint8_t* vb = smem + kOffKV + (j % kStages) * kStageBytes + kKVHalf;
          const int wt = (warp - 2) * 32 + lane;
          for (int idx = wt; idx < 2 * (kBN - first) * 8; idx += 128) {
            const int dh = idx / ((kBN - first) * 8), rem = idx - dh * (kBN - first) * 8;
            *reinterpret_cast<uint4*>(vb + dh * (kKVHalf / 2) + (first + rem / 8) * 128 + (rem & 7) * 16) =
                make_uint4(0, 0, 0, 0);
          }
          // each thread's zeros are made visible to the tensor core before its
          // p_full arrival, and both heads' P.V wait for head A's p_full
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        }
        if constexpr (kPaged) {
          softmax_tile<true>(p, lim, hole_s - e * kBN, hole_e - e * kBN, row, tmem_h + 64 * (j & 1), tmem_o,
                             lane_base, j, &o_done[head_slot], dead, st);
        } else {
          softmax_tile<false>(p, lim, 0, 0, row, tmem_h + 64 * (j & 1), tmem_o, lane_base, j,
                              &o_done[head_slot], dead, st);
        }
        tc_fence_before();  // P's tcgen05.st completed (wait::st) before the arrival
        mbar_arrive_one(&p_full[2 * head_slot + (j & 1)]);
      }
      // epilogue
      const bool o_ok = __all_sync(0xffffffffu, wait_or_abort(o_full, 0, dead, p.err));
      tc_fence_after();
      if (o_ok) {
        // a row that saw no visible key (possible in the code step when the
        // quota and the exclusion hide everything) is written as zeros
        const bool none = !(st.l_run > 0.f);
        const float inv = none ? 0.f : 1.f / st.l_run;
        __nv_bfloat16* orow =
            kPaged ? p.out + (int64_t)(__ldg(p.q_start + b) + q) * p.o_ss + (int64_t)h * p.o_sh
                   : p.out + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + (int64_t)q * p.o_ss;
#pragma unroll 1
        for (int c4 = 0; c4 < 4; ++c4) {
          float t[32];
          tmem_ld32(tmem_o + lane_base + c4 * 32, t);
          tmem_wait_ld();
          if (none) {
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = 0.f;
          }
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            uint4 pk;
            pk.x = pack_bf16x2(t[v8 * 8 + 0] * inv, t[v8 * 8 + 1] * inv);
            pk.y = pack_bf16x2(t[v8 * 8 + 2] * inv, t[v8 * 8 + 3] * inv);
            pk.z = pack_bf16x2(t[v8 * 8 + 4] * inv, t[v8 * 8 + 5] * inv);
            pk.w = pack_bf16x2(t[v8 * 8 + 6] * inv, t[v8 * 8 + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c4 * 32 + v8 * 8) = pk;
          }
        }
        if (!kPaged && p.lse) {
          const float lse2 = st.l_run > 0.f ? st.m_run + log2f(st.l_run) : -INFINITY;
          p.lse[((int64_t)b * p.H + h) * p.S + q] = lse2 * 0.6931471805599453f;  // natural log
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  attn_body<false>(p);
}

__global__ void __launch_bounds__(kThreads, 1) codestep_kernel(const __grid_constant__ PrefillParams p) {
  attn_body<true>(p);
}

// ---------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [B][heads][S][128] bf16 with element strides (sb, sh, ss) -> 4D tensor map,
// box = 64 dims x box_rows rows, 128B swizzle.
int make_map(CUtensorMap* m, const void* base, int B, int heads, int S, const int64_t* strides, int box_rows) {
  cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)S, (cuuint64_t)heads, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2, (cuuint64_t)strides[0] * 2};
  for (int i = 0; i < 3; ++i)
    if (gstr[i] % 16 != 0 || gstr[i] == 0) return ABKV_ERR_INVALID_ARG;
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  // the driver entry point is resolved through the runtime, so the library
  // does not link libcuda and still loads on hosts without a GPU driver
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) != cudaSuccess ||
      qres != cudaDriverEntryPointSuccess || !fn)
    return ABKV_ERR_CUDA;
  CUresult r = reinterpret_cast<EncodeTiled>(fn)(
      m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, gstr, box, es,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ABKV_OK : ABKV_ERR_INVALID_ARG;
}

}  // namespace
}  // namespace abkv

using namespace abkv;

extern "C" int abkv_prefill_masked(const void* q, const int64_t* q_strides, const void* k,
                                   const int64_t* k_strides, const void* v, const int64_t* v_strides,
                                   void* out, const int64_t* out_strides, float* lse,
                                   const int32_t* quota_per_head, const int32_t* prompt_len, int B, int H,
                                   int Hkv, int S, int head_dim, int C, int K_layout, float scale,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !out_strides) return ABKV_ERR_INVALID_ARG;
  if (B <= 0 || H <= 0 || Hkv <= 0 || S <= 0 || H % Hkv != 0 || !(scale > 0.f)) return ABKV_ERR_INVALID_ARG;
  if (head_dim != kD || H > kMaxHeads || B > 65535) return ABKV_ERR_UNSUPPORTED;
  if (C <= 0 || K_layout <= 0 || C % kBM || K_layout % kBM || S % (C + K_layout)) return ABKV_ERR_UNSUPPORTED;
  if (S / kBN > kMaxKeyTiles || C + K_layout > 65535) return ABKV_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return ABKV_ERR_INVALID_ARG;
  if (out_strides[0] % 8 || out_strides[1] % 8 || out_strides[2] % 8) return ABKV_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < 256 || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return ABKV_ERR_WORKSPACE;
  PrefillParams prm;
  std::memset(&prm, 0, sizeof(prm));
  int st = make_map(&prm.tm_q, q, B, H, S, q_strides, kBM);
  if (st == ABKV_OK) st = make_map(&prm.tm_k, k, B, Hkv, S, k_strides, kBN);
  if (st == ABKV_OK) st = make_map(&prm.tm_v, v, B, Hkv, S, v_strides, kBN);
  if (st != ABKV_OK) return st;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.o_sb = out_strides[0];
  prm.o_sh = out_strides[1];
  prm.o_ss = out_strides[2];
  prm.lse = lse;
  prm.prompt_len = prompt_len;
  prm.err = static_cast<int32_t*>(workspace);
  for (int h = 0; h < H; ++h) {
    const int qq = quota_per_head ? quota_per_head[h] : K_layout;
    if (qq < 0) return ABKV_ERR_INVALID_ARG;
    prm.quota[h] = qq;
  }
  prm.B = B;
  prm.H = H;
  prm.Hkv = Hkv;
  prm.G = H / Hkv;
  prm.npairs = (prm.G + 1) / 2;
  prm.S = S;
  prm.C = C;
  prm.KL = K_layout;
  prm.per = C + K_layout;
  prm.n_qtiles = S / kBM;
  prm.scale_log2 = scale * 1.4426950408889634f;
  if (cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
      cudaSuccess)
    return ABKV_ERR_CUDA;
  if (Hkv * prm.npairs > 65535) return ABKV_ERR_UNSUPPORTED;
  dim3 grid(prm.n_qtiles, Hkv * prm.npairs, B);
  prefill_kernel<<<grid, kThreads, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}

namespace abkv {
namespace {
// 4D tensor map over bf16 with byte strides gstr (dims 1..3), 128B swizzle.
int make_map_raw(CUtensorMap* m, const void* base, const cuuint64_t (&dims)[4], const cuuint64_t (&gstr)[3],
                 const cuuint32_t (&box)[4]) {
  for (int i = 0; i < 3; ++i)
    if (gstr[i] % 16 != 0 || gstr[i] == 0) return ABKV_ERR_INVALID_ARG;
  const cuuint32_t es[4] = {1, 1, 1, 1};
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) != cudaSuccess ||
      qres != cudaDriverEntryPointSuccess || !fn)
    return ABKV_ERR_CUDA;
  CUresult r = reinterpret_cast<EncodeTiled>(fn)(
      m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, gstr, box, es,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ABKV_OK : ABKV_ERR_INVALID_ARG;
}
}  // namespace
}  // namespace abkv

extern "C" int abkv_code_step_attention(const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out,
                                        int64_t out_row_stride, int64_t out_head_stride, const int32_t* q_start,
                                        const void* kv_cache, int kv_layout, int64_t num_blocks, int page_size,
                                        const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                                        const int32_t* excluded, const int32_t* quota_per_kv_head, int R, int Hq,
                                        int Hkv, int head_dim, int K_code, int T, float scale, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (!q || !out || !q_start || !kv_cache || !block_table || !seq_lens || !quota_per_kv_head)
    return ABKV_ERR_INVALID_ARG;
  if (R <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || T <= 0 || num_blocks <= 0 || bt_stride <= 0 ||
      !(scale > 0.f) || (kv_layout != 0 && kv_layout != 1))
    return ABKV_ERR_INVALID_ARG;
  if (head_dim != kD || Hq > kMaxHeads || R > 65535 || K_code <= 0 || K_code % kBM || page_size <= 0 ||
      page_size % 16 || 2 * num_blocks > INT32_MAX || K_code > T)
    return ABKV_ERR_UNSUPPORTED;
  if (q_row_stride <= 0 || q_head_stride <= 0 || out_row_stride % 8 || out_head_stride % 8 ||
      out_row_stride <= 0 || out_head_stride <= 0)
    return ABKV_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(kv_cache)) &
      15)
    return ABKV_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < 256 || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return ABKV_ERR_WORKSPACE;
  PrefillParams prm;
  std::memset(&prm, 0, sizeof(prm));
  {
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)Hq, (cuuint64_t)T, 1};
    const cuuint64_t gstr[3] = {(cuuint64_t)q_head_stride * 2, (cuuint64_t)q_row_stride * 2,
                                (cuuint64_t)q_row_stride * 2 * (cuuint64_t)T};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t)kBM, 1};
    const int st = make_map_raw(&prm.tm_q, q, dims, gstr, box);
    if (st != ABKV_OK) return st;
  }
  {
    // K and V planes of the paged cache as one 4D tensor: (dim, kv head, page
    // row, plane) with plane = 2 * block + {0, 1} (FlashInfer) or
    // {0, num_blocks} + block (FlashAttention); both have the same strides
    const cuuint64_t row = (cuuint64_t)Hkv * kD * 2;
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)Hkv, (cuuint64_t)page_size, (cuuint64_t)(2 * num_blocks)};
    const cuuint64_t gstr[3] = {(cuuint64_t)kD * 2, row, row * (cuuint64_t)page_size};
    const cuuint32_t box[4] = {64, 1, 16, 1};
    const int st = make_map_raw(&prm.tm_k, kv_cache, dims, gstr, box);
    if (st != ABKV_OK) return st;
  }
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.o_sh = out_head_stride;
  prm.o_ss = out_row_stride;
  prm.err = static_cast<int32_t*>(workspace);
  const int G = Hq / Hkv;
  for (int h = 0; h < Hq; ++h) {
    const int qq = quota_per_kv_head[h / G];
    if (qq < 0 || qq > K_code) return ABKV_ERR_INVALID_ARG;
    prm.quota[h] = qq;
  }
  prm.B = R;
  prm.H = Hq;
  prm.Hkv = Hkv;
  prm.G = G;
  prm.npairs = (G + 1) / 2;
  prm.n_qtiles = K_code / kBM;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.bt = block_table;
  prm.seq_lens = seq_lens;
  prm.q_start = q_start;
  prm.excl = excluded;
  prm.bt_stride = bt_stride;
  prm.num_blocks = num_blocks;
  prm.page = page_size;
  prm.Kc = K_code;
  prm.T = T;
  prm.fa_layout = kv_layout;
  if (Hkv * prm.npairs > 65535) return ABKV_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(codestep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
      cudaSuccess)
    return ABKV_ERR_CUDA;
  dim3 grid(prm.n_qtiles, Hkv * prm.npairs, R);
  codestep_kernel<<<grid, kThreads, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}
