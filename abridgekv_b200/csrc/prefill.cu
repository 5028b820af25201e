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
// PARTIAL or EMPTY by the analytic classification of prefill_mask.cuh (the
// block structure of _fast_layer_blockmasks, :760-789).  EMPTY tiles are never
// loaded; inside a PARTIAL tile the visible keys of a row are a prefix of the tile.
//
// CTA = one 128-row query tile of TWO query heads of the same KV head.  Their
// masks are the same block structure, so both heads share every K/V tile
// (loaded once into a 4-stage ring); 19 warps:
//   warp 0      TMA producer: Q of both heads, then the K/V tiles of the visited
//               list (cp.async.bulk.tensor, 128B swizzle, no multicast)
//   warp 1      TMEM owner (512 columns: per head two S/P buffers + O); lane 0
//               issues head A's tcgen05.mma: S_A(0) S_A(1) | PV_A(j) S_A(j+2) | ...
//   warp 18     lane 0 issues head B's the same way
//                 S  = Q K^T   (A = Q, B = K, both K-major, fp32 in TMEM)
//                 O += P V     (A = P from TMEM, B = V, MN-major)
//               One issuer per head: an issuing thread's own mbarrier waits stall
//               behind the MMA operand reads it has queued, so one issuer for both
//               heads left the tensor core idle at every wait.
//   warps 2..9  softmax of head A, warps 10..17 softmax of head B: thread = one
//               TMEM lane = one query row, two warps per row quarter, each with 32
//               of the tile's 64 columns (partial row maxima exchanged through
//               shared memory at a named barrier per pair); masked online softmax
//               in fp32 with a lazily updated reference maximum, P (bf16 pairs)
//               stored into the upper half of its S buffer with tcgen05.st -- P is
//               double-buffered with S, so a head's softmax of tile j+1 waits for
//               its P.V of tile j only to rescale O; each warp keeps the row sum of
//               its columns and rescales its half of O; at the end both stage the
//               output tile in the head's (then idle) Q buffer, 128B-swizzled, and one
//               thread stores it with a TMA tensor store per 64-dim box.  The S MMA of
//               tile j+2 overwrites P(j) after P.V(j) read it: tcgen05.mma
//               operations of one thread run in issue order.
// Every mbarrier wait is bounded and records ABKV_DEVERR_TIMEOUT on expiry.
#include <cstring>

#include "prefill_mask.cuh"
#include "tcgen05.cuh"

namespace abkv {
namespace {
using namespace tc;
using mask::tile_class_t;
using mask::tile_limit_t;

constexpr int kBM = 128, kBN = 64;  // head_dim D is 64 or 128 (template parameter)
// warp 0 producer, warp 1 head A's MMA issuer (and TMEM owner), warps 2..17 softmax, warp 18 head B's
// MMA issuer
constexpr int kThreads = 608;
constexpr int kWarpIssuerB = 18;
constexpr int kMaxHeads = 128;
constexpr int kStages = 4;
constexpr uint32_t kTmemCols = 512;  // per head (A at 0, B at 256): S/P buffers [0,64) [64,128), O [128,128+D)
constexpr uint32_t kPCol = 32;       // P (64 bf16 = 32 columns) lives in columns [32, 64) of its S buffer
constexpr uint32_t kIdescQK = idesc_bf16_m128(kBN, false);  // S = Q K^T: N = keys, A and B K-major
constexpr int kOffQ = 0;                        // Q_A, Q_B
constexpr int kMaxKeyTiles = 2048;              // keys up to 2048 x 64 = 128K rows
// exchange between the two warps of a row quarter: partial row maxima [2 parity][2 heads][2 halves][128],
// then partial row sums [2 heads][2 halves][128]
constexpr int kXchgMax = 2 * 2 * 2 * 128 * 4, kXchgSum = 2 * 2 * 128 * 4;

// Dynamic shared memory layout for head_dim D (1024-byte aligned pieces for
// 128B swizzle): a [rows][D] bf16 tile is D / 64 atom columns of [rows][128 B].
template <int D>
struct Layout {
  static constexpr int kAtoms = D / 64;
  static constexpr int kQBytes = kBM * D * 2;        // per head
  static constexpr int kKVHalf = kBN * D * 2;        // K or V tile
  static constexpr int kStageBytes = 2 * kKVHalf;    // K then V
  static constexpr int kOffKV = 2 * kQBytes;
  static constexpr int kOffBar = kOffKV + kStages * kStageBytes;
  static constexpr int kOffList = kOffBar + 256;     // visited key tiles: (kb << 16) | kw0, per key tile
  static constexpr int kOffXchg = kOffList + 4 * kMaxKeyTiles + 16;
  static constexpr int kSmem = kOffXchg + kXchgMax + kXchgSum + 1024;  // + alignment slack
  static constexpr uint32_t kIdescPV = idesc_bf16_m128(D, true);  // O += P V: N = D, B (V) MN-major
};
static_assert(Layout<128>::kSmem <= 227 * 1024, "shared memory");
// mbarriers (u64 slots from kOffBar): q_full, kv_full[kStages], kv_empty[kStages] (one arrival per
// head's P.V), s_full[head][S buffer], p_full[head][S buffer], o_done[head], o_full[head], then the TMEM
// address.  p_full is double-buffered like S: a head's softmax may finish tile j+1 before its issuer
// has taken tile j's P, and one barrier per buffer keeps the two arrivals apart.
constexpr int kBarKvFull = 1, kBarKvEmpty = kBarKvFull + kStages, kBarSFull = kBarKvEmpty + kStages,
              kBarPFull = kBarSFull + 4, kBarODone = kBarPFull + 4, kBarOFull = kBarODone + 2,
              kBarTmem = kBarOFull + 2;
static_assert((kBarTmem + 1) * 8 <= 256, "barrier area");
// Lazy rescaling: a row keeps its reference maximum until a tile's maximum
// exceeds it by more than this (log2 units), so P <= 2^8 and O is rescaled
// only on large jumps (O and the row sum always share the reference).
constexpr float kRescaleThreshold = 8.f;

struct alignas(64) PrefillParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_out;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_ss;
  float* lse;  // [B][H][S] or null
  const int32_t* prompt_len;  // [B] or null
  int32_t* err;
  int quota[kMaxHeads];
  int B, H, Hkv, G, npairs, S, C, KL, per, n_qtiles;
  float scale_log2;
};

// Softmax of one (head, 64-key tile) for query row `row` (= TMEM lane), columns
// [32 half, 32 half + 32) of the tile; the partner warp (same rows, other half)
// does the rest.  The two exchange their partial row maxima through shared
// memory (xm_mine / xm_other, one float per row) at the pair's named barrier,
// so both take the same lazy-rescale decision and reference maximum; each keeps
// the row sum of its own columns and rescales its own half of O (D / 2 columns).
// P (bf16, 16 words) goes into this half's columns of the upper half of the S buffer.
template <int D>
__device__ __forceinline__ void softmax_half(const PrefillParams& p, int lim, int half, int row, uint32_t tmem_s,
                                             uint32_t tmem_o, uint32_t lane_base, int j, uint64_t* o_done,
                                             bool& dead, SoftmaxState& st, float* xm_mine, const float* xm_other,
                                             int pair_bar, bool live) {
  if (!live) {  // this warp gave up waiting for S: it only meets its partner at the pair's barrier
    named_bar_sync(pair_bar, 64);
    return;
  }
  const float sl2 = p.scale_log2;  // lim: visible columns of this row are c < lim
  const int c0 = 32 * half;
  float t[32];
  tmem_ld32(tmem_s + lane_base + c0, t);
  tmem_wait_ld();
  // visible columns of this half as a bit mask (bit i: column c0 + i visible, i.e. c0 + i < lim)
  const int nv = lim - c0;
  const uint32_t vm = nv >= 32 ? 0xFFFFFFFFu : (nv <= 0 ? 0u : ((1u << nv) - 1u));
  auto vis = [&](int c) { return ((vm >> (c - c0)) & 1u) != 0u; };
  const bool full = lim == kBN;
  float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
  if (full) {
#pragma unroll
    for (int i = 0; i < 16; ++i) mxa[i & 3] = fmax3(mxa[i & 3], t[2 * i], t[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      mxa[i & 3] = fmax3(mxa[i & 3], vis(c0 + 2 * i) ? t[2 * i] : -INFINITY,
                         vis(c0 + 2 * i + 1) ? t[2 * i + 1] : -INFINITY);
  }
  const float mpart = fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3]));
  xm_mine[row] = mpart;
  // both warps' S loads are complete (wait::ld) before either stores P over columns [32, 64)
  tc_fence_before();
  named_bar_sync(pair_bar, 64);
  tc_fence_after();
  const float mx = fmaxf(mpart, xm_other[row]) * sl2;  // the row's maximum over both halves
  const bool need = mx > st.m_run + kRescaleThreshold || (st.m_run == -INFINITY && mx > -INFINITY);
  const float m_new = need ? mx : st.m_run;
  const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
  const float alpha = need ? fast_exp2(st.m_run - m_use) : 1.f;
  float rsa[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};  // packed pair accumulators
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = c0 + 2 * i;
    float x0, x1;
    ffma2(x0, x1, t[2 * i], t[2 * i + 1], sl2, -m_use);
    float p0 = fast_exp2(x0);
    float p1 = fast_exp2(x1);
    if (!full) {
      p0 = vis(c) ? p0 : 0.f;
      p1 = vis(c + 1) ? p1 : 0.f;
    }
    fadd2(rsa[i & 3][0], rsa[i & 3][1], p0, p1);
    w[i] = pack_bf16x2(p0, p1);
  }
  fadd2(rsa[0][0], rsa[0][1], rsa[1][0], rsa[1][1]);
  fadd2(rsa[2][0], rsa[2][1], rsa[3][0], rsa[3][1]);
  st.l_run = st.l_run * alpha + ((rsa[0][0] + rsa[0][1]) + (rsa[2][0] + rsa[2][1]));
  st.m_run = m_new;
  // P(j) into this half's columns of the upper half of the tile's S buffer (already read into
  // registers); the buffer's previous P was consumed by P.V(j-2), which completed before S(j)
  // was signalled
  tmem_st16(tmem_s + lane_base + kPCol + 16 * half, w);
  if (j > 0 && __any_sync(0xffffffffu, need)) {
    // O is touched only after the previous P.V of this head completed; the partner warp takes
    // the same branch (same rows, same maxima) and rescales the other half of O's columns
    const bool ok = __all_sync(0xffffffffu, wait_or_abort(o_done, (uint32_t)((j - 1) & 1), dead, p.err));
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c4 = 0; c4 < D / 64; ++c4) {
        float o[32];
        const uint32_t col = tmem_o + lane_base + (D / 2) * half + 32 * c4;
        tmem_ld32(col, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= alpha;
        tmem_st32(col, o);
      }
    }
  }
  tmem_wait_st();
}

__device__ __forceinline__ bool visit_tile(const PrefillParams& p, int hA, int hB, int qt, int kt, int pl) {
  return tile_class_t<kBM, kBN>(p, hA, qt, kt, pl) != 0 || (hB >= 0 && tile_class_t<kBM, kBN>(p, hB, qt, kt, pl) != 0);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  using LY = Layout<D>;
  constexpr int kQBytes = LY::kQBytes, kKVHalf = LY::kKVHalf, kStageBytes = LY::kStageBytes;
  constexpr int kOffKV = LY::kOffKV, kOffBar = LY::kOffBar, kOffList = LY::kOffList, kAtoms = LY::kAtoms;
  constexpr uint32_t kIdescPV = LY::kIdescPV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + kBarKvFull;    // [kStages]
  uint64_t* kv_empty = bar + kBarKvEmpty;  // [kStages]
  uint64_t* s_full = bar + kBarSFull;      // [head][S buffer]
  uint64_t* p_full = bar + kBarPFull;      // [head][S buffer]
  uint64_t* o_done = bar + kBarODone;      // [head]: one phase per P.V
  uint64_t* o_full = bar + kBarOFull;      // [head]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar + kBarTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.n_qtiles - 1 - (int)blockIdx.x;  // heaviest query tiles first
  const int hk = blockIdx.y / p.npairs, hp = blockIdx.y % p.npairs;
  const int hA = hk * p.G + 2 * hp;
  const int hB = (2 * hp + 1 < p.G) ? hA + 1 : -1;  // odd group size: the last pair has one head
  const int b = blockIdx.z;
  const int pl = p.prompt_len ? __ldg(p.prompt_len + b) : 0;
  const int qb = qt * kBM / p.per;
  const int kt_end = (qb + 1) * p.per / kBN;  // key tiles beyond the query's block are never visible

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], hB >= 0 ? 2 : 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);  // the 8 softmax warps of a head
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&o_done[i], 1);
      mbar_init(&o_full[i], 1);
    }
    // Q of both heads right away: its latency overlaps the tile-list build below
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    mbar_expect_tx(q_full, (hB >= 0 ? 2 : 1) * kQBytes);
    for (int a = 0; a < kAtoms; ++a) {
      tma_load_4d(smem + kOffQ + a * (kQBytes / kAtoms), &p.tm_q, 64 * a, qt * kBM, hA, b, q_full);
      if (hB >= 0)
        tma_load_4d(smem + kOffQ + kQBytes + a * (kQBytes / kAtoms), &p.tm_q, 64 * a, qt * kBM, hB, b, q_full);
    }
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
      const bool vis = kt < kt_end && visit_tile(p, hA, hB, qt, kt, pl);
      const uint32_t m = __ballot_sync(0xffffffffu, vis);
      if (vis) {
        const int k0 = kt * kBN, kb = k0 / p.per;
        s_list[n + __popc(m & ((1u << lane) - 1u))] = (kb << 16) | (k0 - kb * p.per);
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
      for (int j = 0; j < n_tiles; ++j) {
        const int e = s_list[j];
        const int k0 = (e >> 16) * p.per + (e & 0xFFFF);
        const int st = j % kStages;
        if (!wait_or_abort(&kv_empty[st], (uint32_t)(((j / kStages) & 1) ^ 1), dead, p.err)) break;
        uint8_t* kbuf = smem + kOffKV + st * kStageBytes;
        mbar_expect_tx(&kv_full[st], kStageBytes);
        for (int a = 0; a < kAtoms; ++a) {
          tma_load_4d(kbuf + a * (kKVHalf / kAtoms), &p.tm_k, 64 * a, k0, hk, b, &kv_full[st]);
          tma_load_4d(kbuf + kKVHalf + a * (kKVHalf / kAtoms), &p.tm_v, 64 * a, k0, hk, b, &kv_full[st]);
        }
      }
    }
  } else if (warp == 1 || warp == kWarpIssuerB) {
    // ---------------- MMA issuers: warp 1 head A, warp 18 head B ----------------
    const int hs = warp == 1 ? 0 : 1;
    if (lane == 0 && (hs == 0 || hB >= 0)) {
      wait_or_abort(q_full, 0, dead, p.err);
      const uint32_t qaddr = smem_u32(smem + kOffQ) + hs * kQBytes;
      const uint32_t sbase = tmem + 256 * hs, obase = sbase + 128;
      auto issue_s = [&](uint32_t sd, int st) {
        const uint64_t dq = desc_kmajor_sw128(qaddr);
        const uint64_t dk = desc_kmajor_sw128(smem_u32(smem + kOffKV + st * kStageBytes));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // over head_dim in steps of 16 (4 per atom column)
          umma(sd, desc_advance(dq, (kk >> 2) * (kQBytes / kAtoms) + (kk & 3) * 32),
               desc_advance(dk, (kk >> 2) * (kKVHalf / kAtoms) + (kk & 3) * 32), kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](uint32_t ptmem, int st, bool first) {
        const uint64_t dv =
            desc_mnmajor_sw128(smem_u32(smem + kOffKV + st * kStageBytes + kKVHalf), kKVHalf / kAtoms);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {  // over the tile's keys in steps of 16 (8 TMEM columns)
          umma_tmem_a(obase, ptmem + kk * 8, desc_advance(dv, kk * 2048), kIdescPV, (!first || kk > 0) ? 1u : 0u);
        }
      };
      // tile sequence; S of tile j goes to S buffer j % 2
      const int n = n_tiles;
      for (int t = 0; t < 2 && t < n && !dead; ++t) {
        if (!wait_or_abort(&kv_full[t], 0, dead, p.err)) break;
        tc_fence_after();
        issue_s(sbase + 64 * t, t);
        umma_commit(&s_full[2 * hs + t]);
      }
      for (int j = 0; j < n && !dead; ++j) {
        const int st = j % kStages, st2 = (j + 2) % kStages;
        const bool more = j + 2 < n;
        // the step's waits first (after the first the queue has drained, so the next cost no
        // further stall), then P(j) V_j and S(j+2) into the S buffer softmax(j) has released
        if (more && !wait_or_abort(&kv_full[st2], (uint32_t)(((j + 2) / kStages) & 1), dead, p.err)) break;
        if (!wait_or_abort(&p_full[2 * hs + (j & 1)], (uint32_t)((j >> 1) & 1), dead, p.err)) break;
        tc_fence_after();
        issue_pv(sbase + 64 * (j & 1) + kPCol, st, j == 0);
        umma_commit(&o_done[hs]);
        umma_commit(&kv_empty[st]);  // this head's last use of the K/V stage
        if (more) {
          issue_s(sbase + 64 * (j & 1), st2);
          umma_commit(&s_full[2 * hs + (j & 1)]);
        }
      }
      umma_commit(&o_full[hs]);
    }
  } else {
    // ---------------- softmax / correction / epilogue ----------------
    const int sw = warp - 2;                         // 0..15
    const int head_slot = sw >> 3;                   // 0: head A (warps 2..9), 1: head B (warps 10..17)
    const int half = (sw >> 2) & 1;                  // columns [32 half, 32 half + 32) of every tile
    const int h = head_slot ? hB : hA;
    const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;             // query row within the tile
    const int q = qt * kBM + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t tmem_h = tmem + (head_slot ? 256 : 0), tmem_o = tmem_h + 128;
    // the two warps of these rows meet at named barrier 1 + head x 4 + quarter, once per tile and
    // twice at the end: neither leaves the tile loop early (a warp that gave up waiting skips the
    // work but not the barriers), so both execute the same barriers
    const int pair_bar = 1 + head_slot * 4 + quarter;
    float* xmax = reinterpret_cast<float*>(smem + LY::kOffXchg);                          // [parity][head][half][128]
    float* xsum = reinterpret_cast<float*>(smem + LY::kOffXchg + kXchgMax) + head_slot * 256;  // [half][128]
    if (h >= 0) {
      SoftmaxState st{-INFINITY, 0.f};  // l_run: the row sum of this warp's columns
      const int qbr = q / p.per, qwr = q - qbr * p.per, quota = p.quota[h];
      for (int j = 0; j < n_tiles; ++j) {
        const int e = s_list[j];
        const int kb = e >> 16, kw0 = e & 0xFFFF;
        const int lim = tile_limit_t<kBN>(p, quota, q, qbr, qwr, kb, kw0, kb * p.per + kw0, pl);
        // warp-uniform (tcgen05.ld is a warp-collective); a warp that gave up waiting keeps
        // going through the tiles without their work, so both warps of the pair meet at the
        // same named barriers
        const bool ok = __all_sync(0xffffffffu,
                                   wait_or_abort(&s_full[2 * head_slot + (j & 1)], (uint32_t)((j >> 1) & 1), dead, p.err));
        if (!ok) dead = true;
        tc_fence_after();
        float* xm = xmax + ((j & 1) * 2 + head_slot) * 256;  // parity j: tile j + 2 reuses it after both
        softmax_half<D>(p, lim, half, row, tmem_h + 64 * (j & 1), tmem_o, lane_base, j, &o_done[head_slot], dead,
                        st, xm + half * 128, xm + (1 - half) * 128, pair_bar, ok);
        tc_fence_before();  // P's tcgen05.st completed (wait::st) before the arrival
        mbar_arrive_one(&p_full[2 * head_slot + (j & 1)]);
      }
      // epilogue: this warp writes dims [D/2 half, D/2 half + D/2) of its row
      const bool o_ok =
          named_bar_and(pair_bar, 64, __all_sync(0xffffffffu, wait_or_abort(&o_full[head_slot], 0, dead, p.err)));
      tc_fence_after();
      xsum[half * 128 + row] = st.l_run;
      named_bar_sync(pair_bar, 64);
      const float l = st.l_run + xsum[(1 - half) * 128 + row];  // the row sum over both halves
      // O -> the head's half of the Q buffer (no S MMA reads it any more: o_full followed the head's
      // last MMAs), 128B-swizzled like the output map's boxes; then one thread stores the head's tile
      uint8_t* stage = smem + kOffQ + head_slot * kQBytes;
      if (o_ok) {
        const bool none = !(l > 0.f);  // no visible key: zeros
        const float inv = none ? 0.f : 1.f / l;
#pragma unroll 1
        for (int c4 = 0; c4 < D / 64; ++c4) {
          float t[32];
          tmem_ld32(tmem_o + lane_base + (D / 2) * half + c4 * 32, t);
          tmem_wait_ld();
          if (none) {
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = 0.f;
          }
          const int d0 = (D / 2) * half + 32 * c4;  // first dim of these 32
          uint8_t* atom = stage + (d0 / 64) * (kQBytes / kAtoms);
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8)
            st_swizzled16(atom, row, (d0 % 64) / 8 + v8, pack_bf16x2(t[v8 * 8 + 0] * inv, t[v8 * 8 + 1] * inv),
                          pack_bf16x2(t[v8 * 8 + 2] * inv, t[v8 * 8 + 3] * inv),
                          pack_bf16x2(t[v8 * 8 + 4] * inv, t[v8 * 8 + 5] * inv),
                          pack_bf16x2(t[v8 * 8 + 6] * inv, t[v8 * 8 + 7] * inv));
        }
        if (p.lse && half == 0) {
          const float lse2 = l > 0.f ? st.m_run + log2f(l) : -INFINITY;
          p.lse[((int64_t)b * p.H + h) * p.S + q] = lse2 * 0.6931471805599453f;  // natural log
        }
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // staged rows visible to the TMA
      named_bar_sync(9 + head_slot, 256);                            // the head's 8 warps have staged
      if ((sw & 7) == 0 && lane == 0) {
        if (o_ok) {
          for (int a = 0; a < kAtoms; ++a)
            tma_store_4d(&p.tm_out, stage + a * (kQBytes / kAtoms), 64 * a, qt * kBM, h, b);
          tma_store_commit();
        }
        tma_store_wait_read();  // the shared memory stays valid until the store has read it
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

// ---------------------------------------------------------------------------
// [B][heads][S][D] bf16 with element strides (sb, sh, ss) -> 4D tensor map,
// box = 64 dims x box_rows rows, 128B swizzle.
int make_map(CUtensorMap* m, const void* base, int B, int heads, int S, int D, const int64_t* strides,
             int box_rows) {
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)heads, (cuuint64_t)B};
  const cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2, (cuuint64_t)strides[0] * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  return tc::encode_tiled_4d(m, base, dims, gstr, box);
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
  if ((head_dim != 64 && head_dim != 128) || H > kMaxHeads || B > 65535) return ABKV_ERR_UNSUPPORTED;
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
  int st = make_map(&prm.tm_q, q, B, H, S, head_dim, q_strides, kBM);
  if (st == ABKV_OK) st = make_map(&prm.tm_k, k, B, Hkv, S, head_dim, k_strides, kBN);
  if (st == ABKV_OK) st = make_map(&prm.tm_v, v, B, Hkv, S, head_dim, v_strides, kBN);
  if (st == ABKV_OK) st = make_map(&prm.tm_out, out, B, H, S, head_dim, out_strides, kBM);
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
  auto kernel = head_dim == 64 ? prefill_kernel<64> : prefill_kernel<128>;
  const int smem = head_dim == 64 ? Layout<64>::kSmem : Layout<128>::kSmem;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return ABKV_ERR_CUDA;
  if (Hkv * prm.npairs > 65535) return ABKV_ERR_UNSUPPORTED;
  dim3 grid(prm.n_qtiles, Hkv * prm.npairs, B);
  kernel<<<grid, kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}

