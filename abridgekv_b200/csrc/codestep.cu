// Code step: the K code queries of every active request over the paged KV
// cache, on 5th-generation tensor cores (tcgen05 + TMEM) for sm_100a.
//
// Semantics: the noncausal branch of PackedKVSidecar._attend_request_vectorized
// (third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:648-741):
// request r's queries (rows q_start[r] .. q_start[r] + Kc - 1 of q) attend to
// rows [0, seq_len) of its block-table row; a KV head with quota q hides its
// own code slots >= q, i.e. sees rows [0, seq_len - (Kc - q)) (:711-720), and
// an optional per-request range [start, end) is hidden as well (:721-726).
// out = softmax(q.k^T * scale + mask) v with an fp32 online softmax.
//
// CTA = one 128-row query tile of TWO query heads of the same KV head (both
// heads share every K/V tile); 64-key tiles; 19 warps:
//   warp 0      TMA producer: Q of both heads, then the tile's four 16-row page
//               slices of K and V into a 4-stage ring (cp.async.bulk.tensor,
//               128B swizzle, no multicast); the block table is read 32 entries
//               at a time, one lane per slice, the next read in flight
//   warp 1      TMEM owner (512 columns: per head two S buffers + O); lane 0
//               issues head A's tcgen05.mma: S_A(0) S_A(1) | PV_A(j) S_A(j+2) | ...
//   warp 18     lane 0 issues head B's the same way
//                 S  = Q K^T   (A = Q, B = K, both K-major, fp32 in TMEM)
//                 O += P V     (A = P from TMEM, B = V, MN-major)
//               One issuer per head: an issuing thread's own mbarrier waits stall
//               behind the MMA operand reads it has queued (a few MMAs deep), so a
//               single issuer for both heads left the tensor core idle at every wait.
//   warps 2..9  softmax of head A, warps 10..17 softmax of head B: thread = one
//               TMEM lane = one query row, two warps per row quarter, each with
//               32 of the tile's 64 columns (they exchange partial row maxima at
//               a named barrier: one warp per row's 64 columns is bound by its own
//               instruction latencies, not by MUFU or the tensor core); masked
//               online softmax in fp32, P (bf16 pairs) stored into the upper half
//               of its own S buffer with tcgen05.st -- P is double-buffered with
//               S, so a head's softmax of tile j+1 waits for its P.V of tile j
//               only to rescale O; the epilogue divides by the row sum and stages a full
//               query tile's output in the head's (then idle) Q buffer for one TMA tensor
//               store per 64-dim box (partial causal tiles: row stores).  The S MMA of tile j+2 overwrites P(j)
//               after P.V(j) read it: tcgen05.mma operations of one thread run
//               in issue order.
// With all tiles full (no causal diagonal), the double-buffered S keeps the
// tensor core busier here than a 128-key tiling with one S buffer per head (which TMEM
// would impose: 2 heads x (128 S + 128 O) = 512 columns).
// Every mbarrier wait is bounded and records ABKV_DEVERR_TIMEOUT on expiry.
#include <algorithm>
#include <cstring>
#include <vector>

#include "tcgen05.cuh"

namespace abkv {
namespace {
using namespace tc;

constexpr int kBM = 128, kBN = 64, kD = 128;
// warp 0 producer, warp 1 head A's MMA issuer (and TMEM owner), warps 2..17 softmax: 8 per head,
// two per TMEM lane quarter (each owns 32 of a tile's 64 columns), warp 18 head B's MMA issuer
constexpr int kThreads = 608;
constexpr int kWarpIssuerB = 18;
constexpr int kMaxHeads = 128;
constexpr int kStages = 4;
constexpr uint32_t kTmemCols = 512;  // per head (A at 0, B at 256): S buffers [0,64) [64,128), O [128,256)
constexpr uint32_t kPCol = 32;       // P (64 bf16 = 32 columns) lives in columns [32, 64) of its S buffer
constexpr uint32_t kIdescQK = idesc_bf16_m128(kBN, false);  // S = Q K^T: N = keys, A and B K-major
constexpr uint32_t kIdescPV = idesc_bf16_m128(kD, true);    // O += P V: N = head_dim, B (V) MN-major

// dynamic shared memory layout (1024-byte aligned pieces for 128B swizzle)
constexpr int kQBytes = kBM * kD * 2;          // 32 KiB: 2 atoms of [128 rows][128 B]
constexpr int kKVHalf = kBN * kD * 2;          // 16 KiB: 2 atoms of [64 rows][128 B]
constexpr int kStageBytes = 2 * kKVHalf;       // K then V
constexpr int kOffQ = 0;                        // Q_A, Q_B
constexpr int kOffKV = 2 * kQBytes;
constexpr int kOffBar = kOffKV + kStages * kStageBytes;
// mbarriers (u64 slots from kOffBar): q_full, kv_full[kStages], kv_empty[kStages] (one
// arrival per head's P.V), s_full[head][S buffer], p_full[head][S buffer], o_done[head],
// o_full[head], v_zero[2] (head A's softmax warps have zeroed the V rows past the valid rows
// of the last sidecar tile / the last cache tile: head B's P.V of that tile waits for it),
// then the TMEM address.  p_full is double-buffered like S: a head's softmax may finish tile j+1
// before the MMA thread has taken tile j's P, and one barrier per buffer keeps the
// two arrivals in different barriers (a parity wait cannot tell phases 2 apart).
constexpr int kBarKvFull = 1, kBarKvEmpty = kBarKvFull + kStages, kBarSFull = kBarKvEmpty + kStages,
              kBarPFull = kBarSFull + 4, kBarODone = kBarPFull + 4, kBarOFull = kBarODone + 2,
              kBarVZero = kBarOFull + 2, kBarTmem = kBarVZero + 2;
static_assert((kBarTmem + 1) * 8 <= 256, "barrier area");
constexpr int kOffList = kOffBar + 256;         // visited key tiles (tile indices)
constexpr int kMaxKeyTiles = 2048;              // keys up to 2048 x 64 = 128K rows
// exchange between the two warps of a row quarter: partial row maxima [2 parity][2 heads][2 halves][128]
// and, at the end, partial row sums [2 heads][2 halves][128]
constexpr int kOffXchg = kOffList + 4 * kMaxKeyTiles + 16;
constexpr int kXchgMax = 2 * 2 * 2 * 128 * 4, kXchgSum = 2 * 2 * 128 * 4;
constexpr int kSmemBytes = kOffXchg + kXchgMax + kXchgSum + 1024;  // + slack for 1024-byte alignment
static_assert(kSmemBytes <= 227 * 1024, "shared memory");
// Lazy rescaling: a row keeps its reference maximum until a tile's maximum
// exceeds it by more than this (log2 units), so P <= 2^8 and O is rescaled
// only on large jumps (O and the row sum always share the reference).
constexpr float kRescaleThreshold = 8.f;

struct alignas(64) CodeStepParams {
  CUtensorMap tm_q, tm_k;  // q [T][H][D]; K/V planes of the paged cache
  CUtensorMap tm_out;      // out [T][H][D] (used when out_tma: full query tiles are stored by TMA)
  int out_tma;
  __nv_bfloat16* out;
  int64_t o_sh, o_ss;
  int32_t* err;
  int quota[kMaxHeads];
  int H, Hkv, G, npairs;
  float scale_log2;
  const int32_t* bt;
  const int32_t* seq_lens;
  const int32_t* q_start;
  const int32_t* excl;  // optional [R][2]: rows [start, end) hidden from the code queries
  int64_t bt_stride, num_blocks;
  int page, Kc, T, fa_layout;
  // optional compaction that follows the code step (abkv_code_step_attention_compact): request r's
  // row copies cops[coff[r] .. coff[r + 1]) ([n][4] = src block, src offset, dst block, dst offset),
  // applied to this layer's cache by the last CTA of the request to finish its reads
  const int32_t* cops;
  const int32_t* coff;
  int32_t* ccount;  // [R] finished CTAs per request (zeroed by the host before the launch)
  char* kv;
  int64_t row_bytes;
  int ctas_per_req;
  // causal mode (abkv_paged_prefill): request r's query rows are q_start[r] .. q_start[r + 1] - 1
  // (qlen rows, any count); row i sees cache rows [0, seq_len - qlen + i + 1), every head alike
  int causal;
  // optional packed sidecar (the *_packed entries): before its paged rows, KV head h of request r
  // attends to head h's slots [side_off[h], side_off[h] + side_q[h]) of each of the request's
  // side_count[r] packed pages (ids side_bt[r * side_bt_stride + i]); every query row sees them all
  CUtensorMap tm_side;  // (dim, 1, slot, plane = 2 * page + {0: K, 1: V}) over [pages][2][slots][D]
  const int32_t* side_bt;
  const int32_t* side_count;
  int64_t side_bt_stride, side_pages;
  int side_off[8], side_q[8];
  int has_side;
};

// The last CTA of request blockIdx.z applies that request's copy ops.  Every CTA of the request
// counts itself once all its reads of the cache are done: its TMA loads were consumed (waited on)
// before its MMAs, and the barrier before this call orders every thread.  A CTA that gave up on a
// wait, or that met an out-of-range page id in the request's block-table row, does not count, so
// the request's ops are not applied and the error word says why.  The host
// checked that no op writes a row any op reads and that destinations are unique, so the copies may
// run in any order.
__device__ __noinline__ void commit_request_ops(const CodeStepParams& p, bool dead) {
  __shared__ int s_last;
  const int any_dead = __syncthreads_or(dead ? 1 : 0);
  if (threadIdx.x == 0) {
    int last = 0;
    if (!any_dead) {
      __threadfence();
      last = atomicAdd(p.ccount + blockIdx.z, 1) == p.ctas_per_req - 1;
      if (last) __threadfence();
    }
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  const int o0 = __ldcg(p.coff + blockIdx.z), o1 = __ldcg(p.coff + blockIdx.z + 1);
  // one warp per op moves its K and V rows, each lane with up to 2 x 4 vectors in flight
  constexpr int kCV = 4;
  const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int64_t vecs = p.row_bytes >> 4;  // 16-byte vectors per K or V row
  for (int op = o0 + (int)(threadIdx.x >> 5); op < o1; op += nw) {
    const int sb = __ldcg(p.cops + 4 * op), so = __ldcg(p.cops + 4 * op + 1);
    const int db = __ldcg(p.cops + 4 * op + 2), dof = __ldcg(p.cops + 4 * op + 3);
    const uint4* src[2];
    uint4* dst[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t ps = p.fa_layout ? (h ? p.num_blocks + sb : sb) : 2 * (int64_t)sb + h;
      const int64_t pd = p.fa_layout ? (h ? p.num_blocks + db : db) : 2 * (int64_t)db + h;
      src[h] = reinterpret_cast<const uint4*>(p.kv + (ps * p.page + so) * p.row_bytes);
      dst[h] = reinterpret_cast<uint4*>(p.kv + (pd * p.page + dof) * p.row_bytes);
    }
    for (int64_t v0 = 0; v0 < vecs; v0 += 32 * kCV) {
      uint4 buf[2][kCV];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < kCV; ++k) {
          const int64_t v = v0 + k * 32 + lane;
          if (v < vecs) buf[h][k] = __ldcg(src[h] + v);
        }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < kCV; ++k) {
          const int64_t v = v0 + k * 32 + lane;
          if (v < vecs) __stcg(dst[h] + v, buf[h][k]);
        }
    }
  }
}

// Softmax of one (head, key tile) for query row `row` (= TMEM lane), columns
// [32 half, 32 half + 32) of the tile; the partner warp (same rows, other half)
// does the rest.  The two exchange their partial row maxima through shared
// memory (xm_mine / xm_other, one float per row) at the pair's named barrier,
// so both take the same lazy-rescale decision and reference maximum; each keeps
// the row sum of its own columns and rescales its own half of O.  P (bf16,
// 16 words) goes into this half's columns of the upper half of the S buffer.
// kHole: columns [hs, he) are hidden as well (the code step's tail exclusion).
template <bool kHole>
__device__ __forceinline__ void softmax_half(const CodeStepParams& p, int lim, int hs, int he, int half, int row,
                                             uint32_t tmem_s, uint32_t tmem_o, uint32_t lane_base, int j,
                                             uint64_t* o_done, bool& dead, SoftmaxState& st, float* xm_mine,
                                             const float* xm_other, int pair_bar, bool live) {
  if (!live) {  // this warp gave up waiting for S: it only meets its partner at the pair's barrier
    named_bar_sync(pair_bar, 64);
    return;
  }
  const float sl2 = p.scale_log2;  // lim: visible columns of this row are c < lim
  const int c0 = 32 * half;
  float t[32];
  tmem_ld32(tmem_s + lane_base + c0, t);
  tmem_wait_ld();
  // visible columns of this half as a bit mask (bit i: column c0 + i): c < lim, outside [hs, he)
  auto span = [](int a, int e) -> uint32_t {  // bits [a, e) of 32, a and e clamped to [0, 32]
    a = a < 0 ? 0 : (a > 32 ? 32 : a);
    e = e < 0 ? 0 : (e > 32 ? 32 : e);
    if (e <= a) return 0u;
    const uint32_t hi = e >= 32 ? 0xFFFFFFFFu : ((1u << e) - 1u);
    const uint32_t lo = (1u << a) - 1u;  // a < 32 here
    return hi & ~lo;
  };
  const bool full = lim == kBN && (!kHole || he <= 0 || hs >= kBN);
  uint32_t vm = 0xFFFFFFFFu;  // only a partial tile needs the mask
  if (!full) {
    vm = span(0, lim - c0);
    if (kHole) vm &= ~span(hs - c0, he - c0);
  }
  auto vis = [&](int c) { return ((vm >> (c - c0)) & 1u) != 0u; };
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
      for (int c4 = 0; c4 < 2; ++c4) {
        float o[32];
        const uint32_t col = tmem_o + lane_base + 64 * half + 32 * c4;
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

__global__ void __launch_bounds__(kThreads, 1) codestep_kernel(const __grid_constant__ CodeStepParams p) {
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
  uint64_t* v_zero = bar + kBarVZero;      // [sidecar, cache]: used at most once each
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar + kBarTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x;  // query tile of the request's code rows
  const int hk = blockIdx.y / p.npairs, hp = blockIdx.y % p.npairs;
  const int hA = hk * p.G + 2 * hp;
  const int hB = (2 * hp + 1 < p.G) ? hA + 1 : -1;  // odd group size: the last pair has one head
  const int b = blockIdx.z;  // request
  int kt_end = 0, seq_len = 0, leffA = 0, leffB = 0, hole_s = 0, hole_e = 0;
  int qlen = p.Kc;  // the request's query rows (all Kc code rows in the code step)
  int n_side = 0, side_tiles = 0;  // sidecar rows of this CTA's KV head, in 64-row tiles
  {
    // every thread reads the same values, so an early return is CTA-uniform and
    // happens before any barrier, TMEM allocation or copy
    const int q0 = __ldg(p.q_start + b);
    if (p.causal) {
      const int q1 = __ldg(p.q_start + b + 1);
      qlen = q1 - q0;
      if (q0 < 0 || qlen < 0 || q1 > p.T) {
        if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_RANGE);
        return;
      }
      // rows past the grid's tiles (max_query_len understated) are not computed
      if (qlen > (int)gridDim.x * kBM && qt == 0 && threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_RANGE);
      if (qt * kBM >= qlen) return;  // no row of this request in this tile
    } else if (q0 < 0 || (int64_t)q0 + p.Kc > p.T) {
      if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_RANGE);
      return;
    }
    // trim identity: a head with quota q sees rows [0, seq_len - (Kc - q)) --
    // its own code slots >= q are the last Kc - q rows of the request
    int sl = __ldg(p.seq_lens + b);
    const int64_t cap = min(p.bt_stride * (int64_t)p.page, (int64_t)kMaxKeyTiles * kBN);
    if (sl < qlen || (int64_t)sl > cap) {
      if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_SEQ_OOB);
      sl = sl < qlen ? qlen : (int)cap;
      // more query rows than the key-tile list holds: nothing of the request is computed
      if ((int64_t)sl > cap) return;
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
    if (p.causal) {
      // the tile's last row (qt * 128 + 127, or the request's last) sees the most keys
      const int last = min(qt * kBM + kBM, qlen);
      leffA = leffB = seq_len - qlen + last;
    } else {
      leffA = min(max(seq_len - (p.Kc - p.quota[hA]), 0), seq_len);
      leffB = hB >= 0 ? min(max(seq_len - (p.Kc - p.quota[hB]), 0), seq_len) : 0;
    }
    kt_end = (max(leffA, leffB) + kBN - 1) / kBN;
    if (p.has_side) {
      int cnt = __ldg(p.side_count + b);
      if (cnt < 0 || (int64_t)cnt > p.side_bt_stride) {
        if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_SEQ_OOB);
        cnt = cnt < 0 ? 0 : (int)p.side_bt_stride;
      }
      n_side = cnt * p.side_q[hk];
    }
    side_tiles = (n_side + kBN - 1) / kBN;
    if (side_tiles + kt_end > kMaxKeyTiles) {  // the tile list would not hold them: skip the request
      if (threadIdx.x == 0) set_error(p.err, ABKV_DEVERR_SEQ_OOB);
      return;
    }
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], hB >= 0 ? 2 : 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&s_full[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&p_full[i], 256);  // the 8 softmax warps of a head
    for (int i = 0; i < 2; ++i) {
      mbar_init(&o_done[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&v_zero[i], 256);
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
    // sidecar tiles first (entry -(t + 1) = sidecar tile t), all visible
    for (int base = 0; base < side_tiles; base += 32) {
      const int t = base + lane;
      const uint32_t m = __ballot_sync(0xffffffffu, t < side_tiles);
      if (t < side_tiles) s_list[n + __popc(m & ((1u << lane) - 1u))] = -(t + 1);
      n += __popc(m);
    }
    for (int base = 0; base < kt_end; base += 32) {
      const int kt = base + lane;
      // tiles entirely inside the exclusion range are skipped for both heads
      const bool vis = kt < kt_end && !(kt * kBN >= hole_s && kt * kBN + kBN <= hole_e);
      const uint32_t m = __ballot_sync(0xffffffffu, vis);
      if (vis) s_list[n + __popc(m & ((1u << lane) - 1u))] = kt;
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
  // set by the producer lane that met an out-of-range page id: the attention
  // still completes (that slice is not loaded), but the request's copy ops
  // are not applied after attention over a bad block table
  bool bad_page = false;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_expect_tx(q_full, (hB >= 0 ? 2 : 1) * kQBytes);
      const int qrow = __ldg(p.q_start + b) + qt * kBM;
      tma_load_4d(smem + kOffQ, &p.tm_q, 0, hA, qrow, 0, q_full);
      tma_load_4d(smem + kOffQ + kQBytes / 2, &p.tm_q, 64, hA, qrow, 0, q_full);
      if (hB >= 0) {
        tma_load_4d(smem + kOffQ + kQBytes, &p.tm_q, 0, hB, qrow, 0, q_full);
        tma_load_4d(smem + kOffQ + kQBytes + kQBytes / 2, &p.tm_q, 64, hB, qrow, 0, q_full);
      }
    }
    {
      // The whole warp: lane i holds the page id of 16-row slice i % 4 of tile
      // j0 + i / 4, so one coalesced block-table read covers 8 tiles and the
      // next batch's read is in flight while this batch's copies are issued.
      // Slices past seq_len (or with an invalid page id) are not loaded; their
      // V rows are zero-filled by the softmax warps.
      auto slice_page = [&](int j0) -> int {
        const int j = j0 + (lane >> 2);
        if (j >= n_tiles) return -1;
        if (s_list[j] < 0) {  // sidecar tile: the page holding this 16-slot slice
          const int row0 = (-s_list[j] - 1) * kBN + 16 * (lane & 3);
          if (row0 >= n_side) return -1;
          const int v = __ldg(p.side_bt + (int64_t)b * p.side_bt_stride + row0 / p.side_q[hk]);
          if (v < 0 || (int64_t)v >= p.side_pages) {
            set_error(p.err, ABKV_DEVERR_PAGE_OOB);
            bad_page = true;
            return -1;
          }
          return v;
        }
        const int row0 = s_list[j] * kBN + 16 * (lane & 3);
        if (row0 >= seq_len) return -1;
        const int v = __ldg(p.bt + (int64_t)b * p.bt_stride + row0 / p.page);
        if (v < 0 || (int64_t)v >= p.num_blocks) {
          set_error(p.err, ABKV_DEVERR_PAGE_OOB);
          bad_page = true;
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
          if (lane < 4 && pg >= 0 && kt < 0) {
            // sidecar slice: 16 slots of head hk's segment of packed page pg (K plane, V plane)
            uint8_t* kbuf = smem + kOffKV + st * kStageBytes + lane * 2048;
            const int row0 = (-kt - 1) * kBN + 16 * lane;
            const int slot = p.side_off[hk] + row0 % p.side_q[hk];
            tma_load_4d(kbuf, &p.tm_side, 0, 0, slot, 2 * pg, &kv_full[st]);
            tma_load_4d(kbuf + kKVHalf / 2, &p.tm_side, 64, 0, slot, 2 * pg, &kv_full[st]);
            tma_load_4d(kbuf + kKVHalf, &p.tm_side, 0, 0, slot, 2 * pg + 1, &kv_full[st]);
            tma_load_4d(kbuf + kKVHalf + kKVHalf / 2, &p.tm_side, 64, 0, slot, 2 * pg + 1, &kv_full[st]);
          } else if (lane < 4 && pg >= 0) {
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
    }
  } else if (warp == 1 || warp == kWarpIssuerB) {
    // ---------------- MMA issuers: warp 1 head A, warp 18 head B ----------------
    // One issuing thread per head: a thread's shared-memory accesses (its mbarrier waits)
    // wait behind the tcgen05.mma operand reads it has queued, so while one issuer waits
    // the other's queued MMAs keep the tensor core busy.
    const int hs = warp == 1 ? 0 : 1;
    if (lane == 0 && (hs == 0 || hB >= 0)) {
      // head B's P.V of a partial tile (the last sidecar tile, the last cache tile) waits
      // until head A's softmax warps have zeroed its V rows past the valid rows; the two
      // tile indices, read before any MMA is issued
      int jz0 = -1, jz1 = -1;
      if (hs == 1) {
        if (n_side % kBN) jz0 = side_tiles - 1;
        if (n_tiles > side_tiles && (seq_len % kBN) && s_list[n_tiles - 1] == (seq_len - 1) / kBN) jz1 = n_tiles - 1;
      }
      wait_or_abort(q_full, 0, dead, p.err);
      const uint32_t qaddr = smem_u32(smem + kOffQ) + hs * kQBytes;
      const uint32_t sbase = tmem + 256 * hs, obase = sbase + 128;
      auto issue_s = [&](uint32_t sd, int st) {
        const uint64_t dq = desc_kmajor_sw128(qaddr);
        const uint64_t dk = desc_kmajor_sw128(smem_u32(smem + kOffKV + st * kStageBytes));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // over head_dim in steps of 16
          umma(sd, desc_advance(dq, (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32),
               desc_advance(dk, (kk >> 2) * (kKVHalf / 2) + (kk & 3) * 32), kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](uint32_t ptmem, int st, bool first) {
        const uint64_t dv = desc_mnmajor_sw128(smem_u32(smem + kOffKV + st * kStageBytes + kKVHalf), kKVHalf / 2);
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
        // all waits of the step first (after the first one the queue has drained, so the
        // next cost no further stall), then P(j) V_j and S(j+2) into the S buffer that
        // softmax(j) has released
        if (more && !wait_or_abort(&kv_full[st2], (uint32_t)(((j + 2) / kStages) & 1), dead, p.err)) break;
        if (!wait_or_abort(&p_full[2 * hs + (j & 1)], (uint32_t)((j >> 1) & 1), dead, p.err)) break;
        if (j == jz0 && !wait_or_abort(&v_zero[0], 0, dead, p.err)) break;
        if (j == jz1 && !wait_or_abort(&v_zero[1], 0, dead, p.err)) break;
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
    // the two warps of these rows (warps w and w + 4) meet at named barrier 1 + head x 4 + quarter,
    // once per tile and twice at the end: neither leaves the tile loop early (a warp that gave up
    // waiting skips the work but not the barriers), so both always execute the same barriers
    const int pair_bar = 1 + head_slot * 4 + quarter;
    float* xmax = reinterpret_cast<float*>(smem + kOffXchg);            // [parity][head][half][128]
    float* xsum = reinterpret_cast<float*>(smem + kOffXchg + kXchgMax) + head_slot * 256;  // [half][128]
    if (h >= 0) {
      SoftmaxState st{-INFINITY, 0.f};  // l_run: the row sum of this warp's columns
      // causal: row q sees seq_len - qlen + q + 1 keys (rows past the request's
      // last row, which are never written, take the last row's limit)
      const int leff = p.causal ? seq_len - qlen + min(q, qlen - 1) + 1 : (head_slot ? leffB : leffA);
      for (int j = 0; j < n_tiles; ++j) {
        const int e = s_list[j];
        const bool side = e < 0;  // sidecar tile -(e + 1): every query row sees its rows
        const int lim = side ? min(max(n_side - (-e - 1) * kBN, 0), kBN) : min(max(leff - e * kBN, 0), kBN);
        // valid rows of the tile: the rest was not loaded (V zeroed below)
        const int valid = side ? n_side - (-e - 1) * kBN : seq_len - e * kBN;
        // warp-uniform (tcgen05.ld is a warp-collective); a warp that gave up waiting keeps
        // going through the tiles without their work, so both warps of the pair meet at the
        // same named barriers
        const bool ok = __all_sync(0xffffffffu,
                                   wait_or_abort(&s_full[2 * head_slot + (j & 1)], (uint32_t)((j >> 1) & 1), dead, p.err));
        if (!ok) dead = true;
        tc_fence_after();
        if (ok && head_slot == 0 && valid < kBN) {
          // V rows at or past seq_len (or the sidecar segment's end): stale page
          // slots or unloaded slices become zeros before either head's P.V reads
          // them (P is 0 there, but 0 * NaN would not be)
          const int first = max(valid, 0);
          uint8_t* vb = smem + kOffKV + (j % kStages) * kStageBytes + kKVHalf;
          const int wt = sw * 32 + lane;  // head A's 256 threads
          for (int idx = wt; idx < 2 * (kBN - first) * 8; idx += 256) {
            const int dh = idx / ((kBN - first) * 8), rem = idx - dh * (kBN - first) * 8;
            *reinterpret_cast<uint4*>(vb + dh * (kKVHalf / 2) + (first + rem / 8) * 128 + (rem & 7) * 16) =
                make_uint4(0, 0, 0, 0);
          }
          // each thread's zeros are made visible to the tensor core before its
          // p_full and v_zero arrivals (head B's P.V waits for v_zero)
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
          mbar_arrive_one(&v_zero[side ? 0 : 1]);
        }
        float* xm = xmax + ((j & 1) * 2 + head_slot) * 256;  // parity j: tile j + 2 reuses it after both
        softmax_half<true>(p, lim, side ? 0 : hole_s - e * kBN, side ? 0 : hole_e - e * kBN, half, row,
                           tmem_h + 64 * (j & 1), tmem_o, lane_base, j, &o_done[head_slot], dead, st,
                           xm + half * 128, xm + (1 - half) * 128, pair_bar, ok);
        tc_fence_before();  // P's tcgen05.st completed (wait::st) before the arrival
        mbar_arrive_one(&p_full[2 * head_slot + (j & 1)]);
      }
      // epilogue: this warp writes dims [64 half, 64 half + 64) of its rows
      const bool o_ok =
          named_bar_and(pair_bar, 64, __all_sync(0xffffffffu, wait_or_abort(&o_full[head_slot], 0, dead, p.err)));
      tc_fence_after();
      xsum[half * 128 + row] = st.l_run;
      named_bar_sync(pair_bar, 64);
      const float l = st.l_run + xsum[(1 - half) * 128 + row];  // the row sum over both halves
      // a full query tile goes through the head's half of the Q buffer (no S MMA reads it any more:
      // o_full followed the head's last MMAs), 128B-swizzled like the output map's boxes, and one
      // thread stores it; a partial tile (causal mode) is stored row by row
      const bool tile_store = p.out_tma && qt * kBM + kBM <= qlen;  // CTA-uniform
      uint8_t* stage = smem + kOffQ + head_slot * kQBytes;
      if (o_ok) {
        // a row that saw no visible key (possible in the code step when the
        // quota and the exclusion hide everything) is written as zeros
        const bool none = !(l > 0.f);
        const float inv = none ? 0.f : 1.f / l;
        __nv_bfloat16* orow =
            p.out + (int64_t)(__ldg(p.q_start + b) + q) * p.o_ss + (int64_t)h * p.o_sh + 64 * half;
#pragma unroll 1
        for (int c4 = 0; c4 < 2; ++c4) {
          float t[32];
          tmem_ld32(tmem_o + lane_base + 64 * half + c4 * 32, t);
          tmem_wait_ld();
          if (none) {
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = 0.f;
          }
          if (tile_store) {
            uint8_t* atom = stage + half * (kQBytes / 2);
#pragma unroll
            for (int v8 = 0; v8 < 4; ++v8)
              st_swizzled16(atom, row, 4 * c4 + v8, pack_bf16x2(t[v8 * 8 + 0] * inv, t[v8 * 8 + 1] * inv),
                            pack_bf16x2(t[v8 * 8 + 2] * inv, t[v8 * 8 + 3] * inv),
                            pack_bf16x2(t[v8 * 8 + 4] * inv, t[v8 * 8 + 5] * inv),
                            pack_bf16x2(t[v8 * 8 + 6] * inv, t[v8 * 8 + 7] * inv));
          } else if (q < qlen) {
            // tcgen05.ld above is warp-collective; only the stores skip rows past
            // the request's last query row (causal mode)
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
        }
      }
      if (tile_store) {
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // staged rows visible to the TMA
        named_bar_sync(9 + head_slot, 256);                            // the head's 8 warps have staged
        if ((sw & 7) == 0 && lane == 0) {
          if (o_ok) {
            const int row0 = __ldg(p.q_start + b) + qt * kBM;
            tma_store_4d(&p.tm_out, stage, 0, h, row0, 0);
            tma_store_4d(&p.tm_out, stage + kQBytes / 2, 64, h, row0, 0);
            tma_store_commit();
          }
          tma_store_wait_read();  // the shared memory stays valid until the store has read it
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
  if (p.cops) commit_request_ops(p, dead || bad_page);
}

}  // namespace
}  // namespace abkv

using namespace abkv;

namespace {
// Copy ops of the compaction that follows the code step, already validated and uploaded.
struct CommitArgs {
  const int32_t* ops;  // device [n][4]
  const int32_t* off;  // device [R + 1]
  int32_t* count;      // device [R], zeroed
};

int code_step_launch(const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out,
                     int64_t out_row_stride, int64_t out_head_stride, const int32_t* q_start,
                     const void* kv_cache, int kv_layout, int64_t num_blocks, int page_size,
                     const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                     const int32_t* excluded, const int32_t* quota_per_kv_head, int R, int Hq,
                     int Hkv, int head_dim, int K_code, int T, float scale, void* workspace,
                     size_t workspace_bytes, void* stream, const CommitArgs* commit, int causal_max_qlen = 0,
                     const abkv_sidecar_t* side = nullptr);

constexpr size_t align256(size_t x) { return (x + 255) / 256 * 256; }
size_t commit_workspace(int R, int64_t n_ops) {
  return 256 + align256((size_t)R * 4) + align256((size_t)(R + 1) * 4) + align256((size_t)n_ops * 16);
}
}  // namespace

extern "C" int abkv_code_step_attention(const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out,
                                        int64_t out_row_stride, int64_t out_head_stride, const int32_t* q_start,
                                        const void* kv_cache, int kv_layout, int64_t num_blocks, int page_size,
                                        const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                                        const int32_t* excluded, const int32_t* quota_per_kv_head, int R, int Hq,
                                        int Hkv, int head_dim, int K_code, int T, float scale, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  return code_step_launch(q, q_row_stride, q_head_stride, out, out_row_stride, out_head_stride, q_start, kv_cache,
                          kv_layout, num_blocks, page_size, block_table, bt_stride, seq_lens, excluded,
                          quota_per_kv_head, R, Hq, Hkv, head_dim, K_code, T, scale, workspace, workspace_bytes,
                          stream, nullptr);
}

extern "C" int abkv_paged_prefill(const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out,
                                  int64_t out_row_stride, int64_t out_head_stride, const int32_t* query_start_loc,
                                  const void* kv_cache, int kv_layout, int64_t num_blocks, int page_size,
                                  const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens, int R,
                                  int Hq, int Hkv, int head_dim, int max_query_len, int T, float scale,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (max_query_len <= 0) return ABKV_ERR_INVALID_ARG;
  return code_step_launch(q, q_row_stride, q_head_stride, out, out_row_stride, out_head_stride, query_start_loc,
                          kv_cache, kv_layout, num_blocks, page_size, block_table, bt_stride, seq_lens, nullptr,
                          nullptr, R, Hq, Hkv, head_dim, 0, T, scale, workspace, workspace_bytes, stream, nullptr,
                          max_query_len);
}

extern "C" int abkv_code_step_attention_packed(
    const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out, int64_t out_row_stride,
    int64_t out_head_stride, const int32_t* q_start, const void* kv_cache, int kv_layout, int64_t num_blocks,
    int page_size, const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens, const int32_t* excluded,
    const int32_t* quota_per_kv_head, int R, int Hq, int Hkv, int head_dim, int K_code, int T, float scale,
    const abkv_sidecar_t* sidecar, void* workspace, size_t workspace_bytes, void* stream) {
  if (!sidecar) return ABKV_ERR_INVALID_ARG;
  return code_step_launch(q, q_row_stride, q_head_stride, out, out_row_stride, out_head_stride, q_start, kv_cache,
                          kv_layout, num_blocks, page_size, block_table, bt_stride, seq_lens, excluded,
                          quota_per_kv_head, R, Hq, Hkv, head_dim, K_code, T, scale, workspace, workspace_bytes,
                          stream, nullptr, 0, sidecar);
}

extern "C" int abkv_paged_prefill_packed(const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out,
                                         int64_t out_row_stride, int64_t out_head_stride,
                                         const int32_t* query_start_loc, const void* kv_cache, int kv_layout,
                                         int64_t num_blocks, int page_size, const int32_t* block_table,
                                         int64_t bt_stride, const int32_t* seq_lens, int R, int Hq, int Hkv,
                                         int head_dim, int max_query_len, int T, float scale,
                                         const abkv_sidecar_t* sidecar, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  if (max_query_len <= 0 || !sidecar) return ABKV_ERR_INVALID_ARG;
  return code_step_launch(q, q_row_stride, q_head_stride, out, out_row_stride, out_head_stride, query_start_loc,
                          kv_cache, kv_layout, num_blocks, page_size, block_table, bt_stride, seq_lens, nullptr,
                          nullptr, R, Hq, Hkv, head_dim, 0, T, scale, workspace, workspace_bytes, stream, nullptr,
                          max_query_len, sidecar);
}

extern "C" size_t abkv_code_step_compact_workspace_size(int num_requests, int64_t n_ops) {
  if (num_requests <= 0 || n_ops < 0 || n_ops > INT32_MAX / 4) return 0;
  return commit_workspace(num_requests, n_ops);
}

extern "C" int abkv_code_step_attention_compact(
    const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out, int64_t out_row_stride,
    int64_t out_head_stride, const int32_t* q_start, void* kv_cache, int kv_layout, int64_t num_blocks,
    int page_size, const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens, const int32_t* excluded,
    const int32_t* quota_per_kv_head, int R, int Hq, int Hkv, int head_dim, int K_code, int T, float scale,
    const int32_t* ops, const int64_t* op_offsets, int64_t n_ops, void* workspace, size_t workspace_bytes,
    void* stream) {
  if (R <= 0 || !op_offsets || n_ops < 0 || n_ops > INT32_MAX / 4 || (n_ops > 0 && !ops) || num_blocks <= 0 ||
      page_size <= 0)
    return ABKV_ERR_INVALID_ARG;
  if (op_offsets[0] != 0 || op_offsets[R] != n_ops) return ABKV_ERR_INVALID_ARG;
  for (int r = 0; r < R; ++r)
    if (op_offsets[r + 1] < op_offsets[r]) return ABKV_ERR_INVALID_ARG;
  // every op in range; destinations unique and never a source, so the copies may run in any order
  // (the same result as the executor's gather-all-then-scatter batch)
  std::vector<int64_t> src((size_t)n_ops), dst((size_t)n_ops);
  for (int64_t i = 0; i < n_ops; ++i) {
    const int32_t sb = ops[4 * i], so = ops[4 * i + 1], db = ops[4 * i + 2], dof = ops[4 * i + 3];
    if (sb < 0 || sb >= num_blocks || db < 0 || db >= num_blocks || so < 0 || so >= page_size || dof < 0 ||
        dof >= page_size)
      return ABKV_ERR_INVALID_ARG;
    src[i] = (int64_t)sb * page_size + so;
    dst[i] = (int64_t)db * page_size + dof;
  }
  std::sort(src.begin(), src.end());
  std::sort(dst.begin(), dst.end());
  if (std::adjacent_find(dst.begin(), dst.end()) != dst.end()) return ABKV_ERR_UNSUPPORTED;
  for (size_t i = 0, j = 0; i < dst.size() && j < src.size();) {
    if (dst[i] == src[j]) return ABKV_ERR_UNSUPPORTED;
    if (dst[i] < src[j]) ++i; else ++j;
  }
  const size_t need = commit_workspace(R, n_ops);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return ABKV_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  CommitArgs c;
  c.count = reinterpret_cast<int32_t*>(ws + 256);
  int32_t* d_off = reinterpret_cast<int32_t*>(ws + 256 + align256((size_t)R * 4));
  int32_t* d_ops = reinterpret_cast<int32_t*>(ws + 256 + align256((size_t)R * 4) + align256((size_t)(R + 1) * 4));
  c.off = d_off;
  c.ops = d_ops;
  std::vector<int32_t> off32((size_t)R + 1);
  for (int r = 0; r <= R; ++r) off32[r] = (int32_t)op_offsets[r];
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // pageable host sources: each copy is staged before the call returns
  if (cudaMemcpyAsync(d_off, off32.data(), off32.size() * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      (n_ops > 0 && cudaMemcpyAsync(d_ops, ops, (size_t)n_ops * 16, cudaMemcpyHostToDevice, s) != cudaSuccess) ||
      cudaMemsetAsync(c.count, 0, (size_t)R * 4, s) != cudaSuccess)
    return ABKV_ERR_CUDA;
  return code_step_launch(q, q_row_stride, q_head_stride, out, out_row_stride, out_head_stride, q_start, kv_cache,
                          kv_layout, num_blocks, page_size, block_table, bt_stride, seq_lens, excluded,
                          quota_per_kv_head, R, Hq, Hkv, head_dim, K_code, T, scale, workspace, workspace_bytes,
                          stream, &c);
}

namespace {
int code_step_launch(const void* q, int64_t q_row_stride, int64_t q_head_stride, void* out,
                     int64_t out_row_stride, int64_t out_head_stride, const int32_t* q_start,
                     const void* kv_cache, int kv_layout, int64_t num_blocks, int page_size,
                     const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                     const int32_t* excluded, const int32_t* quota_per_kv_head, int R, int Hq,
                     int Hkv, int head_dim, int K_code, int T, float scale, void* workspace,
                     size_t workspace_bytes, void* stream, const CommitArgs* commit, int causal_max_qlen,
                     const abkv_sidecar_t* side) {
  const bool causal = causal_max_qlen > 0;  // abkv_paged_prefill: no quotas, no exclusion, no copies
  if (!q || !out || !q_start || !kv_cache || !block_table || !seq_lens || (!causal && !quota_per_kv_head))
    return ABKV_ERR_INVALID_ARG;
  if (R <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || T <= 0 || num_blocks <= 0 || bt_stride <= 0 ||
      !(scale > 0.f) || (kv_layout != 0 && kv_layout != 1))
    return ABKV_ERR_INVALID_ARG;
  if (causal && (excluded || commit || causal_max_qlen > T)) return ABKV_ERR_INVALID_ARG;
  if (head_dim != kD || Hq > kMaxHeads || R > 65535 || page_size <= 0 || page_size % 16 ||
      2 * num_blocks > INT32_MAX)
    return ABKV_ERR_UNSUPPORTED;
  if (!causal && (K_code <= 0 || K_code % kBM || K_code > T)) return ABKV_ERR_UNSUPPORTED;
  if (q_row_stride <= 0 || q_head_stride <= 0 || out_row_stride % 8 || out_head_stride % 8 ||
      out_row_stride <= 0 || out_head_stride <= 0)
    return ABKV_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(kv_cache)) &
      15)
    return ABKV_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < 256 || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return ABKV_ERR_WORKSPACE;
  CodeStepParams prm;
  std::memset(&prm, 0, sizeof(prm));
  {
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)Hq, (cuuint64_t)T, 1};
    const cuuint64_t gstr[3] = {(cuuint64_t)q_head_stride * 2, (cuuint64_t)q_row_stride * 2,
                                (cuuint64_t)q_row_stride * 2 * (cuuint64_t)T};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t)kBM, 1};
    const int st = tc::encode_tiled_4d(&prm.tm_q, q, dims, gstr, box);
    if (st != ABKV_OK) return st;
  }
  {
    // the output map (same shape as q's); without one (strides not multiples of 16 bytes) every
    // tile is stored row by row
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)Hq, (cuuint64_t)T, 1};
    const cuuint64_t gstr[3] = {(cuuint64_t)out_head_stride * 2, (cuuint64_t)out_row_stride * 2,
                                (cuuint64_t)out_row_stride * 2 * (cuuint64_t)T};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t)kBM, 1};
    prm.out_tma = ((out_head_stride | out_row_stride) % 8 == 0 && out_head_stride > 0 && out_row_stride > 0 &&
                   tc::encode_tiled_4d(&prm.tm_out, out, dims, gstr, box) == ABKV_OK)
                      ? 1
                      : 0;
  }
  {
    // K and V planes of the paged cache as one 4D tensor: (dim, kv head, page
    // row, plane) with plane = 2 * block + {0, 1} (FlashInfer) or
    // {0, num_blocks} + block (FlashAttention); both have the same strides
    const cuuint64_t row = (cuuint64_t)Hkv * kD * 2;
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)Hkv, (cuuint64_t)page_size, (cuuint64_t)(2 * num_blocks)};
    const cuuint64_t gstr[3] = {(cuuint64_t)kD * 2, row, row * (cuuint64_t)page_size};
    const cuuint32_t box[4] = {64, 1, 16, 1};
    const int st = tc::encode_tiled_4d(&prm.tm_k, kv_cache, dims, gstr, box);
    if (st != ABKV_OK) return st;
  }
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.o_sh = out_head_stride;
  prm.o_ss = out_row_stride;
  prm.err = static_cast<int32_t*>(workspace);
  const int G = Hq / Hkv;
  for (int h = 0; h < Hq && !causal; ++h) {
    const int qq = quota_per_kv_head[h / G];
    if (qq < 0 || qq > K_code) return ABKV_ERR_INVALID_ARG;
    prm.quota[h] = qq;
  }
  prm.causal = causal ? 1 : 0;
  prm.H = Hq;
  prm.Hkv = Hkv;
  prm.G = G;
  prm.npairs = (G + 1) / 2;
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
  if (side) {
    // pages [num_pages][2][slots][D]; quotas multiples of 16 (a 16-slot slice never leaves its head's
    // segment) summing to slots
    if (!side->pages || !side->page_table || !side->page_count || side->page_table_stride <= 0 ||
        side->num_pages <= 0 || side->num_pages > (INT32_MAX / 2) || commit)
      return ABKV_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(side->pages) & 15) || (reinterpret_cast<uintptr_t>(side->page_table) & 3))
      return ABKV_ERR_INVALID_ARG;
    if (Hkv > 8) return ABKV_ERR_UNSUPPORTED;
    int sum = 0;
    for (int h = 0; h < Hkv; ++h) {
      const int qh = side->quotas[h];
      if (qh <= 0 || qh % 16 || qh >= (1 << 16)) return ABKV_ERR_UNSUPPORTED;
      prm.side_off[h] = sum;
      prm.side_q[h] = qh;
      sum += qh;
    }
    if (sum != side->slots) return ABKV_ERR_INVALID_ARG;
    const cuuint64_t dims[4] = {(cuuint64_t)kD, 1, (cuuint64_t)side->slots, (cuuint64_t)(2 * side->num_pages)};
    const cuuint64_t gstr[3] = {(cuuint64_t)kD * 2, (cuuint64_t)kD * 2, (cuuint64_t)side->slots * kD * 2};
    const cuuint32_t box[4] = {64, 1, 16, 1};
    const int st = tc::encode_tiled_4d(&prm.tm_side, side->pages, dims, gstr, box);
    if (st != ABKV_OK) return st;
    prm.side_bt = side->page_table;
    prm.side_count = side->page_count;
    prm.side_bt_stride = side->page_table_stride;
    prm.side_pages = side->num_pages;
    prm.has_side = 1;
  }
  if (cudaFuncSetAttribute(codestep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
      cudaSuccess)
    return ABKV_ERR_CUDA;
  if (commit) {
    prm.cops = commit->ops;
    prm.coff = commit->off;
    prm.ccount = commit->count;
    prm.kv = static_cast<char*>(const_cast<void*>(kv_cache));
    prm.row_bytes = (int64_t)Hkv * kD * 2;
    prm.ctas_per_req = (K_code / kBM) * Hkv * prm.npairs;
  }
  dim3 grid(causal ? (causal_max_qlen + kBM - 1) / kBM : K_code / kBM, Hkv * prm.npairs, R);
  codestep_kernel<<<grid, kThreads, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}
}  // namespace
