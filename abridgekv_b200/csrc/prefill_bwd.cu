// Backward of the pause-token prefill attention (dQ, dK, dV) on 5th-generation
// tensor cores (tcgen05 + TMEM) for sm_100a: the gradients of the training
// path, which the reference runs through torch FlexAttention's backward with
// the mask of CompressLM._arith_mask_mod (abridgekv/compress_forward.py:248,
// 695-727, 1229; training: sft_ddp.py:1225).
//
// With P = softmax(scale q k^T + mask) recomputed from the forward's log-sum-exp:
//   dV = sum_h P^T dO            dP = dO V^T          Di = rowsum(dO * O)
//   dS = P * (dP - Di)           dQ = scale dS K      dK = scale sum_h dS^T Q
// (sums over the query heads h of a KV head).
//
// CTA = one 128-key tile of one KV head; it walks every (query tile, query head
// of the group) pair whose 128 x 128 tile the mask does not empty, keeping dK and
// dV in TMEM, and adds each pair's dQ tile into an fp32 buffer with TMA tensor
// reductions.  10 warps:
//   warp 0      TMA: the CTA's K and V tiles once, then Q and dO of each pair
//               (cp.async.bulk.tensor, 128B swizzle, no multicast)
//   warp 1      TMEM owner (512 columns) and MMA issuer, per pair:
//                 S^T  = K Q^T  -> [0,128)     dP^T = V dO^T -> [128,256)
//                 (thread phase: P^T, dS^T)
//                 dV  += P^T dO  (A = P^T, bf16 in [32,96))       -> [256,256+D)
//                 dK  += dS^T Q  (A = dS^T, bf16 in [160,224))    -> [384,384+D)
//                 dQ   = dS K    (A = dS from shared memory, MN-major; two
//                                   N = 64 halves into [0,64) and [128,192))
//   warps 2..9  thread = one TMEM lane: a key row for the P / dS phase, a query
//               row when dQ is read back; the two warps of a lane quarter take
//               one half of the 128 query columns (and of dQ's dims) each.  Per
//               pair they stage lse, Di and the row limit of the 128 query rows
//               in shared memory, form P and dS for their key row from S^T and
//               dP^T (the mask is a per-query prefix of the key tile), store
//               P^T / dS^T into TMEM and dS into shared memory (the A operand of
//               dQ), then add dQ into the fp32 buffer by TMA tensor reductions
//               from a staging buffer.  At the end they write dV (first half)
//               and dK (second half).
// The phases of one pair run one after the other (one S^T / dP^T buffer).  This
// pair kernel serves head_dim 64; head_dim 128 runs prefill_bwd_unit_kernel
// further down, which cuts each pair into two 64-query units so that two units
// are in flight in TMEM at once.
// Every mbarrier wait is bounded and records ABKV_DEVERR_TIMEOUT on expiry.
#include <cstring>
#include <type_traits>

#include "prefill_mask.cuh"
#include "tcgen05.cuh"

namespace abkv {
namespace {
using namespace tc;
using mask::tile_class;
using mask::tile_limit_fast;

constexpr int kT = 128;                // key / query tile rows
constexpr int kThreads = 320;
constexpr int kMaxHeads = 128;
constexpr int kMaxPairs = 2048;        // (query tile, head) pairs per key tile
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdescT = idesc_bf16_m128(kT, false);  // S^T, dP^T: N = 128 query rows, both K-major

template <int D>
struct Layout {
  static constexpr int kAtoms = D / 64;
  static constexpr int kTileBytes = kT * D * 2;   // K, V, Q, dO tiles
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kTileBytes;
  static constexpr int kOffQ = kOffV + kTileBytes;
  static constexpr int kOffDO = kOffQ + kTileBytes;
  static constexpr int kOffDS = kOffDO + kTileBytes;  // dS [128 keys][128 q] bf16, MN-major A of dQ
  static constexpr int kOffStage = kOffDS + kT * kT * 2;  // dQ staging: 2 boxes [128 rows][32 f32], 128B swizzle
  static constexpr int kOffRow = kOffStage + 2 * kT * 128;  // lse2[128], di[128], lim[128]
  static constexpr int kOffBar = kOffRow + 3 * kT * 4;
  static constexpr int kOffList = kOffBar + 256;
  static constexpr int kSmem = kOffList + 4 * kMaxPairs + 16 + 1024;
  static constexpr uint32_t kIdescAcc = idesc_bf16_m128(D, true);  // dV, dK: N = D, B MN-major
};
// dQ = dS K: M = 128 query rows, N = 64 dims, A (dS) and B (K) MN-major
constexpr uint32_t kIdescDQ = idesc_bf16_m128(64, true) | (1u << 15);

// barriers: kv_full, qd_full, qd_empty, s_full, p_full, dq_full, tm_free, acc_full, TMEM address
constexpr int kBarKV = 0, kBarQD = 1, kBarQDE = 2, kBarS = 3, kBarP = 4, kBarDQ = 5, kBarFree = 6, kBarAcc = 7,
              kBarTmem = 8;

struct alignas(64) BwdParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_do;
  CUtensorMap tm_dq;  // the fp32 dQ accumulator as [B*H*S rows][D], box [rows][32], 128B swizzle
                      // (rows = 128 for the pair kernel, 64 for the unit kernel; Q / dO likewise)
  const float* lse;   // [B][H][S], natural log (the forward's)
  const float* di;    // [B][H][S], rowsum(dO * O)
  float* dq_acc;      // [B][H][S][D] fp32
  __nv_bfloat16* dk;  // strided [B][Hkv][S][D]
  __nv_bfloat16* dv;
  int64_t dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  const int32_t* prompt_len;
  int32_t* err;
  int quota[kMaxHeads];
  int B, H, Hkv, G, S, C, KL, per, n_tiles;
  float scale, scale_log2;
};

// global[tile at (x, y)] += shared box (f32 add by the TMA engine), tracked by the bulk group.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];\n"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src)
               : "memory");
}
// Packed fp32 pairs: (a0, a1) * (b0, b1) + (c0, c1) and (a0 - b0, a1 - b1) * (c0, c1).
__device__ __forceinline__ void fma2v(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n .reg .b64 x, y, z, r;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %5};\n mov.b64 z, {%6, %7};\n"
      " fma.rn.f32x2 r, x, y, z;\n mov.b64 {%0, %1}, r;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void submul2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                        float c1) {
  asm("{\n .reg .b64 x, y, z, r;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %5};\n mov.b64 z, {%6, %7};\n"
      " sub.rn.f32x2 r, x, y;\n mul.rn.f32x2 r, r, z;\n mov.b64 {%0, %1}, r;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// this thread's bulk operations have read their shared-memory sources / have completed
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 256;\n" ::: "memory"); }
// 16 columns of 32-bit words from this warp's TMEM lanes
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_bwd_kernel(const __grid_constant__ BwdParams p) {
  using LY = Layout<D>;
  constexpr int kAtoms = LY::kAtoms, kTileBytes = LY::kTileBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + LY::kOffBar);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar + kBarTmem);
  float* s_lse2 = reinterpret_cast<float*>(smem + LY::kOffRow);
  float* s_di = s_lse2 + kT;
  int32_t* s_lim = reinterpret_cast<int32_t*>(s_di + kT);
  int32_t* s_list = reinterpret_cast<int32_t*>(smem + LY::kOffList);
  int32_t* s_n = s_list + kMaxPairs;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.G;
  const int pl = p.prompt_len ? __ldg(p.prompt_len + b) : 0;
  const int kb = kt * kT / p.per, kw0 = kt * kT - kb * p.per;
  const int qt_first = kb * p.per / kT;  // query tiles of earlier blocks never see this key tile

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBarTmem; ++i) mbar_init(&bar[i], (i == kBarP || i == kBarFree) ? 256 : 1);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  if (warp == 2) {  // the (query tile, head) pairs this key tile contributes to, by ballot
    int n = 0;
    const int total = (p.n_tiles - qt_first) * G;
    for (int base = 0; base < total; base += 32) {
      const int i = base + lane;
      const int qt = qt_first + i / G, g = i % G;
      const bool vis = i < total && tile_class(p, hk * G + g, qt, kt, pl) != 0;
      const uint32_t m = __ballot_sync(0xffffffffu, vis);
      if (vis && n + __popc(m & ((1u << lane) - 1u)) < kMaxPairs)
        s_list[n + __popc(m & ((1u << lane) - 1u))] = (qt << 8) | g;
      n += __popc(m);
    }
    if (lane == 0) {
      if (n > kMaxPairs) set_error(p.err, ABKV_DEVERR_RANGE);
      *s_n = n < kMaxPairs ? n : kMaxPairs;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_pairs = *s_n;
  bool dead = false;

  if (warp == 0) {
    // ---------------- TMA ----------------
    if (lane == 0) {
      mbar_expect_tx(&bar[kBarKV], 2 * kTileBytes);
      for (int a = 0; a < kAtoms; ++a) {
        tma_load_4d(smem + LY::kOffK + a * (kTileBytes / kAtoms), &p.tm_k, 64 * a, kt * kT, hk, b, &bar[kBarKV]);
        tma_load_4d(smem + LY::kOffV + a * (kTileBytes / kAtoms), &p.tm_v, 64 * a, kt * kT, hk, b, &bar[kBarKV]);
      }
      for (int i = 0; i < n_pairs; ++i) {
        const int e = s_list[i];
        const int qt = e >> 8, h = hk * G + (e & 0xFF);
        if (!wait_or_abort(&bar[kBarQDE], (uint32_t)((i & 1) ^ 1), dead, p.err)) break;
        mbar_expect_tx(&bar[kBarQD], 2 * kTileBytes);
        for (int a = 0; a < kAtoms; ++a) {
          tma_load_4d(smem + LY::kOffQ + a * (kTileBytes / kAtoms), &p.tm_q, 64 * a, qt * kT, h, b, &bar[kBarQD]);
          tma_load_4d(smem + LY::kOffDO + a * (kTileBytes / kAtoms), &p.tm_do, 64 * a, qt * kT, h, b, &bar[kBarQD]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint64_t dk_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffK));   // K as the A of S^T
      const uint64_t dv_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffV));   // V as the A of dP^T
      const uint64_t dq_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffQ));   // Q as the B of S^T
      const uint64_t ddo_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffDO)); // dO as the B of dP^T
      const uint64_t dq_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffQ), kTileBytes / kAtoms);    // B of dK
      const uint64_t ddo_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffDO), kTileBytes / kAtoms);  // B of dV
      const uint64_t dds_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffDS), kT * 128);             // A of dQ
      const uint64_t dk_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffK), kTileBytes / kAtoms);    // B of dQ
      constexpr int kAtomBytes = kTileBytes / kAtoms;
      wait_or_abort(&bar[kBarKV], 0, dead, p.err);
      for (int i = 0; i < n_pairs && !dead; ++i) {
        const uint32_t par = (uint32_t)(i & 1);
        if (!wait_or_abort(&bar[kBarQD], par, dead, p.err)) break;
        // S^T / dP^T overwrite the columns the threads read dQ(i-1) from
        if (i > 0 && !wait_or_abort(&bar[kBarFree], par ^ 1u, dead, p.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtomBytes + (kk & 3) * 32;
          umma(tmem + 0, desc_advance(dk_k, off), desc_advance(dq_k, off), kIdescT, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtomBytes + (kk & 3) * 32;
          umma(tmem + 128, desc_advance(dv_k, off), desc_advance(ddo_k, off), kIdescT, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar[kBarS]);
        if (!wait_or_abort(&bar[kBarP], par, dead, p.err)) break;
        tc_fence_after();
        // dV += P^T dO, dK += dS^T Q over the 128 query rows in steps of 16
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)
          umma_tmem_a(tmem + 256, tmem + 32 + kk * 8, desc_advance(ddo_mn, kk * 2048), LY::kIdescAcc,
                      (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)
          umma_tmem_a(tmem + 384, tmem + 160 + kk * 8, desc_advance(dq_mn, kk * 2048), LY::kIdescAcc,
                      (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bar[kBarQDE]);  // Q and dO may be replaced once these ran
        // dQ = dS K over the 128 keys in steps of 16, per 64-dim half of K (its accumulators overlap
        // P^T / dS^T, which the dV / dK MMAs above read first: one thread's MMAs run in issue order)
#pragma unroll
        for (int hd = 0; hd < D / 64; ++hd)
#pragma unroll
          for (int kk = 0; kk < kT / 16; ++kk)
            umma(tmem + (hd ? 128 : 0), desc_advance(dds_mn, kk * 2048),
                 desc_advance(dk_mn, hd * kAtomBytes + kk * 2048), kIdescDQ, kk > 0 ? 1u : 0u);
        umma_commit(&bar[kBarDQ]);
      }
      umma_commit(&bar[kBarAcc]);
    }
  } else {
    // ---------------- threads of TMEM lanes: P / dS, dQ, then dK and dV ----------------
    // Warps 2..9: the two warps of a lane quarter share its 32 rows; warp half hf takes query
    // columns [64 hf, 64 hf + 64) in the P / dS phase and dims [64 hf, 64 hf + 64) of dQ.
    const int quarter = warp & 3, hf = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;  // key row (P / dS phase), query row (dQ read-back)
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale_log2, scale = p.scale;
    const uint32_t ds_row = smem_u32(smem + LY::kOffDS) + hf * (kT * 128) + row * 128;  // atom column hf
    for (int i = 0; i < n_pairs; ++i) {
      const uint32_t par = (uint32_t)(i & 1);
      const int e = s_list[i];
      const int qt = e >> 8, h = hk * G + (e & 0xFF);
      if (hf == 0) {  // the 128 query rows of this pair: log2-domain lse, Di and the visible-key prefix
        const int q = qt * kT + row;
        const int64_t rr = ((int64_t)b * p.H + h) * p.S + q;
        const int qb = q / p.per, qw = q - qb * p.per;
        s_lse2[row] = __ldg(p.lse + rr) * 1.4426950408889634f;
        s_di[row] = __ldg(p.di + rr);
        s_lim[row] = tile_limit_fast(p, p.quota[h], q, qb, qw, kb, kw0, kt * kT, pl);
      }
      softmax_bar();
      const bool ok = __all_sync(0xffffffffu, wait_or_abort(&bar[kBarS], par, dead, p.err));
      if (!ok) dead = true;
      tc_fence_after();
      // P^T (bf16 pairs) goes to columns 32 + q/2 and dS^T to 160 + q/2: for this warp's query
      // range those are score columns of its own range, so each 32-column chunk is read before the
      // chunk whose words land on it is stored (half 0: chunk 1 first; half 1: chunk 0 first).
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int chunk = hf ? c : 1 - c;
        const int qc = 64 * hf + 32 * chunk;  // first query column of the chunk
        float sv[32], dpv[32];
        tmem_ld32(tmem + lane_base + qc, sv);
        tmem_ld32(tmem + lane_base + 128 + qc, dpv);
        tmem_wait_ld();
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const int q0 = qc + 8 * c8;
          const float4 la = *reinterpret_cast<const float4*>(s_lse2 + q0);
          const float4 lb = *reinterpret_cast<const float4*>(s_lse2 + q0 + 4);
          const float4 da = *reinterpret_cast<const float4*>(s_di + q0);
          const float4 db = *reinterpret_cast<const float4*>(s_di + q0 + 4);
          const int4 ma = *reinterpret_cast<const int4*>(s_lim + q0);
          const int4 mb = *reinterpret_cast<const int4*>(s_lim + q0 + 4);
          const float lse[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
          const float di[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
          const int lim[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
          float pv[8], dsv[8];
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const int cc = 8 * c8 + j;
            float x0, x1;
            fma2v(x0, x1, sv[cc], sv[cc + 1], sl2, sl2, -lse[j], -lse[j + 1]);
            pv[j] = row < lim[j] ? fast_exp2(x0) : 0.f;
            pv[j + 1] = row < lim[j + 1] ? fast_exp2(x1) : 0.f;
            // dS = (dP - Di) * (P * scale)
            submul2(dsv[j], dsv[j + 1], dpv[cc], dpv[cc + 1], di[j], di[j + 1], pv[j] * scale, pv[j + 1] * scale);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            wp[4 * c8 + j] = pack_bf16x2(pv[2 * j], pv[2 * j + 1]);
            wd[4 * c8 + j] = pack_bf16x2(dsv[2 * j], dsv[2 * j + 1]);
          }
          // dS row `row`, query rows q0..q0+7: chunk (q0 % 64) / 8 of atom column hf, 128B swizzle
          const int c16 = (q0 & 63) >> 3;
          sts128(ds_row + ((c16 ^ (row & 7)) << 4), wd[4 * c8], wd[4 * c8 + 1], wd[4 * c8 + 2], wd[4 * c8 + 3]);
        }
        tmem_st16(tmem + lane_base + 32 + qc / 2, wp);
        tmem_st16(tmem + lane_base + 160 + qc / 2, wd);
      }
      tmem_wait_st();
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // dS visible to the tensor core
      tc_fence_before();
      mbar_arrive_one(&bar[kBarP]);
      // dQ of this pair: query row `row`, dims [64 hf, 64 hf + 64) in columns [128 hf, 128 hf + 64).
      // Read into registers and release the TMEM columns; then each 64-dim half in turn goes through
      // the staging buffer (two [128 rows][32 dims] boxes, 128B swizzle) into the fp32 accumulator
      // with TMA tensor reductions issued by one thread.
      const bool okq = __all_sync(0xffffffffu, wait_or_abort(&bar[kBarDQ], par, dead, p.err));
      if (!okq) dead = true;
      tc_fence_after();
      float t[64];
      if (hf < D / 64) {
        tmem_ld32(tmem + lane_base + 128 * hf, *reinterpret_cast<float(*)[32]>(t));
        tmem_ld32(tmem + lane_base + 128 * hf + 32, *reinterpret_cast<float(*)[32]>(t + 32));
        tmem_wait_ld();
      }
      tc_fence_before();
      mbar_arrive_one(&bar[kBarFree]);
      const bool issuer = threadIdx.x == 64;
      const uint32_t stage = smem_u32(smem + LY::kOffStage);
      const int y0 = (int)(((int64_t)b * p.H + h) * p.S + qt * kT);
      if (issuer) bulk_wait_read();  // the previous pair's reductions have read the staging buffer
#pragma unroll 1
      for (int half = 0; half < D / 64; ++half) {
        softmax_bar();  // staging buffer free
        if (hf == half) {
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              sts128(stage + j * (kT * 128) + row * 128 + ((c ^ (row & 7)) << 4), __float_as_uint(t[32 * j + 4 * c]),
                     __float_as_uint(t[32 * j + 4 * c + 1]), __float_as_uint(t[32 * j + 4 * c + 2]),
                     __float_as_uint(t[32 * j + 4 * c + 3]));
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        }
        softmax_bar();  // every row of this half is staged
        if (issuer) {
          if (!dead) {
            tma_reduce_add_2d(&p.tm_dq, stage, 64 * half, y0);
            tma_reduce_add_2d(&p.tm_dq, stage + kT * 128, 64 * half + 32, y0);
            bulk_commit();
          }
          if (half + 1 < D / 64) bulk_wait_read();
        }
      }
      softmax_bar();  // the row arrays are rewritten by the next pair
    }
    if (threadIdx.x == 64) bulk_wait_all();  // every dQ reduction of this CTA has landed
    // dV (warp half 0) and dK (half 1) of this key tile: key row `row`
    const bool oka = __all_sync(0xffffffffu, wait_or_abort(&bar[kBarAcc], 0, dead, p.err));
    tc_fence_after();
    if (oka) {
      const int key = kt * kT + row;
      __nv_bfloat16* outr = hf ? p.dk + (int64_t)b * p.dk_sb + (int64_t)hk * p.dk_sh + (int64_t)key * p.dk_ss
                               : p.dv + (int64_t)b * p.dv_sb + (int64_t)hk * p.dv_sh + (int64_t)key * p.dv_ss;
      const uint32_t col = hf ? 384u : 256u;
#pragma unroll 1
      for (int c4 = 0; c4 < D / 32; ++c4) {
        float t[32];
        tmem_ld32(tmem + lane_base + col + c4 * 32, t);
        tmem_wait_ld();
        if (n_pairs == 0) {
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = 0.f;
        }
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8) {
          uint4 pk;
          pk.x = pack_bf16x2(t[v8 * 8 + 0], t[v8 * 8 + 1]);
          pk.y = pack_bf16x2(t[v8 * 8 + 2], t[v8 * 8 + 3]);
          pk.z = pack_bf16x2(t[v8 * 8 + 4], t[v8 * 8 + 5]);
          pk.w = pack_bf16x2(t[v8 * 8 + 6], t[v8 * 8 + 7]);
          *reinterpret_cast<uint4*>(outr + c4 * 32 + v8 * 8) = pk;
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

// ---------------------------------------------------------------------------
// head_dim 128: the same CTA work (one 128-key tile of one KV head, every
// visible (query tile, head) pair) cut into 64-query units -- the two halves of
// each pair -- so that two units are in flight: the tensor core computes the
// scores of unit u+1 and the gradients of unit u while the threads form P / dS
// of one unit and add the dQ of the previous one.  Per unit u (slot s = u % 2):
//   S^T  = K Q_u^T   -> TMEM [128 s, 128 s + 64)        (N = 64 queries)
//   dP^T = V dO_u^T  -> TMEM [128 s + 64, 128 s + 128)
//   (threads: P^T bf16 -> [128 s + 16, 128 s + 48), dS^T -> [128 s + 80, 128 s + 112),
//    dS -> the shared-memory dS buffer; dS is kept without the softmax scale,
//    which dK's epilogue and the dQ conversion apply)
//   dV  += P^T dO_u  -> [256, 384)      dK += dS^T Q_u -> [384, 512)
//   dQ_u^T = K^T dS_u^T (M = 128 dims, N = 64 queries; both operands MN-major in
//            shared memory) -> [128 s, 128 s + 64), over the consumed S^T / P^T
// Per unit the threads wait for S(u), read dQ^T(u-1) out of TMEM (lane = dim,
// kept in registers), form P / dS of u, then stage dQ^T(u-1) as [64 query
// rows][128 dims] fp32 and add it to the accumulator with four TMA tensor
// reductions.  Reading dQ^T(u-1) first frees its buffer, so the MMA thread
// issues the scores of u + 1 while P(u) is formed, then dV / dK(u) and
// dQ^T(u); and dQ^T(u-1) has read dS before P(u) rewrites it (one dS buffer).
// Q / dO of a unit sit in a three-slot ring ([64 rows][128 dims] each), a slot
// refilled once the dV / dK MMAs of its unit ran.
// ---------------------------------------------------------------------------
constexpr int kU = 64;      // queries per unit
constexpr int kQSlots = 3;  // Q / dO ring depth
constexpr uint32_t kIdescU = idesc_bf16_m128(kU, false);  // S^T, dP^T of a unit: N = 64, both K-major
constexpr uint32_t kIdescAccU = idesc_bf16_m128(128, true);  // dV, dK: N = 128 dims, B MN-major

struct LayoutU {
  static constexpr int kKV = kT * 128 * 2;      // K or V tile: 2 atoms of [128 rows][128 B]
  static constexpr int kSlot = kU * 128 * 2;    // Q or dO of a unit: 2 atoms of [64 rows][128 B]
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kKV;
  static constexpr int kOffQ = kOffV + kKV;                // Q slots
  static constexpr int kOffDO = kOffQ + kQSlots * kSlot;   // dO slots
  static constexpr int kOffDS = kOffDO + kQSlots * kSlot;  // dS of the current unit: [128 keys][64 queries]
  static constexpr int kOffStage = kOffDS + kT * kU * 2;   // dQ staging: 4 boxes [64 rows][32 f32]
  static constexpr int kOffRow = kOffStage + kU * 128 * 4;  // lse2, di, lim: [2 slots][64] each
  static constexpr int kOffBar = kOffRow + 3 * 2 * kU * 4 + 16;  // + [2 slots][2] "all keys visible" flags
  static constexpr int kOffList = kOffBar + 256;
  static constexpr int kSmem = kOffList + 4 * kMaxPairs + 16 + 1024;
};
static_assert(LayoutU::kSmem <= 227 * 1024, "shared memory of the 64-query-unit backward");

// barriers of the unit kernel: QD / QDE one per Q / dO slot; S / P / DQ / Free one per TMEM buffer
constexpr int kUBarKV = 0, kUBarQD = 1, kUBarQDE = kUBarQD + kQSlots, kUBarS = kUBarQDE + kQSlots,
              kUBarP = kUBarS + 2, kUBarDQ = kUBarP + 2, kUBarFree = kUBarDQ + 2, kUBarAcc = kUBarFree + 2,
              kUBarTmem = kUBarAcc + 1;
static_assert((kUBarTmem + 1) * 8 <= 256, "barrier area");

__global__ void __launch_bounds__(kThreads, 1) prefill_bwd_unit_kernel(const __grid_constant__ BwdParams p) {
  using LY = LayoutU;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + LY::kOffBar);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar + kUBarTmem);
  float* s_lse2 = reinterpret_cast<float*>(smem + LY::kOffRow);  // [2][64]
  float* s_di = s_lse2 + 2 * kU;                                   // [2][64]
  int32_t* s_lim = reinterpret_cast<int32_t*>(s_di + 2 * kU);      // [2][64]
  int32_t* s_allvis = s_lim + 2 * kU;                               // [2][2]
  int32_t* s_list = reinterpret_cast<int32_t*>(smem + LY::kOffList);
  int32_t* s_n = s_list + kMaxPairs;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.G;
  const int pl = p.prompt_len ? __ldg(p.prompt_len + b) : 0;
  const int kb = kt * kT / p.per, kw0 = kt * kT - kb * p.per;
  const int qt_first = kb * p.per / kT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kUBarTmem; ++i) {
      const bool threads = (i >= kUBarP && i < kUBarP + 2) || (i >= kUBarFree && i < kUBarFree + 2);
      mbar_init(&bar[i], threads ? 256 : 1);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(s_tmem)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  if (warp == 2) {  // the (query tile, head) pairs this key tile contributes to, by ballot
    int n = 0;
    const int total = (p.n_tiles - qt_first) * G;
    for (int base = 0; base < total; base += 32) {
      const int i = base + lane;
      const int qt = qt_first + i / G, g = i % G;
      const bool vis = i < total && tile_class(p, hk * G + g, qt, kt, pl) != 0;
      const uint32_t m = __ballot_sync(0xffffffffu, vis);
      if (vis && n + __popc(m & ((1u << lane) - 1u)) < kMaxPairs)
        s_list[n + __popc(m & ((1u << lane) - 1u))] = (qt << 8) | g;
      n += __popc(m);
    }
    if (lane == 0) {
      if (n > kMaxPairs) set_error(p.err, ABKV_DEVERR_RANGE);
      *s_n = n < kMaxPairs ? n : kMaxPairs;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_units = 2 * *s_n;
  bool dead = false;

  if (warp == 0) {
    // ---------------- TMA ----------------
    if (lane == 0) {
      mbar_expect_tx(&bar[kUBarKV], 2 * LY::kKV);
      for (int a = 0; a < 2; ++a) {
        tma_load_4d(smem + LY::kOffK + a * (LY::kKV / 2), &p.tm_k, 64 * a, kt * kT, hk, b, &bar[kUBarKV]);
        tma_load_4d(smem + LY::kOffV + a * (LY::kKV / 2), &p.tm_v, 64 * a, kt * kT, hk, b, &bar[kUBarKV]);
      }
      for (int u = 0; u < n_units; ++u) {
        const int e = s_list[u >> 1];
        const int qrow = (e >> 8) * kT + kU * (u & 1), h = hk * G + (e & 0xFF);
        const int qs = u % kQSlots, use = u / kQSlots;
        // slot qs is free once the dV / dK MMAs of unit u - 3 ran (immediate for the first use)
        if (!wait_or_abort(&bar[kUBarQDE + qs], (uint32_t)((use & 1) ^ 1), dead, p.err)) break;
        mbar_expect_tx(&bar[kUBarQD + qs], 2 * LY::kSlot);
        for (int a = 0; a < 2; ++a) {
          tma_load_4d(smem + LY::kOffQ + qs * LY::kSlot + a * (LY::kSlot / 2), &p.tm_q, 64 * a, qrow, h, b,
                      &bar[kUBarQD + qs]);
          tma_load_4d(smem + LY::kOffDO + qs * LY::kSlot + a * (LY::kSlot / 2), &p.tm_do, 64 * a, qrow, h, b,
                      &bar[kUBarQD + qs]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint64_t dk_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffK));                // A of S^T
      const uint64_t dv_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffV));                // A of dP^T
      const uint64_t dk_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffK), LY::kKV / 2);  // A of dQ^T (K^T)
      wait_or_abort(&bar[kUBarKV], 0, dead, p.err);
      // scores of unit u into TMEM buffer u % 2
      auto issue_s = [&](int u) -> bool {
        const int s = u & 1, i = u >> 1, qs = u % kQSlots;
        if (!wait_or_abort(&bar[kUBarQD + qs], (uint32_t)((u / kQSlots) & 1), dead, p.err)) return false;
        // the buffer held dQ^T of unit u - 2: the threads have read it back
        if (!wait_or_abort(&bar[kUBarFree + s], (uint32_t)((i & 1) ^ 1), dead, p.err)) return false;
        tc_fence_after();
        const uint64_t dq_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffQ + qs * LY::kSlot));
        const uint64_t ddo_k = desc_kmajor_sw128(smem_u32(smem + LY::kOffDO + qs * LY::kSlot));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t oa = (kk >> 2) * (LY::kKV / 2) + (kk & 3) * 32, ob = (kk >> 2) * (LY::kSlot / 2) + (kk & 3) * 32;
          umma(tmem + 128 * s, desc_advance(dk_k, oa), desc_advance(dq_k, ob), kIdescU, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t oa = (kk >> 2) * (LY::kKV / 2) + (kk & 3) * 32, ob = (kk >> 2) * (LY::kSlot / 2) + (kk & 3) * 32;
          umma(tmem + 128 * s + 64, desc_advance(dv_k, oa), desc_advance(ddo_k, ob), kIdescU, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar[kUBarS + s]);
        return true;
      };
      // dV / dK of unit u once its P^T / dS^T are in TMEM: the last reads of its Q / dO slot
      auto grad_kv = [&](int u) -> bool {
        const int s = u & 1, i = u >> 1, qs = u % kQSlots;
        if (!wait_or_abort(&bar[kUBarP + s], (uint32_t)(i & 1), dead, p.err)) return false;
        tc_fence_after();
        const uint64_t ddo_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffDO + qs * LY::kSlot), LY::kSlot / 2);
        const uint64_t dq_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffQ + qs * LY::kSlot), LY::kSlot / 2);
#pragma unroll
        for (int kk = 0; kk < kU / 16; ++kk)
          umma_tmem_a(tmem + 256, tmem + 128 * s + 16 + kk * 8, desc_advance(ddo_mn, kk * 2048),
                      kIdescAccU, (u > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kU / 16; ++kk)
          umma_tmem_a(tmem + 384, tmem + 128 * s + 80 + kk * 8, desc_advance(dq_mn, kk * 2048),
                      kIdescAccU, (u > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bar[kUBarQDE + qs]);  // Q / dO slot qs may be refilled once these ran
        return true;
      };
      // dQ^T of unit u over the 128 keys in steps of 16 (its columns overlap P^T, which dV read
      // first: one thread's MMAs run in issue order)
      auto grad_q = [&](int u) {
        const int s = u & 1;
        const uint64_t dds_mn = desc_mnmajor_sw128(smem_u32(smem + LY::kOffDS), kT * 128);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)
          umma(tmem + 128 * s, desc_advance(dk_mn, kk * 2048), desc_advance(dds_mn, kk * 2048), kIdescDQ,
               kk > 0 ? 1u : 0u);
        umma_commit(&bar[kUBarDQ + s]);
      };
      // order: the scores of unit u as soon as the threads have read dQ^T(u - 2) out of its
      // buffer (they do that before forming P of unit u - 1), then dV / dK and dQ^T of unit u - 1
      for (int u = 0; u <= n_units && !dead; ++u) {
        if (u < n_units && !issue_s(u)) break;
        if (u > 0) {
          if (!grad_kv(u - 1)) break;
          grad_q(u - 1);
        }
      }
      umma_commit(&bar[kUBarAcc]);
    }
  } else {
    // ---------------- threads of TMEM lanes ----------------
    // P / dS phase: lane = key row, warp half hf = query columns [32 hf, 32 hf + 32) of the unit.
    // dQ read-back: lane = dim, warp half hf = the same query columns.
    const int quarter = warp & 3, hf = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    const bool issuer = threadIdx.x == 64;
    const uint32_t stage = smem_u32(smem + LY::kOffStage);
    // dQ^T of unit v: read out of its TMEM buffer (lane = dim, query columns [32 hf, 32 hf + 32))
    // before the next unit's P / dS, which frees the buffer for the scores of unit v + 2 early;
    // staged and added to the accumulator after that P / dS.
    float dqt[32];
    auto fetch_dq = [&](int v) {
      const int s = v & 1, i = v >> 1;
      const bool okq = __all_sync(0xffffffffu, wait_or_abort(&bar[kUBarDQ + s], (uint32_t)(i & 1), dead, p.err));
      if (!okq) dead = true;
      tc_fence_after();
      tmem_ld32(tmem + lane_base + 128 * s + 32 * hf, dqt);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive_one(&bar[kUBarFree + s]);
    };
    auto reduce_dq = [&](int v) {
      const int s = v & 1, i = v >> 1;
      const int e = s_list[i];
      const int qt = e >> 8, h = hk * G + (e & 0xFF);
      if (issuer) bulk_wait_read();  // the previous unit's reductions have read the staging buffer
      softmax_bar();
      // dim `row` of query rows 32 hf .. 32 hf + 31: box `quarter` ([64 rows][32 f32], 128B swizzle)
      const uint32_t box = stage + quarter * (kU * 128) + (lane & 3) * 4;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int q = 32 * hf + j;
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(box + q * 128 + (((lane >> 2) ^ (q & 7)) << 4)),
                     "r"(__float_as_uint(dqt[j]))
                     : "memory");
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      softmax_bar();  // the unit's dQ is staged
      if (issuer && !dead) {
        const int y0 = (int)(((int64_t)b * p.H + h) * p.S + qt * kT + kU * s);
#pragma unroll
        for (int c = 0; c < 4; ++c) tma_reduce_add_2d(&p.tm_dq, stage + c * (kU * 128), 32 * c, y0);
        bulk_commit();
      }
    };
    // lse (log2 domain), Di and the visible-key prefix of a unit's 64 query rows: the threads
    // of warp half 0 with row < 64 fetch unit u + 1's values while unit u is computed and store
    // them at the start of unit u + 1, so the global loads' latency stays off the unit's path
    const bool stager = hf == 0 && row < kU;
    float n_lse = 0.f, n_di = 0.f;
    int n_lim = 0;
    auto fetch_rows = [&](int u) {
      const int e = s_list[u >> 1];
      const int qt = e >> 8, h = hk * G + (e & 0xFF);
      const int q = qt * kT + kU * (u & 1) + row;
      const int64_t rr = ((int64_t)b * p.H + h) * p.S + q;
      const int qb = q / p.per, qw = q - qb * p.per;
      n_lse = __ldg(p.lse + rr);
      n_di = __ldg(p.di + rr);
      n_lim = tile_limit_fast(p, p.quota[h], q, qb, qw, kb, kw0, kt * kT, pl);
    };
    if (stager && n_units > 0) fetch_rows(0);
    for (int u = 0; u < n_units; ++u) {
      const int s = u & 1, i = u >> 1;
      if (stager) {
        s_lse2[kU * s + row] = n_lse * 1.4426950408889634f;
        s_di[kU * s + row] = n_di;
        s_lim[kU * s + row] = n_lim;
        // the stagers are lane quarters 0 and 1 (rows 0..63), one warp each
        const bool all = __all_sync(0xffffffffu, n_lim >= kT);
        if (lane == 0) s_allvis[2 * s + quarter] = all;
      }
      softmax_bar();
      const bool allvis = s_allvis[2 * s] && s_allvis[2 * s + 1];  // every key of the tile is visible
      if (stager && u + 1 < n_units) fetch_rows(u + 1);
      const bool ok = __all_sync(0xffffffffu, wait_or_abort(&bar[kUBarS + s], (uint32_t)(i & 1), dead, p.err));
      if (!ok) dead = true;
      // dQ^T(u - 1) out of TMEM; its MMA also finished reading the dS buffer this unit rewrites
      if (u >= 1) fetch_dq(u - 1);
      tc_fence_after();
      {
        const int qc = 32 * hf;
        float sv[32], dpv[32];
        tmem_ld32(tmem + lane_base + 128 * s + qc, sv);
        tmem_ld32(tmem + lane_base + 128 * s + 64 + qc, dpv);
        tmem_wait_ld();
        uint32_t wp[16], wd[16];
        const uint32_t ds_row = smem_u32(smem + LY::kOffDS) + row * 128;
        // dS is stored without the softmax scale (dS' = P (dP - Di)); dK's epilogue and the dQ
        // conversion apply it.  kAll: no query of the unit has a masked key in this tile.
        auto form = [&](auto all_c) {
          constexpr bool kAll = decltype(all_c)::value;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const int q0 = qc + 8 * c8;
            const float4 la = *reinterpret_cast<const float4*>(s_lse2 + kU * s + q0);
            const float4 lb = *reinterpret_cast<const float4*>(s_lse2 + kU * s + q0 + 4);
            const float4 da = *reinterpret_cast<const float4*>(s_di + kU * s + q0);
            const float4 db = *reinterpret_cast<const float4*>(s_di + kU * s + q0 + 4);
            const float lse[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
            const float di[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
            int lim[8];
            if constexpr (!kAll) {
              const int4 ma = *reinterpret_cast<const int4*>(s_lim + kU * s + q0);
              const int4 mb = *reinterpret_cast<const int4*>(s_lim + kU * s + q0 + 4);
              lim[0] = ma.x; lim[1] = ma.y; lim[2] = ma.z; lim[3] = ma.w;
              lim[4] = mb.x; lim[5] = mb.y; lim[6] = mb.z; lim[7] = mb.w;
            }
            float pv[8], dsv[8];
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const int cc = 8 * c8 + j;
              float x0, x1;
              fma2v(x0, x1, sv[cc], sv[cc + 1], sl2, sl2, -lse[j], -lse[j + 1]);
              pv[j] = fast_exp2(x0);
              pv[j + 1] = fast_exp2(x1);
              if constexpr (!kAll) {
                pv[j] = row < lim[j] ? pv[j] : 0.f;
                pv[j + 1] = row < lim[j + 1] ? pv[j + 1] : 0.f;
              }
              submul2(dsv[j], dsv[j + 1], dpv[cc], dpv[cc + 1], di[j], di[j + 1], pv[j], pv[j + 1]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              wp[4 * c8 + j] = pack_bf16x2(pv[2 * j], pv[2 * j + 1]);
              wd[4 * c8 + j] = pack_bf16x2(dsv[2 * j], dsv[2 * j + 1]);
            }
            // dS row `row`, unit query columns q0..q0+7: 16-byte chunk q0 / 8 of the row, 128B swizzle
            const int c16 = q0 >> 3;
            sts128(ds_row + ((c16 ^ (row & 7)) << 4), wd[4 * c8], wd[4 * c8 + 1], wd[4 * c8 + 2], wd[4 * c8 + 3]);
          }
        };
        if (allvis)
          form(std::true_type{});
        else
          form(std::false_type{});
        // P^T / dS^T (bf16 pairs) land on score columns this warp has already read
        tmem_st16(tmem + lane_base + 128 * s + 16 + qc / 2, wp);
        tmem_st16(tmem + lane_base + 128 * s + 80 + qc / 2, wd);
      }
      tmem_wait_st();
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // dS visible to the tensor core
      tc_fence_before();
      mbar_arrive_one(&bar[kUBarP + s]);
      if (u >= 1) reduce_dq(u - 1);
    }
    if (n_units > 0) {
      fetch_dq(n_units - 1);
      reduce_dq(n_units - 1);
    }
    if (issuer) bulk_wait_all();  // every dQ reduction of this CTA has landed
    // dV (warp half 0) and dK (half 1) of this key tile: key row `row`
    const bool oka = __all_sync(0xffffffffu, wait_or_abort(&bar[kUBarAcc], 0, dead, p.err));
    tc_fence_after();
    if (oka) {
      const int key = kt * kT + row;
      __nv_bfloat16* outr = hf ? p.dk + (int64_t)b * p.dk_sb + (int64_t)hk * p.dk_sh + (int64_t)key * p.dk_ss
                               : p.dv + (int64_t)b * p.dv_sb + (int64_t)hk * p.dv_sh + (int64_t)key * p.dv_ss;
      const uint32_t col = hf ? 384u : 256u;
      const float gs = hf ? p.scale : 1.f;  // dK carries the softmax scale (dS is stored unscaled)
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        float t[32];
        tmem_ld32(tmem + lane_base + col + c4 * 32, t);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) t[j] = n_units == 0 ? 0.f : t[j] * gs;
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8) {
          uint4 pk;
          pk.x = pack_bf16x2(t[v8 * 8 + 0], t[v8 * 8 + 1]);
          pk.y = pack_bf16x2(t[v8 * 8 + 2], t[v8 * 8 + 3]);
          pk.z = pack_bf16x2(t[v8 * 8 + 4], t[v8 * 8 + 5]);
          pk.w = pack_bf16x2(t[v8 * 8 + 6], t[v8 * 8 + 7]);
          *reinterpret_cast<uint4*>(outr + c4 * 32 + v8 * 8) = pk;
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

// Di = rowsum(dO * O) in fp32: one warp per row.
__global__ void rowdot_kernel(const __nv_bfloat16* __restrict__ o, int64_t o_sb, int64_t o_sh, int64_t o_ss,
                              const __nv_bfloat16* __restrict__ dout, int64_t d_sb, int64_t d_sh, int64_t d_ss,
                              float* di, int B, int H, int S, int D) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= (int64_t)B * H * S) return;
  const int q = (int)(r % S);
  const int h = (int)((r / S) % H);
  const int b = (int)(r / ((int64_t)S * H));
  const __nv_bfloat16* orow = o + b * o_sb + h * o_sh + q * o_ss;
  const __nv_bfloat16* drow = dout + b * d_sb + h * d_sh + q * d_ss;
  float acc = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(orow + d);
    const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(drow + d);
    acc += __bfloat162float(a.x) * __bfloat162float(g.x) + __bfloat162float(a.y) * __bfloat162float(g.y);
  }
#pragma unroll
  for (int o2 = 16; o2; o2 >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o2);
  if (lane == 0) di[r] = acc;
}

// dq (strided bf16) = scale x dq_acc (contiguous fp32), 8 dims per thread; scale is the softmax
// scale when the accumulator holds unscaled dS K (head_dim 128), else 1.
__global__ void dq_store_kernel(const float* __restrict__ acc, __nv_bfloat16* dq, int64_t sb, int64_t sh, int64_t ss,
                                int B, int H, int S, int D, float scale) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_row = D / 8;
  if (i >= (int64_t)B * H * S * per_row) return;
  const int64_t r = i / per_row;
  const int d0 = (int)(i % per_row) * 8;
  const int q = (int)(r % S);
  const int h = (int)((r / S) % H);
  const int b = (int)(r / ((int64_t)S * H));
  const float4 x = *reinterpret_cast<const float4*>(acc + r * D + d0);
  const float4 y = *reinterpret_cast<const float4*>(acc + r * D + d0 + 4);
  uint4 pk;
  pk.x = pack_bf16x2(x.x * scale, x.y * scale);
  pk.y = pack_bf16x2(x.z * scale, x.w * scale);
  pk.z = pack_bf16x2(y.x * scale, y.y * scale);
  pk.w = pack_bf16x2(y.z * scale, y.w * scale);
  *reinterpret_cast<uint4*>(dq + b * sb + h * sh + q * ss + d0) = pk;
}

int make_map(CUtensorMap* m, const void* base, int B, int heads, int S, int D, const int64_t* strides,
             int box_rows) {
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)heads, (cuuint64_t)B};
  const cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2, (cuuint64_t)strides[0] * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  return tc::encode_tiled_4d(m, base, dims, gstr, box);
}

constexpr size_t kWsHeader = 256;
size_t bwd_workspace(int B, int H, int S, int D) {
  const size_t rows = (size_t)B * H * S;
  return kWsHeader + (rows * D * 4 + 255) / 256 * 256 + (rows * 4 + 255) / 256 * 256;
}

}  // namespace
}  // namespace abkv

using namespace abkv;

extern "C" size_t abkv_prefill_masked_backward_workspace_size(int B, int H, int S, int head_dim) {
  if (B <= 0 || H <= 0 || S <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  return bwd_workspace(B, H, S, head_dim);
}

extern "C" int abkv_prefill_masked_backward(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, const void* v,
    const int64_t* v_strides, const void* out, const int64_t* out_strides, const void* dout,
    const int64_t* dout_strides, const float* lse, void* dq, const int64_t* dq_strides, void* dk,
    const int64_t* dk_strides, void* dv, const int64_t* dv_strides, const int32_t* quota_per_head,
    const int32_t* prompt_len, int B, int H, int Hkv, int S, int head_dim, int C, int K_layout, float scale,
    void* workspace, size_t workspace_bytes, void* stream) {
  const void* ptrs[9] = {q, k, v, out, dout, dq, dk, dv, lse};
  for (const void* x : ptrs)
    if (!x) return ABKV_ERR_INVALID_ARG;
  const int64_t* strs[8] = {q_strides, k_strides, v_strides, out_strides, dout_strides, dq_strides, dk_strides,
                            dv_strides};
  for (const int64_t* x : strs)
    if (!x) return ABKV_ERR_INVALID_ARG;
  if (B <= 0 || H <= 0 || Hkv <= 0 || S <= 0 || H % Hkv != 0 || !(scale > 0.f)) return ABKV_ERR_INVALID_ARG;
  if ((head_dim != 64 && head_dim != 128) || H > kMaxHeads || B > 65535 || Hkv > 65535) return ABKV_ERR_UNSUPPORTED;
  if (H / Hkv > 255) return ABKV_ERR_UNSUPPORTED;
  if (C <= 0 || K_layout <= 0 || C % kT || K_layout % kT || S % (C + K_layout)) return ABKV_ERR_UNSUPPORTED;
  if ((int64_t)(S / kT) * (H / Hkv) > kMaxPairs || S / kT > (1 << 23)) return ABKV_ERR_UNSUPPORTED;
  if ((int64_t)B * H * S > INT32_MAX) return ABKV_ERR_UNSUPPORTED;  // dQ rows are 32-bit TMA coordinates
  for (int i = 0; i < 8; ++i)
    if (reinterpret_cast<uintptr_t>(ptrs[i]) & 15) return ABKV_ERR_INVALID_ARG;
  for (int i = 3; i < 8; ++i)  // rows of out, dout, dq, dk, dv are written or read as 16-byte vectors
    if (strs[i][0] % 8 || strs[i][1] % 8 || strs[i][2] % 8) return ABKV_ERR_INVALID_ARG;
  const size_t need = bwd_workspace(B, H, S, head_dim);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return ABKV_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  const size_t rows = (size_t)B * H * S;
  float* dq_acc = reinterpret_cast<float*>(ws + kWsHeader);
  float* di = reinterpret_cast<float*>(ws + kWsHeader + (rows * head_dim * 4 + 255) / 256 * 256);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  BwdParams prm;
  std::memset(&prm, 0, sizeof(prm));
  // head_dim 128 runs the 64-query-unit kernel: Q, dO and dQ move in 64-row boxes
  const int qrows = head_dim == 128 ? kU : kT;
  int st = make_map(&prm.tm_q, q, B, H, S, head_dim, q_strides, qrows);
  if (st == ABKV_OK) st = make_map(&prm.tm_do, dout, B, H, S, head_dim, dout_strides, qrows);
  if (st == ABKV_OK) st = make_map(&prm.tm_k, k, B, Hkv, S, head_dim, k_strides, kT);
  if (st == ABKV_OK) st = make_map(&prm.tm_v, v, B, Hkv, S, head_dim, v_strides, kT);
  if (st == ABKV_OK) {
    const cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
    const cuuint64_t gstr[1] = {(cuuint64_t)head_dim * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)qrows};
    st = tc::encode_tiled(&prm.tm_dq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dq_acc, dims, gstr, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (st != ABKV_OK) return st;
  for (int h = 0; h < H; ++h) {
    const int qq = quota_per_head ? quota_per_head[h] : K_layout;
    if (qq < 0) return ABKV_ERR_INVALID_ARG;
    prm.quota[h] = qq;
  }
  prm.lse = lse;
  prm.di = di;
  prm.dq_acc = dq_acc;
  prm.dk = static_cast<__nv_bfloat16*>(dk);
  prm.dv = static_cast<__nv_bfloat16*>(dv);
  prm.dk_sb = dk_strides[0];
  prm.dk_sh = dk_strides[1];
  prm.dk_ss = dk_strides[2];
  prm.dv_sb = dv_strides[0];
  prm.dv_sh = dv_strides[1];
  prm.dv_ss = dv_strides[2];
  prm.prompt_len = prompt_len;
  prm.err = reinterpret_cast<int32_t*>(ws);
  prm.B = B;
  prm.H = H;
  prm.Hkv = Hkv;
  prm.G = H / Hkv;
  prm.S = S;
  prm.C = C;
  prm.KL = K_layout;
  prm.per = C + K_layout;
  prm.n_tiles = S / kT;
  prm.scale = scale;
  prm.scale_log2 = scale * 1.4426950408889634f;

  if (cudaMemsetAsync(dq_acc, 0, rows * head_dim * 4, s) != cudaSuccess) return ABKV_ERR_CUDA;
  {
    const int64_t warps_per_block = 8;
    const int64_t blocks = ((int64_t)rows + warps_per_block - 1) / warps_per_block;
    rowdot_kernel<<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(out), out_strides[0], out_strides[1], out_strides[2],
        static_cast<const __nv_bfloat16*>(dout), dout_strides[0], dout_strides[1], dout_strides[2], di, B, H, S,
        head_dim);
  }
  auto kernel = head_dim == 64 ? prefill_bwd_kernel<64> : prefill_bwd_unit_kernel;
  const int smem = head_dim == 64 ? Layout<64>::kSmem : LayoutU::kSmem;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return ABKV_ERR_CUDA;
  kernel<<<dim3(prm.n_tiles, Hkv, B), kThreads, smem, s>>>(prm);
  {
    const int64_t n = (int64_t)rows * (head_dim / 8);
    dq_store_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dq_acc, static_cast<__nv_bfloat16*>(dq),
                                                                  dq_strides[0], dq_strides[1], dq_strides[2], B, H,
                                                                  S, head_dim,
                                                                  head_dim == 128 ? scale : 1.f);
  }
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}
