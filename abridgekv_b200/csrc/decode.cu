// Split-KV, GQA-packed paged decode attention for sm_100a.
//
// Semantics follow the reference's batched PyTorch decode
//   third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:564-616
// (scores = q.K^T * scale over the first seq_len physical rows of the request's
// block table, fp32 softmax, weights rounded to bf16, weighted sum of V), which
// is the PyTorch image of the FlashInfer decode the vLLM overlay runs per KV
// cache group (gpu_model_runner.py:1672-1681, 2184-2204).
//
// Work decomposition.  One CTA = (split-KV chunk, sequence, layer); its eight
// warps cover the KV heads of that chunk (warp w -> head w % Hkv; with fewer
// than eight KV heads the remaining warps take interleaved tiles of the same
// head and are merged through shared memory).  A "tile" is 16 consecutive
// cache rows.  Per tile a warp:
//   * loads K rows g and g+8 (g = lane/4) as four 16-byte vectors each and V
//     rows 2c,2c+1,2c+8,2c+9 (c = lane%4) as two 16-byte vectors each, straight
//     from HBM into registers in mma fragment order (dims are permuted
//     consistently between Q and K, and between V and the output, so no shared
//     memory or ldmatrix is needed; every warp load covers whole 32-byte
//     sectors);
//   * S = Q.K^T with mma.m16n8k16 (rows = the G query heads of the KV head);
//   * online softmax in fp32 (quad shuffles), P rounded to bf16 as the
//     reference does before its P.V product;
//   * O^T += V^T.P^T with mma.m16n8k16: the S accumulator fragment is exactly
//     the B fragment of this product, so P never leaves registers.
// The block-table slice of the chunk is staged into shared memory by one bulk
// copy (cp.async.bulk on the TMA engine, no multicast) completed on an
// mbarrier with a bounded wait.
// Chunks of one (layer, sequence) are merged inside the same launch: each
// chunk CTA stores its normalised partial and log-sum-exp, and the last one
// to finish (a per-(layer, sequence) counter in the workspace, reset by that
// CTA) combines them.  Single-chunk rows are written directly.  Concurrent
// calls must not share a workspace.
#include <cstring>

#include "common.cuh"

namespace abkv {
namespace {

constexpr int kD = 128;
constexpr int kTile = 16;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxLayers = 56;       // layers per launch: keeps params < 4 KB
constexpr int kMaxChunkPages = 256;  // page ids staged per CTA
constexpr int kMaxG = 8;             // query heads per KV head

struct LayerArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  const int32_t* bt;
  const int32_t* seq_lens;
  __nv_bfloat16* out;
  int64_t bt_stride;
  int64_t num_blocks;
};

struct DecodeParams {
  LayerArgs layer[kMaxLayers];
  float* part_o;    // [layers][B][max_chunks][Hq][D]
  float* part_lse;  // [layers][B][max_chunks][Hq]
  int32_t* counters;  // [layers][B] chunks finished; zero between calls
  int32_t* err;
  float scale_log2;
  int B, Hq, Hkv, G, P;
  int chunk_tiles, max_chunks, max_rows;
  int layer_base;
};

__device__ __forceinline__ int clamp_seq_len(const DecodeParams& p, const LayerArgs& L, int b,
                                             bool report) {
  int s = __ldg(L.seq_lens + b);
  int64_t cap = L.bt_stride * (int64_t)p.P;
  if (cap > p.max_rows) cap = p.max_rows;
  if (s < 0 || (int64_t)s > cap) {
    if (report) set_error(p.err, ABKV_DEVERR_SEQ_OOB);
    s = s < 0 ? 0 : (int)cap;
  }
  return s;
}

// Dynamic shared memory layout of decode_split_kernel:
//   [kStages][kStageBytes]  K/V tile groups (a group = nsub tiles, one per
//                           warp slot; tile = 16 cache rows, K then V, all
//                           KV heads) -- 64 KiB per stage for head_dim 128
//   s_pages[kMaxChunkPages + 4]
//   mbarriers: full[kStages], page-list barrier
// After the main loop the stage buffers are reused for the epilogue arrays.
constexpr int kStages = 3;
constexpr int kStageBytes = kWarps * 2 * kTile * kD * 2;  // nsub * Hkv == kWarps
constexpr size_t kSmemBytes =
    (size_t)kStages * kStageBytes + (kMaxChunkPages + 4) * sizeof(int32_t) + (kStages + 1) * 8;

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(smem_u32(p)));
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    decode_split_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  int32_t* s_pages = reinterpret_cast<int32_t*>(smem + (size_t)kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(s_pages + kMaxChunkPages + 4);
  uint64_t* pg_bar = full + kStages;

  const int chunk = blockIdx.x, b = blockIdx.y, li = blockIdx.z;
  const LayerArgs& L = p.layer[li];
  const int seq_len = clamp_seq_len(p, L, b, chunk == 0 && threadIdx.x == 0);
  const int n_tiles = (seq_len + kTile - 1) / kTile;
  const int n_chunks = (n_tiles + p.chunk_tiles - 1) / p.chunk_tiles;

  if (n_chunks == 0) {  // empty sequence: defined as an all-zero row
    if (chunk == 0) {
      __nv_bfloat16* o = L.out + (int64_t)b * p.Hq * kD;
      for (int i = threadIdx.x; i < p.Hq * kD; i += kThreads) o[i] = __float2bfloat16(0.f);
    }
    return;
  }
  if (chunk >= n_chunks) return;

  const int tile0 = chunk * p.chunk_tiles;
  const int tile1 = min(tile0 + p.chunk_tiles, n_tiles);
  const int page0 = tile0 * kTile / p.P;
  const int page1 = (tile1 * kTile + p.P - 1) / p.P;
  const int npages = page1 - page0;

  // ---- stage this chunk's page ids in shared memory --------------------
  const int32_t* src = L.bt + (int64_t)b * L.bt_stride + page0;
  int head = (int)(((16 - (reinterpret_cast<uintptr_t>(src) & 15)) & 15) >> 2);
  if (head > npages) head = npages;
  const int body = ((npages - head) >> 2) << 2;
  const int shift = (4 - head) & 3;  // makes s_pages + shift + head 16-byte aligned
  if (threadIdx.x == 0) {
    for (int s2 = 0; s2 < kStages; ++s2) mbar_init(&full[s2], 1);
    if (body > 0) mbar_init(pg_bar, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0 && body > 0) {
    mbar_expect_tx(pg_bar, (uint32_t)body * 4u);
    bulk_g2s(s_pages + shift + head, src + head, (uint32_t)body * 4u, pg_bar);
  }
  for (int i = threadIdx.x; i < head; i += kThreads) s_pages[shift + i] = __ldg(src + i);
  for (int i = head + body + threadIdx.x; i < npages; i += kThreads)
    s_pages[shift + i] = __ldg(src + i);
  if (body > 0 && !mbar_wait(pg_bar, 0)) set_error(p.err, ABKV_DEVERR_TIMEOUT);
  __syncthreads();

  // ---- bulk-copy pipeline over tile groups --------------------------------
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hkv = p.Hkv, G = p.G, P = p.P;
  const int h = warp % Hkv, sub = warp / Hkv, nsub = kWarps / Hkv;
  const int g = lane >> 2, c = lane & 3;
  const int row_bytes = Hkv * kD * 2;      // one cache row, all KV heads
  const int tile_half = kTile * row_bytes;  // 16 rows of K (or of V)
  const int64_t row_elems = (int64_t)Hkv * kD;
  const int64_t half_elems = (int64_t)P * row_elems;
  const int64_t page_elems = 2 * half_elems;
  const int64_t nblk = L.num_blocks;
  const int ngroups = (tile1 - tile0 + nsub - 1) / nsub;

  auto tile_page = [&](int t, bool& ok) -> int64_t {
    const int pg = s_pages[shift + t * kTile / P - page0];
    ok = pg >= 0 && (int64_t)pg < nblk;
    return pg;
  };
  // thread 0: copy tile group gi (K rows then V rows of each tile) into its stage
  auto issue = [&](int gi) {
    const int st = gi % kStages;
    uint8_t* dst = smem + (size_t)st * kStageBytes;
    uint32_t bytes = 0;
    for (int j = 0; j < nsub; ++j) {
      const int t = tile0 + gi * nsub + j;
      bool ok = false;
      if (t < tile1) tile_page(t, ok);
      if (ok) bytes += 2u * (uint32_t)tile_half;
    }
    mbar_expect_tx(&full[st], bytes);
    for (int j = 0; j < nsub; ++j) {
      const int t = tile0 + gi * nsub + j;
      if (t >= tile1) break;
      bool ok;
      const int64_t pg = tile_page(t, ok);
      if (!ok) {
        set_error(p.err, ABKV_DEVERR_PAGE_OOB);
        continue;
      }
      const __nv_bfloat16* ksrc = L.kv + pg * page_elems + (int64_t)((t * kTile) % P) * row_elems;
      bulk_g2s(dst + (size_t)j * 2 * tile_half, ksrc, (uint32_t)tile_half, &full[st]);
      bulk_g2s(dst + (size_t)j * 2 * tile_half + tile_half, ksrc + half_elems, (uint32_t)tile_half,
               &full[st]);
    }
  };

  uint32_t qr[4][4];
  {
    const __nv_bfloat16* qrow = L.q + ((int64_t)b * p.Hq + h * G + g) * kD + 8 * c;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (g < G) v = __ldg(reinterpret_cast<const uint4*>(qrow + 32 * m));
      qr[m][0] = v.x; qr[m][1] = v.y; qr[m][2] = v.z; qr[m][3] = v.w;
    }
  }

  if (threadIdx.x == 0) {
    for (int gi = 0; gi < kStages && gi < ngroups; ++gi) issue(gi);
  }

  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const float sl2 = p.scale_log2;

  for (int gi = 0; gi < ngroups; ++gi) {
    const int st = gi % kStages;
    if (!mbar_wait(&full[st], (uint32_t)((gi / kStages) & 1))) set_error(p.err, ABKV_DEVERR_TIMEOUT);
    const int t = tile0 + gi * nsub + sub;
    if (t < tile1) {
      bool ok;
      tile_page(t, ok);
      const int tok0 = t * kTile;
      const uint8_t* kb = smem + (size_t)st * kStageBytes + (size_t)sub * 2 * tile_half + h * kD * 2;
      const uint8_t* vb = kb + tile_half;

      // S = Q.K^T : rows = query heads (g < G real), cols = tokens 8nt + 2c + {0,1}
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int T = 8 * nt + g;
        const bool valid = ok && (tok0 + T < seq_len);
        uint32_t kr[4][4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (valid) v = lds128(kb + T * row_bytes + (32 * m + 8 * c) * 2);
          kr[m][0] = v.x; kr[m][1] = v.y; kr[m][2] = v.z; kr[m][3] = v.w;
        }
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          mma_bf16_16816(s[nt], qr[m][0], 0u, qr[m][1], 0u, kr[m][0], kr[m][1]);
          mma_bf16_16816(s[nt], qr[m][2], 0u, qr[m][3], 0u, kr[m][2], kr[m][3]);
        }
      }

      // online softmax (base-2, scale folded in)
      float x[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const bool valid = ok && (tok0 + 8 * nt + 2 * c + j < seq_len);
          x[nt][j] = valid ? s[nt][j] * sl2 : -INFINITY;
        }
      float tmax = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
      const float m_new = fmaxf(m_run, tmax);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(m_run - m_use);
      float pr[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) pr[nt][j] = exp2f(x[nt][j] - m_use);
      l_run = l_run * alpha + ((pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]));
      m_run = m_new;

      // O^T columns held by this lane are heads 2c and 2c+1
      const float a0 = __shfl_sync(0xffffffffu, alpha, 8 * c);
      const float a1 = __shfl_sync(0xffffffffu, alpha, 8 * c + 4);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= a0; o[mt][1] *= a1; o[mt][2] *= a0; o[mt][3] *= a1;
      }
      const uint32_t pb0 = pack_bf16x2(pr[0][0], pr[0][1]);
      const uint32_t pb1 = pack_bf16x2(pr[1][0], pr[1][1]);

      // V rows 2c, 2c+1, 2c+8, 2c+9 (zero when masked: 0 * NaN would poison O)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t vr[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int T = 2 * c + (i & 1) + 8 * (i >> 1);
          uint4 v = make_uint4(0, 0, 0, 0);
          if (ok && (tok0 + T < seq_len)) v = lds128(vb + T * row_bytes + (64 * hh + 8 * g) * 2);
          vr[i][0] = v.x; vr[i][1] = v.y; vr[i][2] = v.z; vr[i][3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int mt = 4 * hh + i;
          const uint32_t v0 = vr[0][i], v1 = vr[1][i], v2 = vr[2][i], v3 = vr[3][i];
          mma_bf16_16816(o[mt], prmt(v0, v1, 0x5410u), prmt(v0, v1, 0x7632u), prmt(v2, v3, 0x5410u),
                         prmt(v2, v3, 0x7632u), pb0, pb1);
        }
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (threadIdx.x == 0 && gi + kStages < ngroups) issue(gi + kStages);
  }

  // epilogue arrays alias the (now idle) stage buffers
  float (*s_o)[kMaxG][kD] = reinterpret_cast<float (*)[kMaxG][kD]>(smem);
  float (*s_m)[kMaxG] = reinterpret_cast<float (*)[kMaxG]>(smem + sizeof(float) * kWarps * kMaxG * kD);
  float (*s_l)[kMaxG] = s_m + kWarps;

  // ---- epilogue: per-warp partials -> shared memory -> merged output -----
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
#pragma unroll
  for (int jh = 0; jh < 2; ++jh) {
    const int head = 2 * c + jh;
    if (head < G) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int hh = mt >> 2, i = mt & 3;
        const int d = 8 * g + 64 * hh + 2 * i;
        s_o[warp][head][d] = o[mt][jh];
        s_o[warp][head][d + 1] = o[mt][2 + jh];
      }
    }
  }
  if (c == 0 && g < G) {
    s_m[warp][g] = m_run;
    s_l[warp][g] = l_run;
  }
  __syncthreads();

  const int items = p.Hq * kD;
  const int64_t lb = (int64_t)(p.layer_base + li) * p.B + b;  // (layer, sequence) slot
  const int64_t prow = (lb * p.max_chunks + chunk) * p.Hq;
  for (int it = threadIdx.x; it < items; it += kThreads) {
    const int d = it % kD, hr = it / kD;
    const int kh = hr / G, r = hr % G;
    float M = -INFINITY;
    for (int s2 = 0; s2 < nsub; ++s2) M = fmaxf(M, s_m[s2 * Hkv + kh][r]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float Ls = 0.f, Os = 0.f;
    for (int s2 = 0; s2 < nsub; ++s2) {
      const int w = s2 * Hkv + kh;
      const float f = exp2f(s_m[w][r] - Mu);
      Ls += s_l[w][r] * f;
      Os += s_o[w][r][d] * f;
    }
    const float val = Ls > 0.f ? Os / Ls : 0.f;
    if (n_chunks == 1) {
      L.out[((int64_t)b * p.Hq + hr) * kD + d] = __float2bfloat16(val);
    } else {
      p.part_o[(prow + hr) * kD + d] = val;
      if (d == 0) p.part_lse[prow + hr] = Ls > 0.f ? Mu + log2f(Ls) : -INFINITY;
    }
  }
  if (n_chunks == 1) return;

  // ---- split-KV merge: the last chunk CTA of this (layer, sequence) combines
  // every chunk's partial with log-sum-exp weights and resets the counter.
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.counters + lb, 1);
    s_last = (prev == n_chunks - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int64_t row0 = lb * p.max_chunks * p.Hq;
  for (int it = threadIdx.x; it < items; it += kThreads) {
    const int d = it % kD, hr = it / kD;
    float M = -INFINITY;
    for (int ch = 0; ch < n_chunks; ++ch) M = fmaxf(M, __ldcg(p.part_lse + row0 + (int64_t)ch * p.Hq + hr));
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float Ls = 0.f, Os = 0.f;
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int64_t rr = row0 + (int64_t)ch * p.Hq + hr;
      const float f = exp2f(__ldcg(p.part_lse + rr) - Mu);
      Ls += f;
      Os += f * __ldcg(p.part_o + rr * kD + d);
    }
    L.out[((int64_t)b * p.Hq + hr) * kD + d] = __float2bfloat16(Ls > 0.f ? Os / Ls : 0.f);
  }
  if (threadIdx.x == 0) p.counters[lb] = 0;  // ready for the next call on this workspace
}

int auto_chunk_tiles(int num_layers, int num_seqs, int max_tiles, int page_tiles) {
  // Aim for >= ~8 waves of two CTAs on 148 SMs, with chunks of 32..128 tiles.
  const int64_t total = (int64_t)num_layers * num_seqs * max_tiles;
  int ct = 128;
  while (ct > 32 && total / ct < 148 * 2 * 8) ct >>= 1;
  if (ct < page_tiles) ct = page_tiles;
  ct = (ct / page_tiles) * page_tiles;
  return ct;
}

struct DecodePlan {
  int chunk_tiles, max_chunks, max_tiles;
  size_t counter_bytes, part_o_bytes, part_lse_bytes, total;
};

constexpr size_t kWsHeader = 256;

int plan_decode(int num_layers, int num_seqs, int num_q_heads, int head_dim, int page_size,
                int max_pages, int chunk_tokens, DecodePlan* plan) {
  if (num_layers <= 0 || num_seqs <= 0 || num_q_heads <= 0 || page_size <= 0 || max_pages <= 0)
    return ABKV_ERR_INVALID_ARG;
  if (head_dim != kD || page_size % kTile != 0) return ABKV_ERR_UNSUPPORTED;
  const int page_tiles = page_size / kTile;
  const int64_t max_tiles = (int64_t)max_pages * page_tiles;
  if (max_tiles > (1 << 26)) return ABKV_ERR_UNSUPPORTED;
  int ct;
  if (chunk_tokens == 0) {
    ct = auto_chunk_tiles(num_layers, num_seqs, (int)max_tiles, page_tiles);
  } else {
    if (chunk_tokens < 0 || chunk_tokens % kTile || chunk_tokens % page_size) return ABKV_ERR_INVALID_ARG;
    ct = chunk_tokens / kTile;
  }
  if (ct * kTile / page_size > kMaxChunkPages - 1) return ABKV_ERR_UNSUPPORTED;
  plan->chunk_tiles = ct;
  plan->max_tiles = (int)max_tiles;
  plan->max_chunks = (int)((max_tiles + ct - 1) / ct);
  if (plan->max_chunks > 1) {
    const size_t rows = (size_t)num_layers * num_seqs * plan->max_chunks * num_q_heads;
    plan->counter_bytes = ((size_t)num_layers * num_seqs * sizeof(int32_t) + 255) / 256 * 256;
    plan->part_o_bytes = rows * kD * sizeof(float);
    plan->part_lse_bytes = ((rows * sizeof(float)) + 255) / 256 * 256;
  } else {
    plan->counter_bytes = plan->part_o_bytes = plan->part_lse_bytes = 0;
  }
  plan->total = kWsHeader + plan->counter_bytes + plan->part_lse_bytes + plan->part_o_bytes;
  return ABKV_OK;
}

}  // namespace
}  // namespace abkv

using namespace abkv;

extern "C" size_t abkv_decode_workspace_size(int num_layers, int num_seqs, int num_q_heads,
                                             int head_dim, int page_size, int max_pages_per_seq,
                                             int chunk_tokens) {
  DecodePlan plan;
  if (plan_decode(num_layers, num_seqs, num_q_heads, head_dim, page_size, max_pages_per_seq,
                  chunk_tokens, &plan) != ABKV_OK)
    return 0;
  return plan.total;
}

extern "C" int abkv_decode(const void* const* q, const void* const* kv,
                           const int32_t* const* block_tables, const int64_t* bt_strides,
                           const int32_t* const* seq_lens, const int64_t* num_blocks,
                           void* const* out, int num_layers, int num_seqs, int num_q_heads,
                           int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
                           float scale, int chunk_tokens, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (!q || !kv || !block_tables || !bt_strides || !seq_lens || !num_blocks || !out)
    return ABKV_ERR_INVALID_ARG;
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return ABKV_ERR_INVALID_ARG;
  if (kWarps % num_kv_heads != 0) return ABKV_ERR_UNSUPPORTED;
  const int G = num_q_heads / num_kv_heads;
  if (G > kMaxG) return ABKV_ERR_UNSUPPORTED;
  if (num_seqs > 65535) return ABKV_ERR_UNSUPPORTED;
  if (!(scale > 0.f)) return ABKV_ERR_INVALID_ARG;
  DecodePlan plan;
  int st = plan_decode(num_layers, num_seqs, num_q_heads, head_dim, page_size, max_pages_per_seq,
                       chunk_tokens, &plan);
  if (st != ABKV_OK) return st;
  if (!workspace || workspace_bytes < plan.total) return ABKV_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return ABKV_ERR_WORKSPACE;
  for (int l = 0; l < num_layers; ++l) {
    if (!q[l] || !kv[l] || !block_tables[l] || !seq_lens[l] || !out[l]) return ABKV_ERR_INVALID_ARG;
    if (bt_strides[l] <= 0 || num_blocks[l] <= 0) return ABKV_ERR_INVALID_ARG;
    // 16-byte vector loads of q / kv rows need 16-byte aligned bases.
    if ((reinterpret_cast<uintptr_t>(q[l]) | reinterpret_cast<uintptr_t>(kv[l])) & 15)
      return ABKV_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(block_tables[l]) & 3) return ABKV_ERR_INVALID_ARG;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  // opt in to > 48 KiB of dynamic shared memory (idempotent, per device)
  if (cudaFuncSetAttribute(decode_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kSmemBytes) != cudaSuccess)
    return ABKV_ERR_CUDA;

  DecodeParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.err = reinterpret_cast<int32_t*>(ws);
  const bool split = plan.max_chunks > 1;
  prm.counters = split ? reinterpret_cast<int32_t*>(ws + kWsHeader) : nullptr;
  prm.part_lse = split ? reinterpret_cast<float*>(ws + kWsHeader + plan.counter_bytes) : nullptr;
  prm.part_o = split ? reinterpret_cast<float*>(ws + kWsHeader + plan.counter_bytes +
                                                plan.part_lse_bytes)
                     : nullptr;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.B = num_seqs;
  prm.Hq = num_q_heads;
  prm.Hkv = num_kv_heads;
  prm.G = G;
  prm.P = page_size;
  prm.chunk_tiles = plan.chunk_tiles;
  prm.max_chunks = plan.max_chunks;
  prm.max_rows = plan.max_tiles * kTile;

  for (int l0 = 0; l0 < num_layers; l0 += kMaxLayers) {
    const int nl = (num_layers - l0) < kMaxLayers ? (num_layers - l0) : kMaxLayers;
    for (int i = 0; i < nl; ++i) {
      LayerArgs& a = prm.layer[i];
      a.q = static_cast<const __nv_bfloat16*>(q[l0 + i]);
      a.kv = static_cast<const __nv_bfloat16*>(kv[l0 + i]);
      a.bt = block_tables[l0 + i];
      a.seq_lens = seq_lens[l0 + i];
      a.out = static_cast<__nv_bfloat16*>(out[l0 + i]);
      a.bt_stride = bt_strides[l0 + i];
      a.num_blocks = num_blocks[l0 + i];
    }
    prm.layer_base = l0;
    dim3 grid(plan.max_chunks, num_seqs, nl);
    decode_split_kernel<<<grid, kThreads, kSmemBytes, s>>>(prm);
  }
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}
