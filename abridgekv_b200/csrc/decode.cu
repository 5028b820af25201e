// Split-KV, GQA-packed paged decode attention for sm_100a.
//
// Semantics follow the reference's batched PyTorch decode
//   third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:564-616
// (scores = q.K^T * scale over the first seq_len physical rows of the request's
// block table, fp32 softmax, weights rounded to bf16, weighted sum of V), which
// is the PyTorch image of the FlashInfer decode the vLLM overlay runs per KV
// cache group (gpu_model_runner.py:1672-1681, 2184-2204).
//
// Structure: a persistent kernel, one CTA per SM (8 consumer warps + 1
// producer warp).  Work items are (split-KV chunk, layer, sequence); the
// producer takes them from a global atomic counter (chunk-major order, empty
// chunks skipped), stages each item's page ids in shared memory and streams
// "tile groups" into a 3-stage shared-memory ring with bulk copies
// (cp.async.bulk on the TMA engine, no multicast) completed on full/empty
// mbarriers, running ahead across item boundaries.  A tile is 16 cache rows;
// a group holds one tile per consumer-warp slot (K rows then V rows, all KV
// heads: 64 KiB for head_dim 128).  Consumer warp w handles KV head w % Hkv
// (with fewer than 8 KV heads, warps of one head take different tiles of a
// group and are merged at the end of the item).  Per tile a warp
//   * reads K rows g and g+8 (g = lane/4) and V rows 2c,2c+1,2c+8,2c+9
//     (c = lane%4) from shared memory in mma fragment order (dims permuted
//     consistently between Q and K, and between V and the output);
//   * S = Q.K^T with mma.m16n8k16 (rows = the G query heads of the KV head);
//   * online softmax in fp32 (quad shuffles), P rounded to bf16 as the
//     reference does before its P.V product;
//   * O^T += V^T.P^T with mma.m16n8k16: the S accumulator fragment is exactly
//     the B fragment of this product, so P never leaves registers.
// At the end of an item the consumers merge warp partials in shared memory
// (named barrier 1, consumers only); single-chunk rows are written directly,
// otherwise each chunk stores a normalised partial + log-sum-exp and the last
// chunk to finish for its (layer, sequence) (a counter in the workspace,
// reset by that chunk) combines them.  The last CTA to run out of work resets
// the work counters; the host clears the chunk counters before each call (a
// call with another plan may find the previous call's partials there), so a
// workspace is ready for any later call on the same stream; concurrent calls
// must not share a workspace.  Every mbarrier wait is bounded.
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace abkv {
namespace {

constexpr int kD = 128;  // largest head_dim (64 and 128 are compiled); buffers are sized for it
constexpr int kTile = 16;
constexpr int kWarps = 8;                  // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + producer warp
constexpr int kConsumerThreads = kWarps * 32;
constexpr int kMaxLayers = 56;       // layers per launch (plain parameters < 4 KB, with sidecars ~9.6 KB)
constexpr int kMaxChunkPages = 512;  // page ids staged per work item
constexpr int kMaxG = 8;             // query heads per KV head
constexpr int kStages = 3;
constexpr int kStageBytes = kWarps * 2 * kTile * kD * 2;  // nsub * Hkv == kWarps -> 64 KiB

struct LayerArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  const int32_t* bt;
  const int32_t* seq_lens;
  __nv_bfloat16* out;
  int64_t bt_stride;
  int64_t num_blocks;
};

// Packed sidecar of per-head code quotas of one layer (null pages = none): page i
// of a request holds, for KV head h, slots [off[h], off[h] + q[h]) of a
// [2][slots][D] page; a head's keys are its slots of every sidecar page of the
// request (in page order), then the main rows.
struct SideArgs {
  const __nv_bfloat16* pages;
  const int32_t* bt;     // [B][bt_stride] page ids into `pages`
  const int32_t* count;  // [B] sidecar pages of each request
  int64_t bt_stride, num_pages;
  int slots;
  int off[kWarps], q[kWarps];
};

// Output placement.  Row (b, h) of a layer goes to out + b * out_row + (head0 + h) * D
// in every rank's copy of the output buffer: world == 1 is the plain decode
// ([B][Hq][D], head0 0); world > 1 is the KV-head-sharded decode whose epilogue
// is also the all-gather -- each rank stores its heads straight into all ranks'
// buffers (peer memory over NVLink), then the last CTA raises this rank's flag
// in every peer's flag array and waits (bounded) until all peers' flags for
// this epoch are up in its own.
constexpr int kMaxPeers = 8;
struct GatherArgs {
  int64_t peer_delta[kMaxPeers];  // element offset from this rank's buffer to rank r's
  uint32_t* peer_flags[kMaxPeers];
  uint32_t* my_flags;
  int64_t out_row;
  uint64_t timeout_ns;
  int world, rank, head0;
  uint32_t epoch;
};

struct DecodeParams {
  LayerArgs layer[kMaxLayers];
  GatherArgs gather;
  float* part_o;      // [layers][B][max_chunks][Hq][D]
  float* part_lse;    // [layers][B][max_chunks][Hq]
  int32_t* counters;  // [layers][B] (CTA epilogue) or [layers][B][Hkv] (warp epilogue) chunks
                      // finished; cleared by the host before each call
  int32_t* work;      // [2]: next item, CTAs done; zero between calls
  int32_t* err;
  float scale_log2;
  int B, Hq, Hkv, G, P;
  int chunk_tiles, max_chunks, max_rows;
  int layer_base, nl;
  int num_items;
  int warp_epi;  // 1: per-warp epilogue (one consumer warp per KV head, 16-byte aligned outputs)
  static constexpr bool kHasSide = false;
};

// Parameters of the packed-sidecar decode.  The plain decode is compiled from
// the same templates with DecodeParams, so it carries neither the sidecar
// parameters nor the sidecar branches.
struct SideDecodeParams : DecodeParams {
  SideArgs side[kMaxLayers];
  static constexpr bool kHasSide = true;
};

// A group is either main tiles (16 rows x all KV heads; ok bit per tile, warp w
// takes head w % Hkv of tile w / Hkv) or sidecar tiles of ONE KV head (the
// item's head, bits 11..13): warp w takes tile w (16 slots); seq_len holds the
// request's sidecar page count.
struct StageMeta {
  int li, b, chunk, n_chunks, seq_len, t0, ntiles, bits;  // bits: ok mask | kFirst | kLast | kSide
};
constexpr int kFirst = 1 << 8;
constexpr int kLast = 1 << 9;
constexpr int kSide = 1 << 10;
constexpr int kSideHeadShift = 11;

// Dynamic shared memory layout.
constexpr size_t kOffStage = 0;
constexpr size_t kOffO = kOffStage + (size_t)kStages * kStageBytes;        // float[8][8][128]
constexpr size_t kOffML = kOffO + sizeof(float) * kWarps * kMaxG * kD;     // float[2][8][8]
constexpr size_t kOffMeta = kOffML + sizeof(float) * 2 * kWarps * kMaxG;   // StageMeta[kStages]
constexpr size_t kOffPages = kOffMeta + sizeof(StageMeta) * kStages;       // int32[kMaxChunkPages]
constexpr size_t kOffBar = kOffPages + sizeof(int32_t) * kMaxChunkPages;   // u64 full[3], empty[3]
constexpr size_t kOffFlag = kOffBar + sizeof(uint64_t) * 2 * kStages;
constexpr size_t kSmemBytes = kOffFlag + 16;

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

__device__ __forceinline__ int clamp_side_count(const DecodeParams& p, const SideArgs& S, int b, bool report) {
  int c = __ldg(S.count + b);
  if (c < 0 || (int64_t)c > S.bt_stride) {
    if (report) set_error(p.err, ABKV_DEVERR_SEQ_OOB);
    c = c < 0 ? 0 : (int)S.bt_stride;
  }
  return c;
}

__device__ __forceinline__ uint4 lds128(const void* ptr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(smem_u32(ptr)));
  return r;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumerThreads) : "memory");
}

template <int D, bool kGather>
__device__ __forceinline__ void store_out(const DecodeParams& p, const LayerArgs& L, int b, int hr, int d,
                                          float val) {
  const __nv_bfloat16 v = __float2bfloat16(val);
  if constexpr (kGather) {
    const GatherArgs& g = p.gather;
    __nv_bfloat16* dst = L.out + (int64_t)b * g.out_row + (int64_t)(g.head0 + hr) * D + d;
    for (int r = 0; r < g.world; ++r) dst[g.peer_delta[r]] = v;
  } else {
    L.out[((int64_t)b * p.Hq + hr) * D + d] = v;
  }
}

// Eight consecutive dims [d0, d0 + 8) of row (b, hr) as one 16-byte store (per rank when gathering).
template <int D, bool kGather>
__device__ __forceinline__ void store_out8(const DecodeParams& p, const LayerArgs& L, int b, int hr, int d0,
                                           const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  if constexpr (kGather) {
    const GatherArgs& g = p.gather;
    __nv_bfloat16* dst = L.out + (int64_t)b * g.out_row + (int64_t)(g.head0 + hr) * D + d0;
    for (int r = 0; r < g.world; ++r) *reinterpret_cast<uint4*>(dst + g.peer_delta[r]) = u;
  } else {
    *reinterpret_cast<uint4*>(L.out + ((int64_t)b * p.Hq + hr) * D + d0) = u;
  }
}

// Chunk count of a (layer, sequence[, KV head]): the release publishes this
// warp's partial stores (ordered before it by __syncwarp), the acquire makes the
// other chunks' partials visible to the warp that sees the final count.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t* ptr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;\n" : "=r"(old) : "l"(ptr), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void st_release_sys(uint32_t* ptr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// End of a gathering launch: every CTA's output stores are fenced system-wide
// before it is counted; the last CTA publishes this rank's epoch to all ranks
// and waits for theirs.  The wait gives up after timeout_ns (or kPeerSpinLimit
// polls, whichever comes first) and records ABKV_DEVERR_TIMEOUT, so a missing
// peer cannot hang the GPU.
constexpr uint32_t kPeerSpinLimit = 1u << 26;
__device__ void gather_barrier(const DecodeParams& p) {
  const GatherArgs& g = p.gather;
  __threadfence_system();
  const int prev = atomicAdd(p.work + 2, 1);
  if (prev != (int)gridDim.x - 1) return;
  p.work[2] = 0;  // ready for the next launch on this workspace
  __threadfence_system();
  for (int r = 0; r < g.world; ++r) st_release_sys(g.peer_flags[r] + g.rank, g.epoch);
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < g.world; ++r) {
    uint32_t i = 0;
    while ((int32_t)(ld_acquire_sys(g.my_flags + r) - g.epoch) < 0) {
      if (++i >= kPeerSpinLimit || globaltimer_ns() - t0 > g.timeout_ns) {
        set_error(p.err, ABKV_DEVERR_TIMEOUT);
        return;
      }
      __nanosleep(128);
    }
  }
}

// ---------------------------------------------------------------------------
template <int D, class Prm>
__device__ void producer(const Prm& p, uint8_t* smem) {
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + kOffMeta);
  int32_t* s_pages = reinterpret_cast<int32_t*>(smem + kOffPages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  const int lane = threadIdx.x & 31;
  const int Hkv = p.Hkv, P = p.P, nsub = kWarps / Hkv;
  const int tile_half = kTile * Hkv * D * 2;
  const int64_t row_elems = (int64_t)Hkv * D;
  const int64_t half_elems = (int64_t)P * row_elems;
  const int64_t page_elems = 2 * half_elems;
  const int lb_items = p.nl * p.B;
  int gq = 0;  // groups issued by this CTA
  bool alive = true;

  while (alive) {
    int li = -1, b = 0, chunk = 0, nch = 0, slen = 0, nside = 0, scount = 0;
    if (lane == 0) {
      for (;;) {
        const int i = atomicAdd(p.work, 1);
        if (i >= p.num_items) break;
        chunk = i / lb_items;
        const int rem = i - chunk * lb_items;
        li = rem / p.B;
        b = rem - li * p.B;
        slen = clamp_seq_len(p, p.layer[li], b, chunk == 0);
        // chunks [0, nside) cover the sidecar rows, head after head; the rest the main rows
        const int ntl = (slen + kTile - 1) / kTile;
        if constexpr (Prm::kHasSide) {
          const SideArgs& S = p.side[li];
          nside = scount = 0;
          if (S.pages) {
            scount = clamp_side_count(p, S, b, chunk == 0);
            for (int hh = 0; hh < Hkv; ++hh)
              nside += ((scount * S.q[hh] + kTile - 1) / kTile + p.chunk_tiles - 1) / p.chunk_tiles;
          }
        }
        nch = max(1, nside + (ntl + p.chunk_tiles - 1) / p.chunk_tiles);
        if (chunk < nch) break;
        li = -1;
      }
    }
    li = __shfl_sync(0xffffffffu, li, 0);
    if (li < 0) break;
    b = __shfl_sync(0xffffffffu, b, 0);
    chunk = __shfl_sync(0xffffffffu, chunk, 0);
    nch = __shfl_sync(0xffffffffu, nch, 0);
    slen = __shfl_sync(0xffffffffu, slen, 0);
    const LayerArgs& L = p.layer[li];
    if constexpr (Prm::kHasSide) {
      nside = __shfl_sync(0xffffffffu, nside, 0);
      scount = __shfl_sync(0xffffffffu, scount, 0);
      if (chunk < nside) {
        const SideArgs& S = p.side[li];
        // ---- sidecar item: tiles of one KV head; lane i < kWarps owns tile i of a group (16
        // consecutive slots of the head; quotas are multiples of 16, so they lie in one page)
        int hs = 0, c0 = 0, stl = 0;
        for (;; ++hs) {
          stl = (scount * S.q[hs] + kTile - 1) / kTile;
          const int nc = (stl + p.chunk_tiles - 1) / p.chunk_tiles;
          if (chunk < c0 + nc || hs == Hkv - 1) break;
          c0 += nc;
        }
        const int qh = S.q[hs];
        const int tile0 = (chunk - c0) * p.chunk_tiles;
        const int tile1 = min(tile0 + p.chunk_tiles, stl);
        const int ntiles = max(0, tile1 - tile0);
        const int ngroups = max(1, (ntiles + kWarps - 1) / kWarps);
        const int head_tile = kTile * D * 2;
        for (int grp = 0; grp < ngroups; ++grp, ++gq) {
          const int st = gq % kStages;
          const int tg0 = tile0 + grp * kWarps;
          const int nt = max(0, min(kWarps, tile1 - tg0));
          int64_t src = -1;
          if (lane < nt) {
            const int row0 = (tg0 + lane) * kTile;
            const int64_t pid = __ldg(S.bt + (int64_t)b * S.bt_stride + row0 / qh);
            if (pid >= 0 && pid < S.num_pages) {
              src = (pid * 2 * S.slots + S.off[hs] + row0 % qh) * D;
            } else {
              set_error(p.err, ABKV_DEVERR_PAGE_OOB);
            }
          }
          const uint32_t okmask = __ballot_sync(0xffffffffu, src >= 0) & ((1u << nt) - 1u);
          if (lane == 0) {
            const uint32_t k = (uint32_t)(gq / kStages);
            if (!mbar_wait(&empty[st], (k & 1u) ^ 1u)) {
              set_error(p.err, ABKV_DEVERR_TIMEOUT);
              alive = false;
            }
          }
          alive = __shfl_sync(0xffffffffu, alive ? 1 : 0, 0) != 0;
          if (!alive) break;
          if (lane == 0) {
            StageMeta m;
            m.li = li; m.b = b; m.chunk = chunk; m.n_chunks = nch; m.seq_len = scount;
            m.t0 = tg0; m.ntiles = nt;
            m.bits = (int)okmask | kSide | (hs << kSideHeadShift) | (grp == 0 ? kFirst : 0) |
                     (grp == ngroups - 1 ? kLast : 0);
            meta[st] = m;
            mbar_expect_tx(&full[st], (uint32_t)__popc(okmask) * 2u * (uint32_t)head_tile);
          }
          __syncwarp();  // the expected byte count is posted before any copy can complete
          if (src >= 0) {
            uint8_t* dst = smem + kOffStage + (size_t)st * kStageBytes + (size_t)lane * 2 * head_tile;
            bulk_g2s(dst, S.pages + src, (uint32_t)head_tile, &full[st]);
            bulk_g2s(dst + head_tile, S.pages + src + (int64_t)S.slots * D, (uint32_t)head_tile, &full[st]);
          }
        }
        continue;
      }
    }
    // ---- main item: tiles of 16 rows x all KV heads through the block table
    const int ntl = (slen + kTile - 1) / kTile;
    const int tile0 = (chunk - nside) * p.chunk_tiles;
    const int tile1 = min(tile0 + p.chunk_tiles, ntl);
    const int ntiles = max(0, tile1 - tile0);
    const int page0 = tile0 * kTile / P;
    const int npages = ntiles ? (tile1 * kTile + P - 1) / P - page0 : 0;
    const int32_t* bt = L.bt + (int64_t)b * L.bt_stride + page0;
    for (int i = lane; i < npages; i += 32) s_pages[i] = __ldg(bt + i);
    __syncwarp();
    const int ngroups = max(1, (ntiles + nsub - 1) / nsub);
    for (int grp = 0; grp < ngroups; ++grp, ++gq) {
      // lane j < nt owns tile j of the group: its page lookup, bounds check and
      // copies run in parallel across the lanes (one tile's latency per group)
      const int st = gq % kStages;
      const int tg0 = tile0 + grp * nsub;
      const int nt = max(0, min(nsub, tile1 - tg0));
      int64_t pg = -1;
      if (lane < nt) {
        const int t = tg0 + lane;
        pg = s_pages[(P == kTile ? t : t * kTile / P) - page0];
        if (pg < 0 || pg >= L.num_blocks) {
          set_error(p.err, ABKV_DEVERR_PAGE_OOB);
          pg = -1;
        }
      }
      const uint32_t okmask = __ballot_sync(0xffffffffu, pg >= 0) & ((1u << nt) - 1u);
      if (lane == 0) {
        const uint32_t k = (uint32_t)(gq / kStages);
        if (!mbar_wait(&empty[st], (k & 1u) ^ 1u)) {
          set_error(p.err, ABKV_DEVERR_TIMEOUT);
          alive = false;
        }
      }
      alive = __shfl_sync(0xffffffffu, alive ? 1 : 0, 0) != 0;
      if (!alive) break;
      if (lane == 0) {
        StageMeta m;
        m.li = li; m.b = b; m.chunk = chunk; m.n_chunks = nch; m.seq_len = slen;
        m.t0 = tg0; m.ntiles = nt;
        m.bits = (int)okmask | (grp == 0 ? kFirst : 0) | (grp == ngroups - 1 ? kLast : 0);
        meta[st] = m;
        // release: meta is visible once the phase completes
        mbar_expect_tx(&full[st], (uint32_t)__popc(okmask) * 2u * (uint32_t)tile_half);
      }
      __syncwarp();  // the expected byte count is posted before any copy can complete
      if (pg >= 0) {
        const int t = tg0 + lane;
        uint8_t* dst = smem + kOffStage + (size_t)st * kStageBytes + (size_t)lane * 2 * tile_half;
        const __nv_bfloat16* ksrc = L.kv + pg * page_elems + (int64_t)((t * kTile) % P) * row_elems;
        bulk_g2s(dst, ksrc, (uint32_t)tile_half, &full[st]);
        bulk_g2s(dst + tile_half, ksrc + half_elems, (uint32_t)tile_half, &full[st]);
      }
    }
    __syncwarp();  // s_pages is rewritten for the next item only after this one is issued
  }
  if (lane == 0) {
    // end-of-work marker for the consumers
    const int st = gq % kStages;
    const uint32_t k = (uint32_t)(gq / kStages);
    if (!mbar_wait(&empty[st], (k & 1u) ^ 1u)) set_error(p.err, ABKV_DEVERR_TIMEOUT);
    meta[st].li = -1;
    mbar_expect_tx(&full[st], 0u);
    // the last CTA to run out of work resets the work counters for the next call
    __threadfence();
    const int prev = atomicAdd(p.work + 1, 1);
    if (prev == (int)gridDim.x - 1) {
      p.work[0] = 0;
      p.work[1] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// End of an item when each consumer warp owns one KV head (8 KV heads): the
// warp's registers hold the item's complete result for its G query heads, so it
// writes the output rows (single-chunk items) or its partial rows + log-sum-exp
// itself, counts the chunk for (layer, sequence, KV head) and, if it finished
// the last one, combines that head's chunk partials -- no shared memory, no CTA
// barrier, so the other warps keep consuming stages meanwhile.  Lane (g, c)
// holds dims [8g, 8g + 8) + 64 hh of query heads 2c and 2c + 1 (o[4 hh + i][jh]
// = dim 8g + 64 hh + 2i, o[4 hh + i][2 + jh] = the next dim); the row statistics
// of query head r sit in lanes 4r..4r+3.  Arithmetic as the shared-memory merge
// (one warp: weight exp2(0) = 1) and combine, so both epilogues give the same bits.
template <int D, bool kGather>
__device__ __forceinline__ void warp_epilogue(const DecodeParams& p, const LayerArgs& L, const StageMeta& M, int h,
                                              int lane, const float (&o)[D / 16][4], float m_run, float l_run) {
  constexpr int kVH = D / 64;
  const int g = lane >> 2, c = lane & 3, G = p.G;
  float lq = l_run;
  lq += __shfl_xor_sync(0xffffffffu, lq, 1);
  lq += __shfl_xor_sync(0xffffffffu, lq, 2);
  float mh[2], lh[2];
  mh[0] = __shfl_sync(0xffffffffu, m_run, 8 * c);
  mh[1] = __shfl_sync(0xffffffffu, m_run, 8 * c + 4);
  lh[0] = __shfl_sync(0xffffffffu, lq, 8 * c);
  lh[1] = __shfl_sync(0xffffffffu, lq, 8 * c + 4);
  const int n_chunks = M.n_chunks;
  const int64_t lb = (int64_t)(p.layer_base + M.li) * p.B + M.b;
  if (n_chunks == 1) {
#pragma unroll
    for (int jh = 0; jh < 2; ++jh) {
      const int head = 2 * c + jh;
      if (head >= G) continue;
      const float Ls = lh[jh];
#pragma unroll
      for (int hh = 0; hh < kVH; ++hh) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[2 * i] = Ls > 0.f ? o[4 * hh + i][jh] / Ls : 0.f;
          v[2 * i + 1] = Ls > 0.f ? o[4 * hh + i][2 + jh] / Ls : 0.f;
        }
        store_out8<D, kGather>(p, L, M.b, h * G + head, 64 * hh + 8 * g, v);
      }
    }
    return;
  }
  const int64_t prow = (lb * p.max_chunks + M.chunk) * p.Hq;
#pragma unroll
  for (int jh = 0; jh < 2; ++jh) {
    const int head = 2 * c + jh;
    if (head >= G) continue;
    const int hr = h * G + head;
    const float Ls = lh[jh];
#pragma unroll
    for (int hh = 0; hh < kVH; ++hh) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = Ls > 0.f ? o[4 * hh + i][jh] / Ls : 0.f;
        v[2 * i + 1] = Ls > 0.f ? o[4 * hh + i][2 + jh] / Ls : 0.f;
      }
      float4* dst = reinterpret_cast<float4*>(p.part_o + (prow + hr) * D + 64 * hh + 8 * g);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (g == 0) p.part_lse[prow + hr] = Ls > 0.f ? mh[jh] + log2f(Ls) : -INFINITY;
  }
  __syncwarp();
  int prev = 0;
  int32_t* counter = p.counters + lb * p.Hkv + h;
  if (lane == 0) prev = atom_add_acq_rel_gpu(counter, 1);
  __syncwarp();
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev != n_chunks - 1) return;
  if (lane == 0) *counter = 0;  // ready for the next call on this workspace
  const int64_t row0 = lb * p.max_chunks * p.Hq;
#pragma unroll
  for (int jh = 0; jh < 2; ++jh) {
    const int head = 2 * c + jh;
    if (head >= G) continue;
    const int hr = h * G + head;
    float Mx = -INFINITY;
    for (int ch = 0; ch < n_chunks; ++ch) Mx = fmaxf(Mx, __ldcg(p.part_lse + row0 + (int64_t)ch * p.Hq + hr));
    const float Mu = (Mx == -INFINITY) ? 0.f : Mx;
    float Ls = 0.f, acc[kVH][8];
#pragma unroll
    for (int hh = 0; hh < kVH; ++hh)
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[hh][k] = 0.f;
#pragma unroll 2
    for (int ch = 0; ch < n_chunks; ++ch) {
      const int64_t rr = row0 + (int64_t)ch * p.Hq + hr;
      const float f = exp2f(__ldcg(p.part_lse + rr) - Mu);
      Ls += f;
#pragma unroll
      for (int hh = 0; hh < kVH; ++hh) {
        const float4* src = reinterpret_cast<const float4*>(p.part_o + rr * D + 64 * hh + 8 * g);
        const float4 a = __ldcg(src), bq = __ldcg(src + 1);
        acc[hh][0] += f * a.x; acc[hh][1] += f * a.y; acc[hh][2] += f * a.z; acc[hh][3] += f * a.w;
        acc[hh][4] += f * bq.x; acc[hh][5] += f * bq.y; acc[hh][6] += f * bq.z; acc[hh][7] += f * bq.w;
      }
    }
#pragma unroll
    for (int hh = 0; hh < kVH; ++hh) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = Ls > 0.f ? acc[hh][k] / Ls : 0.f;
      store_out8<D, kGather>(p, L, M.b, hr, 64 * hh + 8 * g, v);
    }
  }
}

// ---------------------------------------------------------------------------
// D = head_dim: the Q.K^T product runs over D / 32 chunks of 32 dims (8 per lane),
// P.V over D / 64 halves of 64 dims, O^T in D / 16 accumulator tiles.
template <int D, class Prm, bool kGather>
__device__ void consumer(const Prm& p, uint8_t* smem) {
  const StageMeta* meta = reinterpret_cast<const StageMeta*>(smem + kOffMeta);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  float (*s_o)[kMaxG][kD] = reinterpret_cast<float (*)[kMaxG][kD]>(smem + kOffO);
  float (*s_m)[kMaxG] = reinterpret_cast<float (*)[kMaxG]>(smem + kOffML);
  float (*s_l)[kMaxG] = s_m + kWarps;
  int* s_flag = reinterpret_cast<int*>(smem + kOffFlag);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hkv = p.Hkv, G = p.G;
  const int h = warp % Hkv, sub = warp / Hkv, nsub = kWarps / Hkv;
  const int g = lane >> 2, c = lane & 3;
  const int row_bytes = Hkv * D * 2;
  const int tile_half = kTile * row_bytes;
  const float sl2 = p.scale_log2;
  constexpr int kQC = D / 32, kVH = D / 64, kOT = D / 16;

  float o[kOT][4];
  float m_run = -INFINITY, l_run = 0.f;
  uint32_t qr[kQC][4];

  for (int gq = 0;; ++gq) {
    const int st = gq % kStages;
    if (!mbar_wait(&full[st], (uint32_t)((gq / kStages) & 1))) {
      set_error(p.err, ABKV_DEVERR_TIMEOUT);
      break;
    }
    const StageMeta M = meta[st];
    if (M.li < 0) break;
    const LayerArgs& L = p.layer[M.li];
    // sidecar items: every warp works for the item's head, warp w on tile w
    const bool side_grp = Prm::kHasSide && (M.bits & kSide) != 0;
    const int hw = side_grp ? (M.bits >> kSideHeadShift) & 7 : h;  // head of this warp's rows
    const int my_tile = side_grp ? warp : sub;
    if (M.bits & kFirst) {
#pragma unroll
      for (int mt = 0; mt < kOT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      m_run = -INFINITY;
      l_run = 0.f;
      const __nv_bfloat16* qrow = L.q + ((int64_t)M.b * p.Hq + hw * G + g) * D + 8 * c;
#pragma unroll
      for (int m = 0; m < kQC; ++m) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (g < G) v = __ldg(reinterpret_cast<const uint4*>(qrow + 32 * m));
        qr[m][0] = v.x; qr[m][1] = v.y; qr[m][2] = v.z; qr[m][3] = v.w;
      }
    }
    if (my_tile < M.ntiles) {
      // main tile: row T of KV head h at T * row_bytes + h * D * 2 of tile sub, rows < seq_len;
      // sidecar tile w: 16 slots of the item's head, K then V, rows < pages * quota
      const bool ok = (M.bits >> my_tile) & 1;
      const int tok0 = (M.t0 + my_tile) * kTile;
      int seq_len = M.seq_len;
      if constexpr (Prm::kHasSide) {
        if (side_grp) seq_len *= p.side[M.li].q[hw];
      }
      const int rstride = side_grp ? D * 2 : row_bytes;
      const int head_tile = kTile * D * 2;
      const uint8_t* kb = smem + kOffStage + (size_t)st * kStageBytes +
                          (side_grp ? (size_t)warp * 2 * head_tile : (size_t)sub * 2 * tile_half + h * D * 2);
      const uint8_t* vb = kb + (side_grp ? head_tile : tile_half);

      // S = Q.K^T : rows = query heads (g < G real), cols = tokens 8nt + 2c + {0,1}
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int T = 8 * nt + g;
        const bool valid = ok && (tok0 + T < seq_len);
        uint32_t kr[kQC][4];
#pragma unroll
        for (int m = 0; m < kQC; ++m) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (valid) v = lds128(kb + T * rstride + (32 * m + 8 * c) * 2);
          kr[m][0] = v.x; kr[m][1] = v.y; kr[m][2] = v.z; kr[m][3] = v.w;
        }
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int m = 0; m < kQC; ++m) {
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
      for (int mt = 0; mt < kOT; ++mt) {
        o[mt][0] *= a0; o[mt][1] *= a1; o[mt][2] *= a0; o[mt][3] *= a1;
      }
      const uint32_t pb0 = pack_bf16x2(pr[0][0], pr[0][1]);
      const uint32_t pb1 = pack_bf16x2(pr[1][0], pr[1][1]);

      // V rows 2c, 2c+1, 2c+8, 2c+9 (zero when masked: 0 * NaN would poison O)
#pragma unroll
      for (int hh = 0; hh < kVH; ++hh) {
        uint32_t vr[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int T = 2 * c + (i & 1) + 8 * (i >> 1);
          uint4 v = make_uint4(0, 0, 0, 0);
          if (ok && (tok0 + T < seq_len)) v = lds128(vb + T * rstride + (64 * hh + 8 * g) * 2);
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
    if (!(M.bits & kLast)) continue;
    if constexpr (!Prm::kHasSide) {
      if (p.warp_epi) {
        warp_epilogue<D, kGather>(p, L, M, h, lane, o, m_run, l_run);
        continue;
      }
    }

    // ---- end of item: merge warp partials, write output or chunk partial ----
    float lq = l_run;
    lq += __shfl_xor_sync(0xffffffffu, lq, 1);
    lq += __shfl_xor_sync(0xffffffffu, lq, 2);
#pragma unroll
    for (int jh = 0; jh < 2; ++jh) {
      const int head = 2 * c + jh;
      if (head < G) {
#pragma unroll
        for (int mt = 0; mt < kOT; ++mt) {
          const int hh = mt >> 2, i = mt & 3;
          const int d = 8 * g + 64 * hh + 2 * i;
          s_o[warp][head][d] = o[mt][jh];
          s_o[warp][head][d + 1] = o[mt][2 + jh];
        }
      }
    }
    if (c == 0 && g < G) {
      s_m[warp][g] = m_run;
      s_l[warp][g] = lq;
    }
    consumer_sync();
    // four consecutive dims per thread and step: 16-byte shared-memory reads and partial stores
    constexpr int kD4 = D / 4;
    const int items4 = p.Hq * kD4;
    const int n_chunks = M.n_chunks;
    const int64_t lb = (int64_t)(p.layer_base + M.li) * p.B + M.b;  // (layer, sequence) slot
    const int64_t prow = (lb * p.max_chunks + M.chunk) * p.Hq;
    for (int it = threadIdx.x; it < items4; it += kConsumerThreads) {
      const int d0 = (it % kD4) * 4, hr = it / kD4;
      const int kh = hr / G, r = hr % G;
      if (side_grp && kh != hw) {
        // a sidecar item covers one KV head: the other heads' rows of this chunk are empty
        if (d0 == 0 && n_chunks > 1) p.part_lse[prow + hr] = -INFINITY;
        continue;
      }
      // warps holding this row: all of them for a sidecar item, else those of head kh
      const int nw = side_grp ? kWarps : nsub, w0 = side_grp ? 0 : kh, dw = side_grp ? 1 : Hkv;
      float Mx = -INFINITY;
      for (int s2 = 0; s2 < nw; ++s2) Mx = fmaxf(Mx, s_m[w0 + s2 * dw][r]);
      const float Mu = (Mx == -INFINITY) ? 0.f : Mx;
      float Ls = 0.f, Os[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s2 = 0; s2 < nw; ++s2) {
        const int w = w0 + s2 * dw;
        const float f = exp2f(s_m[w][r] - Mu);
        Ls += s_l[w][r] * f;
        const float4 ov = *reinterpret_cast<const float4*>(&s_o[w][r][d0]);
        Os[0] += ov.x * f;
        Os[1] += ov.y * f;
        Os[2] += ov.z * f;
        Os[3] += ov.w * f;
      }
      float val[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) val[k] = Ls > 0.f ? Os[k] / Ls : 0.f;
      if (n_chunks == 1) {
#pragma unroll
        for (int k = 0; k < 4; ++k) store_out<D, kGather>(p, L, M.b, hr, d0 + k, val[k]);
      } else {
        *reinterpret_cast<float4*>(p.part_o + (prow + hr) * D + d0) = make_float4(val[0], val[1], val[2], val[3]);
        if (d0 == 0) p.part_lse[prow + hr] = Ls > 0.f ? Mu + log2f(Ls) : -INFINITY;
      }
    }
    if (n_chunks > 1) {
      // The last chunk of this (layer, sequence) combines all chunk partials.  The barrier
      // orders every thread's partial stores before thread 0's acq_rel count (a cumulative
      // release at GPU scope); the count's acquire side plus the next barrier order the
      // combine's loads after the other chunks' releases.
      consumer_sync();
      if (threadIdx.x == 0) {
        const int prev = atom_add_acq_rel_gpu(p.counters + lb, 1);
        *s_flag = (prev == n_chunks - 1);
      }
      consumer_sync();
      if (*s_flag) {
        const int64_t row0 = lb * p.max_chunks * p.Hq;
        for (int it = threadIdx.x; it < items4; it += kConsumerThreads) {
          const int d0 = (it % kD4) * 4, hr = it / kD4;
          float Mx = -INFINITY;
#pragma unroll 4
          for (int ch = 0; ch < n_chunks; ++ch)
            Mx = fmaxf(Mx, __ldcg(p.part_lse + row0 + (int64_t)ch * p.Hq + hr));
          const float Mu = (Mx == -INFINITY) ? 0.f : Mx;
          float Ls = 0.f, Os[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
          for (int ch = 0; ch < n_chunks; ++ch) {
            const int64_t rr = row0 + (int64_t)ch * p.Hq + hr;
            const float lse = __ldcg(p.part_lse + rr);
            if (Prm::kHasSide && lse == -INFINITY) continue;  // empty sidecar chunk: its O was not written
            const float f = exp2f(lse - Mu);
            Ls += f;
            const float4 ov = __ldcg(reinterpret_cast<const float4*>(p.part_o + rr * D + d0));
            Os[0] += f * ov.x;
            Os[1] += f * ov.y;
            Os[2] += f * ov.z;
            Os[3] += f * ov.w;
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) store_out<D, kGather>(p, L, M.b, hr, d0 + k, Ls > 0.f ? Os[k] / Ls : 0.f);
        }
        if (threadIdx.x == 0) p.counters[lb] = 0;  // ready for the next call on this workspace
      }
    }
    consumer_sync();  // s_o / s_m / s_l / s_flag may be rewritten by the next item
  }
}

template <int D, class Prm, bool kGather>
__global__ void __launch_bounds__(kThreads, 1) decode_split_kernel(const __grid_constant__ Prm p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kWarps);
    }
  }
  __syncthreads();
  if ((threadIdx.x >> 5) == kWarps) {
    producer<D>(p, smem);
  } else {
    consumer<D, Prm, kGather>(p, smem);
  }
  if constexpr (kGather) {
    __threadfence_system();  // this thread's output stores, to every rank
    __syncthreads();
    if (threadIdx.x == 0) gather_barrier(p);
  }
}

constexpr int kMaxAutoChunkTiles = 384;  // 6144 cache rows

int auto_chunk_tiles(int num_layers, int num_seqs, int max_tiles, int page_tiles, int num_kv_heads) {
  // Persistent CTAs take items dynamically: aim for >= ~4 items per SM, with
  // chunks of 16..128 tiles (256..2048 cache rows).  (A launch of one layer of
  // a KV-head shard, 256 sequences x 1 KV head: 2048-row chunks take 203 us per
  // layer, 1024-row chunks -- the choice at >= 8 items per SM -- 221 us; launches
  // of many layers have items to spare and keep 128 tiles either way.)
  const int64_t total = (int64_t)num_layers * num_seqs * max_tiles;
  int ct = 128;
  while (ct > 16 && total / ct < 148 * 4) ct >>= 1;
  if (ct < page_tiles) ct = page_tiles;
  ct = (ct / page_tiles) * page_tiles;
  // A tile of fewer than 8 KV heads carries fewer bytes, so the per-item costs
  // (page-id staging, the chunk merge) weigh more: with enough items, grow the
  // chunk by 8 / num_kv_heads up to kMaxAutoChunkTiles.  Never below the chunk
  // chosen without the head count, so a workspace sized without it still fits.
  if (ct == 128 && num_kv_heads > 0 && num_kv_heads < 8) {
    int big = 128 * (8 / num_kv_heads);
    if (big > kMaxAutoChunkTiles) big = kMaxAutoChunkTiles;
    big = (big / page_tiles) * page_tiles;
    if (big > ct && total / big >= 148 * 8) ct = big;
  }
  return ct;
}

struct DecodePlan {
  int chunk_tiles, max_chunks, max_tiles;
  size_t counter_bytes, part_o_bytes, part_lse_bytes, total;
};

constexpr size_t kWsHeader = 256;

// max_side_rows: an upper bound of the sidecar rows of one (layer, request) over
// all its heads (sidecar pages x slots), 0 without a sidecar.  Sidecar chunks are
// per head, so each head may round up by one chunk (+2 per head of slack).
// num_kv_heads: the launch's KV heads, or 0 where it is not known (workspace
// queries); it only ever enlarges the auto chunk, so 0 gives the larger plan.
int plan_decode(int num_layers, int num_seqs, int num_q_heads, int head_dim, int page_size,
                int max_pages, int chunk_tokens, int64_t max_side_rows, DecodePlan* plan,
                int num_kv_heads = 0) {
  if (num_layers <= 0 || num_seqs <= 0 || num_q_heads <= 0 || page_size <= 0 || max_pages <= 0)
    return ABKV_ERR_INVALID_ARG;
  if ((head_dim != 64 && head_dim != kD) || page_size % kTile != 0) return ABKV_ERR_UNSUPPORTED;
  const int page_tiles = page_size / kTile;
  const int64_t max_tiles = (int64_t)max_pages * page_tiles;
  if (max_side_rows < 0) return ABKV_ERR_INVALID_ARG;
  const int64_t side_tiles = (max_side_rows + kTile - 1) / kTile;
  if (max_tiles > (1 << 26) || side_tiles > (1 << 26)) return ABKV_ERR_UNSUPPORTED;
  int ct;
  if (chunk_tokens == 0) {
    ct = auto_chunk_tiles(num_layers, num_seqs, (int)(max_tiles + side_tiles), page_tiles, num_kv_heads);
  } else {
    if (chunk_tokens < 0 || chunk_tokens % kTile || chunk_tokens % page_size) return ABKV_ERR_INVALID_ARG;
    ct = chunk_tokens / kTile;
  }
  if (ct * kTile / page_size > kMaxChunkPages - 1) return ABKV_ERR_UNSUPPORTED;
  plan->chunk_tiles = ct;
  plan->max_tiles = (int)max_tiles;
  plan->max_chunks = (int)((max_tiles + ct - 1) / ct + (side_tiles ? (side_tiles + ct - 1) / ct + 2 * kWarps : 0));
  if (plan->max_chunks > 1) {
    const size_t rows = (size_t)num_layers * num_seqs * plan->max_chunks * num_q_heads;
    // one counter per (layer, sequence, KV head); num_q_heads bounds the KV heads
    plan->counter_bytes = ((size_t)num_layers * num_seqs * num_q_heads * sizeof(int32_t) + 255) / 256 * 256;
    plan->part_o_bytes = rows * head_dim * sizeof(float);
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
                  chunk_tokens, 0, &plan) != ABKV_OK)
    return 0;
  return plan.total;
}

namespace abkv {
namespace {
template <class Prm, bool kGather>
int launch_kernel(const Prm& prm, int head_dim, int grid, cudaStream_t s) {
  auto kernel = head_dim == 64 ? decode_split_kernel<64, Prm, kGather> : decode_split_kernel<kD, Prm, kGather>;
  // opt in to > 48 KiB of dynamic shared memory (idempotent, per device)
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
    return ABKV_ERR_CUDA;
  kernel<<<grid, kThreads, kSmemBytes, s>>>(prm);
  return ABKV_OK;
}

template <class Prm>
int fill_and_launch(Prm& prm, const DecodePlan& plan, const void* const* q, const void* const* kv,
                    const int32_t* const* block_tables, const int64_t* bt_strides, const int32_t* const* seq_lens,
                    const int64_t* num_blocks, void* const* out, int num_layers, int num_seqs, int num_q_heads,
                    int num_kv_heads, int head_dim, int page_size, float scale, char* ws, void* stream,
                    const GatherArgs& gather, const abkv_sidecar_t* sidecars) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int dev = 0, num_sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || num_sms <= 0)
    return ABKV_ERR_CUDA;
  const bool gathering = gather.my_flags != nullptr;
  prm.err = reinterpret_cast<int32_t*>(ws);
  prm.work = reinterpret_cast<int32_t*>(ws + 64);  // [next item, CTAs done], inside the header
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
  prm.G = num_q_heads / num_kv_heads;
  prm.P = page_size;
  prm.chunk_tiles = plan.chunk_tiles;
  prm.max_chunks = plan.max_chunks;
  prm.max_rows = plan.max_tiles * kTile;
  prm.gather = gather;
  // Per-warp epilogue: one consumer warp per KV head and 16-byte stores into
  // every output (and every rank's copy of it).
  bool warp_epi = !Prm::kHasSide && num_kv_heads == kWarps;
  for (int l = 0; l < num_layers && warp_epi; ++l)
    if (reinterpret_cast<uintptr_t>(out[l]) & 15) warp_epi = false;
  if (gathering)
    for (int r = 0; r < gather.world && warp_epi; ++r)
      if ((gather.peer_delta[r] * 2) & 15) warp_epi = false;
  prm.warp_epi = warp_epi ? 1 : 0;
  // The chunk counters must start at zero.  Each launch resets the ones it used,
  // but a call with a larger plan on the same workspace would also find, in its
  // counter range, the previous plan's partials: clear them on the stream.
  if (split && cudaMemsetAsync(prm.counters, 0, plan.counter_bytes, s) != cudaSuccess) return ABKV_ERR_CUDA;

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
      if constexpr (Prm::kHasSide) {
        SideArgs& sa = prm.side[i];
        sa.pages = nullptr;
        if (sidecars[l0 + i].pages) {
          const abkv_sidecar_t& sc = sidecars[l0 + i];
          sa.pages = static_cast<const __nv_bfloat16*>(sc.pages);
          sa.bt = sc.page_table;
          sa.count = sc.page_count;
          sa.bt_stride = sc.page_table_stride;
          sa.num_pages = sc.num_pages;
          sa.slots = sc.slots;
          for (int h = 0, off = 0; h < num_kv_heads; ++h) {
            sa.off[h] = off;
            sa.q[h] = sc.quotas[h];
            off += sc.quotas[h];
          }
        }
      }
    }
    prm.layer_base = l0;
    prm.nl = nl;
    prm.num_items = plan.max_chunks * nl * num_seqs;
    const int grid = prm.num_items < num_sms ? prm.num_items : num_sms;
    int rc;
    if constexpr (Prm::kHasSide) {
      rc = launch_kernel<Prm, false>(prm, head_dim, grid, s);  // the sidecar decode does not gather
    } else {
      rc = gathering ? launch_kernel<Prm, true>(prm, head_dim, grid, s)
                     : launch_kernel<Prm, false>(prm, head_dim, grid, s);
    }
    if (rc != ABKV_OK) return rc;
  }
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}

int launch_decode(const void* const* q, const void* const* kv, const int32_t* const* block_tables,
                  const int64_t* bt_strides, const int32_t* const* seq_lens, const int64_t* num_blocks,
                  void* const* out, int num_layers, int num_seqs, int num_q_heads, int num_kv_heads,
                  int head_dim, int page_size, int max_pages_per_seq, float scale, int chunk_tokens,
                  void* workspace, size_t workspace_bytes, void* stream, const GatherArgs& gather,
                  const abkv_sidecar_t* sidecars = nullptr) {
  if (!q || !kv || !block_tables || !bt_strides || !seq_lens || !num_blocks || !out)
    return ABKV_ERR_INVALID_ARG;
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return ABKV_ERR_INVALID_ARG;
  if (kWarps % num_kv_heads != 0) return ABKV_ERR_UNSUPPORTED;
  const int G = num_q_heads / num_kv_heads;
  if (G > kMaxG) return ABKV_ERR_UNSUPPORTED;
  if (num_seqs > 65535) return ABKV_ERR_UNSUPPORTED;
  if (!(scale > 0.f)) return ABKV_ERR_INVALID_ARG;
  // sidecars: per layer, pages == NULL means none; quotas multiples of 16 in [16, 2^16)
  int64_t max_side_rows = 0;
  if (sidecars) {
    for (int l = 0; l < num_layers; ++l) {
      const abkv_sidecar_t& sc = sidecars[l];
      if (!sc.pages) continue;
      if (!sc.page_table || !sc.page_count || sc.page_table_stride <= 0 || sc.num_pages <= 0)
        return ABKV_ERR_INVALID_ARG;
      if ((reinterpret_cast<uintptr_t>(sc.pages) & 15) || (reinterpret_cast<uintptr_t>(sc.page_table) & 3))
        return ABKV_ERR_INVALID_ARG;
      int sum = 0;
      for (int h = 0; h < num_kv_heads; ++h) {
        const int qh = sc.quotas[h];
        if (qh <= 0 || qh % kTile || qh >= (1 << 16)) return ABKV_ERR_UNSUPPORTED;
        sum += qh;
      }
      if (sum != sc.slots) return ABKV_ERR_INVALID_ARG;
      const int64_t rows = sc.page_table_stride * sum;
      max_side_rows = rows > max_side_rows ? rows : max_side_rows;
    }
  }
  DecodePlan plan;
  int st = plan_decode(num_layers, num_seqs, num_q_heads, head_dim, page_size, max_pages_per_seq,
                       chunk_tokens, max_side_rows, &plan, num_kv_heads);
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
  char* ws = static_cast<char*>(workspace);
  const bool gathering = gather.my_flags != nullptr;
  if (sidecars) {
    if (gathering) return ABKV_ERR_UNSUPPORTED;
    SideDecodeParams prm;
    memset(&prm, 0, sizeof(prm));
    return fill_and_launch(prm, plan, q, kv, block_tables, bt_strides, seq_lens, num_blocks, out, num_layers,
                           num_seqs, num_q_heads, num_kv_heads, head_dim, page_size, scale, ws, stream, gather,
                           sidecars);
  }
  DecodeParams prm;
  memset(&prm, 0, sizeof(prm));
  return fill_and_launch(prm, plan, q, kv, block_tables, bt_strides, seq_lens, num_blocks, out, num_layers, num_seqs,
                         num_q_heads, num_kv_heads, head_dim, page_size, scale, ws, stream, gather, nullptr);
}

}  // namespace
}  // namespace abkv

extern "C" int abkv_decode(const void* const* q, const void* const* kv,
                           const int32_t* const* block_tables, const int64_t* bt_strides,
                           const int32_t* const* seq_lens, const int64_t* num_blocks,
                           void* const* out, int num_layers, int num_seqs, int num_q_heads,
                           int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
                           float scale, int chunk_tokens, void* workspace, size_t workspace_bytes,
                           void* stream) {
  GatherArgs g;
  memset(&g, 0, sizeof(g));
  g.out_row = (int64_t)num_q_heads * head_dim;
  g.world = 1;
  return launch_decode(q, kv, block_tables, bt_strides, seq_lens, num_blocks, out, num_layers, num_seqs,
                       num_q_heads, num_kv_heads, head_dim, page_size, max_pages_per_seq, scale, chunk_tokens,
                       workspace, workspace_bytes, stream, g);
}

extern "C" size_t abkv_decode_packed_workspace_size(int num_layers, int num_seqs, int num_q_heads, int head_dim,
                                                    int page_size, int max_pages_per_seq, int chunk_tokens,
                                                    int64_t max_side_rows) {
  DecodePlan plan;
  if (plan_decode(num_layers, num_seqs, num_q_heads, head_dim, page_size, max_pages_per_seq, chunk_tokens,
                  max_side_rows, &plan) != ABKV_OK)
    return 0;
  return plan.total;
}

extern "C" int abkv_decode_packed(const void* const* q, const void* const* kv,
                                  const int32_t* const* block_tables, const int64_t* bt_strides,
                                  const int32_t* const* seq_lens, const int64_t* num_blocks,
                                  void* const* out, int num_layers, int num_seqs, int num_q_heads,
                                  int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
                                  float scale, int chunk_tokens, const abkv_sidecar_t* sidecars,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (!sidecars) return ABKV_ERR_INVALID_ARG;
  GatherArgs g;
  memset(&g, 0, sizeof(g));
  g.out_row = (int64_t)num_q_heads * head_dim;
  g.world = 1;
  return launch_decode(q, kv, block_tables, bt_strides, seq_lens, num_blocks, out, num_layers, num_seqs,
                       num_q_heads, num_kv_heads, head_dim, page_size, max_pages_per_seq, scale, chunk_tokens,
                       workspace, workspace_bytes, stream, g, sidecars);
}

extern "C" int abkv_decode_gather(const void* const* q, const void* const* kv,
                                  const int32_t* const* block_tables, const int64_t* bt_strides,
                                  const int32_t* const* seq_lens, const int64_t* num_blocks,
                                  void* const* out, int num_layers, int num_seqs, int num_q_heads,
                                  int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
                                  float scale, int chunk_tokens, const abkv_gather_t* gather,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (!gather || !out) return ABKV_ERR_INVALID_ARG;
  const abkv_gather_t& a = *gather;
  if (a.world < 1 || a.world > kMaxPeers || a.rank < 0 || a.rank >= a.world || a.epoch == 0)
    return ABKV_ERR_INVALID_ARG;
  if (a.hq_total != a.world * num_q_heads) return ABKV_ERR_INVALID_ARG;
  for (int r = 0; r < a.world; ++r)
    if (!a.rank_buffers[r] || (reinterpret_cast<uintptr_t>(a.rank_buffers[r]) & 255)) return ABKV_ERR_INVALID_ARG;
  // every layer's output slot [num_seqs][hq_total][D] lies in this rank's buffer
  // after the flag area (the same offsets are written in the peers' buffers)
  const char* base = static_cast<const char*>(a.rank_buffers[a.rank]);
  const size_t slot = (size_t)num_seqs * a.hq_total * head_dim * 2;
  for (int l = 0; l < num_layers; ++l) {
    const char* o = static_cast<const char*>(out[l]);
    if (!o || o < base + ABKV_GATHER_FLAG_BYTES || o + slot > base + a.buffer_bytes ||
        ((o - base) & 15))
      return ABKV_ERR_INVALID_ARG;
  }
  GatherArgs g;
  memset(&g, 0, sizeof(g));
  for (int r = 0; r < a.world; ++r) {
    g.peer_delta[r] = (static_cast<const char*>(a.rank_buffers[r]) - base) / 2;
    g.peer_flags[r] = static_cast<uint32_t*>(a.rank_buffers[r]);
  }
  g.my_flags = static_cast<uint32_t*>(a.rank_buffers[a.rank]);
  g.out_row = (int64_t)a.hq_total * head_dim;
  g.world = a.world;
  g.rank = a.rank;
  g.head0 = a.rank * num_q_heads;
  g.epoch = a.epoch;
  g.timeout_ns = (a.timeout_us ? (uint64_t)a.timeout_us : 5000000ull) * 1000ull;
  return launch_decode(q, kv, block_tables, bt_strides, seq_lens, num_blocks, out, num_layers, num_seqs,
                       num_q_heads, num_kv_heads, head_dim, page_size, max_pages_per_seq, scale, chunk_tokens,
                       workspace, workspace_bytes, stream, g);
}

// ---------------------------------------------------------------------------
// Decode without any allocation by the caller or by the library.
//
// Some callers cannot allocate device memory at the point where they decode:
// an inference engine that reserves all of HBM for its KV cache up front and
// forbids later cudaMalloc calls, a host loop whose allocator is not
// thread-safe, or code that must not touch the CUDA caching allocator at all.
// For them the split-KV scratch (partials, counters, error word) lives in one
// file-scope device array of kNoAllocScratchBytes that every GPU loading this
// library holds until process exit.  The caller passes only inputs and outputs.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code the
// symbol name is only a host-side stand-in, so its address is looked up once
// per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return ABKV_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return ABKV_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return ABKV_OK;
}
}  // namespace

extern "C" int abkv_decode_noalloc(const void* const* q, const void* const* kv,
                                   const int32_t* const* block_tables, const int64_t* bt_strides,
                                   const int32_t* const* seq_lens, const int64_t* num_blocks,
                                   void* const* out, int num_layers, int num_seqs, int num_q_heads,
                                   int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
                                   float scale, int chunk_tokens, int32_t* device_error, void* stream) {
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return ABKV_ERR_INVALID_ARG;
  // The plan of the launch itself (with its KV-head count), so the limit check
  // refuses exactly the requests whose launch would not fit.
  DecodePlan plan;
  const int st = plan_decode(num_layers, num_seqs, num_q_heads, head_dim, page_size, max_pages_per_seq,
                             chunk_tokens, 0, &plan, num_kv_heads);
  if (st != ABKV_OK) return st;
  if (plan.total > kNoAllocScratchBytes) return ABKV_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int se = noalloc_scratch(&scratch);
  if (se != ABKV_OK) return se;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: clear the error word, the
  // work counters and the per-(layer, sequence) chunk counters.
  if (cudaMemsetAsync(scratch, 0, kWsHeader + plan.counter_bytes, s) != cudaSuccess) return ABKV_ERR_CUDA;
  const int rc = abkv_decode(q, kv, block_tables, bt_strides, seq_lens, num_blocks, out, num_layers,
                             num_seqs, num_q_heads, num_kv_heads, head_dim, page_size, max_pages_per_seq,
                             scale, chunk_tokens, scratch, kNoAllocScratchBytes, stream);
  if (rc != ABKV_OK) return rc;
  if (device_error &&
      cudaMemcpyAsync(device_error, scratch, sizeof(int32_t), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return ABKV_ERR_CUDA;
  return ABKV_OK;
}
