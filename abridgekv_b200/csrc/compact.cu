// KV compaction executor for sm_100a: ordered batches of slot copies applied
// to every layer tensor of a KV-cache group in one launch per batch.
//
// Reference semantics: GPUModelRunner._execute_kv_copy_operations /
// _execute_kv_copy_group (third_party/vllm_overlay/vllm/v1/worker/
// gpu_model_runner.py:1147-1220): for each group, batches are applied in order,
// and within a batch every source row is gathered before any destination row
// is written ("gather-all-then-scatter"), for both paged layouts
//   FlashInfer       [num_blocks, 2, page, Hkv, D]   (layout 0)
//   FlashAttention   [2, num_blocks, page, Hkv, D]   (layout 1).
//
// Plan (host, per batch).  Op i copies row r_i to row w_i.  If op i writes a
// row that op j reads (w_i == r_j), j must read before i writes.  When every
// destination is unique and every row is read by at most one op, these
// constraints form disjoint chains  j -> writer(r_j) -> ...; a chain walked in
// order by ONE thread group, with each lane always handling the same bytes of
// every row, reproduces gather-then-scatter exactly with no grid barrier (no
// op outside a chain reads or writes that chain's rows).  Batches without any
// hazard are chains of length one and run fully parallel (found with a bit per
// pool row for "read" and "written", without hashing, when the pool is small).  A batch with a
// cycle, a row read twice, or a duplicate destination takes the two-phase
// path instead: gather every source row into the workspace, then scatter
// (for duplicate destinations the op listed last wins).
//
// Kernel work item = (chain, layer); one warp per item moves the K and V row
// halves of each op together, 16-byte loads/stores, 64 bytes per lane per
// 2 KiB row half (Hkv*D*2 bytes), both halves' loads in flight before the stores.
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace abkv {
namespace {

constexpr int kMaxLayers = 96;

struct CompactParams {
  char* layer[kMaxLayers];
  const int32_t* ops;      // [n][4] in chain order
  const int32_t* chain;    // [n_chains + 1] offsets into ops
  char* scratch;           // two-phase path: [n][layers][2][row_bytes]
  int32_t* err;
  int64_t blk_stride;      // bytes between consecutive blocks
  int64_t half_stride;     // bytes between the K and V halves of a block
  int64_t row_bytes;       // Hkv * D * 2
  int64_t num_blocks;
  int num_layers, page, n_chains, n_ops;
};

__device__ __forceinline__ bool row_ok(const CompactParams& p, int blk, int off) {
  return blk >= 0 && blk < p.num_blocks && off >= 0 && off < p.page;
}

__device__ __forceinline__ char* row_ptr(const CompactParams& p, int layer, int half, int blk, int off) {
  return p.layer[layer] + (int64_t)blk * p.blk_stride + (int64_t)half * p.half_stride +
         (int64_t)off * p.row_bytes;
}

__device__ __forceinline__ uint4 ld_cg(const void* ptr) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr));
  return r;
}
__device__ __forceinline__ void st_cg(void* ptr, uint4 v) {
  asm volatile("st.global.cg.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"l"(ptr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// One warp walks one chain for one layer, moving each op's K and V row halves
// together: rows are processed in 512-byte slabs (32 lanes x 16 B), and each
// lane keeps up to kVec vectors of each half in flight before its stores.
constexpr int kVec = 4;

__global__ void __launch_bounds__(256) compact_chain_kernel(const __grid_constant__ CompactParams p) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t items = (int64_t)p.n_chains * p.num_layers;
  if (warp >= items) return;
  const int layer = (int)(warp % p.num_layers);
  const int c = (int)(warp / p.num_layers);
  const int o0 = p.chain ? p.chain[c] : c, o1 = p.chain ? p.chain[c + 1] : c + 1;  // null: one op per chain
  const int64_t vecs = p.row_bytes >> 4;  // 16-byte vectors per row half
  for (int i = o0; i < o1; ++i) {
    const int sb = p.ops[4 * i], so = p.ops[4 * i + 1], db = p.ops[4 * i + 2], dof = p.ops[4 * i + 3];
    if (!row_ok(p, sb, so) || !row_ok(p, db, dof)) {
      if (lane == 0) set_error(p.err, ABKV_DEVERR_ROW_OOB);
      continue;
    }
    const char* src = row_ptr(p, layer, 0, sb, so);
    char* dst = row_ptr(p, layer, 0, db, dof);
    for (int64_t v0 = 0; v0 < vecs; v0 += 32 * kVec) {
      uint4 buf[2][kVec];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < kVec; ++k) {
          const int64_t v = v0 + k * 32 + lane;
          if (v < vecs) buf[h][k] = ld_cg(src + h * p.half_stride + 16 * v);
        }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < kVec; ++k) {
          const int64_t v = v0 + k * 32 + lane;
          if (v < vecs) st_cg(dst + h * p.half_stride + 16 * v, buf[h][k]);
        }
    }
  }
}

// Two-phase path.  phase 0: scratch[i][layer][half] <- src row; phase 1: dst
// row <- scratch (ops whose destination is overwritten later in the batch are
// skipped: "last op wins").
__global__ void __launch_bounds__(256) compact_twophase_kernel(const __grid_constant__ CompactParams p,
                                                               int phase) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t items = (int64_t)p.n_ops * p.num_layers * 2;
  if (warp >= items) return;
  const int half = (int)(warp & 1);
  const int layer = (int)((warp >> 1) % p.num_layers);
  const int i = (int)((warp >> 1) / p.num_layers);
  const int sb = p.ops[4 * i], so = p.ops[4 * i + 1], db = p.ops[4 * i + 2], dof = p.ops[4 * i + 3];
  if (!row_ok(p, sb, so) || !row_ok(p, db, dof)) {
    if (lane == 0) set_error(p.err, ABKV_DEVERR_ROW_OOB);
    return;
  }
  char* slot = p.scratch + (((int64_t)i * p.num_layers + layer) * 2 + half) * p.row_bytes;
  const int64_t vecs = p.row_bytes >> 4;
  if (phase == 0) {
    const char* src = row_ptr(p, layer, half, sb, so);
    for (int64_t v = lane; v < vecs; v += 32) st_cg(slot + 16 * v, ld_cg(src + 16 * v));
  } else {
    if (p.chain[i]) return;  // superseded duplicate destination
    char* dst = row_ptr(p, layer, half, db, dof);
    for (int64_t v = lane; v < vecs; v += 32) st_cg(dst + 16 * v, ld_cg(slot + 16 * v));
  }
}

constexpr size_t kWsHeader = 256;

struct BatchPlan {
  std::vector<int32_t> ops;    // reordered, [n][4]
  std::vector<int32_t> chain;  // chain offsets (chain path) or superseded flags (two-phase)
  bool two_phase = false;
  int n_chains = 0;
  const int32_t* singles = nullptr;  // hazard-free batch: the caller's ops, one op per chain
};

// Hazard-free batches (no row read twice, no destination twice, no source row that an op of the
// batch writes) are every op its own chain, in input order: one bit per cache row for "read" and
// one for "written" decide it without hashing, when the pool's rows fit a small bitmap.
bool plan_singles(const int32_t* ops, int64_t n, int page, int64_t num_blocks, BatchPlan* out) {
  const int64_t rows = num_blocks * page;
  if (rows > ((int64_t)1 << 23) || rows > 256 * n + 65536) return false;
  const size_t words = (size_t)((rows + 63) >> 6);
  std::vector<uint64_t> rd(words, 0), wr(words, 0);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t r = (int64_t)ops[4 * i] * page + ops[4 * i + 1];
    const int64_t w = (int64_t)ops[4 * i + 2] * page + ops[4 * i + 3];
    const uint64_t rb = 1ull << (r & 63), wb = 1ull << (w & 63);
    if ((rd[r >> 6] & rb) || (wr[w >> 6] & wb)) return false;  // a row read twice, or written twice
    rd[r >> 6] |= rb;
    wr[w >> 6] |= wb;
  }
  for (int64_t i = 0; i < n; ++i) {
    const int64_t r = (int64_t)ops[4 * i] * page + ops[4 * i + 1];
    if (wr[r >> 6] & (1ull << (r & 63))) return false;  // a source row is overwritten in the batch
  }
  out->ops.clear();
  out->chain.clear();
  out->singles = ops;
  out->n_chains = (int)n;
  out->two_phase = false;
  return true;
}

// Slot (block * page + offset, >= 0) -> op index, open addressing with linear
// probing at load <= 1/4 and Fibonacci (Knuth multiplicative) hashing: the host
// planning of a 4096-op batch stays in the tens of microseconds.
class SlotMap {
 public:
  explicit SlotMap(int64_t n) {
    size_t cap = 16;
    while (cap < (size_t)n * 4) cap <<= 1;
    keys_.assign(cap, -1);
    vals_.resize(cap);
    mask_ = cap - 1;
  }
  // The value slot of `key`; *fresh says whether the key was absent (its value is then unset).
  int64_t& slot(int64_t key, bool* fresh) {
    for (size_t i = index(key);; i = (i + 1) & mask_) {
      if (keys_[i] == key) {
        *fresh = false;
        return vals_[i];
      }
      if (keys_[i] < 0) {
        keys_[i] = key;
        *fresh = true;
        return vals_[i];
      }
    }
  }
  const int64_t* find(int64_t key) const {
    for (size_t i = index(key);; i = (i + 1) & mask_) {
      if (keys_[i] == key) return &vals_[i];
      if (keys_[i] < 0) return nullptr;
    }
  }

 private:
  size_t index(int64_t key) const {
    const uint64_t x = (uint64_t)key * 0x9E3779B97F4A7C15ull;
    return (size_t)(x ^ (x >> 29)) & mask_;
  }
  std::vector<int64_t> keys_, vals_;
  size_t mask_ = 0;
};

// Row (block * page + offset, >= 0) -> the op that reads it and the op that writes it, in one
// 16-byte entry: open addressing with linear probing at load <= 1/2, Fibonacci hashing.  One probe
// per source and per destination row; the source's entry index is kept, so finding the op that
// overwrites a source row needs no second lookup.
class RowMap {
 public:
  struct Entry {
    int64_t key;
    int32_t reader, writer;
  };
  explicit RowMap(int64_t rows) {
    size_t cap = 16;
    while (cap < (size_t)rows * 2) cap <<= 1;
    e_.assign(cap, Entry{-1, -1, -1});
    mask_ = cap - 1;
  }
  // The index of `key`'s entry, inserted (reader and writer unset) when absent.
  size_t locate(int64_t key) {
    const uint64_t x = (uint64_t)key * 0x9E3779B97F4A7C15ull;
    for (size_t i = (size_t)(x ^ (x >> 29)) & mask_;; i = (i + 1) & mask_) {
      if (e_[i].key == key) return i;
      if (e_[i].key < 0) {
        e_[i].key = key;
        return i;
      }
    }
  }
  Entry& operator[](size_t i) { return e_[i]; }

 private:
  std::vector<Entry> e_;
  size_t mask_ = 0;
};

// Split one batch into chains (see file comment); returns false when the
// batch needs the two-phase path.
bool plan_chains(const int32_t* ops, int64_t n, int page, BatchPlan* out) {
  auto key = [page](int32_t blk, int32_t off) -> int64_t { return (int64_t)blk * page + off; };
  RowMap rows(2 * n);
  std::vector<size_t> src_at(n);
  for (int64_t i = 0; i < n; ++i) {
    const size_t a = rows.locate(key(ops[4 * i], ops[4 * i + 1]));
    if (rows[a].reader >= 0) return false;  // a row read twice
    rows[a].reader = (int32_t)i;
    src_at[i] = a;
    const size_t w = rows.locate(key(ops[4 * i + 2], ops[4 * i + 3]));
    if (rows[w].writer >= 0) return false;  // duplicate destination
    rows[w].writer = (int32_t)i;
  }
  // next(j) = the op that overwrites j's source row (other than j itself)
  std::vector<int64_t> next(n, -1);
  std::vector<char> has_prev(n, 0);
  for (int64_t j = 0; j < n; ++j) {
    const int64_t w = rows[src_at[j]].writer;
    if (w >= 0 && w != j) {
      next[j] = w;
      has_prev[w] = 1;
    }
  }
  std::vector<char> seen(n, 0);
  out->ops.clear();
  out->ops.reserve((size_t)n * 4);
  out->chain.assign(1, 0);
  int64_t covered = 0;
  for (int64_t s = 0; s < n; ++s) {
    if (has_prev[s]) continue;
    for (int64_t i = s; i >= 0; i = next[i]) {
      if (seen[i]) return false;
      seen[i] = 1;
      out->ops.insert(out->ops.end(), ops + 4 * i, ops + 4 * i + 4);
      ++covered;
    }
    out->chain.push_back((int32_t)(out->ops.size() / 4));
  }
  if (covered != n) return false;  // the rest lie on cycles
  out->n_chains = (int)out->chain.size() - 1;
  out->two_phase = false;
  return true;
}

void plan_two_phase(const int32_t* ops, int64_t n, int page, BatchPlan* out) {
  out->ops.assign(ops, ops + 4 * n);
  out->chain.assign(n, 0);
  SlotMap last_writer(n);
  for (int64_t i = 0; i < n; ++i) {
    bool fresh;
    last_writer.slot((int64_t)ops[4 * i + 2] * page + ops[4 * i + 3], &fresh) = i;
  }
  for (int64_t i = 0; i < n; ++i)
    out->chain[i] = *last_writer.find((int64_t)ops[4 * i + 2] * page + ops[4 * i + 3]) != i;
  out->two_phase = true;
  out->n_chains = 0;
}

}  // namespace
}  // namespace abkv

using namespace abkv;

extern "C" size_t abkv_compact_workspace_size(int num_layers, int page_size, int num_kv_heads,
                                              int head_dim, int64_t max_ops_per_batch) {
  if (num_layers <= 0 || page_size <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_ops_per_batch < 0)
    return 0;
  const size_t row = (size_t)num_kv_heads * head_dim * 2;
  const size_t n = (size_t)max_ops_per_batch;
  const size_t meta = ((n * 4 + n + 1) * sizeof(int32_t) + 255) / 256 * 256;
  return kWsHeader + meta + n * (size_t)num_layers * 2 * row;
}

extern "C" int abkv_compact(void* const* layer_caches, int num_layers, int layout, int64_t num_blocks,
                            int page_size, int num_kv_heads, int head_dim, const int32_t* ops,
                            const int64_t* batch_offsets, int num_batches, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!layer_caches || num_layers <= 0 || num_layers > kMaxLayers) return ABKV_ERR_INVALID_ARG;
  if (layout != 0 && layout != 1) return ABKV_ERR_INVALID_ARG;
  if (num_blocks <= 0 || page_size <= 0 || num_kv_heads <= 0 || head_dim <= 0) return ABKV_ERR_INVALID_ARG;
  if (num_batches < 0 || (num_batches > 0 && (!ops || !batch_offsets))) return ABKV_ERR_INVALID_ARG;
  const int64_t row_bytes = (int64_t)num_kv_heads * head_dim * 2;
  if (row_bytes % 16) return ABKV_ERR_UNSUPPORTED;
  for (int l = 0; l < num_layers; ++l)
    if (!layer_caches[l] || (reinterpret_cast<uintptr_t>(layer_caches[l]) & 15)) return ABKV_ERR_INVALID_ARG;
  if (num_batches == 0) return ABKV_OK;
  if (batch_offsets[0] != 0) return ABKV_ERR_INVALID_ARG;
  int64_t max_n = 0;
  for (int b = 0; b < num_batches; ++b) {
    const int64_t n = batch_offsets[b + 1] - batch_offsets[b];
    if (n < 0 || n > (int64_t)1 << 30) return ABKV_ERR_INVALID_ARG;
    max_n = std::max(max_n, n);
  }
  const int64_t total = batch_offsets[num_batches];
  for (int64_t i = 0; i < total; ++i) {  // host-side validation of every row
    const int32_t* o = ops + 4 * i;
    if (o[0] < 0 || o[0] >= num_blocks || o[2] < 0 || o[2] >= num_blocks || o[1] < 0 ||
        o[1] >= page_size || o[3] < 0 || o[3] >= page_size)
      return ABKV_ERR_INVALID_ARG;
  }
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255)) return ABKV_ERR_WORKSPACE;
  const size_t meta_bytes = ((size_t)(max_n * 4 + max_n + 1) * sizeof(int32_t) + 255) / 256 * 256;
  const size_t base_need = kWsHeader + meta_bytes;
  if (workspace_bytes < base_need) return ABKV_ERR_WORKSPACE;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  CompactParams prm;
  std::memset(&prm, 0, sizeof(prm));
  for (int l = 0; l < num_layers; ++l) prm.layer[l] = static_cast<char*>(layer_caches[l]);
  prm.err = reinterpret_cast<int32_t*>(ws);
  int32_t* d_ops = reinterpret_cast<int32_t*>(ws + kWsHeader);
  int32_t* d_chain = d_ops + 4 * max_n;
  prm.ops = d_ops;
  prm.chain = d_chain;
  prm.scratch = ws + base_need;
  prm.row_bytes = row_bytes;
  prm.num_blocks = num_blocks;
  prm.page = page_size;
  prm.num_layers = num_layers;
  if (layout == 0) {
    prm.half_stride = (int64_t)page_size * row_bytes;
    prm.blk_stride = 2 * prm.half_stride;
  } else {
    prm.blk_stride = (int64_t)page_size * row_bytes;
    prm.half_stride = num_blocks * prm.blk_stride;
  }

  // Plan every batch first so that a workspace shortfall launches nothing.
  std::vector<BatchPlan> plans(num_batches);
  for (int b = 0; b < num_batches; ++b) {
    const int64_t n = batch_offsets[b + 1] - batch_offsets[b];
    const int32_t* bo = ops + 4 * batch_offsets[b];
    if (!plan_singles(bo, n, page_size, num_blocks, &plans[b]) && !plan_chains(bo, n, page_size, &plans[b]))
      plan_two_phase(bo, n, page_size, &plans[b]);
    if (plans[b].two_phase &&
        workspace_bytes < base_need + (size_t)n * num_layers * 2 * (size_t)row_bytes)
      return ABKV_ERR_WORKSPACE;
  }
  for (int b = 0; b < num_batches; ++b) {
    BatchPlan& pl = plans[b];
    const int64_t n = pl.singles ? pl.n_chains : (int64_t)pl.ops.size() / 4;
    if (n == 0) continue;
    // Pageable-host copies are staged before cudaMemcpyAsync returns, so the
    // plan vectors (and the caller's ops) may be released afterwards; stream order
    // protects the device buffer from the next batch's upload until this batch's kernels ran.
    const int32_t* host_ops = pl.singles ? pl.singles : pl.ops.data();
    if (cudaMemcpyAsync(d_ops, host_ops, (size_t)n * 4 * sizeof(int32_t), cudaMemcpyHostToDevice, s) != cudaSuccess)
      return ABKV_ERR_CUDA;
    if (!pl.singles && cudaMemcpyAsync(d_chain, pl.chain.data(), pl.chain.size() * sizeof(int32_t),
                                       cudaMemcpyHostToDevice, s) != cudaSuccess)
      return ABKV_ERR_CUDA;
    prm.chain = pl.singles ? nullptr : d_chain;
    prm.n_ops = (int)n;
    if (!pl.two_phase) {
      prm.n_chains = pl.n_chains;
      const int64_t warps = (int64_t)pl.n_chains * num_layers;
      const int64_t blocks = (warps * 32 + 255) / 256;
      compact_chain_kernel<<<(unsigned)blocks, 256, 0, s>>>(prm);
    } else {
      prm.n_chains = 0;
      const int64_t warps = n * num_layers * 2;
      const int64_t blocks = (warps * 32 + 255) / 256;
      compact_twophase_kernel<<<(unsigned)blocks, 256, 0, s>>>(prm, 0);
      compact_twophase_kernel<<<(unsigned)blocks, 256, 0, s>>>(prm, 1);
    }
  }
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}

// ---------------------------------------------------------------------------
// Row gather: dst[t][o][j] = src[t][o][keep[j]] for every tensor t, viewed as
// [outer][rows][row_bytes].  This is KVStore.evict(keep_cols)
// (abridgekv/gen_compress.py:72-77: K[:, :, keep_cols, :] for every layer's K
// and V) with all tensors of all layers in one launch.
namespace abkv {
namespace {
constexpr int kMaxGatherTensors = 192;
struct GatherParams {
  const char* src[kMaxGatherTensors];
  char* dst[kMaxGatherTensors];
  const int64_t* keep;
  int32_t* err;
  int64_t outer, src_rows, dst_rows, row_bytes;
  int num_tensors;
};

__global__ void __launch_bounds__(256) gather_rows_kernel(const __grid_constant__ GatherParams p) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t items = (int64_t)p.num_tensors * p.outer * p.dst_rows;
  if (warp >= items) return;
  const int64_t j = warp % p.dst_rows;
  const int64_t o = (warp / p.dst_rows) % p.outer;
  const int t = (int)(warp / (p.dst_rows * p.outer));
  const int64_t r = p.keep[j];
  char* dst = p.dst[t] + (o * p.dst_rows + j) * p.row_bytes;
  const int64_t vecs = p.row_bytes >> 4;
  if (r < 0 || r >= p.src_rows) {
    if (lane == 0) set_error(p.err, ABKV_DEVERR_ROW_OOB);
    for (int64_t v = lane; v < vecs; v += 32) st_cg(dst + 16 * v, make_uint4(0, 0, 0, 0));
    return;
  }
  const char* src = p.src[t] + (o * p.src_rows + r) * p.row_bytes;
  for (int64_t v = lane; v < vecs; v += 32) st_cg(dst + 16 * v, ld_cg(src + 16 * v));
}
// New rows into the paged cache (vLLM's reshape_and_cache_flash, which the backend's
// AttentionImpl.forward runs before attention): token t's K and V rows ([Hkv][D], each head's D
// contiguous, free token / head strides) go to slot slot_mapping[t] = block * page + offset of
// the cache; a negative slot (padding) is skipped.  One warp per (token, K|V), 16-byte vectors.
struct StoreParams {
  const char* src[2];   // key, value
  int64_t src_row[2];   // bytes between tokens
  int64_t src_head[2];  // bytes between heads
  const int64_t* slots;
  char* kv;
  int32_t* err;
  int64_t blk_stride, half_stride, row_bytes, num_slots;
  int T, page, head_vecs;  // head_vecs: 16-byte vectors per head row (D * 2 / 16)
};

__global__ void __launch_bounds__(256) store_kv_kernel(const __grid_constant__ StoreParams p) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= 2 * (int64_t)p.T) return;
  const int t = (int)(warp >> 1), half = (int)(warp & 1);
  const int64_t slot = __ldg(p.slots + t);
  if (slot < 0) return;
  if (slot >= p.num_slots) {
    if (lane == 0) set_error(p.err, ABKV_DEVERR_ROW_OOB);
    return;
  }
  char* dst = p.kv + (slot / p.page) * p.blk_stride + half * p.half_stride + (slot % p.page) * p.row_bytes;
  const char* src = p.src[half] + t * p.src_row[half];
  const int64_t vecs = p.row_bytes >> 4;
  for (int64_t v = lane; v < vecs; v += 32) {
    const int64_t h = v / p.head_vecs, w = v - h * p.head_vecs;
    st_cg(dst + 16 * v, ld_cg(src + h * p.src_head[half] + 16 * w));
  }
}
}  // namespace
}  // namespace abkv

extern "C" int abkv_store_kv(const void* key, int64_t key_row_stride, int64_t key_head_stride, const void* value,
                             int64_t value_row_stride, int64_t value_head_stride, void* kv_cache, int kv_layout,
                             int64_t num_blocks, int page_size, int num_kv_heads, int head_dim,
                             const int64_t* slot_mapping, int T, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (T < 0 || !kv_cache || num_blocks <= 0 || page_size <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      (kv_layout != 0 && kv_layout != 1))
    return ABKV_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < kWsHeader || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return ABKV_ERR_WORKSPACE;
  if (T == 0) return ABKV_OK;
  if (!key || !value || !slot_mapping || key_row_stride <= 0 || value_row_stride <= 0 || key_head_stride <= 0 ||
      value_head_stride <= 0)
    return ABKV_ERR_INVALID_ARG;
  // 16-byte vectors: every head row starts on a 16-byte boundary
  if ((head_dim * 2) % 16 || ((key_row_stride | key_head_stride | value_row_stride | value_head_stride) * 2) % 16 ||
      ((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
        reinterpret_cast<uintptr_t>(kv_cache)) & 15))
    return ABKV_ERR_UNSUPPORTED;
  StoreParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.src[0] = static_cast<const char*>(key);
  prm.src[1] = static_cast<const char*>(value);
  prm.src_row[0] = key_row_stride * 2;
  prm.src_row[1] = value_row_stride * 2;
  prm.src_head[0] = key_head_stride * 2;
  prm.src_head[1] = value_head_stride * 2;
  prm.slots = slot_mapping;
  prm.kv = static_cast<char*>(kv_cache);
  prm.err = static_cast<int32_t*>(workspace);
  prm.row_bytes = (int64_t)num_kv_heads * head_dim * 2;
  const int64_t page_bytes = prm.row_bytes * page_size;
  prm.blk_stride = kv_layout ? page_bytes : 2 * page_bytes;  // [nb][2][page] or [2][nb][page]
  prm.half_stride = kv_layout ? num_blocks * page_bytes : page_bytes;
  prm.num_slots = num_blocks * page_size;
  prm.T = T;
  prm.page = page_size;
  prm.head_vecs = head_dim * 2 / 16;
  const int64_t threads = 2 * (int64_t)T * 32;
  store_kv_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}

extern "C" int abkv_gather_rows(const void* const* src, void* const* dst, int num_tensors, int64_t outer,
                                int64_t src_rows, int64_t dst_rows, int64_t row_bytes, const int64_t* keep,
                                void* workspace, size_t workspace_bytes, void* stream) {
  if (!src || !dst || num_tensors <= 0 || outer <= 0 || src_rows < 0 || dst_rows < 0 || row_bytes <= 0)
    return ABKV_ERR_INVALID_ARG;
  if (row_bytes % 16) return ABKV_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < kWsHeader || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return ABKV_ERR_WORKSPACE;
  if (dst_rows == 0) return ABKV_OK;
  if (!keep) return ABKV_ERR_INVALID_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  GatherParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.keep = keep;
  prm.err = static_cast<int32_t*>(workspace);
  prm.outer = outer;
  prm.src_rows = src_rows;
  prm.dst_rows = dst_rows;
  prm.row_bytes = row_bytes;
  for (int t0 = 0; t0 < num_tensors; t0 += kMaxGatherTensors) {
    const int nt = std::min(kMaxGatherTensors, num_tensors - t0);
    for (int i = 0; i < nt; ++i) {
      if (!src[t0 + i] || !dst[t0 + i]) return ABKV_ERR_INVALID_ARG;
      if ((reinterpret_cast<uintptr_t>(src[t0 + i]) | reinterpret_cast<uintptr_t>(dst[t0 + i])) & 15)
        return ABKV_ERR_INVALID_ARG;
      prm.src[i] = static_cast<const char*>(src[t0 + i]);
      prm.dst[i] = static_cast<char*>(dst[t0 + i]);
    }
    prm.num_tensors = nt;
    const int64_t warps = (int64_t)nt * outer * dst_rows;
    gather_rows_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(prm);
  }
  if (cudaGetLastError() != cudaSuccess) return ABKV_ERR_CUDA;
  return ABKV_OK;
}
