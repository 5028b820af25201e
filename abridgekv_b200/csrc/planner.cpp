// Host-side compaction planner: page tables, free-block queue, span index and
// span -> copy-op planning, bit-exact with the reference's vLLM overlay.
//
//   * FreeQueue / Pool: vLLM's FreeKVCacheBlockQueue + BlockPool semantics
//     (third_party/vllm_overlay/vllm/v1/core/block_pool.py:148-175 init pops
//     the null block 0; get_new_blocks :295-325 = popleft_n from the head;
//     free_blocks :385-399 decrements ref counts and appends the blocks that
//     reach zero, in the given order, to the tail).
//   * Group manager: SingleTypeKVCacheManager.allocate_new_blocks / free
//     (single_type_kv_cache_manager.py:122-187), compact_kv_cache_span
//     (:358-390), _truncate_compacted_blocks (:392-420; trailing blocks are
//     freed in reverse order) and BlockPool.copy_kv_slots (block_pool.py:488-550).
//   * SpanIndex: CompactedSpanIndex (vllm/v1/compacted_spans.py:8-68).
//   * mask_token_span: Scheduler.mask_token_span (core/sched/scheduler.py:2060-2204)
//     including its validation order and messages; copy ops are queued per
//     request, per KV-cache group, as ORDERED batches (one per removal).
//   * finish_block: CompressLMProcessor._compact_response_content for physical
//     per-layer quotas (core/compresslm/processor.py:467-557): the response
//     content span from every group, then [code_start+q, code_end) from the
//     groups of each quota q < K, quotas in increasing order.
#include <algorithm>
#include <array>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "abkv.h"

namespace {

// ---------------------------------------------------------------------------
class FreeQueue {
 public:
  explicit FreeQueue(int n) : prev_(n + 2), next_(n + 2), in_(n, 1), n_(n), size_(n) {
    head_ = n;
    tail_ = n + 1;
    int last = head_;
    for (int i = 0; i < n; ++i) {
      next_[last] = i;
      prev_[i] = last;
      last = i;
    }
    next_[last] = tail_;
    prev_[tail_] = last;
  }
  int size() const { return size_; }
  bool contains(int b) const { return in_[b] != 0; }
  int popleft() {
    const int b = next_[head_];
    unlink(b);
    return b;
  }
  void popleft_n(int k, std::vector<int>* out) {
    for (int i = 0; i < k; ++i) out->push_back(popleft());
  }
  void append(int b) {
    const int last = prev_[tail_];
    next_[last] = b;
    prev_[b] = last;
    next_[b] = tail_;
    prev_[tail_] = b;
    in_[b] = 1;
    ++size_;
  }
  void remove(int b) { unlink(b); }
  void to_vector(std::vector<int>* out) const {
    for (int b = next_[head_]; b != tail_; b = next_[b]) out->push_back(b);
  }

 private:
  void unlink(int b) {
    next_[prev_[b]] = next_[b];
    prev_[next_[b]] = prev_[b];
    in_[b] = 0;
    --size_;
  }
  std::vector<int> prev_, next_;
  std::vector<char> in_;
  int n_, size_, head_, tail_;
};

class Pool {
 public:
  explicit Pool(int n) : q_(n), ref_(n, 0) { null_block_ = q_.popleft(); }
  int null_block() const { return null_block_; }
  int num_free() const { return q_.size(); }
  bool get_new_blocks(int k, std::vector<int>* out) {
    if (k > q_.size()) return false;
    const size_t base = out->size();
    q_.popleft_n(k, out);
    for (size_t i = base; i < out->size(); ++i) ref_[(*out)[i]] += 1;
    return true;
  }
  void free_blocks(const std::vector<int>& ordered) {
    for (int b : ordered) ref_[b] -= 1;
    for (int b : ordered)
      if (ref_[b] == 0 && b != null_block_) q_.append(b);
  }
  void free_queue(std::vector<int>* out) const { q_.to_vector(out); }
  int num_blocks() const { return (int)ref_.size(); }

 private:
  FreeQueue q_;
  std::vector<int> ref_;
  int null_block_;
};

// ---------------------------------------------------------------------------
struct SpanIndex {
  std::vector<std::pair<int64_t, int64_t>> spans;
  std::vector<int64_t> starts, cumulative, gap_physical, gap_logical;
  int64_t total_removed = 0;

  void rebuild() {
    starts.clear();
    cumulative.clear();
    gap_physical.assign(1, 0);
    gap_logical.assign(1, 0);
    total_removed = 0;
    for (auto& s : spans) {
      starts.push_back(s.first);
      total_removed += s.second - s.first;
      cumulative.push_back(total_removed);
      gap_physical.push_back(s.second - total_removed);
      gap_logical.push_back(s.second);
    }
  }
  // index of the last start <= x, or -1
  int rfind(const std::vector<int64_t>& v, int64_t x) const {
    return (int)(std::upper_bound(v.begin(), v.end(), x) - v.begin()) - 1;
  }
  int64_t logical_to_physical(int64_t pos) const {
    if (starts.empty()) return pos;
    const int idx = rfind(starts, pos);
    if (idx < 0) return pos;
    const int64_t end = spans[idx].second;
    if (pos >= end) return pos - cumulative[idx];
    const int64_t prev = idx > 0 ? cumulative[idx - 1] : 0;
    return pos - prev - (pos - starts[idx]);
  }
  int64_t physical_to_logical(int64_t phys) const {
    const int idx = rfind(gap_physical, phys);
    return gap_logical[idx] + (phys - gap_physical[idx]);
  }
  bool is_active(int64_t pos) const {
    if (starts.empty()) return true;
    const int idx = rfind(starts, pos);
    if (idx < 0) return true;
    return pos >= spans[idx].second;
  }
};

std::vector<std::pair<int64_t, int64_t>> merge_spans(std::vector<std::pair<int64_t, int64_t>> s) {
  std::vector<std::pair<int64_t, int64_t>> out;
  if (s.empty()) return out;
  std::sort(s.begin(), s.end());
  out.push_back(s[0]);
  for (size_t i = 1; i < s.size(); ++i) {
    if (s[i].first <= out.back().second) {
      out.back().second = std::max(out.back().second, s[i].second);
    } else {
      out.push_back(s[i]);
    }
  }
  return out;
}

}  // namespace

struct abkv_planner {
  int block_size = 16;
  int num_groups = 1;
  Pool pool;
  // per group: request -> block list
  std::vector<std::map<int64_t, std::vector<int>>> req_blocks;
  struct Req {
    int64_t num_computed = 0;
    std::vector<SpanIndex> groups;
  };
  std::map<int64_t, Req> reqs;
  // pending worker-side operations
  std::map<int64_t, std::vector<std::vector<std::vector<std::array<int32_t, 4>>>>> pending_ops;
  std::map<int64_t, std::vector<int32_t>> pending_trunc;

  abkv_planner(int n, int bs, int g) : block_size(bs), num_groups(g), pool(n), req_blocks(g) {}

  // SingleTypeKVCacheManager.allocate_new_blocks
  int allocate(int g, int64_t req, int64_t num_tokens) {
    auto& blocks = req_blocks[g][req];
    const int64_t need = (num_tokens + block_size - 1) / block_size - (int64_t)blocks.size();
    if (need <= 0) return ABKV_OK;
    std::vector<int> fresh;
    if (!pool.get_new_blocks((int)need, &fresh)) return ABKV_ERR_NO_BLOCKS;
    blocks.insert(blocks.end(), fresh.begin(), fresh.end());
    return ABKV_OK;
  }

  // SingleTypeKVCacheManager._truncate_compacted_blocks
  int truncate(std::vector<int>& blocks, int64_t n_active) {
    const int64_t needed = (n_active + block_size - 1) / block_size;
    std::vector<int> to_free;
    int freed = 0;
    for (int64_t i = needed; i < (int64_t)blocks.size(); ++i) {
      if (blocks[i] != pool.null_block()) {
        to_free.push_back(blocks[i]);
        blocks[i] = pool.null_block();
        ++freed;
      }
    }
    if ((int64_t)blocks.size() > needed) blocks.resize(needed);
    if (!to_free.empty()) {
      std::reverse(to_free.begin(), to_free.end());
      pool.free_blocks(to_free);
    }
    return freed;
  }

  // SingleTypeKVCacheManager.compact_kv_cache_span + BlockPool.copy_kv_slots
  int compact_span(int g, int64_t req, int64_t start, int64_t end, int64_t n_active, int* freed,
                   std::vector<std::array<int32_t, 4>>* ops) {
    *freed = 0;
    auto it = req_blocks[g].find(req);
    if (it == req_blocks[g].end()) return ABKV_OK;
    if (!(0 <= start && start < end && end <= n_active)) return ABKV_ERR_SPAN;
    auto& blocks = it->second;
    if (blocks.empty()) return ABKV_OK;
    const int64_t removed = end - start;
    if ((n_active + block_size - 1) / block_size > (int64_t)blocks.size()) return ABKV_ERR_SPAN;
    ops->reserve(ops->size() + (size_t)(n_active - end));
    // slot s moves to s - removed, for s in [end, n_active): block and offset of both advance by one
    // slot per op (no division per op)
    int64_t sb = end / block_size, d0 = end - removed, db = d0 / block_size;
    int32_t so = (int32_t)(end % block_size), dof = (int32_t)(d0 % block_size);
    for (int64_t s = end; s < n_active; ++s) {
      ops->push_back({blocks[sb], so, blocks[db], dof});
      if (++so == block_size) {
        so = 0;
        ++sb;
      }
      if (++dof == block_size) {
        dof = 0;
        ++db;
      }
    }
    *freed = truncate(blocks, n_active - removed);
    return ABKV_OK;
  }

  void fail(abkv_span_result_t* r, const std::string& msg) {
    r->success = 0;
    r->tokens_removed = 0;
    r->blocks_freed = 0;
    std::snprintf(r->error_message, sizeof(r->error_message), "%s", msg.c_str());
  }

  // Scheduler.mask_token_span
  int mask_token_span(int64_t req, int64_t start, int64_t end, const int32_t* groups, int n_groups,
                      abkv_span_result_t* r) {
    std::memset(r, 0, sizeof(*r));
    auto rit = reqs.find(req);
    if (rit == reqs.end()) {
      fail(r, "Request " + std::to_string(req) + " not found");
      return ABKV_OK;
    }
    Req& rq = rit->second;
    if (start < 0 || end <= start) {
      fail(r, "Invalid span: must have 0 <= start < end");
      return ABKV_OK;
    }
    if (end > rq.num_computed) {
      fail(r, "end_position (" + std::to_string(end) + ") exceeds computed tokens (" +
                  std::to_string(rq.num_computed) + ")");
      return ABKV_OK;
    }
    const int64_t tokens = end - start;
    std::vector<int> target;
    if (groups == nullptr) {
      for (int g = 0; g < num_groups; ++g) target.push_back(g);
    } else {
      target.assign(groups, groups + n_groups);
      std::sort(target.begin(), target.end());
      target.erase(std::unique(target.begin(), target.end()), target.end());
    }
    struct Plan { int g; int64_t ps, pe, n_active; };
    std::vector<Plan> plans;
    for (int g : target) {
      if (g < 0 || g >= num_groups) {
        fail(r, "KV cache group " + std::to_string(g) + " out of range");
        return ABKV_OK;
      }
      const SpanIndex& si = rq.groups[g];
      for (auto& s : si.spans) {
        if (start < s.second && end > s.first) {
          fail(r, "Cannot compact an already-removed token span (group " + std::to_string(g) + ")");
          return ABKV_OK;
        }
      }
      const int64_t ps = si.logical_to_physical(start), pe = si.logical_to_physical(end);
      if (pe - ps != tokens) {
        fail(r, "Logical span does not map to one active physical span (group " + std::to_string(g) +
                    ")");
        return ABKV_OK;
      }
      const int64_t n_active = rq.num_computed - si.total_removed;
      if (n_active == tokens) {
        fail(r, "Cannot compact: all tokens would be removed");
        return ABKV_OK;
      }
      plans.push_back({g, ps, pe, n_active});
    }
    int total_freed = 0;
    for (auto& pl : plans) {
      int freed = 0;
      std::vector<std::array<int32_t, 4>> ops;
      const int st = compact_span(pl.g, req, pl.ps, pl.pe, pl.n_active, &freed, &ops);
      if (st != ABKV_OK) return st;  // unreachable after the validation above
      total_freed += freed;
      if (!ops.empty()) {
        auto& per_group = pending_ops[req];
        if (per_group.empty()) per_group.resize(num_groups);
        per_group[pl.g].push_back(std::move(ops));
      }
      SpanIndex& si = rq.groups[pl.g];
      auto spans = si.spans;
      spans.push_back({start, end});
      si.spans = merge_spans(spans);
      si.rebuild();
    }
    std::vector<int32_t> trunc(num_groups);
    for (int g = 0; g < num_groups; ++g) {
      auto it = req_blocks[g].find(req);
      trunc[g] = it == req_blocks[g].end() ? 0 : (int32_t)it->second.size();
    }
    pending_trunc[req] = trunc;
    r->success = 1;
    r->tokens_removed = tokens;
    r->blocks_freed = total_freed;
    return ABKV_OK;
  }
};

namespace {
abkv_planner::Req* find_req(abkv_planner* p, int64_t req) {
  auto it = p->reqs.find(req);
  return it == p->reqs.end() ? nullptr : &it->second;
}
}  // namespace

// ---------------------------------------------------------------------------
extern "C" {

abkv_planner_t* abkv_planner_create(int num_blocks, int block_size, int num_groups) {
  if (num_blocks < 1 || block_size < 1 || num_groups < 1) return nullptr;
  try {
    return new abkv_planner(num_blocks, block_size, num_groups);
  } catch (...) {
    return nullptr;
  }
}

void abkv_planner_destroy(abkv_planner_t* p) { delete p; }

int abkv_planner_add_request(abkv_planner_t* p, int64_t req) {
  if (!p) return ABKV_ERR_INVALID_ARG;
  if (p->reqs.count(req)) return ABKV_ERR_INVALID_ARG;
  abkv_planner::Req r;
  r.groups.resize(p->num_groups);
  for (auto& g : r.groups) g.rebuild();
  p->reqs[req] = std::move(r);
  return ABKV_OK;
}

int abkv_planner_set_num_computed(abkv_planner_t* p, int64_t req, int64_t num_computed_tokens) {
  if (!p || num_computed_tokens < 0) return ABKV_ERR_INVALID_ARG;
  auto* r = find_req(p, req);
  if (!r) return ABKV_ERR_INVALID_ARG;
  r->num_computed = num_computed_tokens;
  return ABKV_OK;
}

int abkv_planner_allocate_slots(abkv_planner_t* p, int64_t req, int64_t num_tokens) {
  // KVCacheManager.allocate_slots deducts each group's compacted tokens
  // (kv_cache_manager.py:281-299), then every group allocates in order
  // (kv_cache_coordinator.py:126-152).
  if (!p || num_tokens < 0) return ABKV_ERR_INVALID_ARG;
  auto* r = find_req(p, req);
  if (!r) return ABKV_ERR_INVALID_ARG;
  int64_t need_blocks = 0;
  for (int g = 0; g < p->num_groups; ++g) {
    const int64_t n = num_tokens - r->groups[g].total_removed;
    auto it = p->req_blocks[g].find(req);
    const int64_t have = it == p->req_blocks[g].end() ? 0 : (int64_t)it->second.size();
    // summed unclamped, as get_num_blocks_to_allocate does (kv_cache_coordinator.py:70-105)
    need_blocks += (n + p->block_size - 1) / p->block_size - have;
  }
  if (need_blocks > p->pool.num_free()) return ABKV_ERR_NO_BLOCKS;
  for (int g = 0; g < p->num_groups; ++g) {
    const int st = p->allocate(g, req, num_tokens - r->groups[g].total_removed);
    if (st != ABKV_OK) return st;
  }
  return ABKV_OK;
}

int abkv_planner_free_request(abkv_planner_t* p, int64_t req) {
  // SingleTypeKVCacheManager.free: blocks freed in reverse order, group by group.
  if (!p) return ABKV_ERR_INVALID_ARG;
  for (int g = 0; g < p->num_groups; ++g) {
    auto it = p->req_blocks[g].find(req);
    if (it == p->req_blocks[g].end()) continue;
    std::vector<int> rev(it->second.rbegin(), it->second.rend());
    p->req_blocks[g].erase(it);
    p->pool.free_blocks(rev);
  }
  p->reqs.erase(req);
  p->pending_ops.erase(req);
  p->pending_trunc.erase(req);
  return ABKV_OK;
}

int abkv_planner_mask_token_span(abkv_planner_t* p, int64_t req, int64_t start, int64_t end,
                                 const int32_t* groups, int num_groups_given,
                                 abkv_span_result_t* result) {
  if (!p || !result) return ABKV_ERR_INVALID_ARG;
  if (groups && num_groups_given < 0) return ABKV_ERR_INVALID_ARG;
  return p->mask_token_span(req, start, end, groups, num_groups_given, result);
}

int abkv_planner_finish_block(abkv_planner_t* p, int64_t req, int64_t resp_start, int64_t resp_end,
                              int64_t code_start, int64_t code_end, const int32_t* group_quotas,
                              int num_groups, int num_code_tokens, abkv_span_result_t* result) {
  if (!p || !result || !group_quotas || num_groups != p->num_groups) return ABKV_ERR_INVALID_ARG;
  if (code_end - code_start != num_code_tokens) return ABKV_ERR_INVALID_ARG;
  std::memset(result, 0, sizeof(*result));
  int removed = 0, freed = 0;
  if (resp_end > resp_start) {
    abkv_span_result_t r;
    p->mask_token_span(req, resp_start, resp_end, nullptr, 0, &r);
    if (!r.success) {
      *result = r;
      return ABKV_ERR_SPAN;
    }
    removed += r.tokens_removed;
    freed += r.blocks_freed;
  }
  std::vector<int> quotas(group_quotas, group_quotas + num_groups);
  std::vector<int> distinct = quotas;
  std::sort(distinct.begin(), distinct.end());
  distinct.erase(std::unique(distinct.begin(), distinct.end()), distinct.end());
  for (int q : distinct) {
    if (q >= num_code_tokens) continue;
    std::vector<int32_t> gs;
    for (int g = 0; g < num_groups; ++g)
      if (quotas[g] == q) gs.push_back(g);
    abkv_span_result_t r;
    p->mask_token_span(req, code_start + q, code_end, gs.data(), (int)gs.size(), &r);
    if (!r.success) {
      *result = r;
      return ABKV_ERR_SPAN;
    }
    removed += r.tokens_removed;
    freed += r.blocks_freed;
  }
  result->success = 1;
  result->tokens_removed = removed;
  result->blocks_freed = freed;
  return ABKV_OK;
}

int abkv_planner_block_table(const abkv_planner_t* p, int64_t req, int group, int32_t* out, int cap,
                             int* n) {
  if (!p || !n || group < 0 || group >= p->num_groups) return ABKV_ERR_INVALID_ARG;
  auto it = p->req_blocks[group].find(req);
  const int len = it == p->req_blocks[group].end() ? 0 : (int)it->second.size();
  *n = len;
  if (len > cap || (len && !out)) return ABKV_ERR_INVALID_ARG;
  for (int i = 0; i < len; ++i) out[i] = it->second[i];
  return ABKV_OK;
}

int abkv_planner_free_queue(const abkv_planner_t* p, int32_t* out, int cap, int* n) {
  if (!p || !n) return ABKV_ERR_INVALID_ARG;
  std::vector<int> v;
  p->pool.free_queue(&v);
  *n = (int)v.size();
  if ((int)v.size() > cap || (!v.empty() && !out)) return ABKV_ERR_INVALID_ARG;
  std::copy(v.begin(), v.end(), out);
  return ABKV_OK;
}

int abkv_planner_num_free(const abkv_planner_t* p) { return p ? p->pool.num_free() : -1; }

int abkv_planner_span_map(const abkv_planner_t* p, int64_t req, int group, int64_t position,
                          int to_physical, int64_t* out) {
  if (!p || !out || group < 0 || group >= p->num_groups) return ABKV_ERR_INVALID_ARG;
  auto it = p->reqs.find(req);
  if (it == p->reqs.end()) return ABKV_ERR_INVALID_ARG;
  const SpanIndex& si = it->second.groups[group];
  *out = to_physical ? si.logical_to_physical(position) : si.physical_to_logical(position);
  return ABKV_OK;
}

int abkv_planner_compacted_spans(const abkv_planner_t* p, int64_t req, int group, int64_t* out,
                                 int cap, int* n) {
  if (!p || !n || group < 0 || group >= p->num_groups) return ABKV_ERR_INVALID_ARG;
  auto it = p->reqs.find(req);
  if (it == p->reqs.end()) return ABKV_ERR_INVALID_ARG;
  const auto& spans = it->second.groups[group].spans;
  *n = (int)spans.size();
  if ((int)spans.size() > cap || (!spans.empty() && !out)) return ABKV_ERR_INVALID_ARG;
  for (size_t i = 0; i < spans.size(); ++i) {
    out[2 * i] = spans[i].first;
    out[2 * i + 1] = spans[i].second;
  }
  return ABKV_OK;
}

int abkv_planner_pending_requests(const abkv_planner_t* p, int64_t* out, int cap, int* n) {
  if (!p || !n) return ABKV_ERR_INVALID_ARG;
  *n = (int)p->pending_ops.size();
  if (*n > cap || (*n && !out)) return ABKV_ERR_INVALID_ARG;
  int i = 0;
  for (auto& kv : p->pending_ops) out[i++] = kv.first;
  return ABKV_OK;
}

int abkv_planner_pending_num_batches(const abkv_planner_t* p, int64_t req, int group) {
  if (!p || group < 0 || group >= p->num_groups) return -1;
  auto it = p->pending_ops.find(req);
  if (it == p->pending_ops.end() || it->second.empty()) return 0;
  return (int)it->second[group].size();
}

int abkv_planner_pending_batch(const abkv_planner_t* p, int64_t req, int group, int batch,
                               int32_t* ops, int cap_ops, int* n_ops) {
  if (!p || !n_ops || group < 0 || group >= p->num_groups) return ABKV_ERR_INVALID_ARG;
  auto it = p->pending_ops.find(req);
  if (it == p->pending_ops.end() || it->second.empty()) return ABKV_ERR_INVALID_ARG;
  const auto& batches = it->second[group];
  if (batch < 0 || batch >= (int)batches.size()) return ABKV_ERR_INVALID_ARG;
  const auto& b = batches[batch];
  *n_ops = (int)b.size();
  if ((int)b.size() > cap_ops || (!b.empty() && !ops)) return ABKV_ERR_INVALID_ARG;
  for (size_t i = 0; i < b.size(); ++i)
    for (int k = 0; k < 4; ++k) ops[4 * i + k] = b[i][k];
  return ABKV_OK;
}

int abkv_planner_pending_truncation(const abkv_planner_t* p, int64_t req, int32_t* out, int cap,
                                    int* n) {
  if (!p || !n) return ABKV_ERR_INVALID_ARG;
  auto it = p->pending_trunc.find(req);
  if (it == p->pending_trunc.end()) {
    *n = 0;
    return ABKV_OK;
  }
  *n = (int)it->second.size();
  if (*n > cap || !out) return ABKV_ERR_INVALID_ARG;
  std::copy(it->second.begin(), it->second.end(), out);
  return ABKV_OK;
}

int abkv_planner_pending_export(const abkv_planner_t* p, int64_t* req_ids, int32_t* group_batches,
                                int32_t* batch_ops, int32_t* ops, int cap_reqs, int cap_batches, int cap_ops,
                                int* n_reqs, int* n_batches, int* n_ops) {
  if (!p || !n_reqs || !n_batches || !n_ops) return ABKV_ERR_INVALID_ARG;
  const int G = p->num_groups;
  int64_t nr = 0, nbt = 0, no = 0;
  for (const auto& kv : p->pending_ops) {
    ++nr;
    for (const auto& batches : kv.second) {
      nbt += (int64_t)batches.size();
      for (const auto& b : batches) no += (int64_t)b.size();
    }
  }
  if (nr > INT32_MAX || nbt > INT32_MAX || no > INT32_MAX / 4) return ABKV_ERR_INVALID_ARG;
  *n_reqs = (int)nr;
  *n_batches = (int)nbt;
  *n_ops = (int)no;
  const bool query = !req_ids && !group_batches && !batch_ops && !ops && !cap_reqs && !cap_batches && !cap_ops;
  if (query) return ABKV_OK;
  if (nr > cap_reqs || nbt > cap_batches || no > cap_ops || (nr && (!req_ids || !group_batches)) ||
      (nbt && !batch_ops) || (no && !ops))
    return ABKV_ERR_INVALID_ARG;
  int64_t r = 0, bi = 0, oi = 0;
  for (const auto& kv : p->pending_ops) {
    req_ids[r] = kv.first;
    for (int g = 0; g < G; ++g) {
      const bool has = g < (int)kv.second.size();
      group_batches[r * G + g] = has ? (int32_t)kv.second[g].size() : 0;
      if (!has) continue;
      for (const auto& b : kv.second[g]) {
        batch_ops[bi++] = (int32_t)b.size();
        for (const auto& op : b) {
          for (int k = 0; k < 4; ++k) ops[4 * oi + k] = op[k];
          ++oi;
        }
      }
    }
    ++r;
  }
  return ABKV_OK;
}

int abkv_planner_pending_trunc_export(const abkv_planner_t* p, int64_t* req_ids, int32_t* counts, int cap,
                                      int* n) {
  if (!p || !n) return ABKV_ERR_INVALID_ARG;
  const int G = p->num_groups;
  *n = (int)p->pending_trunc.size();
  if (!req_ids && !counts && !cap) return ABKV_OK;
  if (*n > cap || (*n && (!req_ids || !counts))) return ABKV_ERR_INVALID_ARG;
  int r = 0;
  for (const auto& kv : p->pending_trunc) {
    req_ids[r] = kv.first;
    for (int g = 0; g < G; ++g) counts[r * G + g] = g < (int)kv.second.size() ? kv.second[g] : -1;
    ++r;
  }
  return ABKV_OK;
}

int abkv_planner_clear_pending(abkv_planner_t* p) {
  if (!p) return ABKV_ERR_INVALID_ARG;
  p->pending_ops.clear();
  p->pending_trunc.clear();
  return ABKV_OK;
}

}  // extern "C"
