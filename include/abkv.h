/*
 * abkv.h -- C ABI of libabkv.so, the B200 (sm_100a) implementation of
 * AbridgeKV's compressed-cache attention path.
 *
 * Conventions shared by every entry point:
 *   - Return value: 0 (ABKV_OK) on success, otherwise one of ABKV_ERR_*.
 *     Host-side validation happens before any launch; a call that fails
 *     validation launches nothing and leaves every buffer untouched.
 *   - Device pointers are raw CUDA device addresses; host pointers are plain
 *     host memory (read before the call returns).  No torch types cross
 *     this boundary.
 *   - bf16 tensors are passed as `void*` holding IEEE bfloat16 values.
 *   - `stream` is a cudaStream_t (passed as void* so this header does not
 *     need the CUDA headers).  All launches of one call go to that stream in
 *     order; nothing synchronises the host unless stated.
 *   - Nothing here allocates device memory.  Scratch space is a caller-owned
 *     workspace whose minimum size is reported by the matching *_workspace_size
 *     function.  Byte 0..3 of every workspace is a device error word that the
 *     kernels OR error bits into (read it with abkv_workspace_error).
 *   - Entry points are reentrant: no global mutable state, except the fixed
 *     scratch array of abkv_decode_noalloc (whose calls must be serialised;
 *     see there).
 */
#ifndef ABKV_H_
#define ABKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define ABKV_OK 0
#define ABKV_ERR_INVALID_ARG 1   /* a size, shape or pointer failed validation */
#define ABKV_ERR_WORKSPACE 2     /* workspace missing or smaller than required */
#define ABKV_ERR_UNSUPPORTED 3   /* shape outside what the kernels implement   */
#define ABKV_ERR_CUDA 4          /* a CUDA runtime call failed                 */
#define ABKV_ERR_PAGE_OOB 5      /* device: page id outside [0, num_blocks)    */
#define ABKV_ERR_SEQ_OOB 6       /* device: seq_len exceeds its block-table row*/
#define ABKV_ERR_SPAN 7          /* host planner: span rejected                */
#define ABKV_ERR_NO_BLOCKS 8     /* host planner: free queue exhausted         */
#define ABKV_ERR_TIMEOUT 9       /* device: a bounded wait gave up             */
#define ABKV_ERR_SCRATCH_LIMIT 10 /* request needs more than the fixed scratch of
                                     abkv_decode_noalloc (32 MiB)               */

/* Device error-word bits (OR-ed by kernels into workspace bytes 0..3). */
#define ABKV_DEVERR_PAGE_OOB 0x1
#define ABKV_DEVERR_SEQ_OOB 0x2
#define ABKV_DEVERR_TIMEOUT 0x4
#define ABKV_DEVERR_ROW_OOB 0x8
#define ABKV_DEVERR_RANGE 0x10   /* code step: query rows or exclusion range invalid */

/* Human-readable name of a status code (static string, never NULL). */
const char* abkv_status_string(int status);

/* Library version string, e.g. "abkv 0.1 sm_100a". */
const char* abkv_version(void);

/* Copy the device error word of `workspace` to *host_error and clear it.
 * Synchronises `stream`.  Returns ABKV_OK or ABKV_ERR_CUDA. */
int abkv_workspace_error(void* workspace, void* stream, int32_t* host_error);

/* ========================================================================
 * 1. Paged decode attention over per-layer (per-quota-group) page tables.
 *
 * Replaces the decode attention that the reference runs per layer through
 * FlashInfer's BatchDecodeWithPagedKVCacheWrapper over a KV-cache group's
 * block table and physical seq_lens
 *   (third_party/vllm_overlay/vllm/v1/worker/gpu_model_runner.py:1672-1681,
 *    2184-2204; patch_stock_flashinfer.py:120-129),
 * whose in-repo PyTorch image is PackedKVSidecar._attend_decode_batched
 *   (third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:564-616).
 *
 * One call covers `num_layers` layers (1 for a per-layer vLLM-style call).
 * For layer l and sequence b, the query row q_l[b] ([num_q_heads][head_dim])
 * attends to physical KV rows 0 .. seq_lens_l[b]-1, row r living at
 *   kv_l[block_table_l[b*bt_stride_l + r/page_size]][0 (K) | 1 (V)]
 *       [r % page_size][kv_head][:]
 * i.e. the FlashInfer NHD paged layout
 *   kv_l: [num_blocks_l][2][page_size][num_kv_heads][head_dim] bf16.
 * Query head h reads KV head h / (num_q_heads / num_kv_heads).
 * out_l[b][h][:] = softmax(q.K^T * scale) V, fp32 softmax, bf16 output.
 * A sequence with seq_len 0 gets an all-zero output row.
 *
 * All per-layer arguments are HOST arrays of length num_layers holding
 * device pointers (q, kv, block_tables, seq_lens, out) or host integers
 * (bt_strides, num_blocks).
 *
 * Supported: head_dim 64 or 128; num_kv_heads in {1,2,4,8}; group size
 * num_q_heads/num_kv_heads in 1..8; page_size a multiple of 16;
 * max_pages_per_seq >= every ceil(seq_len/page_size) (it bounds the launch
 * grid).  chunk_tokens = tokens per split-KV work item (0 = automatic; else
 * a multiple of 16 and of page_size).
 * ====================================================================== */
size_t abkv_decode_workspace_size(int num_layers, int num_seqs, int num_q_heads,
                                  int head_dim, int page_size,
                                  int max_pages_per_seq, int chunk_tokens);

int abkv_decode(const void* const* q, const void* const* kv,
                const int32_t* const* block_tables, const int64_t* bt_strides,
                const int32_t* const* seq_lens, const int64_t* num_blocks,
                void* const* out, int num_layers, int num_seqs,
                int num_q_heads, int num_kv_heads, int head_dim,
                int page_size, int max_pages_per_seq, float scale,
                int chunk_tokens, void* workspace, size_t workspace_bytes,
                void* stream);

/* Decode that allocates nothing and takes no workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory when
 * they decode (an engine that has reserved all of HBM for its KV cache, an
 * allocator that must not be touched from this thread).  Arguments and
 * results are those of abkv_decode; the split-KV scratch instead lives in a
 * 32 MiB device array inside this library that every GPU loading the library
 * keeps until the process exits.
 *   - The first call on a device looks up that array's device address (with
 *     the device current) and caches it; make that first call before any
 *     stream capture.  The cached address belongs to the device's primary
 *     context: after that context is reset or destroyed
 *     (cudaDeviceReset) it is stale, and the library must be unloaded and
 *     loaded again before the next call.
 *   - A request whose scratch would exceed 32 MiB is rejected with
 *     ABKV_ERR_SCRATCH_LIMIT before anything runs (the scratch grows with
 *     num_layers x num_seqs x split-KV chunks x num_q_heads x head_dim x 4 B;
 *     per-layer calls or a larger chunk_tokens keep it small).
 *   - Every call shares the array and it keeps the last call's contents: each
 *     call clears its counters first, and calls that overlap on the GPU (two
 *     streams, or two host threads) race on it and must be serialised.
 *   - device_error: optional DEVICE int32 that receives the call's device
 *     error bits (ABKV_DEVERR_*); NULL to ignore them. */
int abkv_decode_noalloc(const void* const* q, const void* const* kv,
                        const int32_t* const* block_tables,
                        const int64_t* bt_strides,
                        const int32_t* const* seq_lens,
                        const int64_t* num_blocks, void* const* out,
                        int num_layers, int num_seqs, int num_q_heads,
                        int num_kv_heads, int head_dim, int page_size,
                        int max_pages_per_seq, float scale, int chunk_tokens,
                        int32_t* device_error, void* stream);

/* Decode with a packed sidecar of per-head code quotas.
 *
 * Replaces PackedKVSidecar._attend_decode_batched with sidecar pages
 * (third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:526-616;
 * page layout PackedKVLayout, :13-155): every compressed block of a request
 * stores, per layer, one packed page [2][slots][head_dim] bf16 in which KV head
 * h owns slots [off_h, off_h + quotas[h]) (off_h = sum of the earlier quotas).
 * For KV head h of request b the keys are, in order, head h's slots of each of
 * the request's page_count[b] pages (ids page_table[b][0..]), then main rows
 * [0, seq_lens[b]) of the paged cache as in abkv_decode.  One descriptor per
 * layer; pages == NULL = no sidecar for that layer.  quotas: multiples of 16.
 * Workspace: abkv_decode_packed_workspace_size with max_side_rows = the largest
 * page_table_stride * slots over the layers. */
typedef struct abkv_sidecar {
  const void* pages;           /* DEVICE [num_pages][2][slots][head_dim] bf16 */
  const int32_t* page_table;   /* DEVICE [B][page_table_stride] page ids     */
  const int32_t* page_count;   /* DEVICE [B] sidecar pages of each request  */
  int64_t page_table_stride;
  int64_t num_pages;
  int slots;                   /* sum of quotas                              */
  int quotas[8];               /* per KV head (num_kv_heads entries used)    */
} abkv_sidecar_t;

size_t abkv_decode_packed_workspace_size(int num_layers, int num_seqs,
                                         int num_q_heads, int head_dim,
                                         int page_size, int max_pages_per_seq,
                                         int chunk_tokens, int64_t max_side_rows);

int abkv_decode_packed(const void* const* q, const void* const* kv,
                       const int32_t* const* block_tables,
                       const int64_t* bt_strides,
                       const int32_t* const* seq_lens,
                       const int64_t* num_blocks, void* const* out,
                       int num_layers, int num_seqs, int num_q_heads,
                       int num_kv_heads, int head_dim, int page_size,
                       int max_pages_per_seq, float scale, int chunk_tokens,
                       const abkv_sidecar_t* sidecars, void* workspace,
                       size_t workspace_bytes, void* stream);

/* KV-head-sharded decode with the all-gather fused into the epilogue.
 *
 * BASELINE config 5's optional mode (one process per GPU, rank r holding KV
 * heads [r*Hkv, (r+1)*Hkv) of every sequence; num_q_heads / num_kv_heads are
 * this rank's share).  Where the reference's layout would follow the
 * attention with an all-gather of the [B, world*Hq, D] head outputs, this
 * call's epilogue stores each output row straight into every rank's gather
 * buffer (peer memory mapped with abkv_peer_open), then its last CTA raises
 * this rank's flag (= epoch) in every rank's flag area and waits until all
 * ranks' flags have reached epoch, so when the launch completes the full
 * [B][world*Hq][D] output of every layer is in this rank's buffer.
 *
 * Every rank calls it with the same layers, shapes and epoch, in the same
 * order (like a collective); epochs start at 1 and increase by one per call.
 * Gather buffer layout (identical on all ranks): ABKV_GATHER_FLAG_BYTES of
 * flags (zero at allocation), then the output slots; out[l] must point into
 * this rank's buffer past the flags, at the same offset on every rank, each
 * slot [num_seqs][hq_total][head_dim] contiguous.  A peer that does not arrive
 * within timeout_us sets ABKV_DEVERR_TIMEOUT in the workspace error word; the
 * kernel still returns.  Other arguments as abkv_decode. */
#define ABKV_GATHER_FLAG_BYTES 256
#define ABKV_MAX_PEERS 8
typedef struct abkv_gather {
  void* rank_buffers[ABKV_MAX_PEERS]; /* every rank's gather buffer, as mapped in
                                         this process (index = rank)           */
  size_t buffer_bytes;                /* size of each gather buffer            */
  int world;                          /* ranks, 1..ABKV_MAX_PEERS              */
  int rank;                           /* this rank                             */
  int hq_total;                       /* world * num_q_heads                   */
  uint32_t epoch;                     /* this call's barrier epoch (>= 1)      */
  uint32_t timeout_us;                /* barrier wait limit; 0 = 5 s           */
} abkv_gather_t;

int abkv_decode_gather(const void* const* q, const void* const* kv,
                       const int32_t* const* block_tables,
                       const int64_t* bt_strides,
                       const int32_t* const* seq_lens,
                       const int64_t* num_blocks, void* const* out,
                       int num_layers, int num_seqs, int num_q_heads,
                       int num_kv_heads, int head_dim, int page_size,
                       int max_pages_per_seq, float scale, int chunk_tokens,
                       const abkv_gather_t* gather, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Peer-visible buffers (CUDA IPC; no multicast object).  abkv_peer_alloc
 * allocates `bytes` (>= ABKV_GATHER_FLAG_BYTES) of zeroed device memory on the
 * current device and writes its ABKV_PEER_HANDLE_BYTES-byte handle;
 * abkv_peer_open maps another process's buffer from its handle;
 * abkv_peer_close unmaps it; abkv_peer_free releases an allocation. */
#define ABKV_PEER_HANDLE_BYTES 64
int abkv_peer_alloc(size_t bytes, void** ptr, unsigned char* handle);
int abkv_peer_open(const unsigned char* handle, void** ptr);
int abkv_peer_close(void* ptr);
int abkv_peer_free(void* ptr);


/* ========================================================================
 * 2. Compaction planner (host C++): page tables, free-block queue, span
 *    index and span -> copy-op planning, bit-exact with the reference.
 *
 * One planner = one vLLM KV-cache manager with `num_groups` KV-cache groups
 * (one per distinct code quota under physical per-layer quotas) sharing one
 * block pool of `num_blocks` pages of `block_size` rows.  Block 0 is the null
 * block and is never handed out.  Request ids are caller-chosen int64 keys.
 *
 * Replaces (file:line in the reference's vLLM overlay, vllm/v1/...):
 *   abkv_planner_create          BlockPool.__init__ (core/block_pool.py:148-175)
 *   abkv_planner_allocate_slots  KVCacheManager.allocate_slots' per-group
 *                                compacted-token deduction + allocate_new_blocks
 *                                (core/kv_cache_manager.py:281-299,
 *                                 core/single_type_kv_cache_manager.py:122-145)
 *   abkv_planner_free_request    SingleTypeKVCacheManager.free (:176-187)
 *   abkv_planner_mask_token_span Scheduler.mask_token_span
 *                                (core/sched/scheduler.py:2060-2204) ->
 *                                compact_kv_cache_span_group -> compact_kv_cache_span
 *                                (single_type_kv_cache_manager.py:358-420) ->
 *                                BlockPool.copy_kv_slots (block_pool.py:488-550)
 *   abkv_planner_finish_block    CompressLMProcessor._compact_response_content,
 *                                physical-quota branch (core/compresslm/processor.py:467-557)
 *   abkv_planner_span_map        CompactedSpanIndex.logical_to_physical /
 *                                physical_to_logical (compacted_spans.py:54-68)
 * Like the reference, mask_token_span reports a rejected span in the result
 * (success = 0, error_message set) and returns ABKV_OK; it never partially
 * applies a rejected span.  Copy ops (src_block, src_off, dst_block, dst_off)
 * are queued per request and per group as ORDERED batches, one per removal,
 * exactly as Scheduler.pending_kv_copy_operations; read them with the
 * abkv_planner_pending_* functions and drop them with abkv_planner_clear_pending.
 * A planner is not thread-safe; use one per scheduler thread.
 * ====================================================================== */
typedef struct abkv_planner abkv_planner_t;

typedef struct abkv_span_result {
  int32_t success;          /* 1 = span removed from every target group       */
  int32_t tokens_removed;   /* end - start on success                         */
  int32_t blocks_freed;     /* pages returned to the free queue               */
  char error_message[160];  /* reference wording when success == 0            */
} abkv_span_result_t;

abkv_planner_t* abkv_planner_create(int num_blocks, int block_size, int num_groups);
void abkv_planner_destroy(abkv_planner_t* planner);
int abkv_planner_add_request(abkv_planner_t* planner, int64_t request);
int abkv_planner_set_num_computed(abkv_planner_t* planner, int64_t request,
                                  int64_t num_computed_tokens);
int abkv_planner_allocate_slots(abkv_planner_t* planner, int64_t request,
                                int64_t num_tokens);
int abkv_planner_free_request(abkv_planner_t* planner, int64_t request);
/* groups == NULL removes the span from every group; a non-NULL list of
 * num_groups entries (possibly zero) names the target groups. */
int abkv_planner_mask_token_span(abkv_planner_t* planner, int64_t request,
                                 int64_t start, int64_t end,
                                 const int32_t* groups, int num_groups,
                                 abkv_span_result_t* result);
/* resp_end == resp_start: no response content to remove. */
int abkv_planner_finish_block(abkv_planner_t* planner, int64_t request,
                              int64_t resp_start, int64_t resp_end,
                              int64_t code_start, int64_t code_end,
                              const int32_t* group_quotas, int num_groups,
                              int num_code_tokens, abkv_span_result_t* result);
int abkv_planner_block_table(const abkv_planner_t* planner, int64_t request,
                             int group, int32_t* out, int cap, int* n);
int abkv_planner_free_queue(const abkv_planner_t* planner, int32_t* out,
                            int cap, int* n);
int abkv_planner_num_free(const abkv_planner_t* planner);
int abkv_planner_span_map(const abkv_planner_t* planner, int64_t request,
                          int group, int64_t position, int to_physical,
                          int64_t* out);
int abkv_planner_compacted_spans(const abkv_planner_t* planner, int64_t request,
                                 int group, int64_t* out, int cap, int* n);
int abkv_planner_pending_requests(const abkv_planner_t* planner, int64_t* out,
                                  int cap, int* n);
int abkv_planner_pending_num_batches(const abkv_planner_t* planner,
                                     int64_t request, int group);
int abkv_planner_pending_batch(const abkv_planner_t* planner, int64_t request,
                               int group, int batch, int32_t* ops, int cap_ops,
                               int* n_ops);
int abkv_planner_pending_truncation(const abkv_planner_t* planner,
                                    int64_t request, int32_t* out, int cap,
                                    int* n);
/* Every pending copy op in one call (the same content as the per-request /
 * per-group / per-batch functions above, for hosts that read it all at once):
 * req_ids[n_reqs] in request-id order; group_batches[n_reqs * num_groups] =
 * batches of (request, group); batch_ops[n_batches] = ops per batch, batches
 * in (request, group, order) order; ops[4 * n_ops] the ops themselves.  With
 * every pointer NULL and every cap 0 it only reports the three counts. */
int abkv_planner_pending_export(const abkv_planner_t* planner, int64_t* req_ids,
                                int32_t* group_batches, int32_t* batch_ops,
                                int32_t* ops, int cap_reqs, int cap_batches,
                                int cap_ops, int* n_reqs, int* n_batches,
                                int* n_ops);
/* Every pending truncation in one call: req_ids[n], counts[n * num_groups]
 * (the per-group block counts of abkv_planner_pending_truncation).  With both
 * pointers NULL and cap 0 it only reports n. */
int abkv_planner_pending_trunc_export(const abkv_planner_t* planner,
                                      int64_t* req_ids, int32_t* counts,
                                      int cap, int* n);
int abkv_planner_clear_pending(abkv_planner_t* planner);

/* ========================================================================
 * 3. Compaction executor (device): ordered batches of KV slot copies.
 *
 * Replaces GPUModelRunner._execute_kv_copy_operations /
 * _execute_kv_copy_group (third_party/vllm_overlay/vllm/v1/worker/
 * gpu_model_runner.py:1147-1220) for ONE KV-cache group: `num_batches`
 * ordered batches, batch b = ops[batch_offsets[b] .. batch_offsets[b+1]),
 * each op = (src_block, src_off, dst_block, dst_off) (host int32 [n][4]).
 * Every batch is applied to every layer tensor of the group with
 * gather-all-then-scatter semantics; batches are applied in order.
 *   layout 0: FlashInfer      [num_blocks][2][page][Hkv][D]
 *   layout 1: FlashAttention  [2][num_blocks][page][Hkv][D]
 * Element type is opaque (rows are copied as bytes; Hkv*D*2 must be a
 * multiple of 16, i.e. 2-byte elements).  Every op is validated on the host
 * (blocks in [0, num_blocks), offsets in [0, page)) before anything runs.
 * Up to 96 layer tensors per call.  The call may wait for the stream while
 * it uploads each batch's plan from host memory.
 * ====================================================================== */
size_t abkv_compact_workspace_size(int num_layers, int page_size, int num_kv_heads,
                                   int head_dim, int64_t max_ops_per_batch);

int abkv_compact(void* const* layer_caches, int num_layers, int layout,
                 int64_t num_blocks, int page_size, int num_kv_heads,
                 int head_dim, const int32_t* ops, const int64_t* batch_offsets,
                 int num_batches, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Row gather over many tensors in one launch: each tensor t is viewed as
 * [outer][rows][row_bytes]; dst[t][o][j] = src[t][o][keep[j]] for
 * j < dst_rows.  keep is a DEVICE int64 array; an index outside
 * [0, src_rows) sets ABKV_DEVERR_ROW_OOB and zero-fills that row.
 * Replaces KVStore.evict(keep_cols) (abridgekv/gen_compress.py:72-77), which
 * gathers the kept columns of every layer's K and V ([1, Hkv, T, D]).
 * row_bytes must be a multiple of 16. */
int abkv_gather_rows(const void* const* src, void* const* dst, int num_tensors,
                     int64_t outer, int64_t src_rows, int64_t dst_rows,
                     int64_t row_bytes, const int64_t* keep, void* workspace,
                     size_t workspace_bytes, void* stream);

/* The step's new K / V rows into the paged cache, before attention: the
 * slot write vLLM's attention backend makes at the start of
 * AttentionImpl.forward (reshape_and_cache_flash in vLLM 0.13.0, the
 * third-party version the overlay pins, requirements.txt:10-12; the
 * overlay's forward then reads the rows back through the block table,
 * compresslm_packed_kv.py:744-761).  Token t's rows key[t] / value[t]
 * ([num_kv_heads][head_dim] bf16, element strides row / head, each head's
 * head_dim contiguous) go to slot s = slot_mapping[t] (DEVICE int64):
 * block s / page_size, offset s % page_size, in either paged layout.  A
 * negative slot (padding) is skipped; a slot past the cache sets
 * ABKV_DEVERR_ROW_OOB and is skipped.  Needs 16-byte aligned bases and
 * strides (ABKV_ERR_UNSUPPORTED otherwise). */
int abkv_store_kv(const void* key, int64_t key_row_stride,
                  int64_t key_head_stride, const void* value,
                  int64_t value_row_stride, int64_t value_head_stride,
                  void* kv_cache, int kv_layout, int64_t num_blocks,
                  int page_size, int num_kv_heads, int head_dim,
                  const int64_t* slot_mapping, int T, void* workspace,
                  size_t workspace_bytes, void* stream);

/* ========================================================================
 * 4. Pause-token prefill attention with the compressed-cache mask (tcgen05).
 *
 * Replaces the FlexAttention call CompressLM makes through transformers
 * (abridgekv/compress_forward.py:248,1229) with the per-layer BlockMasks of
 * _arith_mask_mod / _fast_layer_blockmasks (:695-727, :760-789): the mask is
 * evaluated arithmetically from the block layout instead of a BlockMask.
 * q: [B][H][S][head_dim], k, v: [B][Hkv][S][head_dim] bf16, element strides
 * (batch, head, seq) given in *_strides[3], last dim contiguous; out likewise
 * [B][H][S][head_dim] (strides multiples of 8 elements); lse: optional
 * contiguous [B][H][S] f32, natural log.  Sequence layout: blocks of
 * [C content | K_layout code rows]; quota_per_head: HOST [H] code quota of each
 * query head (NULL = K_layout); prompt_len: DEVICE [B] raw prompt lengths
 * (NULL = none).  Supported: head_dim 64 or 128, C and K_layout multiples of 128,
 * S a multiple of C + K_layout, H <= 128, H % Hkv == 0.
 * ====================================================================== */
int abkv_prefill_masked(const void* q, const int64_t* q_strides, const void* k,
                        const int64_t* k_strides, const void* v,
                        const int64_t* v_strides, void* out,
                        const int64_t* out_strides, float* lse,
                        const int32_t* quota_per_head, const int32_t* prompt_len,
                        int B, int H, int Hkv, int S, int head_dim, int C,
                        int K_layout, float scale, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Backward of abkv_prefill_masked: dq, dk, dv for the upstream gradient dout,
 * the gradients torch FlexAttention's backward gives the training path
 * (abridgekv/compress_forward.py:248,1229 with the same mask; sft_ddp.py:1225).
 * q, k, v, quota_per_head, prompt_len, C, K_layout, scale as in the forward;
 * out: the forward's output [B][H][S][head_dim]; dout likewise; lse: the
 * forward's CONTIGUOUS [B][H][S] f32 log-sum-exp (natural log); dq [B][H][S][D],
 * dk / dv [B][Hkv][S][D] bf16 outputs (strides multiples of 8 elements).
 * The workspace holds an fp32 dq accumulator and rowsum(dout * out):
 * abkv_prefill_masked_backward_workspace_size(B, H, S, head_dim) bytes,
 * 256-byte aligned.  Same shape limits as the forward, (S / 128) x (H / Hkv)
 * <= 2048 and B x H x S < 2^31. */
size_t abkv_prefill_masked_backward_workspace_size(int B, int H, int S,
                                                   int head_dim);
int abkv_prefill_masked_backward(
    const void* q, const int64_t* q_strides, const void* k,
    const int64_t* k_strides, const void* v, const int64_t* v_strides,
    const void* out, const int64_t* out_strides, const void* dout,
    const int64_t* dout_strides, const float* lse, void* dq,
    const int64_t* dq_strides, void* dk, const int64_t* dk_strides, void* dv,
    const int64_t* dv_strides, const int32_t* quota_per_head,
    const int32_t* prompt_len, int B, int H, int Hkv, int S, int head_dim, int C,
    int K_layout, float scale, void* workspace, size_t workspace_bytes,
    void* stream);

/* ========================================================================
 * 5. Code step: K_code code queries per request over the paged cache (tcgen05).
 *
 * Replaces the noncausal branch of PackedKVSidecar._attend_request_vectorized
 * (third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:648-741),
 * reached from override_attention (:329-420) when the step holds the K_code
 * code rows of each active request: request r's queries are rows
 * q_start[r] .. q_start[r] + K_code - 1 of q (query_start_loc); its keys are
 * rows [0, seq_lens[r]) gathered through block-table row r; a KV head with
 * quota q sees rows [0, seq_lens[r] - K_code + q) (:711-720), minus the
 * optional per-request exclusion range [excluded[2r], excluded[2r+1])
 * (:721-726; start == end = none).  Scores, softmax and P.V run on the
 * tensor cores with fp32 accumulation and an online softmax.
 *
 * q: [T][Hq][head_dim] bf16 with element strides (q_row_stride,
 * q_head_stride), last dim contiguous; out likewise.  kv_cache: FlashInfer
 * (kv_layout 0, [num_blocks][2][page][Hkv][D]) or FlashAttention (1,
 * [2][num_blocks][page][Hkv][D]).  block_table: DEVICE [R][bt_stride] int32;
 * q_start, seq_lens: DEVICE [R] int32; excluded: DEVICE [R][2] int32 or NULL;
 * quota_per_kv_head: HOST [Hkv] in [0, K_code].  Supported: head_dim 128,
 * K_code a multiple of 128, page a multiple of 16, seq_lens[r] in
 * [K_code, min(bt_stride * page, 131072)].  Invalid device-side values set
 * ABKV_DEVERR_SEQ_OOB / PAGE_OOB / RANGE in the workspace error word (a request
 * whose query rows fall outside [0, T) is skipped).
 * ====================================================================== */
int abkv_code_step_attention(const void* q, int64_t q_row_stride,
                             int64_t q_head_stride, void* out,
                             int64_t out_row_stride, int64_t out_head_stride,
                             const int32_t* q_start, const void* kv_cache,
                             int kv_layout, int64_t num_blocks, int page_size,
                             const int32_t* block_table, int64_t bt_stride,
                             const int32_t* seq_lens, const int32_t* excluded,
                             const int32_t* quota_per_kv_head, int R, int Hq,
                             int Hkv, int head_dim, int K_code, int T,
                             float scale, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Causal attention of ragged query rows over the paged cache: the prompt
 * prefill, chunked prefill and mixed prefill/decode steps of a CompressLM
 * KV-cache group.  Replaces the causal branch of
 * PackedKVSidecar._attend_request_vectorized with no sidecar pages
 * (third_party/vllm_overlay/vllm/v1/worker/compresslm_packed_kv.py:700-707,
 * reached from override_attention :371-399 when query_len > 1) and the
 * stock backend's causal paged prefill of a KV-cache group
 * (gpu_model_runner.py:1872-1886 metadata, causal=True).
 * Request r's query rows are query_start_loc[r] .. query_start_loc[r+1]-1
 * (qlen rows; their keys are already at cache rows [seq_len - qlen,
 * seq_len)); row i attends to cache rows [0, seq_len - qlen + i + 1) of its
 * block-table row, every query head alike (GQA: head h reads KV head
 * h / (Hq / Hkv)).  Same kernel as abkv_code_step_attention in its causal
 * mode (tcgen05, 128 query rows x 2 heads per CTA, 64-key tiles).
 * query_start_loc: DEVICE [R+1] int32; max_query_len: >= every qlen (the
 * grid has ceil(max_query_len / 128) query tiles per request; a longer
 * request sets ABKV_DEVERR_RANGE and its rows past the grid stay
 * unwritten).  Other arguments as abkv_code_step_attention; seq_lens[r] in
 * [qlen, min(bt_stride * page, 131072)].  Rows of out that belong to no
 * request are not written. */
int abkv_paged_prefill(const void* q, int64_t q_row_stride,
                       int64_t q_head_stride, void* out,
                       int64_t out_row_stride, int64_t out_head_stride,
                       const int32_t* query_start_loc, const void* kv_cache,
                       int kv_layout, int64_t num_blocks, int page_size,
                       const int32_t* block_table, int64_t bt_stride,
                       const int32_t* seq_lens, int R, int Hq, int Hkv,
                       int head_dim, int max_query_len, int T, float scale,
                       void* workspace, size_t workspace_bytes,
                       void* stream);

/* The code step and the causal paged attention of requests that hold packed
 * sidecar pages (per-head quotas): PackedKVSidecar._attend_request_vectorized
 * with layer_pages (third_party/vllm_overlay/vllm/v1/worker/
 * compresslm_packed_kv.py:648-741, noncausal :708-733 and causal :700-707).
 * For KV head h of request r the keys are, first, head h's slots of each of
 * the request's sidecar->page_count[r] packed pages (the layout of
 * abkv_decode_packed), visible to every query row, then the paged rows with
 * the masks of abkv_code_step_attention / abkv_paged_prefill.  Arguments as
 * those two entries plus one sidecar descriptor (quotas: multiples of 16,
 * at most 8 KV heads). */
int abkv_code_step_attention_packed(const void* q, int64_t q_row_stride,
                                    int64_t q_head_stride, void* out,
                                    int64_t out_row_stride,
                                    int64_t out_head_stride,
                                    const int32_t* q_start, const void* kv_cache,
                                    int kv_layout, int64_t num_blocks,
                                    int page_size, const int32_t* block_table,
                                    int64_t bt_stride, const int32_t* seq_lens,
                                    const int32_t* excluded,
                                    const int32_t* quota_per_kv_head, int R,
                                    int Hq, int Hkv, int head_dim, int K_code,
                                    int T, float scale,
                                    const abkv_sidecar_t* sidecar,
                                    void* workspace, size_t workspace_bytes,
                                    void* stream);

int abkv_paged_prefill_packed(const void* q, int64_t q_row_stride,
                              int64_t q_head_stride, void* out,
                              int64_t out_row_stride, int64_t out_head_stride,
                              const int32_t* query_start_loc,
                              const void* kv_cache, int kv_layout,
                              int64_t num_blocks, int page_size,
                              const int32_t* block_table, int64_t bt_stride,
                              const int32_t* seq_lens, int R, int Hq, int Hkv,
                              int head_dim, int max_query_len, int T,
                              float scale, const abkv_sidecar_t* sidecar,
                              void* workspace, size_t workspace_bytes,
                              void* stream);

/* The code step fused with the compaction that follows it in the block
 * boundary flow (CompressLMProcessor._compact_response_content,
 * third_party/vllm_overlay/vllm/v1/core/compresslm/processor.py:467-557,
 * whose copy ops GPUModelRunner._execute_kv_copy_group applies,
 * .../v1/worker/gpu_model_runner.py:1194-1220): the same attention as
 * abkv_code_step_attention, then request r's row copies
 * ops[op_offsets[r] .. op_offsets[r+1]) (HOST [n][4] int32 = src_block,
 * src_off, dst_block, dst_off; op_offsets HOST [R+1] int64, from 0 to n) are
 * applied to this layer's kv_cache by the last CTA of the request, once every
 * CTA of the request has finished reading the cache, so the copies overlap
 * the other requests' attention instead of needing a separate launch.
 * Result: out and kv_cache equal abkv_code_step_attention followed by
 * abkv_compact of the same ops as one batch.  The host rejects ops out of
 * range (ABKV_ERR_INVALID_ARG), and a batch in which a destination repeats or
 * is also a source (ABKV_ERR_UNSUPPORTED: use abkv_compact for ordered
 * batches).  Preconditions the caller guarantees (nothing here can check
 * them against device-side tables):
 *   - ordering: the block finishes directly after its code step, i.e. the
 *     configuration has no replay tail (replay_tail == 0; the reference calls
 *     _finish_block at the end of the code role only when the block has no
 *     replay positions, processor.py:236-255), and the ops are the ones the
 *     planner's finish_block produced for that block before this launch;
 *   - ownership: request r's ops read and write only pages of request r's
 *     own block-table row, and no other request of the launch reads those
 *     pages (true without prefix sharing, which CompressLM disables); with
 *     shared pages the copies would race with the other request's loads, so
 *     use abkv_code_step_attention + abkv_compact instead.
 * The Python wrapper (codestep.code_step_attention_compact) requires the
 * replay tail to be stated and checks ownership against a host copy of the
 * block table when one is given.  If any CTA of a request gives up on a
 * wait, meets an out-of-range page id in the request's block-table row, or
 * the request's query rows are out of range, that request's ops are not
 * applied and the error word records why.  Workspace:
 * abkv_code_step_compact_workspace_size(R, n) bytes, 256-byte aligned. */
size_t abkv_code_step_compact_workspace_size(int num_requests, int64_t n_ops);

int abkv_code_step_attention_compact(const void* q, int64_t q_row_stride,
                                     int64_t q_head_stride, void* out,
                                     int64_t out_row_stride,
                                     int64_t out_head_stride,
                                     const int32_t* q_start, void* kv_cache,
                                     int kv_layout, int64_t num_blocks,
                                     int page_size, const int32_t* block_table,
                                     int64_t bt_stride, const int32_t* seq_lens,
                                     const int32_t* excluded,
                                     const int32_t* quota_per_kv_head, int R,
                                     int Hq, int Hkv, int head_dim, int K_code,
                                     int T, float scale, const int32_t* ops,
                                     const int64_t* op_offsets, int64_t n_ops,
                                     void* workspace, size_t workspace_bytes,
                                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ABKV_H_ */
