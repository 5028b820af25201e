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
 *   - Entry points are reentrant: no global mutable state.
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

/* Device error-word bits (OR-ed by kernels into workspace bytes 0..3). */
#define ABKV_DEVERR_PAGE_OOB 0x1
#define ABKV_DEVERR_SEQ_OOB 0x2
#define ABKV_DEVERR_TIMEOUT 0x4
#define ABKV_DEVERR_ROW_OOB 0x8

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
 * Supported: head_dim 128; num_kv_heads in {1,2,4,8}; group size
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

#ifdef __cplusplus
}
#endif

#endif /* ABKV_H_ */
