// Status strings, version and the workspace error word.
#include <cuda_runtime.h>

#include "abkv.h"

extern "C" const char* abkv_status_string(int status) {
  switch (status) {
    case ABKV_OK: return "ok";
    case ABKV_ERR_INVALID_ARG: return "invalid argument";
    case ABKV_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case ABKV_ERR_UNSUPPORTED: return "shape not supported by the sm_100a kernels";
    case ABKV_ERR_CUDA: return "CUDA runtime error";
    case ABKV_ERR_PAGE_OOB: return "page id outside [0, num_blocks)";
    case ABKV_ERR_SEQ_OOB: return "seq_len exceeds the rows its block-table row can address";
    case ABKV_ERR_SPAN: return "span rejected by the compaction planner";
    case ABKV_ERR_NO_BLOCKS: return "free block queue exhausted";
    case ABKV_ERR_TIMEOUT: return "bounded device wait gave up";
    case ABKV_ERR_SCRATCH_LIMIT: return "request exceeds the 32 MiB scratch of abkv_decode_noalloc";
    default: return "unknown status";
  }
}

extern "C" const char* abkv_version(void) { return "abkv 0.1 sm_100a"; }

extern "C" int abkv_workspace_error(void* workspace, void* stream, int32_t* host_error) {
  if (!workspace || !host_error) return ABKV_ERR_INVALID_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return ABKV_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return ABKV_ERR_CUDA;
  *host_error = v;
  if (v != 0) {
    if (cudaMemsetAsync(workspace, 0, sizeof(v), s) != cudaSuccess) return ABKV_ERR_CUDA;
  }
  return ABKV_OK;
}
