// Peer-visible device buffers for the KV-head-sharded decode (one process per
// GPU).  A rank allocates its gather buffer here, exports a CUDA IPC handle,
// and every other rank of the node maps it; the decode epilogue then stores
// each rank's head outputs into all ranks' buffers over NVLink / NVSwitch.
// The buffers are plain cudaMalloc memory: no multicast object is created.
#include <cuda_runtime.h>

#include <cstring>

#include "abkv.h"

extern "C" int abkv_peer_alloc(size_t bytes, void** ptr, unsigned char* handle) {
  if (!ptr || !handle || bytes < ABKV_GATHER_FLAG_BYTES) return ABKV_ERR_INVALID_ARG;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return ABKV_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return ABKV_ERR_CUDA;
  }
  static_assert(sizeof(h) == ABKV_PEER_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return ABKV_OK;
}

extern "C" int abkv_peer_open(const unsigned char* handle, void** ptr) {
  if (!handle || !ptr) return ABKV_ERR_INVALID_ARG;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return ABKV_ERR_CUDA;
  *ptr = p;
  return ABKV_OK;
}

extern "C" int abkv_peer_close(void* ptr) {
  if (!ptr) return ABKV_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? ABKV_OK : ABKV_ERR_CUDA;
}

extern "C" int abkv_peer_free(void* ptr) {
  if (!ptr) return ABKV_ERR_INVALID_ARG;
  return cudaFree(ptr) == cudaSuccess ? ABKV_OK : ABKV_ERR_CUDA;
}
