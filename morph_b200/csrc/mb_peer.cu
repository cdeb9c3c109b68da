// Peer-writable device buffers for one node: a rank allocates its buffer with
// cudaMalloc, publishes the 64-byte IPC handle, and every other rank maps it
// (cudaIpcOpenMemHandle, peer access enabled lazily), so a kernel can store
// straight into another GPU's buffer over NVLink. Used by the fused
// update + all-gather of the sharded AdamW (kernel 1 with peer copies).
#include <cstring>

#include "mb_common.cuh"

extern "C" {

MB_API int mb_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return MB_ERR_ARG;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return MB_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, *ptr) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return MB_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  return MB_OK;
}

MB_API int mb_ipc_free(void* ptr) {
  if (!ptr) return MB_ERR_ARG;
  return cudaFree(ptr) == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

MB_API int mb_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return MB_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

MB_API int mb_ipc_close(void* ptr) {
  if (!ptr) return MB_ERR_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MB_OK : MB_ERR_CUDA;
}

}  // extern "C"
