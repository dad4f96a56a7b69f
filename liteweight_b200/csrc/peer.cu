// Device memory shared between the ranks of a tensor-parallel decode (one
// process per GPU): each rank allocates its exchange block here, exports a
// CUDA IPC handle, and maps the other ranks' blocks from their handles. The
// kernels then store into and poll those mappings directly (NVLink peer
// loads, stores and atomics). Host-only setup calls.
#include <cuda_runtime.h>
#include <string.h>

#include "../../include/liteweight_b200.h"

extern "C" {

int lw_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr) return LW_ERR_NULL_POINTER;
  *ptr = nullptr;
  if (bytes == 0) return LW_ERR_BAD_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return LW_ERR_LAUNCH;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return LW_ERR_LAUNCH;
  }
  *ptr = p;
  return LW_OK;
}

int lw_peer_free(void* ptr) {
  if (!ptr) return LW_ERR_NULL_POINTER;
  return cudaFree(ptr) == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

size_t lw_peer_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int lw_peer_export(void* ptr, void* handle) {
  if (!ptr || !handle) return LW_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return LW_ERR_LAUNCH;
  memcpy(handle, &h, sizeof(h));
  return LW_OK;
}

int lw_peer_import(const void* handle, void** ptr) {
  if (!handle || !ptr) return LW_ERR_NULL_POINTER;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return LW_ERR_LAUNCH;
  *ptr = p;
  return LW_OK;
}

int lw_peer_close(void* ptr) {
  if (!ptr) return LW_ERR_NULL_POINTER;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

}  // extern "C"
