// Device buffers shared between the ranks of one node (CUDA IPC).
//
// The fused row-parallel reduce-scatter (gemm_i8.cu) reads the other ranks'
// partial outputs and flags through these mappings over NVLink.  They are
// plain cudaMalloc allocations, zeroed at creation, allocated once per layer
// shape at set-up and never per call.
#include <cstring>

#include "common.h"

extern "C" {

int tm_peer_handle_size(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int tm_peer_alloc(uint64_t bytes, void** ptr, void* handle_out) {
  if (ptr == nullptr || handle_out == nullptr) return TM_ERR_NULL_POINTER;
  if (bytes == 0) return TM_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return TM_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return TM_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return TM_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return TM_OK;
}

int tm_peer_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return TM_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return TM_ERR_CUDA;
  *ptr = p;
  return TM_OK;
}

int tm_peer_close(void* ptr) {
  if (ptr == nullptr) return TM_ERR_NULL_POINTER;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? TM_OK : TM_ERR_CUDA;
}

int tm_peer_free(void* ptr) {
  if (ptr == nullptr) return TM_ERR_NULL_POINTER;
  return cudaFree(ptr) == cudaSuccess ? TM_OK : TM_ERR_CUDA;
}

}  // extern "C"
