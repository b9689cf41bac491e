// Peer buffers for the sharded GEMM's fused all-gather: device allocations shared between the rank processes of one
// box through CUDA interprocess handles, mapped with peer access so a kernel's plain stores reach them over NVLink.
#include <string.h>

#include "lk_common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == 64, "interprocess handles are 64 bytes");

extern "C" {

int lk_peer_alloc(int64_t bytes, void** ptr, void* handle64) {
  if (bytes <= 0 || !ptr || !handle64) return LK_EINVAL;
  void* p = nullptr;
  if (cudaMalloc(&p, size_t(bytes)) != cudaSuccess) return LK_ECUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return LK_ECUDA;
  }
  memcpy(handle64, &h, sizeof(h));
  *ptr = p;
  return LK_OK;
}

int lk_peer_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return LK_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return LK_ECUDA;
  *ptr = p;
  return LK_OK;
}

int lk_peer_close(void* ptr) {
  if (!ptr) return LK_EINVAL;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? LK_OK : LK_ECUDA;
}

int lk_peer_free(void* ptr) {
  if (!ptr) return LK_EINVAL;
  return cudaFree(ptr) == cudaSuccess ? LK_OK : LK_ECUDA;
}

}  // extern "C"
