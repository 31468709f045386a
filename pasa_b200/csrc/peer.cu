// Peer memory for the fused Ulysses exchange of the DiT step: device buffers
// allocated by the library, shared with the other ranks' processes on the
// node through CUDA IPC handles, so that the q/k/v producer and the attention
// epilogue of one GPU can store straight into another GPU's buffer over
// NVLink (plain peer stores; no multicast object is created).
#include <cstring>

#include "common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == PASA_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" {

int pasa_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle) return PASA_ERR_NULL;
  if (bytes == 0) return PASA_ERR_SHAPE;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return PASA_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return PASA_ERR_CUDA;
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return PASA_OK;
}

int pasa_peer_free(void* ptr) {
  if (!ptr) return PASA_ERR_NULL;
  return cudaFree(ptr) == cudaSuccess ? PASA_OK : PASA_ERR_CUDA;
}

int pasa_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return PASA_ERR_NULL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? PASA_OK : PASA_ERR_CUDA;
}

int pasa_peer_close(void* ptr) {
  if (!ptr) return PASA_ERR_NULL;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? PASA_OK : PASA_ERR_CUDA;
}

}  // extern "C"
