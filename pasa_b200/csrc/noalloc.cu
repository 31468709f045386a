// pasa_forward_noalloc: the whole PASA forward with its scratch memory
// (block statistics, top-k indices, selection bitmask, error word) in a
// fixed array that is part of this library's device image, for callers that
// must not allocate device memory themselves or through us.
//
// The array is a file-scope __device__ variable.  In host code its name is
// only a host-side stand-in, not a device address, so the device address is
// looked up with cudaGetSymbolAddress once per device (with that device
// current) and cached; kernels receive that address.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace {

// Capacity of the built-in scratch.  Every GPU that loads the library holds
// this much device memory until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB

__device__ __align__(256) unsigned char g_pasa_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

}  // namespace

extern "C" PASA_API int pasa_forward_noalloc(void* stream, const void* q, const void* k, const void* v, int64_t B,
                                             int64_t H, int64_t T, int D, int dtype, double density, float scale,
                                             int use_cov_bias, const float* noise, void* o, int kernel) {
  if (B < 1 || H < 1 || T < 1) return PASA_ERR_SHAPE;
  if (!std::isfinite(density)) return PASA_ERR_DENSITY;
  int64_t ns = 0;
  int st = pasa_derive(T, pasa::kBlock, pasa::kGroup, density, nullptr, nullptr, &ns);
  if (st) return st;
  size_t need = 0;
  st = pasa_workspace_size(B, H, T, D, dtype, pasa::kBlock, pasa::kGroup, ns, &need);
  if (st) return st;
  if (need > kNoAllocScratchBytes) return PASA_ERR_WORKSPACE;  // problem too large for the built-in scratch

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PASA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return PASA_ERR_DEVICE;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    scratch = g_scratch_addr[dev];
    if (!scratch) {  // first call on this device: resolve the array's device address
      if (cudaGetSymbolAddress(&scratch, g_pasa_noalloc_scratch) != cudaSuccess || !scratch) return PASA_ERR_CUDA;
      g_scratch_addr[dev] = scratch;
    }
  }
  // pasa_forward writes every scratch region it reads and clears the error
  // word itself, so the previous call's contents do not matter.
  return pasa_forward(stream, q, k, v, B, H, T, D, dtype, density, scale, use_cov_bias, noise, scratch,
                      kNoAllocScratchBytes, o, kernel);
}
