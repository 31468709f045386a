// pasa_forward_noalloc: the whole PASA forward with its scratch memory
// (block statistics, top-k indices, selection bitmask, error word) in a
// fixed array that is part of this library's device image, for callers that
// must not allocate device memory themselves or through us.
//
// The array is a file-scope __device__ variable.  In host code its name is
// only a host-side stand-in, not a device address, so the device address is
// looked up with cudaGetSymbolAddress with the device current and cached;
// kernels receive that address.  The cache is keyed by the current CUDA
// context (a context created by the caller, or the device's primary context
// after a cudaDeviceReset, has its own copy of the module and its own
// address), so a changed context resolves the address again.
#include <cuda.h>
#include <cudaTypedefs.h>

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
struct ScratchEntry {
  CUcontext ctx = nullptr;
  void* addr = nullptr;
};
ScratchEntry g_scratch[kMaxDevices];

// cuCtxGetCurrent through the runtime's driver entry point (the library links
// only the CUDA runtime), looked up once.
PFN_cuCtxGetCurrent_v4000 ctx_get_current_fn() {
  static const PFN_cuCtxGetCurrent_v4000 fn = []() -> PFN_cuCtxGetCurrent_v4000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    return nullptr;
  }();
  return fn;
}

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
  auto get_ctx = ctx_get_current_fn();
  CUcontext ctx = nullptr;
  if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS) return PASA_ERR_CUDA;
  void* scratch = nullptr;
  if (!ctx) {
    // No context bound to this thread yet: the runtime binds the device's
    // primary context on its first call that needs one (this lookup), and
    // that is the context the launches below use.
    if (cudaGetSymbolAddress(&scratch, g_pasa_noalloc_scratch) != cudaSuccess || !scratch) return PASA_ERR_CUDA;
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return PASA_ERR_CUDA;
  }
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchEntry& e = g_scratch[dev];
    if (e.ctx != ctx || !e.addr) {  // first call in this context: resolve the array's device address
      if (cudaGetSymbolAddress(&scratch, g_pasa_noalloc_scratch) != cudaSuccess || !scratch) return PASA_ERR_CUDA;
      e.ctx = ctx;
      e.addr = scratch;
    }
    scratch = e.addr;
  }
  // pasa_forward writes every scratch region it reads and clears the error
  // word itself, so the previous call's contents do not matter.
  return pasa_forward(stream, q, k, v, B, H, T, D, dtype, density, scale, use_cov_bias, noise, scratch,
                      kNoAllocScratchBytes, o, kernel);
}
