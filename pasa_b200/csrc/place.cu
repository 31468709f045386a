// Token-layout permutation of temporal heads.
//
// Restates hunyuan_sparse_head_placement_kernel and
// hunyuan_hidden_states_placement_kernel (svg/models/hyvideo/placement.py:
// 34-121, :285-357).  For a temporal head, video token t = f*S + p (frame f,
// patch p; t < T - context_length) moves to p*F + f (forward) and back
// (inverse); the trailing context_length text tokens stay in place.  Spatial
// heads are copied.  One warp moves one token row with 16-byte accesses, so
// both the gather and the scatter side are full 128-byte lines for D*esize
// >= 128.
#include "common.cuh"

namespace pasa {

__global__ void __launch_bounds__(256) place_kernel(
    const uint4* __restrict__ src, uint4* __restrict__ dst, const int32_t* __restrict__ temporal,
    int64_t H, int64_t T_len, int vec_per_row, int64_t ctx, int64_t F, int64_t S, int inverse,
    int64_t total_rows) {
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (row >= total_rows) return;
  const int64_t t = row % T_len;
  const int64_t ch = row / T_len;  // cfg * H + h
  int64_t t_out = t;
  if (temporal[ch] != 0 && t < T_len - ctx) {
    if (!inverse) {
      const int64_t f = t / S, p = t - f * S;  // placement.py:73-78
      t_out = p * F + f;
    } else {
      const int64_t p = t / F, f = t - p * F;  // placement.py:320-325
      t_out = f * S + p;
    }
  }
  const uint4* s = src + (ch * T_len + t) * vec_per_row;
  uint4* d = dst + (ch * T_len + t_out) * vec_per_row;
  for (int c = lane; c < vec_per_row; c += 32) d[c] = s[c];
}

cudaError_t launch_place(cudaStream_t st, const void* src, void* dst, const int32_t* temporal, int64_t cfg,
                         int64_t H, int64_t T_len, int D, int esize, int64_t ctx, int64_t F, int64_t S,
                         int inverse) {
  const int vec_per_row = D * esize / 16;
  const int64_t rows = cfg * H * T_len;
  const int64_t threads = rows * 32;
  const unsigned blocks = unsigned(cdiv(threads, 256));
  place_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), temporal, H,
                                       T_len, vec_per_row, ctx, F, S, inverse, rows);
  return cudaGetLastError();
}

}  // namespace pasa
