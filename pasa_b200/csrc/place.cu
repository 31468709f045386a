// Token-layout permutation of temporal heads.
//
// Restates hunyuan_sparse_head_placement_kernel and
// hunyuan_hidden_states_placement_kernel (svg/models/hyvideo/placement.py:
// 34-121, :285-357).  For a temporal head, video token t = f*S + p (frame f,
// patch p; t < T - context_length) moves to p*F + f (forward) and back
// (inverse); the trailing context_length text tokens stay in place.  Spatial
// heads are copied.
//
// A pure copy, bound by HBM bandwidth: every thread moves 16-byte pieces of
// kUnroll rows, issuing all its loads before its stores, and the threads of
// a row (D * esize / 16 of them) cover it with consecutive 16-byte accesses,
// so both the gather and the scatter side are whole 128-byte lines.
#include "common.cuh"

namespace pasa {

namespace {
constexpr int kPlaceThreads = 256;
constexpr int kUnroll = 4;
}  // namespace

__global__ void __launch_bounds__(kPlaceThreads) place_kernel(
    const uint4* __restrict__ src, uint4* __restrict__ dst, const int32_t* __restrict__ temporal,
    int64_t T_len, int vec_per_row, int64_t ctx, int64_t F, int64_t S, int inverse, int64_t total_rows) {
  const int rows_per_cta = kPlaceThreads / vec_per_row;  // rows one pass of the CTA covers
  const int r_in = threadIdx.x / vec_per_row, c = threadIdx.x % vec_per_row;
  if (r_in >= rows_per_cta) return;
  const int64_t base = int64_t(blockIdx.x) * rows_per_cta * kUnroll;
  uint4 val[kUnroll];
  int64_t out[kUnroll];
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t row = base + int64_t(u) * rows_per_cta + r_in;
    out[u] = -1;
    if (row < total_rows) {
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
      val[u] = __ldcs(src + row * vec_per_row + c);  // streamed: read once
      out[u] = (ch * T_len + t_out) * vec_per_row + c;
    }
  }
#pragma unroll
  for (int u = 0; u < kUnroll; ++u)
    if (out[u] >= 0) __stcs(dst + out[u], val[u]);
}

cudaError_t launch_place(cudaStream_t st, const void* src, void* dst, const int32_t* temporal, int64_t cfg,
                         int64_t H, int64_t T_len, int D, int esize, int64_t ctx, int64_t F, int64_t S,
                         int inverse) {
  const int vec_per_row = D * esize / 16;
  if (vec_per_row < 1 || vec_per_row > kPlaceThreads) return cudaErrorInvalidValue;
  const int64_t rows = cfg * H * T_len;
  const int64_t rows_per_cta = (kPlaceThreads / vec_per_row) * int64_t(kUnroll);
  const int64_t blocks = cdiv(rows, rows_per_cta);
  if (blocks > 0x7FFFFFFF) return cudaErrorInvalidValue;
  place_kernel<<<unsigned(blocks), kPlaceThreads, 0, st>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst),
                                                           temporal, T_len, vec_per_row, ctx, F, S, inverse, rows);
  return cudaGetLastError();
}

}  // namespace pasa
