// Block statistics of the PASA forward: qc, kc, vc, h_norm and h_group.
//
// Restates fused_chunk_reduce_kernel + compute_h_group
// (svg/kernels/triton/group_pisa_attention.py:75-129, :268-301) as ONE pass:
// a CTA owns one (head, group of 32 blocks), walks its blocks, and keeps the
// running sum of the per-block D x D matrices hc_j in registers, so hc is
// never written to HBM (the reference writes and re-reads B*H*NT*D*D
// elements, 1.55 GB at the Wan2.1-14B shape).
//
// Rounding points follow the reference:
//   * column sums in the input dtype: fp32 adds rows in order (the
//     reference's CPU run, np.sum over axis 0); bf16 uses the halving tree
//     x[r] + x[r+n/2], each partial sum rounded to bf16 (Triton 3.x sums bf16
//     in bf16, :101-103);
//   * qc = dtype(f32(sum) / len), kc likewise; vc = sum (:101-103, :117-119);
//   * hc = k^T v (fp32) - kc_f32 (x) vc (:106-107); h_norm = sqrt(sum hc^2)
//     from the fp32 hc (:110, :287);
//   * h_group = dtype(sum_j dtype(hc_j) / 32) with blocks past NT as zeros
//     (:291-301, the divisor is always 32).
#include "common.cuh"

namespace pasa {

template <typename T, int D>
struct PrepSmem {
  T q[kBlock][D];
  T k[kBlock][D];
  T v[kBlock][D];
  float kc_f[D];
  float vc_f[D];
  float red[32];
};

// Column sum over the 64 rows of one tile, in the reference's rounding.
template <typename T, int D>
__device__ __forceinline__ float column_sum(const T (*tile)[D], int c);

template <>
__device__ __forceinline__ float column_sum<float, 64>(const float (*tile)[64], int c) {
  float s = tile[0][c];
  for (int r = 1; r < kBlock; ++r) s = s + tile[r][c];
  return s;
}
template <>
__device__ __forceinline__ float column_sum<float, 128>(const float (*tile)[128], int c) {
  float s = tile[0][c];
  for (int r = 1; r < kBlock; ++r) s = s + tile[r][c];
  return s;
}

template <int D>
__device__ __forceinline__ float column_sum_bf16(const __nv_bfloat16 (*tile)[D], int c) {
  float x[kBlock];
#pragma unroll
  for (int r = 0; r < kBlock; ++r) x[r] = __bfloat162float(tile[r][c]);
#pragma unroll
  for (int n = kBlock; n > 1; n >>= 1) {
#pragma unroll
    for (int r = 0; r < n / 2; ++r) x[r] = Elem<__nv_bfloat16>::round(x[r] + x[r + n / 2]);
  }
  return x[0];
}
template <>
__device__ __forceinline__ float column_sum<__nv_bfloat16, 64>(const __nv_bfloat16 (*tile)[64], int c) {
  return column_sum_bf16<64>(tile, c);
}
template <>
__device__ __forceinline__ float column_sum<__nv_bfloat16, 128>(const __nv_bfloat16 (*tile)[128], int c) {
  return column_sum_bf16<128>(tile, c);
}

// Copy rows [t0, t0+64) of one head into a shared tile; rows >= T are zero.
template <typename T, int D>
__device__ __forceinline__ void load_tile(T (*dst)[D], const T* src_head, int64_t t0, int64_t T_len) {
  constexpr int kVecPerRow = D * int(sizeof(T)) / 16;
  const int nvec = kBlock * kVecPerRow;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    int r = i / kVecPerRow, c = i % kVecPerRow;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (t0 + r < T_len) val = reinterpret_cast<const uint4*>(src_head + (t0 + r) * D)[c];
    reinterpret_cast<uint4*>(&dst[r][0])[c] = val;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(256) prep_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    int64_t T_len, int64_t NT, int64_t NG,
    T* __restrict__ qc, T* __restrict__ kc, T* __restrict__ vc,
    float* __restrict__ h_norm, T* __restrict__ h_group) {
  constexpr int MT = D / 16;  // micro-tile edge: 16 x 16 threads cover D x D
  extern __shared__ __align__(16) unsigned char smem_raw[];
  auto& S = *reinterpret_cast<PrepSmem<T, D>*>(smem_raw);

  const int64_t g = blockIdx.x, bh = blockIdx.y;
  const int64_t NTP = NG * kGroup;
  const int tid = threadIdx.x;
  const int a0 = (tid / 16) * MT, b0 = (tid % 16) * MT;
  const T* qh = q + bh * T_len * D;
  const T* kh = k + bh * T_len * D;
  const T* vh = v + bh * T_len * D;

  float gsum[MT][MT];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < MT; ++j) gsum[i][j] = 0.f;

  for (int jj = 0; jj < kGroup; ++jj) {
    const int64_t j = g * kGroup + jj;
    T* qc_row = qc + (bh * NTP + j) * D;
    T* kc_row = kc + (bh * NTP + j) * D;
    T* vc_row = vc + (bh * NTP + j) * D;
    if (j >= NT) {  // zero padding rows (compute_h_group pads hc with zeros)
      for (int c = tid; c < D; c += blockDim.x) {
        Elem<T>::store(qc_row + c, 0.f);
        Elem<T>::store(kc_row + c, 0.f);
        Elem<T>::store(vc_row + c, 0.f);
      }
      continue;
    }
    const int64_t t0 = j * kBlock;
    const float len = float((T_len - t0 < kBlock) ? (T_len - t0) : int64_t(kBlock));  // BLOCK_SIZE (:91)
    load_tile<T, D>(S.q, qh, t0, T_len);
    load_tile<T, D>(S.k, kh, t0, T_len);
    load_tile<T, D>(S.v, vh, t0, T_len);
    __syncthreads();

    for (int task = tid; task < 3 * D; task += blockDim.x) {
      const int which = task / D, c = task % D;
      if (which == 0) {
        float s = column_sum<T, D>(S.q, c);
        Elem<T>::store(qc_row + c, __fdiv_rn(s, len));
      } else if (which == 1) {
        float s = column_sum<T, D>(S.k, c);
        float m = __fdiv_rn(s, len);
        S.kc_f[c] = m;
        Elem<T>::store(kc_row + c, m);
      } else {
        float s = column_sum<T, D>(S.v, c);
        S.vc_f[c] = s;
        Elem<T>::store(vc_row + c, s);
      }
    }
    __syncthreads();

    // hc = k^T v - kc (x) vc on a MT x MT micro-tile per thread
    float acc[MT][MT];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int jx = 0; jx < MT; ++jx) acc[i][jx] = 0.f;
    for (int r = 0; r < kBlock; ++r) {
      float ka[MT], vb[MT];
#pragma unroll
      for (int i = 0; i < MT; ++i) ka[i] = Elem<T>::load(&S.k[r][a0 + i]);
#pragma unroll
      for (int i = 0; i < MT; ++i) vb[i] = Elem<T>::load(&S.v[r][b0 + i]);
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int jx = 0; jx < MT; ++jx) acc[i][jx] = fmaf(ka[i], vb[jx], acc[i][jx]);
    }
    float nsq = 0.f;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      const float kci = S.kc_f[a0 + i];
#pragma unroll
      for (int jx = 0; jx < MT; ++jx) {
        const float hc = fmaf(-kci, S.vc_f[b0 + jx], acc[i][jx]);
        nsq = fmaf(hc, hc, nsq);
        gsum[i][jx] += Elem<T>::round(hc);
      }
    }
    // block reduction of the squared norm
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) nsq += __shfl_xor_sync(0xffffffffu, nsq, off);
    if ((tid & 31) == 0) S.red[tid >> 5] = nsq;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int w = 0; w < int(blockDim.x / 32); ++w) tot += S.red[w];
      h_norm[bh * NT + j] = __fsqrt_rn(tot);
    }
    __syncthreads();  // tiles and kc_f/vc_f are rewritten by the next block
  }

  T* hg = h_group + ((bh * NG + g) * D) * D;
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int jx = 0; jx < MT; ++jx)
      Elem<T>::store(hg + (a0 + i) * D + (b0 + jx), gsum[i][jx] * (1.0f / kGroup));
}

template <typename T, int D>
static cudaError_t launch_prep_t(cudaStream_t st, const void* q, const void* k, const void* v,
                                 int64_t BH, int64_t T_len, int64_t NT, int64_t NG,
                                 void* qc, void* kc, void* vc, float* hn, void* hg) {
  const size_t smem = sizeof(PrepSmem<T, D>);
  auto kern = prep_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(NG), unsigned(BH), 1u};
  kern<<<grid, 256, smem, st>>>(static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v),
                                T_len, NT, NG, static_cast<T*>(qc), static_cast<T*>(kc), static_cast<T*>(vc),
                                hn, static_cast<T*>(hg));
  return cudaGetLastError();
}

cudaError_t launch_prep_tc(cudaStream_t st, int D, const void* q, const void* k, const void* v, int64_t BH,
                           int64_t T_len, void* qc, void* kc, void* vc, float* hn, void* hg, uint32_t* err);

cudaError_t launch_prep(cudaStream_t st, int dtype, int D, const void* q, const void* k, const void* v,
                        int64_t BH, int64_t T_len, void* qc, void* kc, void* vc, float* hn, void* hg, uint32_t* err) {
  const int64_t NT = cdiv(T_len, kBlock), NG = cdiv(NT, kGroup);
  // bf16: tensor-core kernels (prep_tc.cu); the CUDA-core kernel below serves fp32 inputs
  if (dtype == PASA_BF16) return launch_prep_tc(st, D, q, k, v, BH, T_len, qc, kc, vc, hn, hg, err);
  if (D == 64) return launch_prep_t<float, 64>(st, q, k, v, BH, T_len, NT, NG, qc, kc, vc, hn, hg);
  return launch_prep_t<float, 128>(st, q, k, v, BH, T_len, NT, NG, qc, kc, vc, hn, hg);
}

}  // namespace pasa
