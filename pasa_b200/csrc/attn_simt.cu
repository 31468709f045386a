// CUDA-core PASA attention: one CTA per (head, 64-query block).
//
// Follows pisa_pg_fwd_kernel (svg/kernels/triton/group_pisa_attention.py:
// 136-262) step by step: Phase 1 walks the selected blocks in top-k order
// with an online softmax (:170-186); Phase 2 walks the 32-block groups,
// applying the zero-order term to every non-selected block and the
// per-group first-order term q.H_g (:212-253); the final division uses
// l + g_l, where g_l is accumulated without the running-max rescale,
// exactly as the reference does (:242-243, :258-259).
//
// This kernel serves fp32 inputs (products in exact fp32) and is the
// reference-structured check for the tcgen05 kernel on bf16 inputs (bf16
// probabilities before the P.V product, fp32 accumulation).
#include "common.cuh"

namespace pasa {

constexpr int kSimtThreads = 256;

template <int D>
struct SimtSmem {
  float q[kBlock][D];
  float a[kBlock][D];      // K block, or kc rows of a group
  float b[kBlock][D];      // V block, or vc rows of a group
  float h[D][D];           // h_group[g]
  float s[kBlock][kBlock + 1];
  float m[kBlock], l[kBlock], gl[kBlock], alpha[kBlock], gps[kBlock];
  uint32_t selw[64];       // selection bits of this query block, word per group
};

template <typename T, int D>
__device__ __forceinline__ void load_rows(float (*dst)[D], const T* src, int64_t row0, int64_t nrows_valid, int nrows) {
  for (int x = threadIdx.x; x < nrows * D; x += blockDim.x) {
    const int r = x / D, c = x % D;
    dst[r][c] = (row0 + r < nrows_valid) ? Elem<T>::load(src + (row0 + r) * D + c) : 0.f;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kSimtThreads) attn_simt_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ kc, const T* __restrict__ vc, const T* __restrict__ hg,
    const int32_t* __restrict__ indices, const uint32_t* __restrict__ sel_mask,
    int64_t T_len, int64_t NT, int64_t NG, int64_t NS, float scale, T* __restrict__ o) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  auto& S = *reinterpret_cast<SimtSmem<D>*>(smem_raw);
  constexpr int CPT = D / 4;  // output columns per thread
  const int tid = threadIdx.x;
  const int64_t it = blockIdx.x, bh = blockIdx.y;
  const int64_t NTP = NG * kGroup;
  const float scale32 = scale;
  const float sm_scale = scale32 * kLog2e;  // :162

  const T* qh = q + bh * T_len * D;
  const T* kh = k + bh * T_len * D;
  const T* vh = v + bh * T_len * D;
  load_rows<T, D>(S.q, qh, it * kBlock, T_len, kBlock);
  for (int w = tid; w < NG; w += blockDim.x) S.selw[w] = sel_mask[(bh * NT + it) * NG + w];
  if (tid < kBlock) { S.m[tid] = -INFINITY; S.l[tid] = 0.f; S.gl[tid] = 0.f; }

  // thread tiles: S-tile 4x4 at (ty, tx); accumulator row ar, columns ac0..ac0+CPT
  const int ty = tid / 16, tx = tid % 16;
  const int ar = tid / 4, ac0 = (tid % 4) * CPT;
  float acc[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) acc[c] = 0.f;

  // -------------------------- Phase 1 ----------------------------------
  for (int64_t n = 0; n < NS; ++n) {
    const int64_t j = indices[(bh * NT + it) * NS + n];
    __syncthreads();
    load_rows<T, D>(S.a, kh, j * kBlock, T_len, kBlock);
    load_rows<T, D>(S.b, vh, j * kBlock, T_len, kBlock);
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < 4; ++rr)
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int r = ty * 4 + rr, c = tx * 4 + cc;
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot = fmaf(S.q[r][d], S.a[c][d], dot);
        float sv = dot * sm_scale;
        if (j * kBlock + c >= T_len) sv = -INFINITY;  // :178
        S.s[r][c] = sv;
      }
    __syncthreads();
    {  // row statistics: 4 threads per row, 16 columns each
      const int r = tid / 4, part = tid % 4;
      float mx = -INFINITY;
      for (int c = part * 16; c < part * 16 + 16; ++c) mx = fmaxf(mx, S.s[r][c]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_old = S.m[r];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int c = part * 16; c < part * 16 + 16; ++c) {
        const float p = fast_exp2(S.s[r][c] - m_new);
        sum += p;
        S.s[r][c] = Elem<T>::round(p);  // score.to(v dtype) before the dot (:185)
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      __syncwarp();
      if (part == 0) {
        const float al = fast_exp2(m_old - m_new);
        S.alpha[r] = al;
        S.l[r] = S.l[r] * al + sum;
        S.m[r] = m_new;
      }
    }
    __syncthreads();
    {
      const float al = S.alpha[ar];
      float pv[CPT];
#pragma unroll
      for (int c = 0; c < CPT; ++c) pv[c] = 0.f;
      for (int u = 0; u < kBlock; ++u) {
        const float p = S.s[ar][u];
#pragma unroll
        for (int c = 0; c < CPT; ++c) pv[c] = fmaf(p, S.b[u][ac0 + c], pv[c]);
      }
#pragma unroll
      for (int c = 0; c < CPT; ++c) acc[c] = acc[c] * al + pv[c];
    }
  }

  // -------------------------- Phase 2 ----------------------------------
  const T* kch = kc + bh * NTP * D;
  const T* vch = vc + bh * NTP * D;
  const int64_t last_len = T_len - (NT - 1) * kBlock;  // :191
  for (int64_t g = 0; g < NG; ++g) {
    __syncthreads();
    load_rows<T, D>(S.a, kch, g * kGroup, NTP, kGroup);
    load_rows<T, D>(S.b, vch, g * kGroup, NTP, kGroup);
    for (int x = tid; x < D * D; x += blockDim.x)
      S.h[x / D][x % D] = Elem<T>::load(hg + (bh * NG + g) * D * D + x);
    __syncthreads();
    // zero-order logits against the 32 block means
    for (int x = tid; x < kBlock * kGroup; x += blockDim.x) {
      const int r = x / kGroup, c = x % kGroup;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(S.q[r][d], S.a[c][d], dot);
      float sv = dot * sm_scale;
      const int64_t jb = g * kGroup + c;
      const bool selected = (S.selw[g] >> c) & 1u;
      if (jb >= NT || selected) sv = -INFINITY;  // :228-229
      S.s[r][c] = sv;
    }
    __syncthreads();
    {
      const int r = tid / 4, part = tid % 4;  // 8 columns each
      float mx = -INFINITY;
      for (int c = part * 8; c < part * 8 + 8; ++c) mx = fmaxf(mx, S.s[r][c]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_old = S.m[r];
      const float m_new = fmaxf(m_old, mx);
      float psum = 0.f, wsum = 0.f;
      for (int c = part * 8; c < part * 8 + 8; ++c) {
        const float p = fast_exp2(S.s[r][c] - m_new);
        const int64_t jb = g * kGroup + c;
        const float len = (jb == NT - 1) ? float(last_len) : float(kBlock);  // :220
        psum += p;
        wsum += p * len;
        S.s[r][c] = Elem<T>::round(p);
      }
      psum += __shfl_xor_sync(0xffffffffu, psum, 1);
      psum += __shfl_xor_sync(0xffffffffu, psum, 2);
      wsum += __shfl_xor_sync(0xffffffffu, wsum, 1);
      wsum += __shfl_xor_sync(0xffffffffu, wsum, 2);
      __syncwarp();
      if (part == 0) {
        const float al = fast_exp2(m_old - m_new);
        S.alpha[r] = al;
        S.l[r] = S.l[r] * al;      // :234
        S.m[r] = m_new;
        S.gl[r] = S.gl[r] + wsum;  // :243, no rescale
        S.gps[r] = psum;           // :252
      }
    }
    __syncthreads();
    {
      const float al = S.alpha[ar];
      const float w = S.gps[ar] * scale32;  // :253
      float pv[CPT], rv[CPT];
#pragma unroll
      for (int c = 0; c < CPT; ++c) { pv[c] = 0.f; rv[c] = 0.f; }
      for (int u = 0; u < kGroup; ++u) {
        const float p = S.s[ar][u];
#pragma unroll
        for (int c = 0; c < CPT; ++c) pv[c] = fmaf(p, S.b[u][ac0 + c], pv[c]);
      }
      for (int d = 0; d < D; ++d) {
        const float qd = S.q[ar][d];
#pragma unroll
        for (int c = 0; c < CPT; ++c) rv[c] = fmaf(qd, S.h[d][ac0 + c], rv[c]);
      }
#pragma unroll
      for (int c = 0; c < CPT; ++c) acc[c] = (acc[c] * al + pv[c]) + rv[c] * w;
    }
  }

  // -------------------------- Final ------------------------------------
  __syncthreads();
  const int64_t t = it * kBlock + ar;
  if (t < T_len) {
    const float denom = S.l[ar] + S.gl[ar];  // :258
    T* orow = o + (bh * T_len + t) * D;
#pragma unroll
    for (int c = 0; c < CPT; ++c) Elem<T>::store(orow + ac0 + c, __fdiv_rn(acc[c], denom));
  }
}

template <typename T, int D>
static cudaError_t launch_simt_t(cudaStream_t st, const void* q, const void* k, const void* v, const void* kc,
                                 const void* vc, const void* hg, const int32_t* idx, const uint32_t* mask,
                                 int64_t BH, int64_t T_len, int64_t NS, float scale, void* o) {
  const int64_t NT = cdiv(T_len, kBlock), NG = cdiv(NT, kGroup);
  const size_t smem = sizeof(SimtSmem<D>);
  auto kern = attn_simt_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(NT), unsigned(BH), 1u};
  kern<<<grid, kSimtThreads, smem, st>>>(
      static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(kc),
      static_cast<const T*>(vc), static_cast<const T*>(hg), idx, mask, T_len, NT, NG, NS, scale,
      static_cast<T*>(o));
  return cudaGetLastError();
}

cudaError_t launch_attn_simt(cudaStream_t st, int dtype, int D, const void* q, const void* k, const void* v,
                             const void* kc, const void* vc, const void* hg, const int32_t* idx,
                             const uint32_t* mask, int64_t BH, int64_t T_len, int64_t NS, float scale,
                             void* o) {
  if (dtype == PASA_BF16) {
    if (D == 64) return launch_simt_t<__nv_bfloat16, 64>(st, q, k, v, kc, vc, hg, idx, mask, BH, T_len, NS, scale, o);
    return launch_simt_t<__nv_bfloat16, 128>(st, q, k, v, kc, vc, hg, idx, mask, BH, T_len, NS, scale, o);
  }
  if (D == 64) return launch_simt_t<float, 64>(st, q, k, v, kc, vc, hg, idx, mask, BH, T_len, NS, scale, o);
  return launch_simt_t<float, 128>(st, q, k, v, kc, vc, hg, idx, mask, BH, T_len, NS, scale, o);
}

}  // namespace pasa
