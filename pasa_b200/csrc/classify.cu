// Head classification on the GPU: per head, the mean squared difference
// between attention under each emulated sparse mask (spatial, temporal) and
// full attention, on a few sampled query rows.  Replaces sample_mse
// (svg/models/hyvideo/attention.py:381-405; the Wan twin at
// svg/models/wan/attention.py:264-288) together with the emulated masks of
// get_attention_mask (svg/models/hyvideo/utils.py:48-94,
// svg/models/wan/utils.py:63-110), which the reference builds as dense T x T
// tensors with a Python double loop.  Here the masks are closed-form
// predicates on (query, key) positions.
//
// Arithmetic follows the reference's torch ops in the input dtype:
//   s   = round(round(q . k) * (1 / sqrt(D)))        matmul, then / dim**0.5
//   p   = round(exp(s - M) / L)                      F.softmax (fp32 inside)
//   h   = round(sum_j p_j v_j)                       matmul (fp32 accumulate)
//   mse = round(mean(round(round(h_m - h_full)^2)))  torch.mean over rows, D
// with round() the cast to the input dtype (bf16: nearest even).
//
// Five launches: (1) per key chunk, the masked row maxima and exponential
// sums of the three variants (full, spatial, temporal); (2) their
// combination per head; (3) per key chunk, the probabilities times V; (4)
// per slice of output elements, the sum over chunks in a fixed order, the
// rounded outputs and the squared differences; (5) per head, the slices in
// order and the two means.  Every sum has a fixed order, so the result is
// deterministic.  bf16 inputs run the scores and the probability-times-V
// products on the tensor cores (mma.sync m16n8k16, bf16 x bf16 -> fp32,
// the reference matmuls' arithmetic); fp32 inputs on CUDA cores.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace pasa {
namespace cls {

constexpr int kRows = 32;        // sampled rows (at most)
constexpr int kVar = 3;          // 0 full, 1 spatial, 2 temporal
constexpr int kTile = 64;        // keys per shared-memory tile
constexpr int kChunk = 2048;     // keys per CTA
constexpr int kThreads = 256;    // 8 warps x 4 rows; lanes take 2 keys of a tile

struct Spec {
  int64_t T, V, F, S;   // tokens, video tokens, frames, tokens per frame
  int64_t width;        // band half-width in 128-token blocks
  int model;            // 0 HunyuanVideo (text tail), 1 Wan (first-frame sink)
  int R;                // sampled rows
  int64_t rows[kRows];  // sampled query positions
  float inv_sqrt_d;
};

// frame-major position f*S + p -> token-major p*F + f (the reference's
// reshape(S, F, S, F).permute(1, 0, 3, 2) of the mask)
__device__ __forceinline__ int64_t token_major(int64_t x, const Spec& m) {
  const int64_t f = x / m.S;
  return (x - f * m.S) * m.F + f;
}

__device__ __forceinline__ bool allowed(int var, int64_t q, int64_t k, const Spec& m) {
  if (var == 0) return true;
  int64_t qm = q, km = k;
  if (var == 2) {
    qm = token_major(q < m.V ? q : m.V - 1, m);
    km = token_major(k < m.V ? k : m.V - 1, m);
  }
  const int64_t d = qm / 128 - km / 128;
  const bool band = (d < 0 ? -d : d) < m.width;
  if (m.model == 0) return (q < m.V && k < m.V) ? band : true;  // text rows and columns attend everything
  return band || km < m.S;                                        // Wan: first-frame sink
}

template <typename T>
__device__ __forceinline__ float rnd(float x) { return Elem<T>::round(x); }

// The mask-relevant facts of one position, computed once per row or key
// (the token-major index needs a division by the frame size): the same
// predicate as allowed(), split in two halves.
struct Pos {
  int32_t b_sp, b_tm;     // 128-token block in frame-major and in token-major order
  bool sink_sp, sink_tm;  // inside the first frame (Wan's sink), in either order
  bool text;              // a HunyuanVideo text token (attends and is attended by all)
};

__device__ __forceinline__ Pos pos_of(int64_t x, const Spec& m) {
  Pos p;
  const int64_t xc = x < m.V ? x : m.V - 1;
  const int64_t tm = token_major(xc, m);
  p.b_sp = int32_t(x / 128);
  p.b_tm = int32_t(tm / 128);
  p.sink_sp = x < m.S;
  p.sink_tm = tm < m.S;
  p.text = (m.model == 0) && x >= m.V;
  return p;
}

__device__ __forceinline__ bool allowed_pos(int var, const Pos& q, const Pos& k, const Spec& m) {
  if (var == 0) return true;
  if (m.model == 0 && (q.text || k.text)) return true;
  const int32_t d = (var == 1) ? q.b_sp - k.b_sp : q.b_tm - k.b_tm;
  const bool band = (d < 0 ? -d : d) < m.width;
  if (m.model == 0) return band;
  return band || (var == 1 ? k.sink_sp : k.sink_tm);
}

// Scores of this thread's 4 rows x 2 keys of the tile at j0 (rows 4*warp..,
// keys j0 + lane and j0 + lane + 32), or -inf past T.
template <typename T, int D>
__device__ __forceinline__ void tile_scores(const float* qs, const float* ks, int warp, int lane, int64_t j0,
                                            const Spec& m, float (&s)[4][2]) {
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const int jl = lane + 32 * kk;
    const float* kr = ks + jl * (D + 1);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const float* qr = qs + (4 * warp + rr) * D;
      float dot = 0.f;
#pragma unroll 8
      for (int c = 0; c < D; ++c) dot = fmaf(qr[c], kr[c], dot);
      s[rr][kk] = (j0 + jl < m.T) ? rnd<T>(rnd<T>(dot) * m.inv_sqrt_d) : -INFINITY;
    }
  }
}

template <typename T, int D>
__device__ __forceinline__ void load_rows(float* qs, const T* q, int64_t bh, const Spec& m) {
  for (int x = threadIdx.x; x < kRows * D; x += kThreads) {
    const int r = x / D, c = x % D;
    qs[x] = (r < m.R) ? Elem<T>::load(q + (bh * m.T + m.rows[r]) * D + c) : 0.f;
  }
}

template <typename T, int D>
__device__ __forceinline__ void load_tile(float* dst, int stride, const T* src, int64_t bh, int64_t j0,
                                          const Spec& m) {
  for (int x = threadIdx.x; x < kTile * D; x += kThreads) {
    const int j = x / D, c = x % D;
    dst[j * stride + c] = (j0 + j < m.T) ? Elem<T>::load(src + (bh * m.T + j0 + j) * D + c) : 0.f;
  }
}

// (1) per chunk: masked maximum and sum of exp(s - max) per (variant, row)
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) mse_stats_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                             const __grid_constant__ Spec m,
                                                             float2* __restrict__ part) {
  extern __shared__ float sm[];
  float* qs = sm;                  // [32][D]
  float* ks = qs + kRows * D;      // [64][D+1]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y, c = blockIdx.x;
  load_rows<T, D>(qs, q, bh, m);
  float mx[4][kVar], sum[4][kVar];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr)
#pragma unroll
    for (int v = 0; v < kVar; ++v) { mx[rr][v] = -INFINITY; sum[rr][v] = 0.f; }
  const int64_t jend = (c + 1) * kChunk < m.T ? (c + 1) * kChunk : m.T;
  for (int64_t j0 = c * kChunk; j0 < jend; j0 += kTile) {
    __syncthreads();
    load_tile<T, D>(ks, D + 1, k, bh, j0, m);
    __syncthreads();
    float s[4][2];
    tile_scores<T, D>(qs, ks, warp, lane, j0, m, s);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const int r = 4 * warp + rr;
      if (r >= m.R) continue;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int64_t j = j0 + lane + 32 * kk;
        if (j >= m.T) continue;
#pragma unroll
        for (int v = 0; v < kVar; ++v) {
          if (!allowed(v, m.rows[r], j, m)) continue;
          const float x = s[rr][kk];
          if (x > mx[rr][v]) {
            sum[rr][v] = sum[rr][v] * expf(mx[rr][v] - x) + 1.f;
            mx[rr][v] = x;
          } else {
            sum[rr][v] += expf(x - mx[rr][v]);
          }
        }
      }
    }
  }
  // combine the lanes (fixed butterfly order)
#pragma unroll
  for (int rr = 0; rr < 4; ++rr)
#pragma unroll
    for (int v = 0; v < kVar; ++v) {
      float a = mx[rr][v], b = sum[rr][v];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, a, off), ob = __shfl_xor_sync(0xffffffffu, b, off);
        const float nm = fmaxf(a, oa);
        b = (nm == -INFINITY) ? 0.f : b * expf(a - nm) + ob * expf(oa - nm);
        a = nm;
      }
      const int r = 4 * warp + rr;
      if (lane == 0) part[((bh * gridDim.x + c) * kVar + v) * kRows + r] = make_float2(a, b);
    }
}

// (2) per head: the row maxima M and sums L over all chunks
__global__ void mse_combine_kernel(const float2* __restrict__ part, int64_t nchunks, float2* __restrict__ ml) {
  const int64_t bh = blockIdx.x;
  const int t = threadIdx.x;  // v * 32 + r
  if (t >= kVar * kRows) return;
  float M = -INFINITY;
  for (int64_t c = 0; c < nchunks; ++c) M = fmaxf(M, part[(bh * nchunks + c) * kVar * kRows + t].x);
  float L = 0.f;
  for (int64_t c = 0; c < nchunks; ++c) {
    const float2 p = part[(bh * nchunks + c) * kVar * kRows + t];
    if (p.x != -INFINITY) L += p.y * expf(p.x - M);
  }
  ml[bh * kVar * kRows + t] = make_float2(M, L);
}

// (3) per chunk: sum_j round(exp(s - M) / L) v_j for the three variants
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) mse_pv_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                          const T* __restrict__ v, const __grid_constant__ Spec m,
                                                          const float2* __restrict__ ml, float* __restrict__ acc_out) {
  extern __shared__ float sm[];
  float* qs = sm;                        // [32][D]
  float* ks = qs + kRows * D;            // [64][D+1]
  float* vs = ks + kTile * (D + 1);      // [64][D]
  float* ps = vs + kTile * D;            // [3][32][64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y, c = blockIdx.x;
  load_rows<T, D>(qs, q, bh, m);
  // output elements of this thread: column col of rows rg*16 .. rg*16+15, every variant
  constexpr int kRG = kThreads / D;         // row groups (2 for D = 128, 4 for D = 64)
  constexpr int kRPT = kRows / kRG;         // rows per thread
  const int col = threadIdx.x % D, rg = threadIdx.x / D;
  float acc[kVar][kRPT];
#pragma unroll
  for (int x = 0; x < kVar; ++x)
#pragma unroll
    for (int r = 0; r < kRPT; ++r) acc[x][r] = 0.f;
  float2 mlr[4][kVar];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr)
#pragma unroll
    for (int x = 0; x < kVar; ++x) mlr[rr][x] = ml[(bh * kVar + x) * kRows + 4 * warp + rr];
  const int64_t jend = (c + 1) * kChunk < m.T ? (c + 1) * kChunk : m.T;
  for (int64_t j0 = c * kChunk; j0 < jend; j0 += kTile) {
    __syncthreads();
    load_tile<T, D>(ks, D + 1, k, bh, j0, m);
    load_tile<T, D>(vs, D, v, bh, j0, m);
    __syncthreads();
    float s[4][2];
    tile_scores<T, D>(qs, ks, warp, lane, j0, m, s);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const int r = 4 * warp + rr;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int jl = lane + 32 * kk;
        const int64_t j = j0 + jl;
#pragma unroll
        for (int x = 0; x < kVar; ++x) {
          float p = 0.f;
          if (r < m.R && j < m.T && allowed(x, m.rows[r], j, m))
            p = rnd<T>(expf(s[rr][kk] - mlr[rr][x].x) / mlr[rr][x].y);
          ps[(x * kRows + r) * kTile + jl] = p;
        }
      }
    }
    __syncthreads();
    for (int jl = 0; jl < kTile; ++jl) {
      const float vj = vs[jl * D + col];
#pragma unroll
      for (int x = 0; x < kVar; ++x)
#pragma unroll
        for (int r = 0; r < kRPT; ++r) acc[x][r] = fmaf(ps[(x * kRows + rg * kRPT + r) * kTile + jl], vj, acc[x][r]);
    }
  }
#pragma unroll
  for (int x = 0; x < kVar; ++x)
#pragma unroll
    for (int r = 0; r < kRPT; ++r)
      acc_out[(((bh * gridDim.x + c) * kVar + x) * kRows + rg * kRPT + r) * D + col] = acc[x][r];
}

// (4a) per slice of 256 output elements (row, column) of a head: the sum over
// chunks in order, the rounded outputs of the three variants and the two
// squared differences, summed over the slice in a fixed tree
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) mse_finish_part_kernel(const float* __restrict__ acc, int64_t nchunks,
                                                                   int R, float2* __restrict__ partial) {
  __shared__ float red[2][kThreads];
  const int64_t bh = blockIdx.y;
  const int e = blockIdx.x * kThreads + threadIdx.x;
  float part[2] = {0.f, 0.f};
  if (e < R * D) {
    float h[kVar];
#pragma unroll
    for (int x = 0; x < kVar; ++x) {
      float a = 0.f;
      for (int64_t c = 0; c < nchunks; ++c) a += acc[((bh * nchunks + c) * kVar + x) * kRows * D + e];
      h[x] = rnd<T>(a);
    }
#pragma unroll
    for (int x = 1; x < kVar; ++x) {
      const float d = rnd<T>(h[x] - h[0]);
      part[x - 1] = rnd<T>(d * d);
    }
  }
  red[0][threadIdx.x] = part[0];
  red[1][threadIdx.x] = part[1];
  __syncthreads();
  for (int w = kThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      red[0][threadIdx.x] += red[0][threadIdx.x + w];
      red[1][threadIdx.x] += red[1][threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[bh * gridDim.x + blockIdx.x] = make_float2(red[0][0], red[1][0]);
}

// (4b) per head: the slices in order, the mean, the class
template <typename T, int D>
__global__ void mse_finish_kernel(const float2* __restrict__ partial, int nslices, int R, int64_t BH,
                                  T* __restrict__ mse_out, int32_t* __restrict__ best) {
  const int64_t bh = blockIdx.x;
  if (threadIdx.x != 0) return;
  float s0 = 0.f, s1 = 0.f;
  for (int i = 0; i < nslices; ++i) {
    const float2 p = partial[bh * nslices + i];
    s0 += p.x;
    s1 += p.y;
  }
  const float inv_n = 1.0f / float(R * D);
  const float a = rnd<T>(s0 * inv_n), b = rnd<T>(s1 * inv_n);
  if (mse_out) {
    Elem<T>::store(mse_out + bh, a);       // [2, cfg*H]: spatial
    Elem<T>::store(mse_out + BH + bh, b);  // temporal
  }
  if (best) best[bh] = (b < a) ? 1 : 0;    // argmin, first index on ties
}

// ---------------------------------------------------------------------------
// tensor-core path (bf16): scores and probability-times-V on mma.sync
// m16n8k16 (bf16 x bf16 -> fp32, the reference matmuls' arithmetic) over the
// 32 sampled rows; 8 warps, a 64-key tile per step.
// ---------------------------------------------------------------------------
namespace tcp {

constexpr int kRS = 128 + 8;  // padded row stride (elements) of the bf16 tiles: conflict-free ldmatrix

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// rows [r][D] of a bf16 tensor into a padded shared tile (16-byte pieces)
template <int D>
__device__ __forceinline__ void load_rows_bf16(__nv_bfloat16* dst, const __nv_bfloat16* src, int64_t bh,
                                               int64_t T, const int64_t* rows, int nrows) {
  constexpr int kVec = D / 8;
  for (int x = threadIdx.x; x < kRows * kVec; x += kThreads) {
    const int r = x / kVec, c = x % kVec;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < nrows) val = reinterpret_cast<const uint4*>(src + (bh * T + rows[r]) * D)[c];
    *reinterpret_cast<uint4*>(dst + r * kRS + c * 8) = val;
  }
}
// A tile of keys (or values) staged by cp.async (16-byte pieces; rows >= T
// are zero-filled), so that the next tile's loads run while the current one
// is used.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
               :: "r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
template <int D>
__device__ __forceinline__ void async_tile_bf16(__nv_bfloat16* dst, const __nv_bfloat16* src, int64_t bh, int64_t T,
                                                int64_t j0) {
  constexpr int kVec = D / 8;
  for (int x = threadIdx.x; x < kTile * kVec; x += kThreads) {
    const int j = x / kVec, c = x % kVec;
    const bool valid = j0 + j < T;
    cp_async16(dst + j * kRS + c * 8, src + (valid ? (bh * T + j0 + j) * D + c * 8 : 0), valid);
  }
}

// Scores of the warp's 8 keys (keys 8*warp .. +7 of the tile) for all 32
// rows: s[mt][e] is row 16*mt + gq + 8*(e >= 2), key 8*warp + 2*tq + (e & 1),
// already rounded as the reference rounds them (-inf past T).
template <int D>
__device__ __forceinline__ void tile_scores_tc(const __nv_bfloat16* qs, const __nv_bfloat16* ks, int warp, int lane,
                                               int64_t j0, const Spec& m, float (&s)[2][4]) {
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[mt][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t b[2];
    {
      const int mat = (lane >> 3) & 1, i = lane & 7;
      ldsm_x2(b, ks + (8 * warp + i) * kRS + kk * 16 + mat * 8);
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      uint32_t a[4];
      const int mat = lane >> 3, i = lane & 7;
      ldsm_x4(a, qs + (16 * mt + i + ((mat & 1) ? 8 : 0)) * kRS + kk * 16 + ((mat >= 2) ? 8 : 0));
      mma16816(s[mt], a, b[0], b[1]);
    }
  }
  const int tq = lane & 3;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t j = j0 + 8 * warp + 2 * tq + (e & 1);
      s[mt][e] = (j < m.T) ? rnd<__nv_bfloat16>(rnd<__nv_bfloat16>(s[mt][e]) * m.inv_sqrt_d) : -INFINITY;
    }
}

template <int D>
__global__ void __launch_bounds__(kThreads) mse_stats_tc_kernel(const __nv_bfloat16* __restrict__ q,
                                                                const __nv_bfloat16* __restrict__ k,
                                                                const __grid_constant__ Spec m,
                                                                float2* __restrict__ part) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem_raw);     // [32][kRS]
  __nv_bfloat16* ks2 = qs + kRows * kRS;                                // [2 buffers][64][kRS]
  float2* red = reinterpret_cast<float2*>(ks2 + 2 * kTile * kRS);      // [8 warps][3][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  const int64_t bh = blockIdx.y, c = blockIdx.x;
  load_rows_bf16<D>(qs, q, bh, m.T, m.rows, m.R);
  Pos qp[4];  // this lane's rows 16*mt + gq + 8*h, x = 2*mt + h
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int r = 16 * (x >> 1) + gq + 8 * (x & 1);
    qp[x] = pos_of(m.rows[r < m.R ? r : 0], m);
  }
  // per lane: rows 16*mt + gq + 8*h (mt, h in {0, 1}), three variants
  float mx[4][kVar], sum[4][kVar];
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int v = 0; v < kVar; ++v) { mx[x][v] = -INFINITY; sum[x][v] = 0.f; }
  const int64_t jend = (c + 1) * kChunk < m.T ? (c + 1) * kChunk : m.T;
  int buf = 0;
  async_tile_bf16<D>(ks2, k, bh, m.T, c * kChunk);
  cp_async_commit();
  for (int64_t j0 = c * kChunk; j0 < jend; j0 += kTile, buf ^= 1) {
    __syncthreads();  // the tile before was read by every warp: its buffer may be refilled
    if (j0 + kTile < jend) async_tile_bf16<D>(ks2 + (buf ^ 1) * kTile * kRS, k, bh, m.T, j0 + kTile);
    cp_async_commit();
    cp_async_wait1();  // this thread's copies of tile j0 have landed
    __syncthreads();
    const __nv_bfloat16* ks = ks2 + buf * kTile * kRS;
    float s[2][4];
    tile_scores_tc<D>(qs, ks, warp, lane, j0, m, s);
    const Pos kp[2] = {pos_of(j0 + 8 * warp + 2 * tq, m), pos_of(j0 + 8 * warp + 2 * tq + 1, m)};
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rr = 2 * mt + (e >> 1), r = 16 * mt + gq + 8 * (e >> 1);
        const int64_t j = j0 + 8 * warp + 2 * tq + (e & 1);
        if (r >= m.R || j >= m.T) continue;
        const float xv = s[mt][e];
#pragma unroll
        for (int v = 0; v < kVar; ++v) {
          if (!allowed_pos(v, qp[rr], kp[e & 1], m)) continue;
          if (xv > mx[rr][v]) {
            sum[rr][v] = sum[rr][v] * expf(mx[rr][v] - xv) + 1.f;
            mx[rr][v] = xv;
          } else {
            sum[rr][v] += expf(xv - mx[rr][v]);
          }
        }
      }
  }
  // combine the 4 lanes of a row (fixed butterfly), then the 8 warps in order
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int v = 0; v < kVar; ++v) {
      float a = mx[x][v], b = sum[x][v];
#pragma unroll
      for (int off = 1; off < 4; off <<= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, a, off), ob = __shfl_xor_sync(0xffffffffu, b, off);
        const float nm = fmaxf(a, oa);
        b = (nm == -INFINITY) ? 0.f : b * expf(a - nm) + ob * expf(oa - nm);
        a = nm;
      }
      const int r = 16 * (x >> 1) + gq + 8 * (x & 1);
      if (tq == 0) red[(warp * kVar + v) * kRows + r] = make_float2(a, b);
    }
  __syncthreads();
  if (threadIdx.x < kVar * kRows) {
    const int t = threadIdx.x;  // v * 32 + r
    float a = -INFINITY, b = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) {
      const float2 p = red[w * kVar * kRows + t];
      const float nm = fmaxf(a, p.x);
      b = (nm == -INFINITY) ? 0.f : b * expf(a - nm) + p.y * expf(p.x - nm);
      a = nm;
    }
    part[(bh * gridDim.x + c) * kVar * kRows + t] = make_float2(a, b);
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads) mse_pv_tc_kernel(const __nv_bfloat16* __restrict__ q,
                                                             const __nv_bfloat16* __restrict__ k,
                                                             const __nv_bfloat16* __restrict__ v,
                                                             const __grid_constant__ Spec m,
                                                             const float2* __restrict__ ml,
                                                             float* __restrict__ acc_out) {
  constexpr int kPS = kTile + 8;  // padded stride of the probability tiles
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem_raw);     // [32][kRS]
  __nv_bfloat16* ks2 = qs + kRows * kRS;                                // [2 buffers][64][kRS]
  __nv_bfloat16* vs2 = ks2 + 2 * kTile * kRS;                           // [2 buffers][64][kRS]
  __nv_bfloat16* ps = vs2 + 2 * kTile * kRS;                            // [3][32][kPS]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  const int64_t bh = blockIdx.y, c = blockIdx.x;
  load_rows_bf16<D>(qs, q, bh, m.T, m.rows, m.R);
  float2 mlr[4][kVar];  // (M, L) of this lane's rows
  Pos qp[4];
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int r = 16 * (x >> 1) + gq + 8 * (x & 1);
    qp[x] = pos_of(m.rows[r < m.R ? r : 0], m);
#pragma unroll
    for (int vv = 0; vv < kVar; ++vv) mlr[x][vv] = ml[(bh * kVar + vv) * kRows + r];
  }
  // output columns of this warp: D / 8 warps, 16 (D=128) or 8 (D=64) per warp
  constexpr int kNT = D / 64;  // n-tiles of 8 columns per warp
  float acc[kVar][2][kNT][4];
#pragma unroll
  for (int vv = 0; vv < kVar; ++vv)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[vv][mt][nt][e] = 0.f;
  const int64_t jend = (c + 1) * kChunk < m.T ? (c + 1) * kChunk : m.T;
  int buf = 0;
  async_tile_bf16<D>(ks2, k, bh, m.T, c * kChunk);
  async_tile_bf16<D>(vs2, v, bh, m.T, c * kChunk);
  cp_async_commit();
  for (int64_t j0 = c * kChunk; j0 < jend; j0 += kTile, buf ^= 1) {
    __syncthreads();  // the tile before (and its probabilities) were read by every warp
    if (j0 + kTile < jend) {
      async_tile_bf16<D>(ks2 + (buf ^ 1) * kTile * kRS, k, bh, m.T, j0 + kTile);
      async_tile_bf16<D>(vs2 + (buf ^ 1) * kTile * kRS, v, bh, m.T, j0 + kTile);
    }
    cp_async_commit();
    cp_async_wait1();  // this thread's copies of tile j0 have landed
    __syncthreads();
    const __nv_bfloat16* ks = ks2 + buf * kTile * kRS;
    const __nv_bfloat16* vs = vs2 + buf * kTile * kRS;
    float s[2][4];
    tile_scores_tc<D>(qs, ks, warp, lane, j0, m, s);
    const Pos kp[2] = {pos_of(j0 + 8 * warp + 2 * tq, m), pos_of(j0 + 8 * warp + 2 * tq + 1, m)};
    // p = round(exp(s - M) / L), 0 where the mask (or T) excludes the key
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int x = 2 * mt + h, r = 16 * mt + gq + 8 * h;
        const int jl = 8 * warp + 2 * tq;
#pragma unroll
        for (int vv = 0; vv < kVar; ++vv) {
          float p2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int64_t j = j0 + jl + u;
            p2[u] = (r < m.R && j < m.T && allowed_pos(vv, qp[x], kp[u], m))
                        ? expf(s[mt][2 * h + u] - mlr[x][vv].x) / mlr[x][vv].y : 0.f;
          }
          *reinterpret_cast<uint32_t*>(ps + (vv * kRows + r) * kPS + jl) = pack_bf16x2(p2[0], p2[1]);
        }
      }
    __syncthreads();
    // acc[vv] += P[vv] (32 x 64) . V (64 x D): this warp's columns
#pragma unroll
    for (int kk = 0; kk < kTile / 16; ++kk) {
      uint32_t bf[kNT == 2 ? 4 : 2];
      {
        const int mat = lane >> 3, i = lane & 7;
        const int row = kk * 16 + i + ((mat & 1) ? 8 : 0);
        const int col = warp * 8 * kNT + ((mat >= 2) ? 8 : 0);
        if constexpr (kNT == 2) {
          ldsm_x4_trans(bf, vs + row * kRS + col);
        } else {
          uint32_t t4[4];
          ldsm_x4_trans(t4, vs + row * kRS + col);
          bf[0] = t4[0];
          bf[1] = t4[1];
        }
      }
#pragma unroll
      for (int vv = 0; vv < kVar; ++vv)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t a[4];
          const int mat = lane >> 3, i = lane & 7;
          ldsm_x4(a, ps + (vv * kRows + 16 * mt + i + ((mat & 1) ? 8 : 0)) * kPS + kk * 16 + ((mat >= 2) ? 8 : 0));
          mma16816(acc[vv][mt][0], a, bf[0], bf[1]);
          if constexpr (kNT == 2) mma16816(acc[vv][mt][1], a, bf[2], bf[3]);
        }
    }
  }
#pragma unroll
  for (int vv = 0; vv < kVar; ++vv)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = 16 * mt + gq + 8 * (e >> 1);
          const int col = warp * 8 * kNT + 8 * nt + 2 * tq + (e & 1);
          acc_out[(((bh * gridDim.x + c) * kVar + vv) * kRows + r) * D + col] = acc[vv][mt][nt][e];
        }
}

template <int D>
size_t stats_smem() { return size_t(kRows + 2 * kTile) * kRS * 2 + size_t(kThreads / 32) * kVar * kRows * 8; }
template <int D>
size_t pv_smem() { return size_t(kRows + 4 * kTile) * kRS * 2 + size_t(kVar) * kRows * (kTile + 8) * 2; }

}  // namespace tcp

template <int D>
size_t stats_smem() { return sizeof(float) * (kRows * D + kTile * (D + 1)); }
template <int D>
size_t pv_smem() { return sizeof(float) * (kRows * D + kTile * (D + 1) + kTile * D + kVar * kRows * kTile); }

}  // namespace cls

// workspace: chunk statistics | (M, L) | chunk partial outputs | slice sums
size_t sample_mse_workspace(int64_t BH, int64_t T, int D) {
  const int64_t nc = cdiv(T, cls::kChunk);
  size_t o = align256(size_t(BH) * nc * cls::kVar * cls::kRows * sizeof(float2));
  o += align256(size_t(BH) * cls::kVar * cls::kRows * sizeof(float2));
  o += align256(size_t(BH) * nc * cls::kVar * cls::kRows * D * sizeof(float));
  o += align256(size_t(BH) * cdiv(cls::kRows * D, cls::kThreads) * sizeof(float2));
  return o;
}

template <typename T, int D>
static cudaError_t launch_sample_mse_t(cudaStream_t st, const void* q, const void* k, const void* v, int64_t BH,
                                       const cls::Spec& m, void* ws, void* mse_out, int32_t* best) {
  using namespace cls;
  const int64_t nc = cdiv(m.T, kChunk);
  char* w = static_cast<char*>(ws);
  float2* part = reinterpret_cast<float2*>(w);
  w += align256(size_t(BH) * nc * kVar * kRows * sizeof(float2));
  float2* ml = reinterpret_cast<float2*>(w);
  w += align256(size_t(BH) * kVar * kRows * sizeof(float2));
  float* acc = reinterpret_cast<float*>(w);
  w += align256(size_t(BH) * nc * kVar * kRows * D * sizeof(float));
  float2* slices = reinterpret_cast<float2*>(w);
  const int nslices = int(cdiv(kRows * D, kThreads));
  const dim3 grid{unsigned(nc), unsigned(BH), 1u};
  const T* qt = static_cast<const T*>(q);
  const T* kt = static_cast<const T*>(k);
  const T* vt = static_cast<const T*>(v);
  cudaError_t e;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {  // scores and P.V on the tensor cores
    auto k1 = tcp::mse_stats_tc_kernel<D>;
    auto k3 = tcp::mse_pv_tc_kernel<D>;
    e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(tcp::stats_smem<D>()));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, int(tcp::pv_smem<D>()));
    if (e != cudaSuccess) return e;
    k1<<<grid, kThreads, tcp::stats_smem<D>(), st>>>(qt, kt, m, part);
    mse_combine_kernel<<<unsigned(BH), 128, 0, st>>>(part, nc, ml);
    k3<<<grid, kThreads, tcp::pv_smem<D>(), st>>>(qt, kt, vt, m, ml, acc);
  } else {
    auto k1 = mse_stats_kernel<T, D>;
    auto k3 = mse_pv_kernel<T, D>;
    e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(stats_smem<D>()));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, int(pv_smem<D>()));
    if (e != cudaSuccess) return e;
    k1<<<grid, kThreads, stats_smem<D>(), st>>>(qt, kt, m, part);
    mse_combine_kernel<<<unsigned(BH), 128, 0, st>>>(part, nc, ml);
    k3<<<grid, kThreads, pv_smem<D>(), st>>>(qt, kt, vt, m, ml, acc);
  }
  mse_finish_part_kernel<T, D><<<dim3(unsigned(nslices), unsigned(BH), 1u), kThreads, 0, st>>>(acc, nc, m.R, slices);
  mse_finish_kernel<T, D><<<unsigned(BH), 32, 0, st>>>(slices, nslices, m.R, BH, static_cast<T*>(mse_out), best);
  return cudaGetLastError();
}

cudaError_t launch_sample_mse(cudaStream_t st, int dtype, int D, const void* q, const void* k, const void* v,
                              int64_t BH, int64_t T, const int64_t* rows, int R, int model, int64_t ctx,
                              int64_t num_frame, int64_t frame_size, void* ws, void* mse_out, int32_t* best) {
  cls::Spec m{};
  m.T = T;
  m.V = num_frame * frame_size;
  m.F = num_frame;
  m.S = frame_size;
  // (factor * frame_size) // 128 with factor 1.5 (HunyuanVideo) or 2 (Wan)
  m.width = (model == 0) ? (3 * frame_size) / 256 : frame_size / 64;
  m.model = model;
  m.R = R;
  for (int r = 0; r < R; ++r) m.rows[r] = rows[r];
  m.inv_sqrt_d = 1.0f / float(std::sqrt(double(D)));
  if (dtype == PASA_BF16) {
    if (D == 64) return launch_sample_mse_t<__nv_bfloat16, 64>(st, q, k, v, BH, m, ws, mse_out, best);
    return launch_sample_mse_t<__nv_bfloat16, 128>(st, q, k, v, BH, m, ws, mse_out, best);
  }
  if (D == 64) return launch_sample_mse_t<float, 64>(st, q, k, v, BH, m, ws, mse_out, best);
  return launch_sample_mse_t<float, 128>(st, q, k, v, BH, m, ws, mse_out, best);
}

}  // namespace pasa
