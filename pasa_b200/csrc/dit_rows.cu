// Row kernels of the Wan2.1 DiT block around the attention op: the
// elementwise work between the GEMMs, fused so that each activation row
// crosses HBM once per use.  All are HBM-bound.
//
// row_norm_kernel — optional gated residual, then LayerNorm (centered) or
// RMSNorm, optional affine, optional (1 + scale) / shift modulation:
//     x'  = bf16(x + add * gate)          (custom_models.py:58-65, :82-83,
//                                          modulate.py:90-122)
//     y   = bf16(((x' - mean) * rstd) [* w + b] [* (1 + scale) + shift])
//                                         (layernorm.py:13-58, :113-155,
//                                          modulate.py:12-42, rmsnorm.py:8-48)
//     mean = sum(x') / C,  var = sum((x' - mean)^2) / C,  rstd = 1 / sqrt(var + eps)
// (optionally with the reference Triton LayerNorm's padding term: its rows are
// padded with zeros to the next power of two and every padding column adds
// (0 - mean)^2 to the sum of squares, layernorm.py:40-42)
// The reference runs these as separate Triton kernels with fp32
// intermediates in HBM; here the fp32 intermediates stay in registers, so the
// values are the same while the traffic drops to one read and one write.
//
// qkv_rope_kernel — the self-attention producer: RMSNorm of the q and k rows
// over the hidden dimension (rmsnorm.py:8-48, rounded to bf16), the rotary
// embedding of each head's (2i, 2i+1) pairs as a complex multiply in fp64
// (the reference's fallback, svg/models/wan/attention.py:49-57: bf16 ->
// float64, times cos + i sin, -> bf16 through float32 as torch casts), and the
// [B, T, H*D] -> [B, H, T, D] transpose of q, k and v (attention.py:136-141),
// all in one pass.
//
// Data movement (B200): one 128-thread CTA per token row; every thread
// issues all of its 16-byte loads of the row (and of the residual branch /
// the k and v rows) before using any, and holds the row between the two
// reduction passes as packed bf16 (the values are bf16-exact), which keeps the
// register footprint small enough for 12 CTAs per SM: rows of many CTAs are
// in flight at once, which is what an HBM-bound row op needs.  Outputs are
// written with 16-byte stores straight from registers.  (A variant that
// staged rows through a shared-memory ring filled by bulk copies, with fewer
// CTAs per SM, was slower: per row the work is a few thousand warp
// instructions, so the kernel needs many resident rows, not deep prefetch.)
//
// Arithmetic is written with explicit round-to-nearest intrinsics (no fused
// multiply-add) and a fixed reduction order: per thread in vector order
// (thread t owns the 16-byte vectors t, t + 128, ...), then an xor butterfly
// over the warp, then the four warp sums in order.  The CPU restatement in the
// test oracle follows the same order, so the results compare bit for bit.
#include "common.cuh"

namespace pasa {
namespace {

constexpr int kRowThreads = 128;
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kMaxVec = 8;        // 16-byte vectors per thread: cols <= 8 * 8 * 128
constexpr int kRowMinBlocks = 8;  // resident CTAs per SM the register budget is cut for (row_norm)
constexpr int kQkvMinBlocks = 6;  // the same for qkv_rope (two rows in registers)
// Kernels are instantiated for V = ceil(cols / (8 * 128)) vectors per thread,
// so the register arrays are no larger than the row needs (V = 5 at C = 5120).

__device__ __forceinline__ void unpack8(const uint4 u, float* out) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Round eight floats to bf16 (nearest even) and pack them.
__device__ __forceinline__ uint4 pack8(const float* in) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint4 ld16(const __nv_bfloat16* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void st16(__nv_bfloat16* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

__device__ __forceinline__ void load8f(const float* p, float* out) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

// Sum over the CTA in a fixed order; every thread gets the same value.
__device__ __forceinline__ float block_sum(float acc, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < kRowWarps; ++w) t = __fadd_rn(t, red[w]);
  __syncthreads();  // red is reused by the next reduction
  return t;
}

// Two independent sums with one pair of barriers (same order as block_sum).
__device__ __forceinline__ float2 block_sum2(float a, float b, float2* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, off));
    b = __fadd_rn(b, __shfl_xor_sync(0xffffffffu, b, off));
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(a, b);
  __syncthreads();
  float2 t = red[0];
#pragma unroll
  for (int w = 1; w < kRowWarps; ++w) {
    t.x = __fadd_rn(t.x, red[w].x);
    t.y = __fadd_rn(t.y, red[w].y);
  }
  __syncthreads();
  return t;
}

struct RowNormArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* add;  // residual branch, or null
  const float* gate;         // [B, C] gate of the residual branch, or null (plain add)
  __nv_bfloat16* x_out;      // updated residual stream (may alias x), or null
  const float* w;            // [C] affine weight, or null
  const float* b;            // [C] affine bias, or null
  const float* scale;        // [B, C] modulation, or null (then shift is ignored)
  const float* shift;        // [B, C]
  __nv_bfloat16* y;
  int64_t batch_rows;        // rows per batch entry of gate / scale / shift
  int cols;
  float eps;
  int center;                // 1: LayerNorm, 0: RMSNorm
  int pad_cols;              // > 0: add pad_cols * mean^2 to the sum of squares
};

template <int V>
__global__ void __launch_bounds__(kRowThreads, kRowMinBlocks) row_norm_kernel(RowNormArgs a) {
  __shared__ float red[kRowWarps];
  const int64_t row = blockIdx.x;
  const int nvec = a.cols >> 3;
  const int tid = threadIdx.x;
  const int64_t base = row * a.cols;
  const int64_t vb = (row / a.batch_rows) * a.cols;
  const bool has_add = a.add != nullptr;

  uint4 xv[V], av[V];
#pragma unroll
  for (int k = 0; k < V; ++k) {  // every load of the row in flight before any use
    const int j = tid + k * kRowThreads;
    if (j < nvec) {
      xv[k] = ld16(a.x + base + 8 * j);
      if (has_add) av[k] = ld16(a.add + base + 8 * j);
    }
  }
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int j = tid + k * kRowThreads;
    if (j < nvec) {
      float v[8];
      unpack8(xv[k], v);
      if (has_add) {
        float r[8];
        unpack8(av[k], r);
        if (a.gate != nullptr) {
          float g[8];
          load8f(a.gate + vb + 8 * j, g);
#pragma unroll
          for (int e = 0; e < 8; ++e) r[e] = __fmul_rn(r[e], g[e]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], r[e]);
        xv[k] = pack8(v);  // x' = bf16(x + add * gate)
        unpack8(xv[k], v);
        if (a.x_out != nullptr) st16(a.x_out + base + 8 * j, xv[k]);
      }
      if (a.center) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = __fadd_rn(acc, v[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = __fadd_rn(acc, __fmul_rn(v[e], v[e]));
      }
    }
  }
  const float first = block_sum(acc, red);
  float mean = 0.f, ssq = first;
  if (a.center) {
    mean = __fdiv_rn(first, float(a.cols));
    float acc2 = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      if (tid + k * kRowThreads < nvec) {
        float v[8];
        unpack8(xv[k], v);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = __fsub_rn(v[e], mean);
          acc2 = __fadd_rn(acc2, __fmul_rn(d, d));
        }
      }
    }
    ssq = block_sum(acc2, red);
    if (a.pad_cols > 0) ssq = __fadd_rn(ssq, __fmul_rn(float(a.pad_cols), __fmul_rn(mean, mean)));
  }
  const float var = __fdiv_rn(ssq, float(a.cols));
  const float rstd = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, a.eps)));
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int j = tid + k * kRowThreads;
    if (j < nvec) {
      float o[8];
      unpack8(xv[k], o);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(__fsub_rn(o[e], mean), rstd);
      if (a.w != nullptr) {
        float w[8];
        load8f(a.w + 8 * j, w);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(o[e], w[e]);
      }
      if (a.b != nullptr) {
        float b[8];
        load8f(a.b + 8 * j, b);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = __fadd_rn(o[e], b[e]);
      }
      if (a.scale != nullptr) {
        float sc[8], sh[8];
        load8f(a.scale + vb + 8 * j, sc);
        load8f(a.shift + vb + 8 * j, sh);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = __fadd_rn(__fmul_rn(o[e], __fadd_rn(1.f, sc[e])), sh[e]);
      }
      st16(a.y + base + 8 * j, pack8(o));
    }
  }
}

struct QkvArgs {
  const __nv_bfloat16* xq;
  const __nv_bfloat16* xk;  // or null
  const __nv_bfloat16* xv;  // or null
  const float* wq;
  const float* wk;
  const double* cos;        // [tokens, D/2] or null (no rotation)
  const double* sin;
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  int64_t tokens;
  int cols, head_dim;
  float eps;
  int head_major;           // 1: [B, H, tokens, D]; 0: [B, tokens, H*D]
  __nv_bfloat16* const* peer;  // scatter mode: device table of the ranks' [3][H/P][P*tokens][D] buffers
  int npeer;                // 0: write q, k, v; P > 0: scatter to the P ranks
  int rank;                 // scatter mode: this rank (its tokens start at rank * tokens)
};

// Destination of the 8 values at column c of token t (which: 0 q, 1 k, 2 v).
__device__ __forceinline__ __nv_bfloat16* out_ptr(const QkvArgs& a, int which, int64_t bidx, int64_t t, int c) {
  const int h = c / a.head_dim, d = c - h * a.head_dim;
  if (a.npeer > 0) {
    const int hl = (a.cols / a.head_dim) / a.npeer;
    const int dst = h / hl, hh = h - dst * hl;
    const int64_t rows = a.tokens * a.npeer;
    return a.peer[dst] + ((int64_t(which) * hl + hh) * rows + int64_t(a.rank) * a.tokens + t) * a.head_dim + d;
  }
  __nv_bfloat16* base = which == 0 ? a.q : (which == 1 ? a.k : a.v);
  if (!a.head_major) return base + (bidx * a.tokens + t) * a.cols + c;
  const int64_t H = a.cols / a.head_dim;
  return base + ((bidx * H + h) * a.tokens + t) * a.head_dim + d;
}

// bf16(x * rstd * w), then the rotation of its four pairs by the token's
// angles (fp64 complex multiply, rounded through fp32), packed.
__device__ __forceinline__ uint4 norm_rope8(bool rotate, uint4 xp, float rstd, const float* w, const double* cs,
                                            const double* sn) {
  float o[8];
  unpack8(xp, o);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(__fmul_rn(o[e], rstd), w[e]);
  uint4 n = pack8(o);
  if (!rotate) return n;
  unpack8(n, o);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const double re = o[2 * p], im = o[2 * p + 1];
    o[2 * p] = __double2float_rn(__dsub_rn(__dmul_rn(re, cs[p]), __dmul_rn(im, sn[p])));
    o[2 * p + 1] = __double2float_rn(__dadd_rn(__dmul_rn(re, sn[p]), __dmul_rn(im, cs[p])));
  }
  return pack8(o);
}

template <int V>
__global__ void __launch_bounds__(kRowThreads, kQkvMinBlocks) qkv_rope_kernel(QkvArgs a) {
  __shared__ float2 red[kRowWarps];
  const int64_t row = blockIdx.x;
  const int64_t bidx = row / a.tokens, t = row - bidx * a.tokens;
  const int nvec = a.cols >> 3;
  const int tid = threadIdx.x;
  const int64_t base = row * a.cols;
  const bool has_k = a.xk != nullptr, rotate = a.cos != nullptr;

  uint4 qv[V], kv[V];
#pragma unroll
  for (int k = 0; k < V; ++k) {  // q and k rows in flight together
    const int j = tid + k * kRowThreads;
    if (j < nvec) {
      qv[k] = ld16(a.xq + base + 8 * j);
      if (has_k) kv[k] = ld16(a.xk + base + 8 * j);
    }
  }
  if (a.xv != nullptr) {  // v: a transposing copy
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int j = tid + k * kRowThreads;
      if (j < nvec) st16(out_ptr(a, 2, bidx, t, 8 * j), ld16(a.xv + base + 8 * j));
    }
  }
  float accq = 0.f, acck = 0.f;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    if (tid + k * kRowThreads < nvec) {
      float v[8];
      unpack8(qv[k], v);
#pragma unroll
      for (int e = 0; e < 8; ++e) accq = __fadd_rn(accq, __fmul_rn(v[e], v[e]));
      if (has_k) {
        unpack8(kv[k], v);
#pragma unroll
        for (int e = 0; e < 8; ++e) acck = __fadd_rn(acck, __fmul_rn(v[e], v[e]));
      }
    }
  }
  const float2 sums = block_sum2(accq, acck, red);
  const float rq = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sums.x, float(a.cols)), a.eps)));
  const float rk = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sums.y, float(a.cols)), a.eps)));
  const int half = a.head_dim >> 1;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int j = tid + k * kRowThreads;
    if (j < nvec) {
      const int c = 8 * j;
      double cs[4] = {0, 0, 0, 0}, sn[4] = {0, 0, 0, 0};
      if (rotate) {
        const int p0 = (c % a.head_dim) >> 1;
        const double2* cp = reinterpret_cast<const double2*>(a.cos + t * half + p0);
        const double2* sp = reinterpret_cast<const double2*>(a.sin + t * half + p0);
        const double2 c01 = __ldg(cp), c23 = __ldg(cp + 1), s01 = __ldg(sp), s23 = __ldg(sp + 1);
        cs[0] = c01.x; cs[1] = c01.y; cs[2] = c23.x; cs[3] = c23.y;
        sn[0] = s01.x; sn[1] = s01.y; sn[2] = s23.x; sn[3] = s23.y;
      }
      float w[8];
      load8f(a.wq + c, w);
      st16(out_ptr(a, 0, bidx, t, c), norm_rope8(rotate, qv[k], rq, w, cs, sn));
      if (has_k) {
        load8f(a.wk + c, w);
        st16(out_ptr(a, 1, bidx, t, c), norm_rope8(rotate, kv[k], rk, w, cs, sn));
      }
    }
  }
  // peer stores are complete at system scope before the kernel's end (the
  // caller's barrier collective follows it on the stream)
  if (a.npeer > 0) __threadfence_system();
}

int vectors_per_thread(int cols) { return int(cdiv(cols / 8, kRowThreads)); }

}  // namespace

int dit_row_threads() { return kRowThreads; }
int dit_max_cols() { return kMaxVec * 8 * kRowThreads; }

cudaError_t launch_row_norm(cudaStream_t stream, const void* x, const void* add, const float* gate, void* x_out,
                            const float* w, const float* b, const float* scale, const float* shift, int64_t rows,
                            int64_t batch_rows, int cols, float eps, int center, int pad_cols, void* y) {
  RowNormArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.add = static_cast<const __nv_bfloat16*>(add);
  a.gate = gate;
  a.x_out = static_cast<__nv_bfloat16*>(x_out);
  a.w = w;
  a.b = b;
  a.scale = scale;
  a.shift = shift;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.batch_rows = batch_rows;
  a.cols = cols;
  a.eps = eps;
  a.center = center;
  a.pad_cols = pad_cols;
  const dim3 grid{unsigned(rows)};
  switch (vectors_per_thread(cols)) {
    case 1: row_norm_kernel<1><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 2: row_norm_kernel<2><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 3: row_norm_kernel<3><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 4: row_norm_kernel<4><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 5: row_norm_kernel<5><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 6: row_norm_kernel<6><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 7: row_norm_kernel<7><<<grid, kRowThreads, 0, stream>>>(a); break;
    default: row_norm_kernel<8><<<grid, kRowThreads, 0, stream>>>(a); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_qkv_rope(cudaStream_t stream, const void* xq, const void* xk, const void* xv, const float* wq,
                            const float* wk, const double* cos, const double* sin, int64_t batch, int64_t tokens,
                            int cols, int head_dim, float eps, int head_major, void* q, void* k, void* v,
                            void* const* peer, int npeer, int rank) {
  QkvArgs a;
  a.peer = reinterpret_cast<__nv_bfloat16* const*>(peer);
  a.npeer = npeer;
  a.rank = rank;
  a.xq = static_cast<const __nv_bfloat16*>(xq);
  a.xk = static_cast<const __nv_bfloat16*>(xk);
  a.xv = static_cast<const __nv_bfloat16*>(xv);
  a.wq = wq;
  a.wk = wk;
  a.cos = cos;
  a.sin = sin;
  a.q = static_cast<__nv_bfloat16*>(q);
  a.k = static_cast<__nv_bfloat16*>(k);
  a.v = static_cast<__nv_bfloat16*>(v);
  a.tokens = tokens;
  a.cols = cols;
  a.head_dim = head_dim;
  a.eps = eps;
  a.head_major = head_major;
  const dim3 grid{unsigned(batch * tokens)};
  switch (vectors_per_thread(cols)) {
    case 1: qkv_rope_kernel<1><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 2: qkv_rope_kernel<2><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 3: qkv_rope_kernel<3><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 4: qkv_rope_kernel<4><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 5: qkv_rope_kernel<5><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 6: qkv_rope_kernel<6><<<grid, kRowThreads, 0, stream>>>(a); break;
    case 7: qkv_rope_kernel<7><<<grid, kRowThreads, 0, stream>>>(a); break;
    default: qkv_rope_kernel<8><<<grid, kRowThreads, 0, stream>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace pasa
