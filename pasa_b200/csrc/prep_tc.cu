// Block statistics for bf16 inputs on the tensor cores.
//
// Same outputs and rounding points as prep.cu (fused_chunk_reduce +
// compute_h_group, svg/kernels/triton/group_pisa_attention.py:75-129,
// :268-301): a CTA owns one (head, group of 32 blocks); k^T v of every block
// runs on mma.sync (bf16 x bf16 -> fp32, like the reference's tl.dot), the
// group's sum of bf16(hc_j) stays in registers and h_group is written once.
// Tiles stream through a two-stage cp.async pipeline so the next block's
// 48 KB of q, k, v load while the current block computes.  hc itself never
// reaches HBM.
#include "common.cuh"

namespace pasa {

namespace prep_tc {

constexpr int kThreads = 512;  // 16 warps: a 4 x 4 grid of (a, b) sub-tiles of hc

template <int D>
struct Cfg {
  static constexpr int kRS = D + 8;                    // padded row stride (elements): conflict-free ldmatrix
  static constexpr int kTile = kBlock * kRS;           // elements per tile
  static constexpr int kStage = 3 * kTile;             // q, k, v
  static constexpr int kSmem = 2 * kStage * 2 + 2 * D * 4 + 64 * 4;
  static constexpr int WM = D / 4, WN = D / 4;         // per-warp sub-tile of the D x D matrix
  static constexpr int MI = WM / 16, NI = WN / 8;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
               :: "r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int D>
__device__ __forceinline__ void load_block(__nv_bfloat16* stage, const __nv_bfloat16* qh, const __nv_bfloat16* kh,
                                           const __nv_bfloat16* vh, int64_t t0, int64_t T_len) {
  using C = Cfg<D>;
  constexpr int kVec = D / 8;  // 16-byte chunks per row
  for (int i = threadIdx.x; i < 3 * kBlock * kVec; i += kThreads) {
    const int which = i / (kBlock * kVec), rem = i % (kBlock * kVec), r = rem / kVec, c = rem % kVec;
    const __nv_bfloat16* src = (which == 0 ? qh : which == 1 ? kh : vh);
    const bool valid = t0 + r < T_len;
    const __nv_bfloat16* g = src + (valid ? (t0 + r) * D + c * 8 : 0);
    cp_async16(stage + which * C::kTile + r * C::kRS + c * 8, g, valid);
  }
}

// bf16 addition of two pairs, rounded to nearest even: for bf16 inputs the
// same value as adding in fp32 and rounding the sum to bf16 (an exact sum of
// two 8-bit significands that differ by up to 15 binary places fits fp32;
// beyond that the smaller one lies below half a bf16 step, so the fp32
// rounding cannot create a tie).
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Halving-tree column sums in bf16 (each partial sum rounded, as prep.cu)
// of columns c and c + 1 at once; returns them packed (c in the low half).
template <int D>
__device__ __forceinline__ uint32_t tree_sum2(const __nv_bfloat16* tile, int c) {
  using C = Cfg<D>;
  uint32_t x[kBlock];
#pragma unroll
  for (int r = 0; r < kBlock; ++r) x[r] = *reinterpret_cast<const uint32_t*>(tile + r * C::kRS + c);
#pragma unroll
  for (int n = kBlock; n > 1; n >>= 1)
#pragma unroll
    for (int r = 0; r < n / 2; ++r) x[r] = add_bf16x2(x[r], x[r + n / 2]);
  return x[0];
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prep_tc_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    int64_t T_len, int64_t NT, int64_t NG, __nv_bfloat16* __restrict__ qc, __nv_bfloat16* __restrict__ kc,
    __nv_bfloat16* __restrict__ vc, float* __restrict__ h_norm, __nv_bfloat16* __restrict__ h_group) {
  using C = Cfg<D>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* stages = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  float* kc_f = reinterpret_cast<float*>(smem_raw + 2 * C::kStage * 2);
  float* vc_f = kc_f + D;
  float* red = vc_f + D;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t g = blockIdx.x, bh = blockIdx.y, NTP = NG * kGroup;
  const __nv_bfloat16* qh = q + bh * T_len * D;
  const __nv_bfloat16* kh = k + bh * T_len * D;
  const __nv_bfloat16* vh = v + bh * T_len * D;
  const int am = (warp % 4) * C::WM, bn = (warp / 4) * C::WN;
  const int gq = lane >> 2, tq = lane & 3;

  float gsum[C::MI][C::NI][4];
#pragma unroll
  for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
    for (int ni = 0; ni < C::NI; ++ni)
#pragma unroll
      for (int e = 0; e < 4; ++e) gsum[mi][ni][e] = 0.f;

  const int64_t j_first = g * kGroup;
  const int nvalid = int((NT - j_first) < kGroup ? (NT - j_first) : kGroup);  // blocks of this group < NT
  // h_norm of block b from the per-warp partial sums, double-buffered by b's
  // parity; thread 0 finishes it after the next barrier
  auto finish_norm = [&](int b) {
    float tot = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) tot += red[(b & 1) * (kThreads / 32) + w];
    h_norm[bh * NT + j_first + b] = __fsqrt_rn(tot);  // :287
  };
  if (nvalid > 0) load_block<D>(stages, qh, kh, vh, j_first * kBlock, T_len);
  cp_async_commit();

  for (int jj = 0; jj < kGroup; ++jj) {
    const int64_t j = j_first + jj;
    __nv_bfloat16* qc_row = qc + (bh * NTP + j) * D;
    __nv_bfloat16* kc_row = kc + (bh * NTP + j) * D;
    __nv_bfloat16* vc_row = vc + (bh * NTP + j) * D;
    if (jj >= nvalid) {  // zero padding rows (compute_h_group pads hc with zeros)
      for (int c = tid; c < 3 * D; c += kThreads) {
        __nv_bfloat16* row = c < D ? qc_row : (c < 2 * D ? kc_row : vc_row);
        row[c % D] = __float2bfloat16_rn(0.f);
      }
      continue;
    }
    // prefetch the next block into the other stage
    if (jj + 1 < nvalid)
      load_block<D>(stages + ((jj + 1) & 1) * C::kStage, qh, kh, vh, (j + 1) * kBlock, T_len);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (tid == 0 && jj > 0) finish_norm(jj - 1);  // every warp wrote its part of block jj-1 before this barrier
    const __nv_bfloat16* st = stages + (jj & 1) * C::kStage;
    const __nv_bfloat16* sq = st;
    const __nv_bfloat16* sk = st + C::kTile;
    const __nv_bfloat16* sv = st + 2 * C::kTile;
    const int64_t t0 = j * kBlock;
    const float len = float((T_len - t0 < kBlock) ? (T_len - t0) : int64_t(kBlock));  // BLOCK_SIZE (:91)

    for (int task = tid; task < 3 * (D / 2); task += kThreads) {  // two columns per task
      const int which = task / (D / 2), c = 2 * (task % (D / 2));
      const uint32_t sum2 = tree_sum2<D>(which == 0 ? sq : (which == 1 ? sk : sv), c);
      const float s0 = __uint_as_float(sum2 << 16), s1 = __uint_as_float(sum2 & 0xFFFF0000u);
      if (which == 0) {
        *reinterpret_cast<uint32_t*>(qc_row + c) = pack_bf16x2(__fdiv_rn(s0, len), __fdiv_rn(s1, len));
      } else if (which == 1) {
        const float m0 = __fdiv_rn(s0, len), m1 = __fdiv_rn(s1, len);
        kc_f[c] = m0;
        kc_f[c + 1] = m1;
        *reinterpret_cast<uint32_t*>(kc_row + c) = pack_bf16x2(m0, m1);
      } else {
        vc_f[c] = s0;
        vc_f[c + 1] = s1;
        *reinterpret_cast<uint32_t*>(vc_row + c) = sum2;
      }
    }

    // k^T v on the warp's (a, b) sub-tile: A[a][r] = k[r][a], B[r][b] = v[r][b]
    float acc[C::MI][C::NI][4];
#pragma unroll
    for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
      for (int ni = 0; ni < C::NI; ++ni)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mi][ni][e] = 0.f;
#pragma unroll
    for (int kr = 0; kr < kBlock; kr += 16) {
      uint32_t af[C::MI][4];
#pragma unroll
      for (int mi = 0; mi < C::MI; ++mi) {
        const int mat = lane >> 3, i = lane & 7;
        const int row = kr + i + ((mat >= 2) ? 8 : 0), col = am + mi * 16 + ((mat & 1) ? 8 : 0);
        ldsm_x4_trans(af[mi], sk + row * C::kRS + col);
      }
#pragma unroll
      for (int np = 0; np < C::NI; np += 2) {
        uint32_t bf[4];
        const int mat = lane >> 3, i = lane & 7;
        const int row = kr + i + ((mat & 1) ? 8 : 0), col = bn + np * 8 + ((mat >= 2) ? 8 : 0);
        ldsm_x4_trans(bf, sv + row * C::kRS + col);
#pragma unroll
        for (int mi = 0; mi < C::MI; ++mi) {
          mma_bf16_16816(acc[mi][np], af[mi], bf[0], bf[1]);
          if (np + 1 < C::NI) mma_bf16_16816(acc[mi][np + 1], af[mi], bf[2], bf[3]);
        }
      }
    }
    __syncthreads();  // kc_f / vc_f written above

    // elements e, e+1 of a fragment are columns b, b+1 of one row: packed
    // fp32 pair instructions (per-lane results as the scalar forms)
    float2 nsq2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
      for (int ni = 0; ni < C::NI; ++ni) {
        const int b = bn + ni * 8 + 2 * tq;
        const float2 vb = make_float2(vc_f[b], vc_f[b + 1]);
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const float nk = -kc_f[am + mi * 16 + gq + ((e >= 2) ? 8 : 0)];
          const float2 hc = __ffma2_rn(make_float2(nk, nk), vb,
                                       make_float2(acc[mi][ni][e], acc[mi][ni][e + 1]));  // :106-107
          nsq2 = __ffma2_rn(hc, hc, nsq2);                                                // :110
          // hc stored in v dtype (:125): both roundings in one conversion
          const float2 hr = __bfloat1622float2(__floats2bfloat162_rn(hc.x, hc.y));
          const float2 gs = __fadd2_rn(make_float2(gsum[mi][ni][e], gsum[mi][ni][e + 1]), hr);
          gsum[mi][ni][e] = gs.x;
          gsum[mi][ni][e + 1] = gs.y;
        }
      }
    float nsq = nsq2.x + nsq2.y;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) nsq += __shfl_xor_sync(0xffffffffu, nsq, off);
    if (lane == 0) red[(jj & 1) * (kThreads / 32) + warp] = nsq;
    // No barrier here.  The next block's first barrier orders red and the
    // next writes of kc_f / vc_f after this epilogue.  This block's stage was
    // last read (tree sums, MMA fragments) before the kc_f / vc_f barrier
    // above, so the next block's prefetch may refill it.
  }
  cp_async_wait<0>();
  __syncthreads();
  if (tid == 0 && nvalid > 0) finish_norm(nvalid - 1);

  __nv_bfloat16* hg = h_group + ((bh * NG + g) * D) * D;
#pragma unroll
  for (int mi = 0; mi < C::MI; ++mi)
#pragma unroll
    for (int ni = 0; ni < C::NI; ++ni)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int a = am + mi * 16 + gq + ((e >= 2) ? 8 : 0);
        const int b = bn + ni * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(hg + a * D + b) =
            pack_bf16x2(gsum[mi][ni][e] * (1.0f / kGroup), gsum[mi][ni][e + 1] * (1.0f / kGroup));
      }
}

}  // namespace prep_tc

template <int D>
static cudaError_t launch_prep_tc_t(cudaStream_t st, const void* q, const void* k, const void* v, int64_t BH,
                                    int64_t T_len, void* qc, void* kc, void* vc, float* hn, void* hg) {
  using C = prep_tc::Cfg<D>;
  const int64_t NT = cdiv(T_len, kBlock), NG = cdiv(NT, kGroup);
  auto kern = prep_tc::prep_tc_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(NG), unsigned(BH), 1u};
  kern<<<grid, prep_tc::kThreads, C::kSmem, st>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v), T_len, NT, NG, static_cast<__nv_bfloat16*>(qc),
      static_cast<__nv_bfloat16*>(kc), static_cast<__nv_bfloat16*>(vc), hn, static_cast<__nv_bfloat16*>(hg));
  return cudaGetLastError();
}

cudaError_t launch_prep_tc(cudaStream_t st, int D, const void* q, const void* k, const void* v, int64_t BH,
                           int64_t T_len, void* qc, void* kc, void* vc, float* hn, void* hg) {
  if (D == 64) return launch_prep_tc_t<64>(st, q, k, v, BH, T_len, qc, kc, vc, hn, hg);
  return launch_prep_tc_t<128>(st, q, k, v, BH, T_len, qc, kc, vc, hn, hg);
}

}  // namespace pasa
