// Block statistics for bf16 inputs on the tensor cores.
//
// Same outputs and rounding points as prep.cu (fused_chunk_reduce +
// compute_h_group, svg/kernels/triton/group_pisa_attention.py:75-129,
// :268-301): a CTA owns one (head, group of 32 blocks), forms k^T v of every
// block on the tensor core (bf16 x bf16 -> fp32, like the reference's
// tl.dot), keeps the group's sum of bf16(hc_j) on chip and writes h_group
// once; hc itself never reaches HBM.  Two kernels:
//   * prep_tc_kernel (D = 64): k^T v on mma.sync, the group sum in
//     registers, tiles through a two-stage cp.async pipeline;
//   * prep_umma_kernel (D = 128, below): TMA tiles, k^T v on tcgen05 into
//     TMEM, warp-specialised.
#include <cuda.h>

#include "common.cuh"

namespace pasa {

namespace tc {
// 3-D bf16 tensor map over [batch][rows][D], (64 x box_rows x 1) box, 128-byte swizzle (attn_tc.cu)
bool make_map(CUtensorMap* m, const void* base, int D, int64_t rows, int64_t batch, int box_rows);
}  // namespace tc

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

// ---------------------------------------------------------------------------
// D = 128: k^T v on tcgen05 (UMMA), tiles staged by TMA.
//
// A CTA owns one (head, group of 32 blocks), as above, with the same outputs
// and rounding points; only the order in which h_norm's squares are summed
// differs.  Warp-specialised, per block:
//   * warp 0 loads q, k, v (48 KB) by TMA into a 4-deep ring;
//   * warp 1 issues k^T v (M = 128 dims of k, N = 128 dims of v, K = 64
//     tokens; both operands MN-major) into one of two TMEM accumulators;
//   * six tree-sum warps take the bf16 column sums (qc, kc, vc) from the
//     ring and leave kc, vc in fp32 for the epilogue (double-buffered);
//   * four epilogue warps, one accumulator row per thread, form
//     hc = acc - kc (x) vc, its squared norm and the group sum of bf16(hc),
//     which stays in TMEM (128 more columns) until h_group is written.
// So the tree sums of block j+1, the MMA of block j+1 and the epilogue of
// block j run at the same time, with up to four blocks' loads in flight.
// ---------------------------------------------------------------------------
namespace prep_umma {

constexpr int D = 128;
constexpr int kThreads = 384;             // warp 0 TMA, 1 MMA + TMEM, 2-7 tree sums, 8-11 epilogue
constexpr int kSumWarp0 = 2, kSumWarps = 6;
constexpr int kEpiWarp0 = 8, kEpiWarps = 4;
constexpr int kStages = 4;
constexpr int kBox = kBlock * 128;        // [64 rows][64 columns] bf16, 128-byte swizzled rows
constexpr int kTileBytes = 2 * kBox;      // q, k or v of one block
constexpr int kStageBytes = 3 * kTileBytes;
constexpr int kOffF = kStages * kStageBytes;                 // kc_f, vc_f: f32 [2 blocks][2][D]
constexpr int kOffRed = kOffF + 2 * 2 * D * 4;               // h_norm partials: f32 [2 blocks][4 warps]
constexpr int kOffBar = kOffRed + 2 * kEpiWarps * 4;
constexpr int kNumBars = 2 * kStages + 2 + 2 + 2 + 2;
constexpr int kOffSlot = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffSlot + 16 + 1024;                  // + alignment slack
constexpr uint32_t kColAcc = 0;           // accumulator b at column 128 b
constexpr uint32_t kColSum = 256;         // group sum of bf16(hc)
constexpr uint32_t kTmemCols = 512;
constexpr int kBarEpi = 1;                // named barrier of the epilogue warps
static_assert(kSumWarps * 32 == 3 * (D / 2), "one column pair of q, k or v per tree-sum thread");
static_assert(kSmem <= 232448, "shared memory budget");

struct Maps {
  CUtensorMap q, k, v;
};

__device__ uint32_t g_prep_timeout;       // set when a bounded wait gave up and no error word was passed

__device__ __forceinline__ void report_timeout(uint32_t* err) {
  atomicOr(err ? err : &g_prep_timeout, PASA_DEVERR_WAIT_TIMEOUT);
}

__global__ void __launch_bounds__(kThreads, 1) prep_umma_kernel(
    const __grid_constant__ Maps maps, int64_t T_len, int64_t NT, int64_t NG, __nv_bfloat16* __restrict__ qc,
    __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, float* __restrict__ h_norm,
    __nv_bfloat16* __restrict__ h_group, uint32_t* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* kc_f = reinterpret_cast<float*>(sm + kOffF);   // [2][D]: then vc_f at + 2 * D
  float* vc_f = kc_f + 2 * D;
  float* red = reinterpret_cast<float*>(sm + kOffRed);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* empty = full + kStages;         // the stage's k, v read by the MMA and its tree sums taken
  uint64_t* acc_full = empty + kStages;     // [2] k^T v of a block in accumulator b
  uint64_t* acc_empty = acc_full + 2;       // [2] the epilogue warps have read accumulator b
  uint64_t* stats_full = acc_empty + 2;     // [2] kc_f, vc_f of a block in buffer b
  uint64_t* stats_empty = stats_full + 2;   // [2] the epilogue warps are done with buffer b
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffSlot);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t g = blockIdx.x, bh = blockIdx.y, NTP = NG * kGroup;
  const int64_t j_first = g * kGroup;
  const int nvalid = int((NT - j_first) < kGroup ? (NT - j_first) : kGroup);  // blocks of this group < NT

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1 + kSumWarps); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], kEpiWarps);
      mbar_init(&stats_full[b], kSumWarps); mbar_init(&stats_empty[b], kEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) { tmem_alloc(tmem_slot, kTmemCols); tmem_relinquish(); }
  if (warp == 0 && lane == 0) { prefetch_tmap(&maps.q); prefetch_tmap(&maps.k); prefetch_tmap(&maps.v); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int jj = 0; jj < nvalid && ok; ++jj) {
        const int s = jj % kStages;
        if (!mbar_wait_bounded(&empty[s], uint32_t((jj / kStages) & 1) ^ 1u)) { ok = false; break; }
        unsigned char* st = sm + s * kStageBytes;
        const int32_t t0 = int32_t((j_first + jj) * kBlock);  // rows >= T_len load as zeros
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        for (int bx = 0; bx < 2; ++bx) {
          tma_load_3d(st + bx * kBox, &maps.q, &full[s], bx * 64, t0, int32_t(bh));
          tma_load_3d(st + kTileBytes + bx * kBox, &maps.k, &full[s], bx * 64, t0, int32_t(bh));
          tma_load_3d(st + 2 * kTileBytes + bx * kBox, &maps.v, &full[s], bx * 64, t0, int32_t(bh));
        }
        issued = jj + 1;
      }
      if (!ok) report_timeout(err);
      // drain: the last copies land before the CTA can exit
      for (int jj = (issued > kStages ? issued - kStages : 0); jj < issued; ++jj)
        mbar_wait_bounded(&full[jj % kStages], uint32_t((jj / kStages) & 1));
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, 128, true, true);
      bool ok = true;
      for (int jj = 0; jj < nvalid && ok; ++jj) {
        const int s = jj % kStages, b = jj & 1;
        if (!mbar_wait_bounded(&full[s], uint32_t((jj / kStages) & 1))) { ok = false; break; }
        if (!mbar_wait_bounded(&acc_empty[b], uint32_t((jj >> 1) & 1) ^ 1u)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = smem_u32(sm + s * kStageBytes);
        // A[a][r] = k[r][a] and B[r][b] = v[r][b]: both tiles are [tokens][dims]
        // with the dims contiguous, i.e. MN-major; 64-dim boxes kBox apart,
        // 8-row groups 1024 bytes apart, and each K16 slice 16 rows further on
        const uint64_t kd = umma_desc_sw128(st + kTileBytes, kBox, 1024);
        const uint64_t vd = umma_desc_sw128(st + 2 * kTileBytes, kBox, 1024);
#pragma unroll
        for (int kk = 0; kk < kBlock / 16; ++kk)
          mma_ss(tmem + kColAcc + 128u * uint32_t(b), kd + uint64_t((kk * 2048) >> 4), vd + uint64_t((kk * 2048) >> 4),
                 idesc, kk > 0 ? 1u : 0u);
        tc_commit(&empty[s]);
        tc_commit(&acc_full[b]);
      }
      if (!ok) report_timeout(err);
    }
  } else if (warp < kEpiWarp0) {
    // ================= tree sums =================
    const int ct = (warp - kSumWarp0) * 32 + lane;  // q, k, v x 64 column pairs; a warp's pairs are one box
    const int which = ct / (D / 2), c = 2 * (ct % (D / 2));
    bool ok = true;
    for (int jj = 0; jj < kGroup; ++jj) {
      const int64_t j = j_first + jj;
      __nv_bfloat16* row = (which == 0 ? qc : which == 1 ? kc : vc) + (bh * NTP + j) * D;
      if (jj >= nvalid) {  // zero padding rows (compute_h_group pads hc with zeros)
        *reinterpret_cast<uint32_t*>(row + c) = 0u;
        continue;
      }
      const int s = jj % kStages, b = jj & 1;
      if (ok && !mbar_wait_bounded(&full[s], uint32_t((jj / kStages) & 1))) { ok = false; report_timeout(err); }
      // kc_f / vc_f buffer b was last read by the epilogue of block jj - 2
      if (ok && !mbar_wait_bounded(&stats_empty[b], uint32_t((jj >> 1) & 1) ^ 1u)) { ok = false; report_timeout(err); }
      const unsigned char* box = sm + s * kStageBytes + which * kTileBytes + (c >> 6) * kBox;
      const int cc = c & 63;
      uint32_t x[kBlock];
#pragma unroll
      for (int r = 0; r < kBlock; ++r)
        x[r] = *reinterpret_cast<const uint32_t*>(box + r * 128 + ((((cc >> 3) ^ (r & 7)) << 4) | ((cc & 7) * 2)));
      // halving tree in bf16, each partial rounded (as prep.cu)
#pragma unroll
      for (int n = kBlock; n > 1; n >>= 1)
#pragma unroll
        for (int r = 0; r < n / 2; ++r) x[r] = prep_tc::add_bf16x2(x[r], x[r + n / 2]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // this warp's reads of the stage are done
      const uint32_t sum2 = x[0];
      const float s0 = __uint_as_float(sum2 << 16), s1 = __uint_as_float(sum2 & 0xFFFF0000u);
      const int64_t t0 = j * kBlock;
      const float len = float((T_len - t0 < kBlock) ? (T_len - t0) : int64_t(kBlock));  // BLOCK_SIZE (:91)
      if (which == 0) {
        *reinterpret_cast<uint32_t*>(row + c) = pack_bf16x2(__fdiv_rn(s0, len), __fdiv_rn(s1, len));
      } else if (which == 1) {
        const float m0 = __fdiv_rn(s0, len), m1 = __fdiv_rn(s1, len);
        kc_f[b * D + c] = m0;
        kc_f[b * D + c + 1] = m1;
        *reinterpret_cast<uint32_t*>(row + c) = pack_bf16x2(m0, m1);
      } else {
        vc_f[b * D + c] = s0;
        vc_f[b * D + c + 1] = s1;
        *reinterpret_cast<uint32_t*>(row + c) = sum2;
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&stats_full[b]);  // release: kc_f / vc_f above precede it
    }
  } else {
    // ================= epilogue =================
    const int ew = warp - kEpiWarp0;          // 0..3 == warp & 3, the TMEM lane quadrant
    const int a = ew * 32 + lane;             // accumulator row: dimension a of k
    const uint32_t lane_base = uint32_t(ew * 32) << 16;
    bool ok = true;
    auto wait_bar = [&](uint64_t* bar, uint32_t parity) {
      if (ok && !mbar_wait_bounded(bar, parity)) { ok = false; report_timeout(err); }
    };
    {  // the group sum starts at zero
      uint32_t z[16];
#pragma unroll
      for (int x = 0; x < 16; ++x) z[x] = 0u;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) tmem_st16(tmem + lane_base + kColSum + c0, z);
      tmem_wait_st();
    }
    for (int jj = 0; jj < nvalid; ++jj) {
      const int b = jj & 1;
      wait_bar(&stats_full[b], uint32_t((jj >> 1) & 1));
      wait_bar(&acc_full[b], uint32_t((jj >> 1) & 1));
      tc_fence_after();
      const float* kcf = kc_f + b * D;
      const float* vcf = vc_f + b * D;
      const float nk = -kcf[a];
      const float2 nk2 = make_float2(nk, nk);
      float2 nsq2 = make_float2(0.f, 0.f);
#pragma unroll 2
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t acc[16], gs[16];
        tmem_ld16(tmem + lane_base + kColAcc + 128u * uint32_t(b) + c0, acc);
        tmem_ld16(tmem + lane_base + kColSum + c0, gs);
        tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 16; x += 2) {
          const float2 vb = make_float2(vcf[c0 + x], vcf[c0 + x + 1]);
          const float2 hc = __ffma2_rn(nk2, vb, make_float2(__uint_as_float(acc[x]), __uint_as_float(acc[x + 1])));  // :106-107
          nsq2 = __ffma2_rn(hc, hc, nsq2);                                                                     // :110
          // hc stored in v dtype (:125): both roundings in one conversion
          const float2 hr = __bfloat1622float2(__floats2bfloat162_rn(hc.x, hc.y));
          const float2 sum = __fadd2_rn(make_float2(__uint_as_float(gs[x]), __uint_as_float(gs[x + 1])), hr);
          gs[x] = __float_as_uint(sum.x);
          gs[x + 1] = __float_as_uint(sum.y);
        }
        tmem_st16(tmem + lane_base + kColSum + c0, gs);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) { mbar_arrive(&acc_empty[b]); mbar_arrive(&stats_empty[b]); }
      float nsq = nsq2.x + nsq2.y;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) nsq += __shfl_xor_sync(0xffffffffu, nsq, off);
      if (lane == 0) red[b * kEpiWarps + ew] = nsq;
      // h_norm of block jj from the four warps' partials, in warp order
      named_bar_sync(kBarEpi, 32 * kEpiWarps);
      if (ew == 0 && lane == 0) {
        float tot = 0.f;
        for (int w = 0; w < kEpiWarps; ++w) tot += red[b * kEpiWarps + w];
        h_norm[bh * NT + j_first + jj] = __fsqrt_rn(tot);  // :287
      }
    }
    // h_group = bf16(group sum / 32), row a (256 contiguous bytes)
    __nv_bfloat16* hrow = h_group + ((bh * NG + g) * D + a) * D;
#pragma unroll 2
    for (int c0 = 0; c0 < D; c0 += 16) {
      uint32_t gs[16];
      tmem_ld16(tmem + lane_base + kColSum + c0, gs);
      tmem_wait_ld();
      uint4 out[2];
      uint32_t* ow = reinterpret_cast<uint32_t*>(out);
#pragma unroll
      for (int x = 0; x < 8; ++x)
        ow[x] = pack_bf16x2(__uint_as_float(gs[2 * x]) * (1.0f / kGroup), __uint_as_float(gs[2 * x + 1]) * (1.0f / kGroup));
      reinterpret_cast<uint4*>(hrow + c0)[0] = out[0];
      reinterpret_cast<uint4*>(hrow + c0)[1] = out[1];
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace prep_umma

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

static cudaError_t launch_prep_umma(cudaStream_t st, const void* q, const void* k, const void* v, int64_t BH,
                                    int64_t T_len, void* qc, void* kc, void* vc, float* hn, void* hg, uint32_t* err) {
  using namespace prep_umma;
  const int64_t NT = cdiv(T_len, kBlock), NG = cdiv(NT, kGroup);
  Maps maps;
  if (!tc::make_map(&maps.q, q, D, T_len, BH, kBlock) || !tc::make_map(&maps.k, k, D, T_len, BH, kBlock) ||
      !tc::make_map(&maps.v, v, D, T_len, BH, kBlock))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(prep_umma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(NG), unsigned(BH), 1u};
  prep_umma_kernel<<<grid, kThreads, kSmem, st>>>(maps, T_len, NT, NG, static_cast<__nv_bfloat16*>(qc),
                                                  static_cast<__nv_bfloat16*>(kc), static_cast<__nv_bfloat16*>(vc),
                                                  hn, static_cast<__nv_bfloat16*>(hg), err);
  return cudaGetLastError();
}

// bf16 block statistics: tcgen05 at D = 128, mma.sync at D = 64.  err
// (nullable, device) receives PASA_DEVERR_WAIT_TIMEOUT if a bounded wait of
// the tcgen05 kernel gives up.
cudaError_t launch_prep_tc(cudaStream_t st, int D, const void* q, const void* k, const void* v, int64_t BH,
                           int64_t T_len, void* qc, void* kc, void* vc, float* hn, void* hg, uint32_t* err) {
  if (D == 128) return launch_prep_umma(st, q, k, v, BH, T_len, qc, kc, vc, hn, hg, err);
  return launch_prep_tc_t<64>(st, q, k, v, BH, T_len, qc, kc, vc, hn, hg);
}

}  // namespace pasa
