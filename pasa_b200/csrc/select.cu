// Covariance-aware top-k block selection.
//
// Restates svg/kernels/triton/group_pisa_attention.py:365-375:
//   score[i, j] = dtype(qc_i . dtype(kc_j * scale))            (bf16 einsum)
//               + log(h_norm_j + 1e-6) [+ noise_j]              (fp32 bias)
//   indices[i]  = topk(score[i], NS).indices, largest first
// without materialising the NT x NT score matrix in HBM: a CTA scores
// kRows query blocks of one head against all key blocks into shared
// memory, then each warp selects its row's top NS with a 4-pass radix
// select over order-preserving uint32 keys and places the winners by rank.
// Equal scores are ordered by lower block index (torch leaves the order of
// exact ties unspecified).  The same pass writes the row's selection bitmask
// (one 32-bit word per group of 32 key blocks), which the attention kernels
// use instead of the reference's NS-long membership loop (:223-226).
#include "common.cuh"

namespace pasa {

constexpr int kRows = 8;        // query blocks per CTA (one per warp)
constexpr int kChunk = 64;      // key blocks staged per pass
constexpr int kSelThreads = 256;
constexpr int kCompactMax = 1024;  // NS up to this sorts from a compact list

__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct SelectDims {
  int64_t NT, NG, NTP, NS;
  int D;
};

// Winners placed by rank: a warp bitonic sort (descending) of the NS <= 32 P
// composites (key, then lower index), P per lane at positions P * lane + u;
// padding 0 sorts last (every composite is > 0: its low word is
// 0xFFFFFFFF - j with j < 2^24).  Writes the NS indices, best first.
template <int P>
__device__ __forceinline__ void bitonic_place(const uint64_t* cl, int64_t NS, int32_t* out) {
  constexpr int kN = 32 * P;
  const int lane = threadIdx.x & 31;
  uint64_t v[P];
#pragma unroll
  for (int u = 0; u < P; ++u) {
    const int64_t i = P * lane + u;
    v[u] = (i < NS) ? cl[i] : 0ull;
  }
#pragma unroll
  for (int k = 2; k <= kN; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= P) {  // partner in lane ^ (j / P), same slot
        const int lm = j / P;
        const bool lower = (lane & lm) == 0;
#pragma unroll
        for (int u = 0; u < P; ++u) {
          const uint64_t o = __shfl_xor_sync(0xffffffffu, v[u], lm);
          const bool desc = ((P * lane + u) & k) == 0;
          v[u] = (lower == desc) ? (v[u] > o ? v[u] : o) : (v[u] < o ? v[u] : o);
        }
      } else {       // partner in this lane: slot u ^ j
#pragma unroll
        for (int u = 0; u < P; ++u) {
          if ((u & j) != 0) continue;
          const int w = u | j;
          const bool desc = ((P * lane + u) & k) == 0;
          const uint64_t a = v[u], b = v[w];
          const bool swap = desc ? (a < b) : (a > b);
          v[u] = swap ? b : a;
          v[w] = swap ? a : b;
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < P; ++u) {
    const int64_t i = P * lane + u;
    if (i < NS) out[i] = int32_t(0xFFFFFFFFu - uint32_t(v[u] & 0xFFFFFFFFu));
  }
}

// Top-NS of one row of order keys, by one warp: 4-pass radix select of the
// NS-th largest key, ties at that key taken by ascending block index, then
// every winner placed at its rank (key descending, index ascending).  Writes
// the row's indices and, when sel_mask is non-NULL, its selection bitmask.
__device__ __forceinline__ void row_topk(const uint32_t* rk, int64_t NT, int64_t NG, int64_t NS, uint32_t* h,
                                         uint32_t* mw, uint64_t* cl, int32_t* out, uint32_t* mask_out) {
  const int lane = threadIdx.x & 31;
  // The keys of a row share their high bits (the scores of a head lie in a
  // narrow range): start the radix passes below the common prefix of the
  // row's smallest and largest key, so the first histogram is spread over
  // its bins instead of piling every key into one (whose shared-memory
  // atomics serialise) and fewer passes are needed.
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  for (int64_t j = lane; j < NT; j += 32) {
    const uint32_t kj = rk[j];
    kmin = kj < kmin ? kj : kmin;
    kmax = kj > kmax ? kj : kmax;
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  const uint32_t diff = kmin ^ kmax;
  int hi = diff ? 31 - __clz(diff) : -1;  // highest bit in which the keys differ
  // the bits above it (all of them when every key is equal)
  const uint32_t fixed = hi < 0 ? 0xFFFFFFFFu : (hi >= 31 ? 0u : ~((2u << hi) - 1u));
  uint32_t prefix = kmin & fixed, pmask = fixed;
  uint32_t remaining = uint32_t(NS);
  while (hi >= 0) {
    const int shift = hi >= 7 ? hi - 7 : 0;  // digit: bits [shift, shift + 8), those above hi already fixed
    hi = shift - 1;
    for (int b = lane; b < 256; b += 32) h[b] = 0;
    __syncwarp();
    for (int64_t j = lane; j < NT; j += 32) {
      const uint32_t kj = rk[j];
      if ((kj & pmask) == prefix) atomicAdd(&h[(kj >> shift) & 255u], 1u);
    }
    __syncwarp();
    // lane owns buckets 255-8*lane ... 248-8*lane (descending)
    uint32_t cnt[8], tot = 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) { cnt[u] = h[255 - 8 * lane - u]; tot += cnt[u]; }
    uint32_t incl = tot;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += y;
    }
    const uint32_t excl = incl - tot;
    const uint32_t hit = __ballot_sync(0xffffffffu, incl >= remaining);
    const int src = __ffs(hit) - 1;  // first lane whose range reaches `remaining`
    uint32_t bucket = 0, above = 0, bcount = 0;
    if (lane == src) {
      uint32_t c = excl;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (c + cnt[u] >= remaining) { bucket = 255 - 8 * lane - u; above = c; bcount = cnt[u]; break; }
        c += cnt[u];
      }
    }
    bucket = __shfl_sync(0xffffffffu, bucket, src);
    above = __shfl_sync(0xffffffffu, above, src);
    bcount = __shfl_sync(0xffffffffu, bcount, src);
    remaining -= above;
    prefix |= bucket << shift;
    pmask |= 0xFFu << shift;
    __syncwarp();
    if (hi >= 0 && bcount <= 32u) {
      // The boundary bucket holds at most 32 keys: gather them, one per lane
      // (the histogram is free now), and sort them descending across the
      // warp; the remaining-th of them is the NS-th largest key of the row.
      uint32_t got = 0;
      for (int64_t j0 = 0; j0 < NT; j0 += 32) {
        const int64_t j = j0 + lane;
        const uint32_t kj = (j < NT) ? rk[j] : 0u;
        const bool in = (j < NT) && ((kj & pmask) == prefix);
        const uint32_t b = __ballot_sync(0xffffffffu, in);
        if (in) h[got + __popc(b & ((1u << lane) - 1u))] = kj;
        got += __popc(b);
      }
      __syncwarp();
      // absent lanes hold 0, below every key (an order key of 0 would be a NaN score)
      uint32_t c = (uint32_t(lane) < bcount) ? h[lane] : 0u;
#pragma unroll
      for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
        for (int jx = k >> 1; jx > 0; jx >>= 1) {
          const uint32_t o = __shfl_xor_sync(0xffffffffu, c, jx);
          const bool lower = (lane & jx) == 0, desc = (lane & k) == 0;
          c = (lower == desc) ? (c > o ? c : o) : (c < o ? c : o);
        }
      const uint32_t kv = __shfl_sync(0xffffffffu, c, int(remaining) - 1);
      // candidates above the NS-th key are taken whole; ties at it by index
      remaining -= uint32_t(__popc(__ballot_sync(0xffffffffu, c > kv)));
      prefix = kv;
      pmask = 0xFFFFFFFFu;
      hi = -1;
      __syncwarp();
    }
  }
  const uint32_t kth = prefix;  // key of the NS-th largest score
  // ties at kth: take the `remaining` lowest block indices; the same pass
  // writes the mask words and (NS <= kCompactMax) the compact list of
  // (key, index) composites of the selected blocks
  const bool compact = NS <= kCompactMax;
  uint32_t taken = 0, base = 0;
  for (int64_t j0 = 0; j0 < NT; j0 += 32) {
    const int64_t j = j0 + lane;
    const uint32_t kj = (j < NT) ? rk[j] : 0u;
    const bool eq = (j < NT) && (kj == kth);
    const uint32_t eqb = __ballot_sync(0xffffffffu, eq);
    const uint32_t rank_eq = taken + __popc(eqb & ((1u << lane) - 1u));
    const bool sel = (j < NT) && (kj > kth || (eq && rank_eq < remaining));
    const uint32_t selb = __ballot_sync(0xffffffffu, sel);
    taken += __popc(eqb);
    if (lane == 0) mw[j0 >> 5] = selb;  // j0 is a multiple of 32: one word per step
    if (compact && sel)  // larger composite = better: key, then lower index
      cl[base + __popc(selb & ((1u << lane) - 1u))] = (uint64_t(kj) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(j));
    base += __popc(selb);
  }
  __syncwarp();

  if (compact) {
    // place the compacted winners by rank
    if (NS <= 128) {
      bitonic_place<4>(cl, NS, out);
    } else if (NS <= 256) {
      bitonic_place<8>(cl, NS, out);
    } else {
      for (int64_t e = lane; e < NS; e += 32) {
        const uint64_t me = cl[e];
        int64_t rank = 0;
        for (int64_t f = 0; f < NS; ++f) rank += (cl[f] > me) ? 1 : 0;
        out[rank] = int32_t(0xFFFFFFFFu - uint32_t(me & 0xFFFFFFFFu));
      }
    }
  } else {
    for (int64_t j = lane; j < NT; j += 32) {
      if (!((mw[j >> 5] >> (j & 31)) & 1u)) continue;
      const uint64_t me = (uint64_t(rk[j]) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(j));
      int64_t rank = 0;
      for (int64_t f = 0; f < NT; ++f) {
        if (!((mw[f >> 5] >> (f & 31)) & 1u)) continue;
        const uint64_t o = (uint64_t(rk[f]) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(f));
        rank += (o > me) ? 1 : 0;
      }
      out[rank] = int32_t(j);
    }
  }
  if (mask_out)
    for (int64_t w = lane; w < NG; w += 32) mask_out[w] = mw[w];
}

// Dynamic shared memory: qrow[kRows][D] f32 | kch[kChunk][D+1] f32 |
// keys[kRows][NT] u32 | hist[kRows][256] u32 | mask[kRows][NG] u32 |
// compact[kRows][NS] u64 (when NS <= kCompactMax)
template <typename T, int D>
__global__ void __launch_bounds__(kSelThreads) select_kernel(
    const T* __restrict__ qc, const T* __restrict__ kc, const float* __restrict__ h_norm,
    const float* __restrict__ noise, SelectDims dm, float scale, int use_cov_bias,
    int32_t* __restrict__ indices, uint32_t* __restrict__ sel_mask) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int64_t NT = dm.NT, NG = dm.NG, NTP = dm.NTP, NS = dm.NS;
  float* qrow = reinterpret_cast<float*>(smem_raw);
  float* kch = qrow + kRows * D;
  uint32_t* keys = reinterpret_cast<uint32_t*>(kch + kChunk * (D + 1));
  uint32_t* hist = keys + kRows * NT;
  uint32_t* maskw = hist + kRows * 256;
  uint64_t* compact = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(maskw + kRows * NG) + 7) & ~uintptr_t(7));

  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t bh = blockIdx.y;
  const int64_t i0 = int64_t(blockIdx.x) * kRows;
  const int nrows = int((NT - i0 < kRows) ? (NT - i0) : int64_t(kRows));
  const float scale32 = scale;

  for (int x = tid; x < kRows * D; x += kSelThreads) {
    const int r = x / D, c = x % D;
    qrow[x] = (r < nrows) ? Elem<T>::load(qc + (bh * NTP + i0 + r) * D + c) : 0.f;
  }

  // ---- scores ---------------------------------------------------------
  const int jl = tid % kChunk;          // key within chunk
  const int rg = tid / kChunk;          // rows rg*2, rg*2+1
  for (int64_t j0 = 0; j0 < NT; j0 += kChunk) {
    __syncthreads();
    for (int x = tid; x < kChunk * D; x += kSelThreads) {
      const int jj = x / D, c = x % D;
      float val = 0.f;
      if (j0 + jj < NT) val = Elem<T>::round(Elem<T>::load(kc + (bh * NTP + j0 + jj) * D + c) * scale32);
      kch[jj * (D + 1) + c] = val;
    }
    __syncthreads();
    const int64_t j = j0 + jl;
    if (j < NT) {
      float bias = 0.f;
      if (use_cov_bias) {
        bias = logf(h_norm[bh * NT + j] + 1e-6f);
        if (noise) bias = bias + noise[bh * NT + j];
      }
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int r = rg * 2 + rr;
        if (r < nrows) {
          const float* qv = qrow + r * D;
          const float* kv = kch + jl * (D + 1);
          float dot = 0.f;
#pragma unroll 16
          for (int c = 0; c < D; ++c) dot = fmaf(qv[c], kv[c], dot);
          float s = Elem<T>::round(dot);
          if (use_cov_bias) s = s + bias;
          keys[r * NT + j] = order_key(s);
        }
      }
    }
  }
  __syncthreads();

  // ---- per-row radix select + rank placement (one warp per row) --------
  if (warp >= nrows) return;
  const int64_t row = i0 + warp;
  row_topk(keys + warp * NT, NT, NG, NS, hist + warp * 256, maskw + warp * NG, compact + int64_t(warp) * NS,
           indices + (bh * NT + row) * NS, sel_mask ? sel_mask + (bh * NT + row) * NG : nullptr);
}


// ---------------------------------------------------------------------------
// bf16: scores on the tensor cores (mma.sync, fp32 accumulation, rounded to
// bf16 like the reference's bf16 einsum), 16 query blocks per CTA.
// ---------------------------------------------------------------------------
namespace sel_tc {
constexpr int kRowsTC = 16;      // query blocks per CTA, one warp each for the top-k
constexpr int kThreadsTC = 512;
// Two configurations: 64 key blocks per scoring pass (8 scoring warps) with
// two CTAs per SM where the shared memory of two fits (the Wan shapes), so
// that one CTA's top-k overlaps the other's scoring loads; else 128 key
// blocks per pass (all 16 warps score) and one CTA per SM.
constexpr size_t kTwoPerSmSmem = 113 * 1024;  // per-CTA limit for two CTAs per SM

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Shared memory: q rows, a chunk of scaled kc rows and their bias (the
// scoring stage); histograms and compact lists (the top-k stage); the row
// keys and mask words.  With kShare the two stages share one region, which
// makes two CTAs per SM fit at the Wan shapes, so that one CTA's top-k
// overlaps the other's scoring loads.
template <int D, int kKeyChunk, bool kShare>
struct Layout {
  static constexpr int kRS = D + 8;  // padded row stride (elements): conflict-free ldmatrix
  __host__ __device__ static size_t bytes(int64_t NT, int64_t NG, int64_t NS, size_t* off) {
    size_t a = 0;
    off[0] = a; a += size_t(kRowsTC) * kRS * 2;           // qs  bf16 [16][RS]
    off[1] = a; a += size_t(kKeyChunk) * kRS * 2;         // ks  bf16 [chunk][RS]
    off[2] = a; a += size_t(kKeyChunk) * 4;               // bias f32 [chunk]
    if (!kShare) {  // one region after the other
      off[3] = a; a += size_t(kRowsTC) * NT * 4;          // keys u32 [16][NT]
      off[4] = a; a += size_t(kRowsTC) * 256 * 4;         // hist
      off[5] = a; a += size_t(kRowsTC) * NG * 4;          // mask words
      a = (a + 7) & ~size_t(7);
      off[6] = a; if (NS <= kCompactMax) a += size_t(kRowsTC) * NS * 8;  // compact lists
      return a;
    }
    size_t b = 0;
    off[4] = b; b += size_t(kRowsTC) * 256 * 4;           // hist (top-k stage)
    b = (b + 7) & ~size_t(7);
    off[6] = b; if (NS <= kCompactMax) b += size_t(kRowsTC) * NS * 8;  // compact lists (top-k stage)
    size_t o = ((a > b ? a : b) + 15) & ~size_t(15);
    off[3] = o; o += size_t(kRowsTC) * NT * 4;            // keys u32 [16][NT]
    off[5] = o; o += size_t(kRowsTC) * NG * 4;            // mask words
    return o;
  }
};

template <int D, int kKeyChunk, int kMinBlocks>
__global__ void __launch_bounds__(kThreadsTC, kMinBlocks) select_tc_kernel(
    const __nv_bfloat16* __restrict__ qc, const __nv_bfloat16* __restrict__ kc, const float* __restrict__ h_norm,
    const float* __restrict__ noise, SelectDims dm, float scale, int use_cov_bias,
    int32_t* __restrict__ indices, uint32_t* __restrict__ sel_mask) {
  using L = Layout<D, kKeyChunk, (kMinBlocks > 1)>;
  constexpr int RS = L::kRS;
  constexpr int kScoreWarps = kKeyChunk / 8;  // one m16n8 tile of 8 key blocks per scoring warp
  static_assert(kScoreWarps >= 1 && kScoreWarps <= kThreadsTC / 32, "scoring warps");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int64_t NT = dm.NT, NG = dm.NG, NTP = dm.NTP, NS = dm.NS;
  size_t off[7];
  L::bytes(NT, NG, NS, off);
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem_raw + off[0]);
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem_raw + off[1]);
  float* bias = reinterpret_cast<float*>(smem_raw + off[2]);
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw + off[3]);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem_raw + off[4]);
  uint32_t* maskw = reinterpret_cast<uint32_t*>(smem_raw + off[5]);
  uint64_t* compact = reinterpret_cast<uint64_t*>(smem_raw + off[6]);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t bh = blockIdx.y;
  const int64_t i0 = int64_t(blockIdx.x) * kRowsTC;
  const int nrows = int((NT - i0 < kRowsTC) ? (NT - i0) : int64_t(kRowsTC));
  const float scale32 = scale;
  constexpr int kVec = D / 8;

  for (int x = tid; x < kRowsTC * kVec; x += kThreadsTC) {
    const int r = x / kVec, c = x % kVec;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < nrows) val = reinterpret_cast<const uint4*>(qc + (bh * NTP + i0 + r) * D)[c];
    *reinterpret_cast<uint4*>(qs + r * RS + c * 8) = val;
  }

  const int gq = lane >> 2, tq = lane & 3;
  // the kc rows of the next chunk are loaded into registers while the current
  // chunk is scored, so the L2 latency of the staging overlaps the MMAs
  constexpr int kLoads = kKeyChunk * kVec / kThreadsTC;
  static_assert(kKeyChunk * kVec % kThreadsTC == 0, "staging split");
  uint4 pre[kLoads];
  float hpre = 0.f, npre = 0.f;  // h_norm and noise of key block j0 + tid (tid < kKeyChunk)
  auto fetch = [&](int64_t j0) {
#pragma unroll
    for (int it = 0; it < kLoads; ++it) {
      const int x = tid + it * kThreadsTC, jj = x / kVec, c = x % kVec;
      pre[it] = (j0 + jj < NT) ? reinterpret_cast<const uint4*>(kc + (bh * NTP + j0 + jj) * D)[c]
                               : make_uint4(0, 0, 0, 0);
    }
    if (use_cov_bias && tid < kKeyChunk && j0 + tid < NT) {
      hpre = h_norm[bh * NT + j0 + tid];
      if (noise) npre = noise[bh * NT + j0 + tid];
    }
  };
  fetch(0);
  for (int64_t j0 = 0; j0 < NT; j0 += kKeyChunk) {
    __syncthreads();
    // kc * scale rounded to bf16 (:365), staged for the MMA (rows >= NT: zero)
#pragma unroll
    for (int it = 0; it < kLoads; ++it) {
      const int x = tid + it * kThreadsTC, jj = x / kVec, c = x % kVec;
      const uint32_t w[4] = {pre[it].x, pre[it].y, pre[it].z, pre[it].w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
        o[e] = pack_bf16x2(f.x * scale32, f.y * scale32);
      }
      *reinterpret_cast<uint4*>(ks + jj * RS + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if (tid < kKeyChunk) {
      float b = 0.f;
      if (use_cov_bias && j0 + tid < NT) {
        b = logf(hpre + 1e-6f);  // :368
        if (noise) b = b + npre;  // :370
      }
      bias[tid] = b;
    }
    if (j0 + kKeyChunk < NT) fetch(j0 + kKeyChunk);
    __syncthreads();
    if (warp >= kScoreWarps) continue;  // warp-uniform; the loop's barrier is at its top
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int kb = warp * 8;  // this scoring warp's 8 key blocks within the chunk
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4], b[2];
      {
        const int mat = lane >> 3, i = lane & 7;
        ldsm_x4(a, qs + (i + ((mat & 1) ? 8 : 0)) * RS + kk * 16 + ((mat >= 2) ? 8 : 0));
      }
      {
        const int mat = (lane >> 3) & 1, i = lane & 7;
        ldsm_x2(b, ks + (kb + i) * RS + kk * 16 + mat * 8);
      }
      mma16816(acc, a, b);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = gq + ((e >= 2) ? 8 : 0);
      const int key = kb + 2 * tq + (e & 1);
      const int64_t j = j0 + key;
      if (r < nrows && j < NT) {
        float sc = Elem<__nv_bfloat16>::round(acc[e]);  // einsum output in bf16
        if (use_cov_bias) sc = sc + bias[key];          // :371
        keys[r * NT + j] = order_key(sc);
      }
    }
  }
  __syncthreads();
  if (warp >= nrows) return;
  const int64_t row = i0 + warp;
  row_topk(keys + warp * NT, NT, NG, NS, hist + warp * 256, maskw + warp * NG, compact + int64_t(warp) * NS,
           indices + (bh * NT + row) * NS, sel_mask ? sel_mask + (bh * NT + row) * NG : nullptr);
}
}  // namespace sel_tc

template <int D, int kKeyChunk, int kMinBlocks>
static size_t select_tc_smem(const SelectDims& dm) {
  size_t off[7];
  return sel_tc::Layout<D, kKeyChunk, (kMinBlocks > 1)>::bytes(dm.NT, dm.NG, dm.NS, off);
}

template <int D, int kKeyChunk, int kMinBlocks>
static cudaError_t launch_select_tc_t(cudaStream_t st, const void* qc, const void* kc, const float* hn,
                                      const float* noise, int64_t BH, SelectDims dm, float scale, int use_cov_bias,
                                      int32_t* idx, uint32_t* mask) {
  const size_t smem = select_tc_smem<D, kKeyChunk, kMinBlocks>(dm);
  auto kern = sel_tc::select_tc_kernel<D, kKeyChunk, kMinBlocks>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(cdiv(dm.NT, sel_tc::kRowsTC)), unsigned(BH), 1u};
  kern<<<grid, sel_tc::kThreadsTC, smem, st>>>(static_cast<const __nv_bfloat16*>(qc),
                                               static_cast<const __nv_bfloat16*>(kc), hn, noise, dm, scale,
                                               use_cov_bias, idx, mask);
  return cudaGetLastError();
}

// The tensor-core selection of one head dimension: two CTAs per SM when
// they fit, else one, else (rows too long for shared memory) false.
template <int D>
static bool launch_select_tc_any(cudaError_t* err, cudaStream_t st, const void* qc, const void* kc, const float* hn,
                                 const float* noise, int64_t BH, SelectDims dm, float scale, int use_cov_bias,
                                 int32_t* idx, uint32_t* mask) {
  constexpr size_t kMaxSmem = 227 * 1024;
  if (select_tc_smem<D, 64, 2>(dm) <= sel_tc::kTwoPerSmSmem)
    *err = launch_select_tc_t<D, 64, 2>(st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask);
  else if (select_tc_smem<D, 128, 1>(dm) <= kMaxSmem)
    *err = launch_select_tc_t<D, 128, 1>(st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask);
  else
    return false;
  return true;
}

size_t select_smem_bytes(int D, int64_t NT, int64_t NG, int64_t NS) {
  size_t b = sizeof(float) * (kRows * D + kChunk * (D + 1));
  b += sizeof(uint32_t) * (kRows * NT + kRows * 256 + kRows * NG);
  b = (b + 7) & ~size_t(7);
  if (NS <= kCompactMax) b += sizeof(uint64_t) * kRows * NS;
  return b;
}

template <typename T, int D>
static cudaError_t launch_select_t(cudaStream_t st, const void* qc, const void* kc, const float* hn,
                                   const float* noise, int64_t BH, SelectDims dm, float scale,
                                   int use_cov_bias, int32_t* idx, uint32_t* mask) {
  const size_t smem = select_smem_bytes(D, dm.NT, dm.NG, dm.NS);
  auto kern = select_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(cdiv(dm.NT, kRows)), unsigned(BH), 1u};
  kern<<<grid, kSelThreads, smem, st>>>(static_cast<const T*>(qc), static_cast<const T*>(kc), hn, noise, dm,
                                        scale, use_cov_bias, idx, mask);
  return cudaGetLastError();
}

cudaError_t launch_select(cudaStream_t st, int dtype, int D, const void* qc, const void* kc,
                          const float* hn, const float* noise, int64_t BH, int64_t NT, int64_t NS,
                          float scale, int use_cov_bias, int32_t* idx, uint32_t* mask) {
  SelectDims dm;
  dm.NT = NT; dm.NG = cdiv(NT, kGroup); dm.NTP = dm.NG * kGroup; dm.NS = NS; dm.D = D;
  if (dtype == PASA_BF16) {
    cudaError_t e = cudaSuccess;
    if (D == 64 && launch_select_tc_any<64>(&e, st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask))
      return e;
    if (D == 128 && launch_select_tc_any<128>(&e, st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask))
      return e;
    if (D == 64) return launch_select_t<__nv_bfloat16, 64>(st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask);
    return launch_select_t<__nv_bfloat16, 128>(st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask);
  }
  if (D == 64) return launch_select_t<float, 64>(st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask);
  return launch_select_t<float, 128>(st, qc, kc, hn, noise, BH, dm, scale, use_cov_bias, idx, mask);
}

}  // namespace pasa
