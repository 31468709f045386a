// tcgen05 PASA attention for bf16 (sm_100a): TMA-staged tiles, tensor-core
// MMAs into TMEM, one online-softmax pass over exact and corrected blocks.
//
// Semantics: pisa_pg_fwd_kernel (svg/kernels/triton/group_pisa_attention.py:
// 136-262).  For query row t with selected set S_i and running max m:
//   exact      : sum_{j in S_i} sum_{u in j} 2^(s_tu - m) v_u          (:170-186)
//   zero order : sum_{j not in S_i} 2^(a_tj - m) vc_j,  a = q.kc*scale  (:212-240)
//   first order: sum_g (q_t H_g) * scale * sum_{j in g} 2^(a_tj - m)     (:246-253)
//   o = acc / (l_exact + g_l), where g_l = sum 2^(a_tj - m_g) len_j uses
//   the running max m_g at group g and is never rescaled (:242-243, :258).
//
// B200 mapping:
//   * a CTA owns a PAIR of adjacent 64-query blocks (128 rows), so every MMA
//     is M=128 (the full tcgen05 datapath).  Phase 1 walks the union of the
//     two blocks' selected key blocks, TWO key blocks per step: the score MMA
//     is N=128 (full rate; N=64 runs at ~55%) and P.V is K=128.  Steps pair a
//     block only query block A selected with one only B selected where
//     possible, so both halves of the softmax carry equal work.  Rows whose query block did not select a key block get P = 0
//     and skip its exponentials.  Phase 2 (shared by both query blocks) walks
//     the 32-block groups with each half's own selection bits.
//   * Q lives in TMEM as the A operand of every score MMA, so shared memory
//     carries only K/V (or kc/vc/H) tiles: TMA writes them once, the tensor
//     core reads them once.
//   * warp 0: TMA producer (ring 1: K/V of block pairs, 3 slots; ring 2,
//     aliased on the same memory: kc/vc rows and H of a group); warp 1: TMEM
//     owner and score-MMA issuer; warp 2: P.V / correction MMA issuer (one
//     thread issues a tcgen05.mma only every ~90 cycles, so a single issuer
//     would cap the tensor core at ~70% for these shapes); warps 3-10:
//     softmax, two threads per query row (TMEM lane), each owning half of
//     every key block's columns; the two warps of a lane quadrant
//     combine row maxima and probability sums through shared memory.
//   * TMEM: O (fp32), Q (bf16), P (bf16) and two S buffers of 128 columns.
//     The softmax frees an S buffer as soon as its scores are in registers,
//     so the score MMAs of step n+2 overlap the softmax and P.V of step n.
//     In phase 2 the first-order operand U = bf16(w_t q_t) (w_t = scale *
//     sum of the group's probabilities) sits in the upper half of the other
//     S buffer (group scores are only 32 columns wide) and U.H_g is
//     accumulated straight into O; P_g alternates between two 16-column
//     slots, so a group's softmax never waits for the previous group's P.V.
//   * softmax rescales O only when a row max grows by more than 2^8
//     (exact either way: O and l share the stale max); the exact running max
//     is tracked separately to reproduce g_l.
//   * every barrier wait is bounded; on timeout the kernel sets
//     PASA_DEVERR_WAIT_TIMEOUT in the caller's error word and winds down.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace pasa {

namespace tc {

constexpr int kParts = 2;              // softmax threads per query row
constexpr int kSoftmaxWarps = 4 * kParts;
constexpr int kThreads = 32 * (3 + kSoftmaxWarps);  // TMA, S issuer, P.V issuer, softmax
constexpr int kRowsPerTile = 128;      // two query blocks
constexpr float kRescaleThresh = 8.0f; // log2 units
constexpr int kMaxNT = 4096;           // union list capacity (entries)
constexpr int kMaxNG = kMaxNT / kGroup;
constexpr uint64_t kPollLimit = kWaitLimitCycles;  // SM cycles a barrier wait may take before giving up

template <int D>
struct Cfg {
  static constexpr int kBoxes = D / 64;                 // 64-column TMA boxes per row
  static constexpr int kQBytes = kRowsPerTile * D * 2;
  static constexpr int kKVBytes = kBlock * D * 2;       // one K (or V) block
  static constexpr int kCBytes = kGroup * D * 2;        // kc (or vc) rows of one group
  static constexpr int kHBytes = D * D * 2;
  // ring 1 (phase 1) slots: K of two blocks, then V of two blocks, each as
  // kBoxes boxes of [128 rows][64 cols]; ring 2 (phase 2) slots, aliased on
  // the same memory: kc rows, vc rows, H of one group
  static constexpr int kSlot1 = 4 * kKVBytes;
  static constexpr int kSlot2 = 2 * kCBytes + kHBytes;
  static constexpr int kS1 = 3;
  static constexpr int kRingBytes = kS1 * kSlot1;
  static constexpr int kS2 = kRingBytes / kSlot2;
  static constexpr int kPairBox = 2 * kBlock * 128;     // one [128 rows][64 cols] box
  static constexpr uint32_t kTxP1 = kSlot1;
  static constexpr uint32_t kTxP2 = kSlot2;
  // TMEM columns
  static constexpr uint32_t kColO = 0;
  static constexpr uint32_t kColQ = 128;
  static constexpr uint32_t kColP = 192;                // P (packed bf16) of the step in flight
  static constexpr uint32_t kColS0 = 256;               // S buffer b at kColS0 + 128 b
  static constexpr uint32_t kColU = 64;                 // phase 2: U of step n in S buffer (n + 1) & 1
  static constexpr uint32_t kTmemCols = 512;
  // shared memory carve-up (offsets from a 1024-aligned base).  Q is staged
  // inside ring slot 2 and copied to TMEM before that slot is first filled.
  static constexpr int kOffRing = 0;
  static constexpr int kOffQ = 2 * kSlot1;
  static constexpr int kOffUnion = kOffRing + kRingBytes;            // u16 [kMaxNT]
  static constexpr int kOffMask = kOffUnion + kMaxNT * 2;            // u32 [2][kMaxNG]
  static constexpr int kOffXch = kOffMask + 2 * kMaxNG * 4;          // f32 [2 slots][kParts][128]
  static constexpr int kOffHand = kOffXch + 2 * kParts * kRowsPerTile * 4;  // f32 [2 parts][m_used, m_true][128]
  static constexpr int kOffBar = kOffHand + 2 * 2 * kRowsPerTile * 4;
  static constexpr int kNumBars = 2 * kS1 + 2 * kS2 + 2 + 2 + 2 + 2 + 2 + 2 + 2;
  static constexpr int kOffSlot = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffSlot + 16 + 1024;  // + alignment slack
  static_assert(kOffQ + kQBytes <= kRingBytes, "Q staging must fit in the ring");
  static_assert(kS2 >= 2, "ring too small");
  static_assert(kColS0 + 2 * 128 <= kTmemCols, "TMEM budget");
  static_assert(kColU + D / 2 <= 128, "U must fit in the S buffer");
};

struct Maps {
  CUtensorMap q, k, v, kc, vc, h;
};

struct Params {
  int64_t T, NT, NG, NTP;
  float scale;
  __nv_bfloat16* o;
  const uint32_t* sel_mask;
  uint32_t* err;
};

// Optional step tracer (compile with -DPASA_TRACE): the CTA at grid (0, 0)
// records SM clock stamps of its pipeline events for the first kTraceSteps
// steps into g_pasa_trace[event][step]: 0 producer issue, 1 S issue, 2 P.V
// issue, 3 data landed, 4+w softmax warp w sees S, 12+w softmax warp w done;
// pasa_trace_read() copies them out.
#ifdef PASA_TRACE
constexpr int kTraceSteps = 1024;
__device__ unsigned long long g_pasa_trace[30][kTraceSteps];
__device__ unsigned int g_pasa_trace_cta[2];  // (blockIdx.x, blockIdx.y) of the traced CTA
__device__ unsigned long long g_pasa_trace_ctl[8];  // entry, set-up done, softmax done, exit (per traced CTA)
#define PASA_TRACE_CTL(i) do { if (pasa_traced) g_pasa_trace_ctl[(i)] = clock64(); } while (0)
// pasa_traced: a bool computed once per CTA at kernel entry
#define PASA_TRACE_MARK(ev, step)                                                        \
  do {                                                                                    \
    if (pasa_traced && (step) < kTraceSteps) g_pasa_trace[(ev)][(step)] = clock64();      \
  } while (0)
#else
#define PASA_TRACE_MARK(ev, step) do { } while (0)
#define PASA_TRACE_CTL(i) do { } while (0)
#endif

__device__ __forceinline__ void report(uint32_t* err) {
  if (err) atomicOr(err, PASA_DEVERR_WAIT_TIMEOUT);
}

// Set the raw fp32 scores of columns c >= nvalid to -inf.
template <int N>
__device__ __forceinline__ void mask_tail(uint32_t (&sv)[N], int nvalid) {
#pragma unroll
  for (int c = 0; c < N; ++c)
    if (c >= nvalid) sv[c] = __float_as_uint(-INFINITY);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const __grid_constant__ Maps maps, Params P) {
  using C = Cfg<D>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint16_t* ulist = reinterpret_cast<uint16_t*>(sm + C::kOffUnion);  // (block << 2) | half bits
  uint32_t* maskw = reinterpret_cast<uint32_t*>(sm + C::kOffMask);  // [2][kMaxNG]
  float* xch = reinterpret_cast<float*>(sm + C::kOffXch);
  float* hand = reinterpret_cast<float*>(sm + C::kOffHand);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::kOffBar);
  uint64_t* full1 = bars;
  uint64_t* empty1 = full1 + C::kS1;
  uint64_t* full2 = empty1 + C::kS1;
  uint64_t* empty2 = full2 + C::kS2;
  uint64_t* q_full = empty2 + C::kS2;
  uint64_t* q_tmem = q_full + 1;   // Q copied into TMEM by the softmax warps
  uint64_t* s_full = q_tmem + 1;   // [2]
  uint64_t* p_ready = s_full + 2;  // [2]
  uint64_t* o_done = p_ready + 2;  // [2]
  uint64_t* s_free = o_done + 2;   // [2] the buffer's scores are in registers (phase 1)
  uint64_t* s2_free = s_free + 2;  // [2 parts] phase 2: the part's group scores are in registers
  uint64_t* p2_ready = s2_free + 2;  // [2 parts] phase 2: the part's P_g and U are in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::kOffSlot);
  __shared__ uint32_t s_nu;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#ifdef PASA_TRACE
  const bool pasa_traced = blockIdx.x == g_pasa_trace_cta[0] && blockIdx.y == g_pasa_trace_cta[1];
  if (tid == 0) PASA_TRACE_CTL(0);
#endif
  const int64_t pair = blockIdx.x, bh = blockIdx.y;
  const int64_t NT = P.NT, NG = P.NG;
  const int64_t blkA = 2 * pair, blkB = 2 * pair + 1;
  const bool hasB = blkB < NT;

  // ---- set-up: barriers, TMEM, selection bits, union list -------------
  if (tid == 0) {
    for (int s = 0; s < C::kS1; ++s) { mbar_init(&full1[s], 1); mbar_init(&empty1[s], 1); }
    for (int s = 0; s < C::kS2; ++s) { mbar_init(&full2[s], 1); mbar_init(&empty2[s], 1); }
    mbar_init(q_full, 1);
    mbar_init(q_tmem, kSoftmaxWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1); mbar_init(&p_ready[b], kSoftmaxWarps); mbar_init(&o_done[b], 1);
      mbar_init(&s_free[b], kSoftmaxWarps);
      mbar_init(&s2_free[b], kSoftmaxWarps / 2); mbar_init(&p2_ready[b], kSoftmaxWarps / 2);
    }
    fence_barrier_init();
  }
  if (warp == 1) { tmem_alloc(tmem_slot, C::kTmemCols); tmem_relinquish(); }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&maps.q); prefetch_tmap(&maps.k); prefetch_tmap(&maps.v);
    prefetch_tmap(&maps.kc); prefetch_tmap(&maps.vc); prefetch_tmap(&maps.h);
  }
  for (int64_t w = tid; w < NG; w += kThreads) {
    maskw[w] = P.sel_mask[(bh * NT + blkA) * NG + w];
    maskw[kMaxNG + w] = hasB ? P.sel_mask[(bh * NT + blkB) * NG + w] : 0u;
  }
  __syncthreads();
  if (warp == 0) {
    // Union of the two selections, ordered so that consecutive pairs (one
    // phase-1 step) balance the two halves: blocks only A selected alternate
    // with blocks only B selected, then the leftover single-half blocks, then
    // the blocks both selected.  Within each category the order is ascending.
    // (The softmax is order-independent, so any order gives the same result
    // up to floating-point rounding.)
    uint32_t na = 0, nb = 0, nboth = 0;
    for (int64_t w0 = 0; w0 < NG; w0 += 32) {
      const int64_t w = w0 + lane;
      const uint32_t ma = (w < NG) ? maskw[w] : 0u, mb = (w < NG) ? maskw[kMaxNG + w] : 0u;
      na += __popc(ma & ~mb); nb += __popc(mb & ~ma); nboth += __popc(ma & mb);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      na += __shfl_xor_sync(0xffffffffu, na, off);
      nb += __shfl_xor_sync(0xffffffffu, nb, off);
      nboth += __shfl_xor_sync(0xffffffffu, nboth, off);
    }
    const uint32_t m = na < nb ? na : nb;
    uint32_t ka = 0, kb = 0, kab = 0;  // running counts per category
    for (int64_t w0 = 0; w0 < NG; w0 += 32) {
      const int64_t w = w0 + lane;
      const uint32_t ma = (w < NG) ? maskw[w] : 0u, mb = (w < NG) ? maskw[kMaxNG + w] : 0u;
      const uint32_t ua = ma & ~mb, ub = mb & ~ma, uab = ma & mb;
      uint32_t ca = __popc(ua), cb = __popc(ub), cab = __popc(uab);
      uint32_t ia = ca, ib = cb, iab = cab;  // inclusive scans over lanes
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t ya = __shfl_up_sync(0xffffffffu, ia, off);
        const uint32_t yb = __shfl_up_sync(0xffffffffu, ib, off);
        const uint32_t yab = __shfl_up_sync(0xffffffffu, iab, off);
        if (lane >= off) { ia += ya; ib += yb; iab += yab; }
      }
      uint32_t pa = ka + ia - ca, pb = kb + ib - cb, pab = kab + iab - cab;  // category ranks
      for (uint32_t rem = ua | ub | uab; rem; rem &= rem - 1) {
        const int bit = __ffs(rem) - 1;
        const uint32_t j = uint32_t(w * 32 + bit);
        uint32_t pos;
        if ((ua >> bit) & 1u) {
          pos = (pa < m) ? 2 * pa : 2 * m + (pa - m);
          ++pa;
          ulist[pos] = uint16_t((j << 2) | 1u);
        } else if ((ub >> bit) & 1u) {
          pos = (pb < m) ? 2 * pb + 1 : 2 * m + (na - m) + (pb - m);
          ++pb;
          ulist[pos] = uint16_t((j << 2) | 2u);
        } else {
          pos = na + nb + pab;
          ++pab;
          ulist[pos] = uint16_t((j << 2) | 3u);
        }
      }
      ka += __shfl_sync(0xffffffffu, ia, 31);
      kb += __shfl_sync(0xffffffffu, ib, 31);
      kab += __shfl_sync(0xffffffffu, iab, 31);
    }
    if (lane == 0) s_nu = na + nb + nboth;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) PASA_TRACE_CTL(1);
  const int64_t nU = s_nu;
  const int64_t nP = (nU + 1) / 2;  // phase-1 steps: two union blocks each (a lone last block pairs with itself)
  const int64_t total = nP + NG;

  if (warp == 0) {
    // ================= TMA producer =================
#ifdef PASA_TRACE
    if (lane == 1 && pasa_traced) {  // trace only: stamp data arrival (event 3)
      for (int64_t n = 0; n < nP && n < kTraceSteps; ++n)
        if (mbar_wait_bounded(&full1[n % C::kS1], uint32_t((n / C::kS1) & 1), kPollLimit)) PASA_TRACE_MARK(3, n);
    }
#endif
    if (lane == 0) {
      bool ok = true;
      int64_t issued = 0;
      const int32_t row0 = int32_t(pair * kRowsPerTile);
      mbar_arrive_expect_tx(q_full, C::kQBytes);
      for (int bx = 0; bx < C::kBoxes; ++bx)
        tma_load_3d(sm + C::kOffQ + bx * (kRowsPerTile * 128), &maps.q, q_full, bx * 64, row0, int32_t(bh));
      bool q_released = false;  // Q's staging area (ring slot 2) is free once Q sits in TMEM
      auto release_q = [&]() {
        if (!q_released) { ok = ok && mbar_wait_bounded(q_tmem, 0, kPollLimit); q_released = true; }
      };
      // Phase 1: K and V of every union block pair through ring 1
      for (int64_t p = 0; p < nP && ok; ++p) {
        const int s = int(p % C::kS1);
        if (!mbar_wait_bounded(&empty1[s], uint32_t((p / C::kS1) & 1) ^ 1u, kPollLimit)) { ok = false; break; }
        if (s == 2) { release_q(); if (!ok) break; }
        PASA_TRACE_MARK(0, p);
        unsigned char* st = sm + C::kOffRing + s * C::kSlot1;
        const int32_t j0 = int32_t(ulist[2 * p] >> 2);
        const int32_t j1 = (2 * p + 1 < nU) ? int32_t(ulist[2 * p + 1] >> 2) : j0;
        mbar_arrive_expect_tx(&full1[s], C::kTxP1);
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          unsigned char* kb = st + bx * C::kPairBox;
          unsigned char* vb = st + 2 * C::kKVBytes + bx * C::kPairBox;
          tma_load_3d(kb, &maps.k, &full1[s], bx * 64, j0 * kBlock, int32_t(bh));
          tma_load_3d(kb + kBlock * 128, &maps.k, &full1[s], bx * 64, j1 * kBlock, int32_t(bh));
          tma_load_3d(vb, &maps.v, &full1[s], bx * 64, j0 * kBlock, int32_t(bh));
          tma_load_3d(vb + kBlock * 128, &maps.v, &full1[s], bx * 64, j1 * kBlock, int32_t(bh));
        }
        issued = p + 1;
      }
      // ring 2 aliases ring 1 (and Q's staging area): all of it must be free
      for (int64_t p = (nP > C::kS1 ? nP - C::kS1 : 0); p < nP && ok; ++p)
        if (!mbar_wait_bounded(&empty1[p % C::kS1], uint32_t((p / C::kS1) & 1), kPollLimit)) ok = false;
      if (ok) release_q();
      // Phase 2: kc, vc rows and H of every group through ring 2
      for (int64_t g = 0; g < NG && ok; ++g) {
        const int s = int(g % C::kS2);
        if (!mbar_wait_bounded(&empty2[s], uint32_t((g / C::kS2) & 1) ^ 1u, kPollLimit)) { ok = false; break; }
        PASA_TRACE_MARK(0, nP + g);
        unsigned char* st = sm + C::kOffRing + s * C::kSlot2;
        mbar_arrive_expect_tx(&full2[s], C::kTxP2);
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          tma_load_3d(st + bx * (kGroup * 128), &maps.kc, &full2[s], bx * 64, int32_t(g * kGroup), int32_t(bh));
          tma_load_3d(st + C::kCBytes + bx * (kGroup * 128), &maps.vc, &full2[s], bx * 64, int32_t(g * kGroup),
                      int32_t(bh));
          tma_load_3d(st + 2 * C::kCBytes + bx * (D * 128), &maps.h, &full2[s], bx * 64, 0, int32_t(bh * NG + g));
        }
        issued = nP + g + 1;
      }
      if (!ok) report(P.err);
      // drain: let this thread's last copies land before the CTA can exit
      for (int64_t n = (issued > 3 ? issued - 3 : 0); n < issued; ++n) {
        if (n < nP) mbar_wait_bounded(&full1[n % C::kS1], uint32_t((n / C::kS1) & 1), kPollLimit);
        else mbar_wait_bounded(&full2[(n - nP) % C::kS2], uint32_t(((n - nP) / C::kS2) & 1), kPollLimit);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ================= MMA issuers =================
    // One thread can issue a tcgen05.mma only every ~90 cycles, slower than
    // the tensor core retires an M128 N128 K16 step, so the score MMAs
    // (warp 1) and the P.V / correction MMAs (warp 2) have an issuer each.
    // Their only shared resource is the S buffer: S(n) may overwrite buffer
    // n & 1 once the softmax has pulled the scores of step n-2 into registers
    // (s_free).  Phase-2 score MMAs are N = 32 and leave the buffer's upper
    // half to U of step n-1.
    if (lane == 0) {
      constexpr uint32_t idS128 = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idS32 = umma_idesc_bf16(128, 32, false, false);
      constexpr uint32_t idPV = umma_idesc_bf16(128, D, false, true);
      bool ok = mbar_wait_bounded(q_tmem, 0, kPollLimit);
      tc_fence_after();
      const uint32_t tQ = tmem + C::kColQ;

      auto slot_addr = [&](int64_t n) -> uint32_t {
        return (n < nP) ? smem_u32(sm + C::kOffRing + int(n % C::kS1) * C::kSlot1)
                        : smem_u32(sm + C::kOffRing + int((n - nP) % C::kS2) * C::kSlot2);
      };
      if (warp == 1) {
        for (int64_t n = 0; n < total && ok; ++n) {
          if (n >= 2) {
            const int64_t m = n - 2;
            const int64_t g2 = m - nP;  // phase-2 group of step m, if any
            const bool freed = (m < nP) ? mbar_wait_bounded(&s_free[m & 1], uint32_t((m >> 1) & 1), kPollLimit)
                                        : mbar_wait_bounded(&s2_free[g2 & 1], uint32_t((g2 >> 1) & 1), kPollLimit);
            if (!freed) { ok = false; break; }
          }
          const bool landed = (n < nP)
              ? mbar_wait_bounded(&full1[n % C::kS1], uint32_t((n / C::kS1) & 1), kPollLimit)
              : mbar_wait_bounded(&full2[(n - nP) % C::kS2], uint32_t(((n - nP) / C::kS2) & 1), kPollLimit);
          if (!landed) { ok = false; break; }
          PASA_TRACE_MARK(1, n);
          tc_fence_after();
          const uint32_t st = slot_addr(n);
          const uint32_t tS = tmem + C::kColS0 + 128u * uint32_t(n & 1);
          if (n < nP) {  // S = Q . [K_j0; K_j1]^T, N = 128
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int bx = kk / 4, ko = (kk % 4) * 32;
              const uint64_t bd = umma_desc_sw128(st + bx * C::kPairBox + ko, 16, 1024);
              mma_ts(tS, tQ + kk * 8, bd, idS128, kk > 0 ? 1u : 0u);
            }
          } else {       // S = Q . kc_g^T, N = 32
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int bx = kk / 4, ko = (kk % 4) * 32;
              const uint64_t bd = umma_desc_sw128(st + bx * (kGroup * 128) + ko, 16, 1024);
              mma_ts(tS, tQ + kk * 8, bd, idS32, kk > 0 ? 1u : 0u);
            }
          }
          PASA_TRACE_MARK(28, n);
          tc_commit(&s_full[n & 1]);
        }
      } else {
        for (int64_t m = 0; m < total && ok; ++m) {
          const int64_t g2 = m - nP;  // phase-2 group of step m, if any
          const bool ready = (m < nP) ? mbar_wait_bounded(&p_ready[m & 1], uint32_t((m >> 1) & 1), kPollLimit)
                                      : mbar_wait_bounded(&p2_ready[g2 & 1], uint32_t((g2 >> 1) & 1), kPollLimit);
          if (!ready) { ok = false; break; }
          PASA_TRACE_MARK(2, m);
          tc_fence_after();
          const uint32_t st = slot_addr(m);
          if (m < nP) {  // O += P . [V_j0; V_j1], K = 128
#pragma unroll
            for (int kk = 0; kk < 2 * kBlock / 16; ++kk) {
              const uint64_t bd = umma_desc_sw128(st + 2 * C::kKVBytes + kk * 2048, C::kPairBox, 1024);
              mma_ts(tmem + C::kColO, tmem + C::kColP + kk * 8, bd, idPV, (m > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(&empty1[m % C::kS1]);
          } else {       // O += P_g . vc_g + U_g . H_g
            const uint32_t tPg = tmem + C::kColP + 16u * uint32_t(m & 1);
            const uint32_t tU = tmem + C::kColS0 + 128u * uint32_t((m + 1) & 1) + C::kColU;
#pragma unroll
            for (int kk = 0; kk < kGroup / 16; ++kk) {
              const uint64_t bd = umma_desc_sw128(st + C::kCBytes + kk * 2048, C::kCBytes / C::kBoxes, 1024);
              mma_ts(tmem + C::kColO, tPg + kk * 8, bd, idPV, 1u);
            }
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t bd = umma_desc_sw128(st + 2 * C::kCBytes + kk * 2048, C::kHBytes / C::kBoxes, 1024);
              mma_ts(tmem + C::kColO, tU + kk * 8, bd, idPV, 1u);
            }
            tc_commit(&empty2[(m - nP) % C::kS2]);
          }
          tc_commit(&o_done[m & 1]);
          PASA_TRACE_MARK(29, m);
        }
      }
      if (!ok) report(P.err);
    }
    __syncwarp();
  } else {
    // ================= softmax / correction (warps 3 .. 3 + kSoftmaxWarps) =================
    // kParts threads per query row (TMEM lane): thread `part` owns columns
    // [kPC part, kPC part + kPC) of both key blocks of a phase-1 step and
    // output columns [DQ part, DQ part + DQ); in phase 2 it owns every other
    // group of its row.  The kParts warps of a lane quadrant combine
    // row maxima and sums through shared memory.
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may access
    const int part = (warp - 3) >> 2;          // column part of this warp
    const int r = quad * 32 + lane;            // tile row == TMEM lane
    const int half = r >> 6;                   // 0: block A, 1: block B
    const bool live = (half == 0) || hasB;     // uniform per warp
    const int bar_id = 1 + quad;               // named barrier of the quadrant's kParts warps
    const uint32_t lane_base = uint32_t(quad * 32) << 16;
    const float scale32 = P.scale;
    const float sm_scale = scale32 * kLog2e;
    const int64_t last_len = P.T - (NT - 1) * kBlock;
    constexpr int DQ = D / kParts;             // Q / output columns per thread
    constexpr int kPC = kBlock / kParts;       // score columns per key block per thread
    float m_true = -INFINITY, m_used = -INFINITY, l1 = 0.f, gl = 0.f;
    uint32_t xslot = 0;
    // combine one value per thread across the row's kParts threads (fixed order)
    auto row_reduce = [&](float v, bool is_max) -> float {
      xch[(xslot * kParts + part) * kRowsPerTile + r] = v;
      named_bar_sync(bar_id, 32 * kParts);
      float o = xch[(xslot * kParts) * kRowsPerTile + r];
#pragma unroll
      for (int q2 = 1; q2 < kParts; ++q2) {
        const float x = xch[(xslot * kParts + q2) * kRowsPerTile + r];
        o = is_max ? fmaxf(o, x) : o + x;
      }
      xslot ^= 1u;
      return o;
    };
    bool ok = mbar_wait_bounded(q_full, 0, kPollLimit);
    {  // copy this row's part of Q into TMEM, the A operand of the score MMAs
      uint32_t qpk[DQ / 2];
#pragma unroll
      for (int x = 0; x < DQ / 8; ++x) {
        const int d = part * DQ + x * 8, bx = d / 64, c = (d % 64) / 8;
        const uint4 v = *reinterpret_cast<const uint4*>(sm + C::kOffQ + bx * (kRowsPerTile * 128) + r * 128 +
                                                       ((c ^ (r & 7)) << 4));
        qpk[x * 4 + 0] = v.x; qpk[x * 4 + 1] = v.y; qpk[x * 4 + 2] = v.z; qpk[x * 4 + 3] = v.w;
      }
      tmem_st<DQ / 2>(tmem + lane_base + C::kColQ + part * (DQ / 2), qpk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_tmem);
    }

    auto rescale_o = [&](int64_t n, float alpha) -> bool {
      // O is consistent once the MMAs of step n-1 have completed
      if (n >= 1) {
        const int64_t m = n - 1;
        if (!mbar_wait_bounded(&o_done[m & 1], uint32_t((m >> 1) & 1), kPollLimit)) return false;
        tc_fence_after();
      }
#pragma unroll
      for (int c0 = 0; c0 < DQ; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_base + C::kColO + part * DQ + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 16; ++x) v[x] = __float_as_uint(__uint_as_float(v[x]) * alpha);
        tmem_st16(tmem + lane_base + C::kColO + part * DQ + c0, v);
      }
      tmem_wait_st();
      return true;
    };

    // phase 2: one thread owns the row, so it rescales all D columns of O
    auto rescale_o_all = [&](int64_t n, float alpha) -> bool {
      if (n >= 1) {
        const int64_t m = n - 1;
        if (!mbar_wait_bounded(&o_done[m & 1], uint32_t((m >> 1) & 1), kPollLimit)) return false;
        tc_fence_after();
      }
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_base + C::kColO + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 16; ++x) v[x] = __float_as_uint(__uint_as_float(v[x]) * alpha);
        tmem_st16(tmem + lane_base + C::kColO + c0, v);
      }
      tmem_wait_st();
      return true;
    };

    // wait for the scores of step n; returns this thread's S-buffer address
    auto wait_scores = [&](int64_t n, uint32_t& tS) -> bool {
      const int b = int(n & 1);
      if (!mbar_wait_bounded(&s_full[b], uint32_t((n >> 1) & 1), kPollLimit)) return false;
      if (lane == 0 && warp < 11) PASA_TRACE_MARK(4 + (warp - 3), n);
      tc_fence_after();
      tS = tmem + lane_base + C::kColS0 + 128u * uint32_t(b);
      return true;
    };
    // After a failed wait (ok false) the loops keep going without waiting, so
    // every warp still takes part in every named barrier and none is stranded.
    // P of a phase-1 step fills the P region, so the P.V of step n-1 must be
    // done with it.  A phase-2 step n writes P_g to half n & 1 of the region's
    // first 32 columns and U to S buffer (n + 1) & 1, both last read by the
    // P.V of step n-2 (of step n-1 for the first group, after the full-width P).
    const uint32_t tP = tmem + lane_base + C::kColP;
    auto wait_p_free = [&](int64_t n) -> bool {
      const int64_t lag = (n <= nP) ? 1 : 2;
      if (n < lag) return true;
      const int64_t m = n - lag;
      if (!mbar_wait_bounded(&o_done[m & 1], uint32_t((m >> 1) & 1), kPollLimit)) return false;
      tc_fence_after();
      return true;
    };
    // hand P (and U) of step n to the MMA warp
    auto release_step = [&](int64_t n) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && warp < 11) PASA_TRACE_MARK(12 + (warp - 3), n);
      if (lane == 0) mbar_arrive(&p_ready[n & 1]);
    };

    for (int64_t n = 0; n < nP; ++n) {
      uint32_t tS = tmem + lane_base + C::kColS0 + 128u * uint32_t(n & 1);
      if (ok && !wait_scores(n, tS)) ok = false;
      {
        // ---------------- Phase 1: a pair of exact blocks ----------------
        const uint32_t e0 = ulist[2 * n];
        const uint32_t e1 = (2 * n + 1 < nU) ? uint32_t(ulist[2 * n + 1]) : 0u;  // lone last block: no bits
        const bool act0 = live && ((e0 >> half) & 1u);  // uniform per warp (and per quadrant)
        const bool act1 = live && ((e1 >> half) & 1u);
        uint32_t pk0[kPC / 2], pk1[kPC / 2];
        uint32_t s0[kPC], s1[kPC];
        if (act0) tmem_ld<kPC>(tS + part * kPC, s0);
        if (act1) tmem_ld<kPC>(tS + 64 + part * kPC, s1);
        tmem_wait_ld();
        // the scores are in registers: the S buffer may take the scores of step n + 2
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[n & 1]);
        if (act0 || act1) {
          if (warp == 3 && lane == 0) PASA_TRACE_MARK(24, n);
          // key rows >= T are masked (:178); only the last block has them
          if (act0 && int(e0 >> 2) == int(NT) - 1) mask_tail<kPC>(s0, int(last_len) - part * kPC);
          if (act1 && int(e1 >> 2) == int(NT) - 1) mask_tail<kPC>(s1, int(last_len) - part * kPC);
          float mx = -INFINITY;
          if (act0) mx = max_tree<kPC>(s0);
          if (act1) mx = fmaxf(mx, max_tree<kPC>(s1));
          if (warp == 3 && lane == 0) PASA_TRACE_MARK(25, n);
          mx = row_reduce(mx, true) * sm_scale;  // max commutes with the positive scale
          if (warp == 3 && lane == 0) PASA_TRACE_MARK(26, n);
          m_true = fmaxf(m_true, mx);
          const bool grow = mx > m_used + kRescaleThresh;
          const bool need = grow && (m_used != -INFINITY);
          const float alpha = need ? fast_exp2(m_used - mx) : 1.0f;
          if (__any_sync(0xffffffffu, need)) {  // tcgen05.ld/st are warp-collective
            if (ok && !rescale_o(n, alpha)) ok = false;
          }
          l1 *= alpha;
          if (grow) m_used = mx;
          if (act0) {
            l1 += exp2_pack<kPC>(s0, sm_scale, -m_used, pk0);
          } else {
#pragma unroll
            for (int c = 0; c < kPC / 2; ++c) pk0[c] = 0u;
          }
          if (act1) {
            l1 += exp2_pack<kPC>(s1, sm_scale, -m_used, pk1);
          } else {
#pragma unroll
            for (int c = 0; c < kPC / 2; ++c) pk1[c] = 0u;
          }
        } else {
#pragma unroll
          for (int c = 0; c < kPC / 2; ++c) { pk0[c] = 0u; pk1[c] = 0u; }
        }
        if (warp == 3 && lane == 0) PASA_TRACE_MARK(27, n);
        if (ok && !wait_p_free(n)) ok = false;
        tmem_st<kPC / 2>(tP + part * (kPC / 2), pk0);       // keys [kPC part, kPC part + kPC) of block 0
        tmem_st<kPC / 2>(tP + 32 + part * (kPC / 2), pk1);  // the same keys of block 1
        tmem_wait_st();
      }
      release_step(n);
    }

    // ---------------- Phase 2: groups, ping-pong between the two column parts ----------------
    // The warps of part p take the groups g with g % 2 == p, one thread per row
    // owning all kGroup columns of its group, so consecutive groups overlap.
    // The reference's running maxima are sequential over groups (:237-243):
    // each group hands (m_used, m_true) of its rows to the next group's warps
    // through shared memory and a named barrier per lane quadrant and
    // direction (arrive by the producer, sync by the consumer).
    static_assert(kParts == 2, "phase-2 ping-pong pairs the two column parts");
    float m_applied = m_used;  // the maximum this thread's l1 is scaled to
    const int hand_to = 5 + quad * 2 + part;          // barrier this part arrives on
    const int hand_from = 5 + quad * 2 + (part ^ 1);  // barrier this part waits on
    float* hand_out = hand + part * 2 * kRowsPerTile;
    const float* hand_in = hand + (part ^ 1) * 2 * kRowsPerTile;
    for (int64_t g = part; g < NG; g += 2) {
      const int64_t n = nP + g;
      uint32_t tS = tmem + lane_base + C::kColS0 + 128u * uint32_t(n & 1);
      if (ok && !wait_scores(n, tS)) ok = false;
      uint32_t sv[kGroup];
      if (live) tmem_ld<kGroup>(tS, sv);
      tmem_wait_ld();
      // the scores are in registers: the S buffer may take the scores of step n + 2
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s2_free[part]);
      uint32_t pk[kGroup / 2];
      float w = 0.f;
      if (live) {  // uniform per lane quadrant: both parts of a quadrant take this branch
        // columns of selected blocks or of blocks >= NT are masked (:228)
        const int jb0 = int(g) * kGroup;  // NT <= kMaxNT fits in int
        const int lim = int(NT) - jb0;
        const uint32_t word = maskw[half * kMaxNG + g];
#pragma unroll
        for (int c = 0; c < kGroup; ++c)
          if (c >= lim || ((word >> c) & 1u)) sv[c] = __float_as_uint(-INFINITY);
        float mx = max_tree<kGroup>(sv);
        mx = (mx == -INFINITY) ? mx : mx * sm_scale;
        if (g >= 1) {  // running maxima after group g - 1
          named_bar_sync(hand_from, 64);
          m_used = hand_in[r];
          m_true = hand_in[kRowsPerTile + r];
        }
        const float m_used_prev = m_used;
        const float m_true_new = fmaxf(m_true, mx);
        const bool grow = mx > m_used + kRescaleThresh;  // m_used is finite for live rows here
        if (grow) m_used = mx;
        if (g + 1 < NG) {
          hand_out[r] = m_used;
          hand_out[kRowsPerTile + r] = m_true_new;
          named_bar_arrive(hand_to, 64);
        }
        if (__any_sync(0xffffffffu, grow)) {  // O holds steps <= n-1 in units of m_used_prev
          const float alpha = grow ? fast_exp2(m_used_prev - m_used) : 1.0f;
          if (ok && !rescale_o_all(n, alpha)) ok = false;
        }
        if (m_applied != m_used) { l1 *= fast_exp2(m_applied - m_used); m_applied = m_used; }
        float p[kGroup];
        const float negm = -m_used;
#pragma unroll
        for (int c = 0; c < kGroup; ++c) p[c] = exp2_ftz(fmaf(__uint_as_float(sv[c]), sm_scale, negm));
        float psum, wsum;
        {
          float a0 = 0.f, a1 = 0.f, extra = 0.f;
          // bit of the ragged last block's column, if it is in this group
          // (a bit test, not an index: p[] must stay in registers)
          const uint32_t lastbit = (lim >= 1 && lim <= kGroup) ? (1u << (lim - 1)) : 0u;
#pragma unroll
          for (int c = 0; c < kGroup; c += 2) {
            a0 += p[c]; a1 += p[c + 1];
            extra += ((lastbit >> c) & 1u) ? p[c] : (((lastbit >> (c + 1)) & 1u) ? p[c + 1] : 0.f);
          }
          psum = a0 + a1;
          // the ragged last block has its own length (:220)
          wsum = psum * float(kBlock) + extra * float(last_len - kBlock);
        }
#pragma unroll
        for (int c = 0; c < kGroup; c += 2) pk[c / 2] = pack_bf16x2(p[c], p[c + 1]);
        // the reference's probabilities use the exact running max (:237, :243)
        gl += wsum * fast_exp2(m_used - m_true_new);
        m_true = m_true_new;
        w = psum * scale32;  // :253
      } else {
#pragma unroll
        for (int c = 0; c < kGroup / 2; ++c) pk[c] = 0u;
      }
      if (ok && !wait_p_free(n)) ok = false;
      tmem_st<kGroup / 2>(tP + 16u * uint32_t(n & 1), pk);
      // U = bf16(w q) over all D columns, 32 packed columns at a time (Q read back from TMEM)
      const uint32_t tU = tmem + lane_base + C::kColS0 + 128u * uint32_t((n + 1) & 1) + C::kColU;
#pragma unroll
      for (int c0 = 0; c0 < D / 2; c0 += 32) {
        uint32_t qv[32];
        tmem_ld32(tmem + lane_base + C::kColQ + c0, qv);
        tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          const float2 qf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qv[x]));
          qv[x] = pack_bf16x2(qf.x * w, qf.y * w);
        }
        tmem_st32(tU + c0, qv);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && warp < 11) PASA_TRACE_MARK(12 + (warp - 3), n);
      if (lane == 0) mbar_arrive(&p2_ready[part]);
    }
    // Each part ends with the maxima of the last group it saw; the maxima only
    // grow, so the larger pair is the final one.
    if (live) {
      m_used = row_reduce(m_used, true);
      m_true = row_reduce(m_true, true);
      if (m_applied != m_used) l1 *= fast_exp2(m_applied - m_used);
    }

    // ---------------- Final: o = O / (l + g_l) ----------------
    if (ok && total >= 1) {
      const int64_t m = total - 1;
      ok = mbar_wait_bounded(&o_done[m & 1], uint32_t((m >> 1) & 1), kPollLimit);
      tc_fence_after();
    }
    const int64_t blk = (half == 0) ? blkA : blkB;
    const int64_t t = blk * kBlock + (r & 63);
    const bool wok = __all_sync(0xffffffffu, ok);
    if (live) {
      // the row's threads combine their partial sums (all take part even after a failure)
      const float l_tot = row_reduce(l1, false);
      const float g_tot = row_reduce(gl, false);
      if (wok) {  // warp-uniform: tcgen05.ld is warp-collective
        const bool store = t < P.T;
        const float denom = l_tot + g_tot * fast_exp2(m_true - m_used);
        const float inv = 1.0f / denom;
        __nv_bfloat16* orow = P.o + (bh * P.T + t) * D + part * DQ;
#pragma unroll
        for (int c0 = 0; c0 < DQ; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tmem + lane_base + C::kColO + part * DQ + c0, v);
          tmem_wait_ld();
          uint4 out[2];
          uint32_t* ow = reinterpret_cast<uint32_t*>(out);
#pragma unroll
          for (int x = 0; x < 8; ++x)
            ow[x] = pack_bf16x2(__uint_as_float(v[2 * x]) * inv, __uint_as_float(v[2 * x + 1]) * inv);
          if (store) {
            reinterpret_cast<uint4*>(orow + c0)[0] = out[0];
            reinterpret_cast<uint4*>(orow + c0)[1] = out[1];
          }
        }
      }
    }
    if (!ok) report(P.err);
    if (warp == 3 && lane == 0) PASA_TRACE_CTL(2);
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0) PASA_TRACE_CTL(3);
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D bf16 map over [batch][rows][D] with a (64 x box_rows x 1) box, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, int D, int64_t rows, int64_t batch, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(rows), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(D) * 2, cuuint64_t(rows) * cuuint64_t(D) * 2};
  cuuint32_t box[3] = {64u, cuuint32_t(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int D>
cudaError_t launch_tc_t(cudaStream_t st, const void* q, const void* k, const void* v, const void* kc,
                        const void* vc, const void* hg, const uint32_t* mask, int64_t BH, int64_t T_len,
                        float scale, void* o, uint32_t* err) {
  using C = Cfg<D>;
  const int64_t NT = cdiv(T_len, kBlock), NG = cdiv(NT, kGroup), NTP = NG * kGroup;
  if (NT > kMaxNT) return cudaErrorInvalidValue;
  Maps maps;
  if (!make_map(&maps.q, q, D, T_len, BH, kRowsPerTile) || !make_map(&maps.k, k, D, T_len, BH, kBlock) ||
      !make_map(&maps.v, v, D, T_len, BH, kBlock) || !make_map(&maps.kc, kc, D, NTP, BH, kGroup) ||
      !make_map(&maps.vc, vc, D, NTP, BH, kGroup) || !make_map(&maps.h, hg, D, D, BH * NG, D))
    return cudaErrorInvalidValue;
  Params p;
  p.T = T_len; p.NT = NT; p.NG = NG; p.NTP = NTP; p.scale = scale;
  p.o = static_cast<__nv_bfloat16*>(o); p.sel_mask = mask; p.err = err;
  auto kern = attn_tc_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(cdiv(NT, 2)), unsigned(BH), 1u};
  kern<<<grid, kThreads, C::kSmemBytes, st>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace tc

cudaError_t launch_attn_tc(cudaStream_t st, int D, const void* q, const void* k, const void* v, const void* kc,
                           const void* vc, const void* hg, const uint32_t* mask, int64_t BH, int64_t T_len,
                           int64_t /*NS*/, float scale, void* o, uint32_t* err) {
  if (D == 64) return tc::launch_tc_t<64>(st, q, k, v, kc, vc, hg, mask, BH, T_len, scale, o, err);
  return tc::launch_tc_t<128>(st, q, k, v, kc, vc, hg, mask, BH, T_len, scale, o, err);
}

}  // namespace pasa

#ifdef PASA_TRACE
extern "C" PASA_API int pasa_trace_read(void* host_dst, size_t bytes) {
  return cudaMemcpyFromSymbol(host_dst, pasa::tc::g_pasa_trace, bytes) == cudaSuccess ? 0 : PASA_ERR_CUDA;
}
extern "C" PASA_API int pasa_trace_ctl_read(void* host_dst, size_t bytes) {
  return cudaMemcpyFromSymbol(host_dst, pasa::tc::g_pasa_trace_ctl, bytes) == cudaSuccess ? 0 : PASA_ERR_CUDA;
}
extern "C" PASA_API int pasa_trace_select(unsigned int x, unsigned int y) {
  const unsigned int v[2] = {x, y};
  return cudaMemcpyToSymbol(pasa::tc::g_pasa_trace_cta, v, sizeof(v)) == cudaSuccess ? 0 : PASA_ERR_CUDA;
}
#endif
