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
//     is N=128 and P.V is K=128.  Steps pair a block only query block A
//     selected with one only B selected where possible, so both halves of the
//     softmax carry equal work; rows whose query block did not select a key
//     block get P = 0 and skip its exponentials.  Phase 2 (shared by both
//     query blocks) walks the 32-block groups with each half's own selection
//     bits, one group per step.
//   * Q stays in shared memory as the A operand of every score MMA; K and V
//     of a step have separate rings (K runs three steps ahead, V two).
//     Phase 2's rings are aliased on the same memory: kc rows (five groups,
//     freed by the score MMAs) and vc rows + H (three groups, freed by the
//     correction MMAs), so the score MMAs of later groups never wait for an
//     earlier group's correction to free a slot.
//   * TMEM (512 columns): O (128, fp32), two P regions (64 each, bf16) and
//     two S buffers (128 each).  Step n uses S buffer n & 1 and P region n & 1.
//   * warp 0: TMA producer; warp 1: TMEM owner and score-MMA issuer; warp 2:
//     P.V / correction MMA issuer (one thread issues a tcgen05.mma only every
//     ~90 cycles, so one issuer would cap the tensor core at ~70% for these
//     shapes); warps 3-6 and 7-10: the two softmax sets.
//   * The softmax sets ping-pong over steps: set s takes the steps n with
//     n % 2 == s, one thread per query row (TMEM lane) holding all of the
//     step's scores, so one set's loads, maxima and stores overlap the other
//     set's exponentials.  The reference's running maxima are sequential
//     over steps, so each step hands (m_used, m_true) of its rows to the next
//     step's set through shared memory and a named barrier per lane quadrant
//     and direction.  A set frees its S buffer as soon as the scores are in
//     registers, so the score MMAs of step n+2 run during the softmax of n.
//   * Phase 2: group scores are 32 columns; P_g sits in the step's P region
//     and the first-order operand U = bf16(w_t q_t) (w_t = scale * sum of the
//     group's probabilities) in the upper half of the step's own S buffer
//     (the group score MMAs write only its first 32 columns), and U.H_g is
//     accumulated straight into O by the tensor core.
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

// K and V ring depths (slots of two key blocks) and how many phase-1 steps
// the producer issues K ahead of V.
#ifndef PASA_ATTN_SK
#define PASA_ATTN_SK 3
#endif
#ifndef PASA_ATTN_SV
#define PASA_ATTN_SV 2
#endif
#ifndef PASA_ATTN_KV_LAG
#define PASA_ATTN_KV_LAG 2
#endif
#ifndef PASA_ATTN_LAG_H
#define PASA_ATTN_LAG_H 2
#endif

constexpr int kSetWarps = 4;               // warps per softmax set (one per TMEM lane quadrant)
constexpr int kSoftmaxWarps = 2 * kSetWarps;
constexpr int kThreads = 32 * (3 + kSoftmaxWarps);  // TMA, S issuer, P.V issuer, two softmax sets
constexpr int kRowsPerTile = 128;      // two query blocks
constexpr float kRescaleThresh = 8.0f; // log2 units
constexpr int kMaxNT = 4096;           // union list capacity (entries)
constexpr int kMaxNG = kMaxNT / kGroup;
constexpr uint64_t kPollLimit = kWaitLimitCycles;  // SM cycles a barrier wait may take before giving up

template <int D>
struct Cfg {
  static constexpr int kBoxes = D / 64;                 // 64-column TMA boxes per row
  static constexpr int kRowBox = kRowsPerTile * 128;    // one [128 rows][64 cols] SW128 box
  static constexpr int kQBytes = kBoxes * kRowBox;      // Q of the tile
  static constexpr int kPairBytes = kBoxes * kRowBox;   // K (or V) of two key blocks
  static constexpr int kCBytes = kGroup * D * 2;        // kc (or vc) rows of one group
  static constexpr int kHBytes = D * D * 2;
  static constexpr int kSK = PASA_ATTN_SK;              // K ring slots
  static constexpr int kSV = PASA_ATTN_SV;              // V ring slots
  static constexpr int kKVRegion = (kSK + kSV) * kPairBytes;
  // Phase 2 has two rings: vc rows + H (read by the P.V issuer), aliased
  // on the K and V rings, and kc rows (read by the score MMAs) in memory of
  // their own.  Each is released by its own reader, so the next groups' kc
  // need not wait for the correction MMAs of an earlier group to free a
  // shared slot.  The vc/H ring takes the whole K/V region: a group's 40 KB
  // land ~3000 cycles after their slot frees, and the P.V issuer waits for
  // them, so the ring depth sets the phase-2 period (three slots: ~1450
  // cycles per group; four: the issue rate).  Its own kc ring also lets the
  // first groups' kc load while phase 1 still runs.
  static constexpr int kSlotH = kCBytes + kHBytes;      // vc rows and H of one group
  static constexpr int kSHFit = kKVRegion / kSlotH;
  static constexpr int kSH = kSHFit < 6 ? kSHFit : 6;   // vc/H ring slots
  static constexpr int kSC = 2;                         // kc ring slots
  static constexpr int kLagH = PASA_ATTN_LAG_H;         // kc loads run this many groups ahead of vc/H
  // TMEM columns
  static constexpr uint32_t kColO = 0;
  static constexpr uint32_t kColP = 128;                // P region b at kColP + 64 b
  static constexpr uint32_t kColS0 = 256;               // S buffer b at kColS0 + 128 b
  static constexpr uint32_t kColU = 64;                 // phase 2: U of step n in S buffer n & 1
  static constexpr uint32_t kTmemCols = 512;
  // shared memory carve-up (offsets from a 1024-aligned base)
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;                      // K ring, then V ring
  static constexpr int kOffV = kOffK + kSK * kPairBytes;
  static constexpr int kOffRingH = kOffK;                            // aliased on the K and V rings
  static constexpr int kOffRingC = kOffK + kKVRegion;                // kc ring, its own memory
  static constexpr int kOffUnion = kOffRingC + kSC * kCBytes;        // u16 [kMaxNT]
  static constexpr int kOffMask = kOffUnion + kMaxNT * 2;            // u32 [2][kMaxNG]
  static constexpr int kOffXch = kOffMask + 2 * kMaxNG * 4;          // f32 [2 slots][2 sets][128]
  static constexpr int kOffHand = kOffXch + 2 * 2 * kRowsPerTile * 4;  // f32 [2 sets][m_used, m_true][128]
  static constexpr int kOffBar = kOffHand + 2 * 2 * kRowsPerTile * 4;
  static constexpr int kNumBars = 2 * kSK + 2 * kSV + 2 * kSC + 2 * kSH + 1 + 2 + 2 + 2 + 2;
  static constexpr int kOffSlot = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffSlot + 16 + 1024;  // + alignment slack
  // (the producer issues kc(i) before vc/H(i - kLagH); kc(i) waits for the
  // score MMAs of group i - kSC, whose chain of waits reaches back only to
  // vc/H loads issued before it while kLagH <= kSC + 3)
  static_assert(kLagH <= kSC + 3 && kSH >= 3 && kOffRingH + kSH * kSlotH <= kOffK + kKVRegion, "phase-2 rings");
  static_assert(kColS0 + 2 * 128 <= kTmemCols, "TMEM budget");
  static_assert(kColO + D <= kColP, "O must fit below P");
  static_assert(kColU + D / 2 <= 128, "U must fit in the S buffer");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
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
  int dense;  // every key block selected for every query block (sel_mask unused, no phase 2)
  int64_t o_heads;  // 0: o is [B*H, T, D]; H > 0: o is [B, T, H, D] (token-major, bh = b*H + h)
  // scatter mode (o_npeer > 0, B = 1): the row of local head bh and token t
  // goes to o_peer[t / o_tokens] at [(t % o_tokens) * o_heads_total + o_head0 + bh]
  __nv_bfloat16* const* o_peer;
  int o_npeer;
  int64_t o_tokens, o_heads_total, o_head0;
  // CTA p works on the query-block pair pair0 + p and stores only the rows
  // of query blocks in [blk_lo, blk_hi) (a block range of the head)
  int64_t pair0, blk_lo, blk_hi;
};

// Optional step tracer (compile with -DPASA_TRACE): one CTA, chosen with
// pasa_trace_select(), records SM clock stamps of its pipeline events for
// the first kTraceSteps steps into g_pasa_trace[event][step]: 0 producer
// issue (K; kc in phase 2), 1 S issue, 28 S issued, 2 P.V issue, 29 P.V issued, 3 V issue (vc/H in phase 2),
// 4+w softmax warp w (0-7) sees S, 12+w softmax warp w done, 20-27 set-0
// sub-stages; pasa_trace_read() copies them out.
#ifdef PASA_TRACE
constexpr int kTraceSteps = 1024;
__device__ unsigned long long g_pasa_trace[30][kTraceSteps];
__device__ unsigned int g_pasa_trace_cta[2];  // (blockIdx.x, blockIdx.y) of the traced CTA
__device__ unsigned long long g_pasa_trace_ctl[8];  // entry, set-up done, softmax done, exit (per traced CTA)
// every CTA: global timer (ns) at entry and exit, SM clock cycles from entry
// to exit, SM id and union size, at [blockIdx.y * gridDim.x + blockIdx.x]
constexpr int kTraceCtas = 65536;
__device__ unsigned long long g_pasa_trace_cta_rec[kTraceCtas][4];
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
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
  uint64_t* full_k = bars;
  uint64_t* empty_k = full_k + C::kSK;
  uint64_t* full_v = empty_k + C::kSK;
  uint64_t* empty_v = full_v + C::kSV;
  uint64_t* full_c = empty_v + C::kSV;
  uint64_t* empty_c = full_c + C::kSC;
  uint64_t* full_h = empty_c + C::kSC;
  uint64_t* empty_h = full_h + C::kSH;
  uint64_t* q_full = empty_h + C::kSH;
  uint64_t* s_full = q_full + 1;   // [2] scores of S buffer b are in TMEM
  uint64_t* s_free = s_full + 2;   // [2] set b holds the scores of its step in registers
  uint64_t* p_ready = s_free + 2;  // [2] set b's P (and U) of its step are in TMEM
  uint64_t* o_done = p_ready + 2;  // [2] the P.V (and correction) MMAs of a step with parity b completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::kOffSlot);
  __shared__ uint32_t s_nu, s_cnt[2];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#ifdef PASA_TRACE
  const bool pasa_traced = blockIdx.x == g_pasa_trace_cta[0] && blockIdx.y == g_pasa_trace_cta[1];
  if (tid == 0) PASA_TRACE_CTL(0);
  const unsigned long long pasa_t0_ns = global_ns(), pasa_t0_clk = clock64();
#endif
  const int64_t pair = blockIdx.x + P.pair0, bh = blockIdx.y;
  const int64_t NT = P.NT, NG = P.NG;
  const int64_t blkA = 2 * pair, blkB = 2 * pair + 1;
  const bool hasB = blkB < NT;

  // ---- set-up: barriers, TMEM, selection bits, union list -------------
  if (tid == 0) {
    for (int s = 0; s < C::kSK; ++s) { mbar_init(&full_k[s], 1); mbar_init(&empty_k[s], 1); }
    for (int s = 0; s < C::kSV; ++s) { mbar_init(&full_v[s], 1); mbar_init(&empty_v[s], 1); }
    for (int s = 0; s < C::kSC; ++s) { mbar_init(&full_c[s], 1); mbar_init(&empty_c[s], 1); }
    for (int s = 0; s < C::kSH; ++s) { mbar_init(&full_h[s], 1); mbar_init(&empty_h[s], 1); }
    mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1); mbar_init(&s_free[b], kSetWarps);
      mbar_init(&p_ready[b], kSetWarps); mbar_init(&o_done[b], 1);
    }
    fence_barrier_init();
    // Q of the tile needs nothing else: it loads while the union list is built
    mbar_arrive_expect_tx(q_full, C::kQBytes);
    for (int bx = 0; bx < C::kBoxes; ++bx)
      tma_load_3d(sm + C::kOffQ + bx * C::kRowBox, &maps.q, q_full, bx * 64, int32_t(pair * kRowsPerTile),
                  int32_t(bh));
  }
  if (warp == 1) { tmem_alloc(tmem_slot, C::kTmemCols); tmem_relinquish(); }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&maps.q); prefetch_tmap(&maps.k); prefetch_tmap(&maps.v);
    prefetch_tmap(&maps.kc); prefetch_tmap(&maps.vc); prefetch_tmap(&maps.h);
  }
  for (int64_t w = tid; w < NG; w += kThreads) {
    if (P.dense) {  // all blocks < NT
      const int64_t left = NT - w * 32;
      const uint32_t all = left >= 32 ? 0xFFFFFFFFu : ((1u << left) - 1u);
      maskw[w] = all;
      maskw[kMaxNG + w] = hasB ? all : 0u;
    } else {
      maskw[w] = P.sel_mask[(bh * NT + blkA) * NG + w];
      maskw[kMaxNG + w] = hasB ? P.sel_mask[(bh * NT + blkB) * NG + w] : 0u;
    }
  }
  __syncthreads();
  // Union of the two selections, ordered so that consecutive pairs (one
  // phase-1 step) balance the two halves: blocks only A selected alternate
  // with blocks only B selected, then the leftover single-half blocks, then
  // the blocks both selected.  Within each category the order is ascending.
  // (The softmax is order-independent, so any order gives the same result
  // up to floating-point rounding.)  Warp 0 counts each category per mask
  // word and scans the counts over the words; then every thread places
  // blocks j = tid, tid + kThreads, ... at their positions in parallel.
  uint32_t* pre = reinterpret_cast<uint32_t*>(xch);  // [3][kMaxNG] exclusive counts (xch is free until the steps)
  if (warp == 0) {
    uint32_t ka = 0, kb = 0, kab = 0;  // running counts per category
    for (int64_t w0 = 0; w0 < NG; w0 += 32) {
      const int64_t w = w0 + lane;
      const uint32_t ma = (w < NG) ? maskw[w] : 0u, mb = (w < NG) ? maskw[kMaxNG + w] : 0u;
      const uint32_t ca = __popc(ma & ~mb), cb = __popc(mb & ~ma), cab = __popc(ma & mb);
      uint32_t ia = ca, ib = cb, iab = cab;  // inclusive scans over lanes
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t ya = __shfl_up_sync(0xffffffffu, ia, off);
        const uint32_t yb = __shfl_up_sync(0xffffffffu, ib, off);
        const uint32_t yab = __shfl_up_sync(0xffffffffu, iab, off);
        if (lane >= off) { ia += ya; ib += yb; iab += yab; }
      }
      if (w < NG) {
        pre[w] = ka + ia - ca;
        pre[kMaxNG + w] = kb + ib - cb;
        pre[2 * kMaxNG + w] = kab + iab - cab;
      }
      ka += __shfl_sync(0xffffffffu, ia, 31);
      kb += __shfl_sync(0xffffffffu, ib, 31);
      kab += __shfl_sync(0xffffffffu, iab, 31);
    }
    if (lane == 0) { s_cnt[0] = ka; s_cnt[1] = kb; s_nu = ka + kb + kab; }
  }
  __syncthreads();
  {
    const uint32_t na = s_cnt[0], nb = s_cnt[1];
    const uint32_t m = na < nb ? na : nb;
    for (int64_t j = tid; j < NT; j += kThreads) {
      const int64_t w = j >> 5;
      const uint32_t bitm = 1u << (j & 31), below = bitm - 1u;
      const uint32_t ma = maskw[w], mb = maskw[kMaxNG + w];
      const uint32_t ua = ma & ~mb, ub = mb & ~ma, uab = ma & mb;
      if (ua & bitm) {
        const uint32_t pa = pre[w] + __popc(ua & below);
        ulist[(pa < m) ? 2 * pa : 2 * m + (pa - m)] = uint16_t((uint32_t(j) << 2) | 1u);
      } else if (ub & bitm) {
        const uint32_t pb = pre[kMaxNG + w] + __popc(ub & below);
        ulist[(pb < m) ? 2 * pb + 1 : 2 * m + (na - m) + (pb - m)] = uint16_t((uint32_t(j) << 2) | 2u);
      } else if (uab & bitm) {
        const uint32_t pab = pre[2 * kMaxNG + w] + __popc(uab & below);
        ulist[na + nb + pab] = uint16_t((uint32_t(j) << 2) | 3u);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) PASA_TRACE_CTL(1);
  const int64_t nU = s_nu;
  const int64_t nP = (nU + 1) / 2;  // phase-1 steps: two union blocks each (a lone last block pairs with itself)
  // phase 2 corrects the blocks a query block did not select; with every
  // block selected (dense) there are none and its terms are exactly zero
  const int64_t NG2 = P.dense ? 0 : NG;
  const int64_t total = nP + NG2;


  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      bool ok = true;
      // K and V of phase-1 step p: the two union blocks, each [64 rows] of every 64-column box
      auto load_pair = [&](const CUtensorMap* map, unsigned char* dst, uint64_t* bar, int64_t p) {
        const int32_t j0 = int32_t(ulist[2 * p] >> 2);
        const int32_t j1 = (2 * p + 1 < nU) ? int32_t(ulist[2 * p + 1] >> 2) : j0;
        mbar_arrive_expect_tx(bar, C::kPairBytes);
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          tma_load_3d(dst + bx * C::kRowBox, map, bar, bx * 64, j0 * kBlock, int32_t(bh));
          tma_load_3d(dst + bx * C::kRowBox + kBlock * 128, map, bar, bx * 64, j1 * kBlock, int32_t(bh));
        }
      };
      auto load_k = [&](int64_t p) {
        const int s = int(p % C::kSK);
        if (!mbar_wait_bounded(&empty_k[s], uint32_t((p / C::kSK) & 1) ^ 1u, kPollLimit)) { ok = false; return; }
        PASA_TRACE_MARK(0, p);
        load_pair(&maps.k, sm + C::kOffK + s * C::kPairBytes, &full_k[s], p);
      };
      auto load_v = [&](int64_t p) {
        const int s = int(p % C::kSV);
        if (!mbar_wait_bounded(&empty_v[s], uint32_t((p / C::kSV) & 1) ^ 1u, kPollLimit)) { ok = false; return; }
        PASA_TRACE_MARK(3, p);
        load_pair(&maps.v, sm + C::kOffV + s * C::kPairBytes, &full_v[s], p);
      };
      // K runs two steps ahead of V in issue order, so a V slot still held by
      // a P.V never holds back the K that the score MMAs need next.
      for (int64_t p = 0; p < nP + PASA_ATTN_KV_LAG && ok; ++p) {
        if (p < nP) load_k(p);
        if (ok && p >= PASA_ATTN_KV_LAG) load_v(p - PASA_ATTN_KV_LAG);
      }
      // the kc ring has memory of its own: its first groups load while the
      // last phase-1 steps still run
      int64_t issued_c = 0, issued_h = 0;
      auto load_c = [&](int64_t i) {
        const int s = int(i % C::kSC);
        if (!mbar_wait_bounded(&empty_c[s], uint32_t((i / C::kSC) & 1) ^ 1u, kPollLimit)) { ok = false; return; }
        PASA_TRACE_MARK(0, nP + i);
        unsigned char* st = sm + C::kOffRingC + s * C::kCBytes;
        mbar_arrive_expect_tx(&full_c[s], C::kCBytes);
        for (int bx = 0; bx < C::kBoxes; ++bx)
          tma_load_3d(st + bx * (kGroup * 128), &maps.kc, &full_c[s], bx * 64, int32_t(i * kGroup), int32_t(bh));
        issued_c = i + 1;
      };
      for (int64_t i = 0; i < NG2 && i < C::kSC && ok; ++i) load_c(i);
      // the vc/H ring aliases the K and V rings: all of them must be free
      for (int64_t p = (nP > C::kSK ? nP - C::kSK : 0); p < nP && ok; ++p)
        if (!mbar_wait_bounded(&empty_k[p % C::kSK], uint32_t((p / C::kSK) & 1), kPollLimit)) ok = false;
      for (int64_t p = (nP > C::kSV ? nP - C::kSV : 0); p < nP && ok; ++p)
        if (!mbar_wait_bounded(&empty_v[p % C::kSV], uint32_t((p / C::kSV) & 1), kPollLimit)) ok = false;
      // Phase 2: kc rows of every group through ring C, vc rows and H
      // through ring H, the kc loads kLagH groups ahead in issue order (ring
      // C is released by the score MMAs, which run ahead of the P.V issuer)
      for (int64_t i = 0; i < NG2 + C::kLagH && ok; ++i) {
        if (i < NG2 && i >= issued_c) {
          load_c(i);
          if (!ok) break;
        }
        const int64_t g = i - C::kLagH;
        if (g >= 0) {
          const int s = int(g % C::kSH);
          if (!mbar_wait_bounded(&empty_h[s], uint32_t((g / C::kSH) & 1) ^ 1u, kPollLimit)) { ok = false; break; }
          PASA_TRACE_MARK(3, nP + g);
          unsigned char* st = sm + C::kOffRingH + s * C::kSlotH;
          mbar_arrive_expect_tx(&full_h[s], C::kSlotH);
          for (int bx = 0; bx < C::kBoxes; ++bx) {
            tma_load_3d(st + bx * (kGroup * 128), &maps.vc, &full_h[s], bx * 64, int32_t(g * kGroup), int32_t(bh));
            tma_load_3d(st + C::kCBytes + bx * (D * 128), &maps.h, &full_h[s], bx * 64, 0, int32_t(bh * NG + g));
          }
          issued_h = g + 1;
        }
      }
      if (!ok) report(P.err);
      // drain: let this thread's last phase-2 copies land before the CTA can exit
      for (int64_t g = (issued_c > C::kSC ? issued_c - C::kSC : 0); g < issued_c; ++g)
        mbar_wait_bounded(&full_c[g % C::kSC], uint32_t((g / C::kSC) & 1), kPollLimit);
      for (int64_t g = (issued_h > C::kSH ? issued_h - C::kSH : 0); g < issued_h; ++g)
        mbar_wait_bounded(&full_h[g % C::kSH], uint32_t((g / C::kSH) & 1), kPollLimit);
    }
  } else if (warp == 1 || warp == 2) {
    // ================= MMA issuers =================
    // One thread can issue a tcgen05.mma only every ~90 cycles, slower than
    // the tensor core retires an M128 N128 K16 step, so the score MMAs
    // (warp 1) and the P.V / correction MMAs (warp 2) have an issuer each.
    if (lane == 0) {
      constexpr uint32_t idS128 = umma_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idS32 = umma_idesc_bf16(128, 32, false, false);
      constexpr uint32_t idPV = umma_idesc_bf16(128, D, false, true);
      bool ok = true;
      if (warp == 1) {
        // S(n) = Q . K^T into S buffer n & 1, which is free once the set of
        // step n-2 holds that step's scores in registers (s_free)
        ok = mbar_wait_bounded(q_full, 0, kPollLimit);
        const uint32_t q_base = smem_u32(sm + C::kOffQ);
        // Descriptors of the k-th K16 slice are the base descriptor plus the
        // slice's byte offset >> 4: the address field is the low 14 bits
        // (shared addresses < 256 KB), so the add never carries out of it.
        const uint64_t qd0 = umma_desc_sw128(q_base, 16, 1024);
        for (int64_t n = 0; n < total && ok; ++n) {
          if (n >= 2) {
            const int64_t m = n - 2;
            if (!mbar_wait_bounded(&s_free[m & 1], uint32_t((m >> 1) & 1), kPollLimit)) { ok = false; break; }
          }
          const int64_t g = n - nP;  // phase-2 group, if any
          const bool landed = (n < nP)
              ? mbar_wait_bounded(&full_k[n % C::kSK], uint32_t((n / C::kSK) & 1), kPollLimit)
              : mbar_wait_bounded(&full_c[g % C::kSC], uint32_t((g / C::kSC) & 1), kPollLimit);
          if (!landed) { ok = false; break; }
          PASA_TRACE_MARK(1, n);
          tc_fence_after();
          const uint32_t tS = tmem + C::kColS0 + 128u * uint32_t(n & 1);
          if (n < nP) {  // S = Q . [K_j0; K_j1]^T, N = 128
            const uint64_t kd0 =
                umma_desc_sw128(smem_u32(sm + C::kOffK + int(n % C::kSK) * C::kPairBytes), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t off = uint64_t(((kk / 4) * C::kRowBox + (kk % 4) * 32) >> 4);
              mma_ss(tS, qd0 + off, kd0 + off, idS128, kk > 0 ? 1u : 0u);
            }
            tc_commit(&empty_k[n % C::kSK]);
          } else {       // S = Q . kc_g^T, N = 32
            const uint64_t cd0 =
                umma_desc_sw128(smem_u32(sm + C::kOffRingC + int(g % C::kSC) * C::kCBytes), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t aoff = uint64_t(((kk / 4) * C::kRowBox + (kk % 4) * 32) >> 4);
              const uint64_t boff = uint64_t(((kk / 4) * (kGroup * 128) + (kk % 4) * 32) >> 4);
              mma_ss(tS, qd0 + aoff, cd0 + boff, idS32, kk > 0 ? 1u : 0u);
            }
            tc_commit(&empty_c[g % C::kSC]);
          }
          PASA_TRACE_MARK(28, n);
          tc_commit(&s_full[n & 1]);
        }
      } else {
        // O += P(m) . V(m) (phase 1) or P_g . vc_g + U_g . H_g (phase 2)
        for (int64_t m = 0; m < total && ok; ++m) {
          if (!mbar_wait_bounded(&p_ready[m & 1], uint32_t((m >> 1) & 1), kPollLimit)) { ok = false; break; }
          const int64_t g = m - nP;
          const bool landed = (m < nP)
              ? mbar_wait_bounded(&full_v[m % C::kSV], uint32_t((m / C::kSV) & 1), kPollLimit)
              : mbar_wait_bounded(&full_h[g % C::kSH], uint32_t((g / C::kSH) & 1), kPollLimit);
          if (!landed) { ok = false; break; }
          PASA_TRACE_MARK(2, m);
          tc_fence_after();
          const uint32_t tP = tmem + C::kColP + 64u * uint32_t(m & 1);
          if (m < nP) {  // K = 128: the two key blocks of the step
            const uint64_t vd0 =
                umma_desc_sw128(smem_u32(sm + C::kOffV + int(m % C::kSV) * C::kPairBytes), C::kRowBox, 1024);
#pragma unroll
            for (int kk = 0; kk < 2 * kBlock / 16; ++kk)
              mma_ts(tmem + C::kColO, tP + kk * 8, vd0 + uint64_t((kk * 2048) >> 4), idPV,
                     (m > 0 || kk > 0) ? 1u : 0u);
            tc_commit(&empty_v[m % C::kSV]);
          } else {
            const uint32_t st = smem_u32(sm + C::kOffRingH + int(g % C::kSH) * C::kSlotH);
            const uint32_t tU = tmem + C::kColS0 + 128u * uint32_t(m & 1) + C::kColU;
            const uint64_t vcd0 = umma_desc_sw128(st, C::kCBytes / C::kBoxes, 1024);
            const uint64_t hd0 = umma_desc_sw128(st + C::kCBytes, C::kHBytes / C::kBoxes, 1024);
#pragma unroll
            for (int kk = 0; kk < kGroup / 16; ++kk)
              mma_ts(tmem + C::kColO, tP + kk * 8, vcd0 + uint64_t((kk * 2048) >> 4), idPV, 1u);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              mma_ts(tmem + C::kColO, tU + kk * 8, hd0 + uint64_t((kk * 2048) >> 4), idPV, 1u);
            tc_commit(&empty_h[g % C::kSH]);
          }
          tc_commit(&o_done[m & 1]);
          PASA_TRACE_MARK(29, m);
        }
      }
      if (!ok) report(P.err);
    }
    __syncwarp();
  } else {
    // ================= softmax sets (warps 3-6: set 0, warps 7-10: set 1) =================
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may access
    const int set = (warp - 3) >> 2;           // this warp's set: steps n with n % 2 == set
    const int r = quad * 32 + lane;            // tile row == TMEM lane
    const int half = r >> 6;                   // 0: block A, 1: block B
    const bool live = (half == 0) || hasB;     // uniform per lane quadrant
    const int xbar = 1 + quad;                 // both sets of the quadrant (final combine)
    const int hand_to = 5 + quad * 2 + set;          // barrier this set arrives on when handing over
    const int hand_from = 5 + quad * 2 + (set ^ 1);  // barrier this set waits on
    float* hand_out = hand + set * 2 * kRowsPerTile;
    const float* hand_in = hand + (set ^ 1) * 2 * kRowsPerTile;
    const uint32_t lane_base = uint32_t(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + C::kColS0 + 128u * uint32_t(set);  // this set's S buffer
    const uint32_t tP = tmem + lane_base + C::kColP + 64u * uint32_t(set);    // this set's P region
    const uint32_t tU = tmem + lane_base + C::kColS0 + 128u * uint32_t(set) + C::kColU;  // U (phase 2)
    const float scale32 = P.scale;
    const float sm_scale = scale32 * kLog2e;
    const int64_t last_len = P.T - (NT - 1) * kBlock;
    constexpr int DH = D / 2;                  // output columns this set stores
    float m_true = -INFINITY, m_used = -INFINITY, l1 = 0.f, gl = 0.f;
    float m_applied = -INFINITY;  // the maximum this thread's l1 is scaled to
    bool ok = true;
    uint32_t xslot = 0;
    // combine one value per row across the two sets (fixed order: set 0 + set 1)
    auto row_reduce = [&](float v, bool is_max) -> float {
      xch[(xslot * 2 + set) * kRowsPerTile + r] = v;
      named_bar_sync(xbar, 64);
      const float a = xch[(xslot * 2) * kRowsPerTile + r], b = xch[(xslot * 2 + 1) * kRowsPerTile + r];
      xslot ^= 1u;
      return is_max ? fmaxf(a, b) : a + b;
    };
    auto wait_bar = [&](uint64_t* bar, int64_t k) {  // k-th completion of `bar`
      if (ok && !mbar_wait_bounded(bar, uint32_t(k & 1), kPollLimit)) ok = false;
    };
    // O holds the steps <= n-1 once their MMAs completed; one thread owns the
    // row, so it rescales all D columns
    // A parity wait for the k-th completion of a barrier is only sound once
    // its (k-1)-th completion has happened: with the barrier two phases
    // behind, the parity already matches and the wait returns at once.  This
    // set follows o_done[n & 1] step by step (its P-region waits), but not
    // o_done[(n - 1) & 1]; so it first waits for step n-2 on its own barrier,
    // after which step n-3 (issued earlier, completed in order) has completed
    // too, and only then for step n-1 on the other barrier.  (Without the
    // first wait, a rescale at step 3 could start while the P.V of step 0 was
    // still accumulating into O, and corrupt those rows.)
    auto rescale_o = [&](int64_t n, float alpha) {
      if (n >= 2) wait_bar(&o_done[n & 1], (n - 2) >> 1);
      if (n >= 1) { wait_bar(&o_done[(n - 1) & 1], (n - 1) >> 1); tc_fence_after(); }
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
    };
    // running maxima across steps: receive those after step n-1, update with
    // this step's maximum mx (log2 units), pass them on to step n+1
    auto advance_max = [&](int64_t n, float mx, float& m_prev) {
      if (n >= 1) {
        named_bar_sync(hand_from, 64);
        tc_fence_after();  // the handing set's TMEM loads of step n-1 precede this point
        m_used = hand_in[r];
        m_true = hand_in[kRowsPerTile + r];
      }
      m_prev = m_used;
      m_true = fmaxf(m_true, mx);
      if (mx > m_used + kRescaleThresh) m_used = mx;
      if (n + 1 < total) {
        hand_out[r] = m_used;
        hand_out[kRowsPerTile + r] = m_true;
        named_bar_arrive(hand_to, 64);
      }
    };
    wait_bar(q_full, 0);  // phase 2 reads this tile's Q rows from shared memory
    // After a failed wait (ok false) the loop keeps going without waiting, so
    // every warp still takes part in every named barrier and none is stranded.
    for (int64_t n = set; n < total; n += 2) {
      wait_bar(&s_full[set], n >> 1);
      tc_fence_after();
      if (lane == 0) PASA_TRACE_MARK(4 + (warp - 3), n);
      if (n < nP) {
        // ---------------- Phase 1: a pair of exact blocks ----------------
        const uint32_t e0 = ulist[2 * n];
        const uint32_t e1 = (2 * n + 1 < nU) ? uint32_t(ulist[2 * n + 1]) : 0u;  // lone last block: no bits
        const bool act0 = live && ((e0 >> half) & 1u);  // uniform per warp
        const bool act1 = live && ((e1 >> half) & 1u);
        const bool last0 = int(e0 >> 2) == int(NT) - 1, last1 = int(e1 >> 2) == int(NT) - 1;
        // scores of one block (64 columns), with key rows >= T masked (:178);
        // only the last block has them
        uint32_t sa[32], sb[32];
        auto load_block = [&](int blk, bool last) {
          tmem_ld32(tS + 64 * blk, sa);
          tmem_ld32(tS + 64 * blk + 32, sb);
          tmem_wait_ld();
          if (last) { mask_tail<32>(sa, int(last_len)); mask_tail<32>(sb, int(last_len) - 32); }
        };
        auto free_s = [&]() {  // the step's last read of its S buffer is done
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[set]);
        };
        // pass 1: the row maximum over the step's active blocks
        float mx = -INFINITY;
        if (act0) { load_block(0, last0); mx = fmaxf(max_tree32(sa), max_tree32(sb)); }
        if (act1) { load_block(1, last1); mx = fmax3(mx, max_tree32(sa), max_tree32(sb)); }
        if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(24, n);
        mx *= sm_scale;  // max commutes with the positive scale
        float m_prev = m_used;
        if (live) advance_max(n, mx, m_prev);  // uniform per lane quadrant
        if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(25, n);
        const bool need = (m_used != m_prev) && (m_prev != -INFINITY);
        if (__any_sync(0xffffffffu, need)) rescale_o(n, need ? fast_exp2(m_prev - m_used) : 1.0f);
        if (m_applied != m_used) {
          if (m_applied != -INFINITY) l1 *= fast_exp2(m_applied - m_used);
          m_applied = m_used;
        }
        // pass 2: probabilities of both blocks into registers (block 0: keys
        // 0-63 -> P columns 0-31, block 1 -> columns 32-63).  The S buffer is
        // free after the last load, before any wait, and the exponentials run
        // while the P.V of step n-2 still reads this set's P region.
        const float negm = -m_used;
        uint32_t p0a[16], p0b[16], p1a[16], p1b[16];
        if (!act0 && !act1) free_s();
        if (act0) {
          load_block(0, last0);
          if (!act1) free_s();
          l1 += exp2_pack<32>(sa, sm_scale, negm, p0a);
          l1 += exp2_pack<32>(sb, sm_scale, negm, p0b);
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) { p0a[c] = 0u; p0b[c] = 0u; }
        }
        if (act1) {  // block 1 in two halves: block 0's P is held meanwhile
          tmem_ld32(tS + 64, sa);
          tmem_wait_ld();
          if (last1) mask_tail<32>(sa, int(last_len));
          l1 += exp2_pack<32>(sa, sm_scale, negm, p1a);
          tmem_ld32(tS + 96, sb);
          tmem_wait_ld();
          free_s();
          if (last1) mask_tail<32>(sb, int(last_len) - 32);
          l1 += exp2_pack<32>(sb, sm_scale, negm, p1b);
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) { p1a[c] = 0u; p1b[c] = 0u; }
        }
        // this set's P region was last read by the P.V of step n-2
        if (n >= 2) { wait_bar(&o_done[n & 1], (n - 2) >> 1); tc_fence_after(); }
        if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(26, n);
        tmem_st16(tP, p0a);
        tmem_st16(tP + 16, p0b);
        tmem_st16(tP + 32, p1a);
        tmem_st16(tP + 48, p1b);
        if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(27, n);
        tmem_wait_st();
      } else {
        // ---------------- Phase 2: group g ----------------
        const int64_t g = n - nP;
        uint32_t sv[kGroup];
        if (live) tmem_ld32(tS, sv);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[set]);
        uint32_t pk[kGroup / 2];
        float w = 0.f;
        if (live) {  // uniform per lane quadrant
          // columns of selected blocks or of blocks >= NT are masked (:228)
          const int jb0 = int(g) * kGroup;  // NT <= kMaxNT fits in int
          const int lim = int(NT) - jb0;
          const uint32_t dead = maskw[half * kMaxNG + g] |
                                (lim >= kGroup ? 0u : (lim <= 0 ? ~0u : ~((1u << lim) - 1u)));
#pragma unroll
          for (int c = 0; c < kGroup; ++c)
            if ((dead >> c) & 1u) sv[c] = __float_as_uint(-INFINITY);
          float mx = max_tree32(sv);
          mx = (mx == -INFINITY) ? mx : mx * sm_scale;
          float m_prev = m_used;
          advance_max(n, mx, m_prev);
          if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(25, n);
          const float m_true_g = m_true;  // the reference's m at this group (:237, :243)
          const bool grow = m_used != m_prev;  // m_used is finite for live rows here
          if (__any_sync(0xffffffffu, grow)) rescale_o(n, grow ? fast_exp2(m_prev - m_used) : 1.0f);
          if (m_applied != m_used) { l1 *= fast_exp2(m_applied - m_used); m_applied = m_used; }
          float p[kGroup];
          const float negm = -m_used;
          float2 acc = make_float2(0.f, 0.f);  // even / odd column sums
          {
            const float2 sc2 = make_float2(sm_scale, sm_scale), nm2 = make_float2(negm, negm);
#pragma unroll
            for (int c = 0; c < kGroup; c += 2) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])), sc2, nm2);
              p[c] = exp2_ftz(x.x);
              p[c + 1] = exp2_ftz(x.y);
              acc = __fadd2_rn(acc, make_float2(p[c], p[c + 1]));
            }
          }
          const float psum = acc.x + acc.y;
          float extra = 0.f;
          // bit of the ragged last block's column, if it is in this group
          // (a bit test, not an index: p[] must stay in registers); the
          // branch is uniform and taken in one group at most
          const uint32_t lastbit = (lim >= 1 && lim <= kGroup) ? (1u << (lim - 1)) : 0u;
          if (lastbit) {
#pragma unroll
            for (int c = 0; c < kGroup; ++c) extra += ((lastbit >> c) & 1u) ? p[c] : 0.f;
          }
          // the ragged last block has its own length (:220)
          const float wsum = psum * float(kBlock) + extra * float(last_len - kBlock);
#pragma unroll
          for (int c = 0; c < kGroup; c += 2) pk[c / 2] = pack_bf16x2(p[c], p[c + 1]);
          gl += wsum * fast_exp2(m_used - m_true_g);
          w = psum * scale32;  // :253
        } else {
#pragma unroll
          for (int c = 0; c < kGroup / 2; ++c) pk[c] = 0u;
        }
        // P region and U slot were last read by the P.V of step n-2.  U goes to
        // columns 64-127 of this set's own S buffer: the group score MMAs
        // write only columns 0-31, and this set read its last full-width
        // scores there at step n-2.  (The other set's buffer would not do: at
        // the first group that set may still be reading the full-width
        // scores of step n-1 for its probabilities.)
        // U = bf16(q * bf16(w)) over all D columns (one packed bf16 multiply
        // per column pair), from this row of Q in shared memory, built before
        // the wait so that it overlaps the P.V of n-2
        uint32_t u[C::kBoxes][32];
        const __nv_bfloat162 w2 = __float2bfloat162_rn(w);
#pragma unroll
        for (int bx = 0; bx < C::kBoxes; ++bx) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 qv = *reinterpret_cast<const uint4*>(sm + C::kOffQ + bx * C::kRowBox + r * 128 +
                                                            ((c ^ (r & 7)) << 4));
            const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
            for (int x = 0; x < 4; ++x) {
              const __nv_bfloat162 prod = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&qw[x]), w2);
              u[bx][c * 4 + x] = *reinterpret_cast<const uint32_t*>(&prod);
            }
          }
        }
        if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(24, n);
        if (n >= 2) { wait_bar(&o_done[n & 1], (n - 2) >> 1); tc_fence_after(); }
        if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(26, n);
        tmem_st16(tP, pk);
#pragma unroll
        for (int bx = 0; bx < C::kBoxes; ++bx) tmem_st32(tU + bx * 32, u[bx]);
        tmem_wait_st();
        if ((warp & 3) == 3 && lane == 0) PASA_TRACE_MARK(27, n);
      }
      // hand P (and U) of step n to the P.V issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) PASA_TRACE_MARK(12 + (warp - 3), n);
      if (lane == 0) mbar_arrive(&p_ready[set]);
    }

    // ---------------- Final: o = O / (l + g_l) ----------------
    // Each set ends with the maxima after the last step it took; the maxima
    // only grow, so the larger pair is the final one.
    if (live) {
      m_used = row_reduce(m_used, true);
      m_true = row_reduce(m_true, true);
      if (m_applied != m_used && m_applied != -INFINITY) l1 *= fast_exp2(m_applied - m_used);
    }
    if (total >= 1) {
      const int64_t m = total - 1;
      wait_bar(&o_done[m & 1], m >> 1);
      tc_fence_after();
    }
    const int64_t blk = (half == 0) ? blkA : blkB;
    const int64_t t = blk * kBlock + (r & 63);
    const bool wok = __all_sync(0xffffffffu, ok);
    if (live) {
      const float l_tot = row_reduce(l1, false);
      const float g_tot = row_reduce(gl, false);
      if (wok) {  // warp-uniform: tcgen05.ld is warp-collective
        const bool store = t < P.T && blk >= P.blk_lo && blk < P.blk_hi;
        const float denom = l_tot + g_tot * fast_exp2(m_true - m_used);
        const float inv = 1.0f / denom;
        __nv_bfloat16* orow;
        if (P.o_npeer > 0) {
          const int64_t ts = store ? t : 0;
          const int64_t dst = ts / P.o_tokens;
          orow = P.o_peer[dst] + ((ts - dst * P.o_tokens) * P.o_heads_total + P.o_head0 + bh) * D + set * DH;
        } else {
          const int64_t orow_idx = P.o_heads > 0
                                       ? ((bh / P.o_heads) * P.T + t) * P.o_heads + bh % P.o_heads
                                       : bh * P.T + t;
          orow = P.o + orow_idx * D + set * DH;
        }
#pragma unroll
        for (int c0 = 0; c0 < DH; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tmem + lane_base + C::kColO + set * DH + c0, v);
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
        if (P.o_npeer > 0) __threadfence_system();  // peer stores done before the kernel ends
      }
    }
    if (!ok) report(P.err);
    if (warp == 3 && lane == 0) PASA_TRACE_CTL(2);
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0) PASA_TRACE_CTL(3);
#ifdef PASA_TRACE
  if (tid == 0) {
    const unsigned long long idx = (unsigned long long)blockIdx.y * gridDim.x + blockIdx.x;
    if (idx < kTraceCtas) {
      unsigned int smid;
      asm volatile("mov.u32 %0, %smid;" : "=r"(smid));
      g_pasa_trace_cta_rec[idx][0] = pasa_t0_ns;
      g_pasa_trace_cta_rec[idx][1] = global_ns();
      g_pasa_trace_cta_rec[idx][2] = clock64() - pasa_t0_clk;
      g_pasa_trace_cta_rec[idx][3] = ((unsigned long long)smid << 32) | (unsigned long long)nU;
    }
  }
#endif
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
// The driver's tensor-map encoder, looked up once (a function-local static:
// its initialisation is thread-safe, so concurrent first calls from several
// host threads are fine).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return nullptr;
  }();
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
                        float scale, void* o, uint32_t* err, int dense, int64_t o_heads,
                        const OutScatter& sc, int64_t blk_lo, int64_t blk_hi) {
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
  p.o = static_cast<__nv_bfloat16*>(o); p.sel_mask = mask; p.err = err; p.dense = dense;
  p.o_heads = o_heads;
  p.o_peer = reinterpret_cast<__nv_bfloat16* const*>(sc.peer);
  p.o_npeer = sc.npeer;
  p.o_tokens = sc.tokens;
  p.o_heads_total = sc.heads_total;
  p.o_head0 = sc.head0;
  // the pairs that hold blocks [blk_lo, blk_hi)
  if (blk_hi < 0) blk_hi = NT;
  if (blk_lo < 0 || blk_lo >= blk_hi || blk_hi > NT) return cudaErrorInvalidValue;
  p.pair0 = blk_lo / 2;
  p.blk_lo = blk_lo;
  p.blk_hi = blk_hi;
  const int64_t npairs = cdiv(blk_hi, 2) - p.pair0;
  auto kern = attn_tc_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  dim3 grid{unsigned(npairs), unsigned(BH), 1u};
  kern<<<grid, kThreads, C::kSmemBytes, st>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace tc

cudaError_t launch_attn_tc(cudaStream_t st, int D, const void* q, const void* k, const void* v, const void* kc,
                           const void* vc, const void* hg, const uint32_t* mask, int64_t BH, int64_t T_len,
                           int64_t /*NS*/, float scale, void* o, uint32_t* err, int dense, int64_t o_heads,
                           const OutScatter& sc, int64_t blk_lo, int64_t blk_hi) {
  if (D == 64)
    return tc::launch_tc_t<64>(st, q, k, v, kc, vc, hg, mask, BH, T_len, scale, o, err, dense, o_heads, sc, blk_lo,
                               blk_hi);
  return tc::launch_tc_t<128>(st, q, k, v, kc, vc, hg, mask, BH, T_len, scale, o, err, dense, o_heads, sc, blk_lo,
                              blk_hi);
}

}  // namespace pasa

#ifdef PASA_TRACE
extern "C" PASA_API int pasa_trace_read(void* host_dst, size_t bytes) {
  return cudaMemcpyFromSymbol(host_dst, pasa::tc::g_pasa_trace, bytes) == cudaSuccess ? 0 : PASA_ERR_CUDA;
}
extern "C" PASA_API int pasa_trace_ctl_read(void* host_dst, size_t bytes) {
  return cudaMemcpyFromSymbol(host_dst, pasa::tc::g_pasa_trace_ctl, bytes) == cudaSuccess ? 0 : PASA_ERR_CUDA;
}
extern "C" PASA_API int pasa_trace_cta_read(void* host_dst, size_t bytes) {
  return cudaMemcpyFromSymbol(host_dst, pasa::tc::g_pasa_trace_cta_rec, bytes) == cudaSuccess ? 0 : PASA_ERR_CUDA;
}
extern "C" PASA_API int pasa_trace_select(unsigned int x, unsigned int y) {
  const unsigned int v[2] = {x, y};
  return cudaMemcpyToSymbol(pasa::tc::g_pasa_trace_cta, v, sizeof(v)) == cudaSuccess ? 0 : PASA_ERR_CUDA;
}
#endif
