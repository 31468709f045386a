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
//     two blocks' selected key blocks in ascending order; rows whose block
//     did not select the key block get P = 0 and skip the exponentials.
//     Phase 2 (shared by both blocks) walks the 32-block groups with each
//     half's own selection bits.
//   * warp 0: TMA producer (Q once, then K/V blocks or kc/vc/H_g of a group
//     per step through a ring of stages); warp 1: TMEM owner and MMA issuer
//     (one thread); warps 2-5: softmax, one thread per query row (TMEM lane).
//   * TMEM: O accumulator (D cols), two S/P buffers (64 cols; P is written
//     back as packed bf16 over S), two U buffers (D/2 cols).  The first-order
//     term is an MMA: U = bf16(w_t * q_t) (A operand from TMEM, w_t = scale *
//     sum of the group's probabilities) times H_g (B from shared memory),
//     accumulated straight into O.
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

constexpr int kThreads = 192;          // 6 warps
constexpr int kRowsPerTile = 128;      // two query blocks
constexpr float kRescaleThresh = 8.0f; // log2 units
constexpr int kMaxNT = 4096;           // union list capacity (entries)
constexpr int kMaxNG = kMaxNT / kGroup;
constexpr uint64_t kPollLimit = 2000000000ull;  // ns a barrier wait may take before giving up

template <int D>
struct Cfg {
  static constexpr int kBoxes = D / 64;                 // 64-column TMA boxes per row
  static constexpr int kQBytes = kRowsPerTile * D * 2;
  static constexpr int kKVBytes = kBlock * D * 2;       // one K (or V) block
  static constexpr int kCBytes = kGroup * D * 2;        // kc (or vc) rows of one group
  static constexpr int kHBytes = D * D * 2;
  static constexpr int kStageBytes = (2 * kKVBytes > 2 * kCBytes + kHBytes) ? 2 * kKVBytes : 2 * kCBytes + kHBytes;
  static constexpr int kStages = (D == 128) ? 3 : 6;
  static constexpr uint32_t kTxP1 = 2 * kKVBytes;
  static constexpr uint32_t kTxP2 = 2 * kCBytes + kHBytes;
  // TMEM columns
  static constexpr uint32_t kColO = 0;
  static constexpr uint32_t kColS0 = 128;
  static constexpr uint32_t kColU0 = 256;
  static constexpr uint32_t kTmemCols = 512;
  // shared memory carve-up (offsets from a 1024-aligned base)
  static constexpr int kOffQ = 0;
  static constexpr int kOffStages = kQBytes;
  static constexpr int kOffUnion = kOffStages + kStages * kStageBytes;
  static constexpr int kOffMask = kOffUnion + kMaxNT * 4;
  static constexpr int kOffBar = kOffMask + 2 * kMaxNG * 4;
  static constexpr int kNumBars = 2 * kStages + 1 + 2 + 2 + 2;
  static constexpr int kOffSlot = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffSlot + 16 + 1024;  // + alignment slack
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

__device__ __forceinline__ void report(uint32_t* err) {
  if (err) atomicOr(err, PASA_DEVERR_WAIT_TIMEOUT);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const __grid_constant__ Maps maps, Params P) {
  using C = Cfg<D>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* ulist = reinterpret_cast<uint32_t*>(sm + C::kOffUnion);
  uint32_t* maskw = reinterpret_cast<uint32_t*>(sm + C::kOffMask);  // [2][kMaxNG]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kStages;
  uint64_t* q_full = bars + 2 * C::kStages;
  uint64_t* s_full = q_full + 1;   // [2]
  uint64_t* p_ready = s_full + 2;  // [2]
  uint64_t* o_done = p_ready + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::kOffSlot);
  __shared__ uint32_t s_nu;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t pair = blockIdx.x, bh = blockIdx.y;
  const int64_t NT = P.NT, NG = P.NG;
  const int64_t blkA = 2 * pair, blkB = 2 * pair + 1;
  const bool hasB = blkB < NT;

  // ---- set-up: barriers, TMEM, selection bits, union list -------------
  if (tid == 0) {
    for (int s = 0; s < C::kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(q_full, 1);
    for (int b = 0; b < 2; ++b) { mbar_init(&s_full[b], 1); mbar_init(&p_ready[b], 4); mbar_init(&o_done[b], 1); }
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
  if (warp == 0) {  // union of the two selections, ascending block index
    uint32_t base = 0;
    for (int64_t w0 = 0; w0 < NG; w0 += 32) {
      const int64_t w = w0 + lane;
      const uint32_t ma = (w < NG) ? maskw[w] : 0u, mb = (w < NG) ? maskw[kMaxNG + w] : 0u;
      const uint32_t u = ma | mb;
      const uint32_t cnt = __popc(u);
      uint32_t incl = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      uint32_t pos = base + incl - cnt;
      uint32_t rem = u;
      while (rem) {
        const int b = __ffs(rem) - 1;
        rem &= rem - 1;
        const uint32_t j = uint32_t(w * 32 + b);
        ulist[pos++] = (j << 2) | ((ma >> b) & 1u) | (((mb >> b) & 1u) << 1);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_nu = base;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t nU = s_nu;
  const int64_t total = nU + NG;

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      bool ok = true;
      int64_t issued = 0;
      const int32_t row0 = int32_t(pair * kRowsPerTile);
      mbar_arrive_expect_tx(q_full, C::kQBytes);
      for (int bx = 0; bx < C::kBoxes; ++bx)
        tma_load_3d(sm + C::kOffQ + bx * (kRowsPerTile * 128), &maps.q, q_full, bx * 64, row0, int32_t(bh));
      for (int64_t n = 0; n < total && ok; ++n) {
        const int s = int(n % C::kStages);
        const uint32_t ph = uint32_t((n / C::kStages) & 1);
        if (!mbar_wait_bounded(&empty[s], ph ^ 1u, kPollLimit)) { ok = false; break; }
        unsigned char* st = sm + C::kOffStages + s * C::kStageBytes;
        if (n < nU) {
          const int32_t j = int32_t(ulist[n] >> 2);
          mbar_arrive_expect_tx(&full[s], C::kTxP1);
          for (int bx = 0; bx < C::kBoxes; ++bx) {
            tma_load_3d(st + bx * (kBlock * 128), &maps.k, &full[s], bx * 64, j * kBlock, int32_t(bh));
            tma_load_3d(st + C::kKVBytes + bx * (kBlock * 128), &maps.v, &full[s], bx * 64, j * kBlock, int32_t(bh));
          }
        } else {
          const int32_t g = int32_t(n - nU);
          mbar_arrive_expect_tx(&full[s], C::kTxP2);
          for (int bx = 0; bx < C::kBoxes; ++bx) {
            tma_load_3d(st + bx * (kGroup * 128), &maps.kc, &full[s], bx * 64, g * kGroup, int32_t(bh));
            tma_load_3d(st + C::kCBytes + bx * (kGroup * 128), &maps.vc, &full[s], bx * 64, g * kGroup, int32_t(bh));
            tma_load_3d(st + 2 * C::kCBytes + bx * (D * 128), &maps.h, &full[s], bx * 64, 0,
                        int32_t(bh * NG + g));
          }
        }
        issued = n + 1;
      }
      if (!ok) report(P.err);
      // drain: let this thread's last copies land before the CTA can exit
      const int64_t first = issued > C::kStages ? issued - C::kStages : 0;
      for (int64_t n = first; n < issued; ++n) {
        const int s = int(n % C::kStages);
        mbar_wait_bounded(&full[s], uint32_t((n / C::kStages) & 1), kPollLimit);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t idS64 = umma_idesc_bf16(128, 64, false, false);
      constexpr uint32_t idS32 = umma_idesc_bf16(128, 32, false, false);
      constexpr uint32_t idPV = umma_idesc_bf16(128, D, false, true);
      const uint32_t qaddr = smem_u32(sm + C::kOffQ);
      bool ok = mbar_wait_bounded(q_full, 0, kPollLimit);

      auto issue_pv = [&](int64_t m) -> bool {
        const int b = int(m & 1);
        if (!mbar_wait_bounded(&p_ready[b], uint32_t((m >> 1) & 1), kPollLimit)) return false;
        tc_fence_after();
        const int s = int(m % C::kStages);
        const uint32_t st = smem_u32(sm + C::kOffStages + s * C::kStageBytes);
        const uint32_t tS = tmem + C::kColS0 + 64u * b;
        const uint32_t tU = tmem + C::kColU0 + 64u * b;
        if (m < nU) {
#pragma unroll
          for (int kk = 0; kk < kBlock / 16; ++kk) {
            const uint64_t bd = umma_desc_sw128(st + C::kKVBytes + kk * 2048, C::kKVBytes / C::kBoxes, 1024);
            mma_ts(tmem + C::kColO, tS + kk * 8, bd, idPV, (m > 0 || kk > 0) ? 1u : 0u);
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < kGroup / 16; ++kk) {
            const uint64_t bd = umma_desc_sw128(st + C::kCBytes + kk * 2048, C::kCBytes / C::kBoxes, 1024);
            mma_ts(tmem + C::kColO, tS + kk * 8, bd, idPV, 1u);
          }
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t bd = umma_desc_sw128(st + 2 * C::kCBytes + kk * 2048, C::kHBytes / C::kBoxes, 1024);
            mma_ts(tmem + C::kColO, tU + kk * 8, bd, idPV, 1u);
          }
        }
        tc_commit(&empty[s]);
        tc_commit(&o_done[b]);
        return true;
      };

      for (int64_t n = 0; n < total && ok; ++n) {
        const int s = int(n % C::kStages);
        const uint32_t ph = uint32_t((n / C::kStages) & 1);
        const int b = int(n & 1);
        if (!mbar_wait_bounded(&full[s], ph, kPollLimit)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = smem_u32(sm + C::kOffStages + s * C::kStageBytes);
        const uint32_t tS = tmem + C::kColS0 + 64u * b;
        if (n < nU) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int bx = kk / 4, ko = (kk % 4) * 32;
            const uint64_t ad = umma_desc_sw128(qaddr + bx * (kRowsPerTile * 128) + ko, 16, 1024);
            const uint64_t bd = umma_desc_sw128(st + bx * (kBlock * 128) + ko, 16, 1024);
            mma_ss(tS, ad, bd, idS64, kk > 0 ? 1u : 0u);
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int bx = kk / 4, ko = (kk % 4) * 32;
            const uint64_t ad = umma_desc_sw128(qaddr + bx * (kRowsPerTile * 128) + ko, 16, 1024);
            const uint64_t bd = umma_desc_sw128(st + bx * (kGroup * 128) + ko, 16, 1024);
            mma_ss(tS, ad, bd, idS32, kk > 0 ? 1u : 0u);
          }
        }
        tc_commit(&s_full[b]);
        if (n >= 1 && !issue_pv(n - 1)) { ok = false; break; }
      }
      if (ok && total >= 1) ok = issue_pv(total - 1);
      if (!ok) report(P.err);
    }
    __syncwarp();
  } else {
    // ================= softmax / correction (warps 2..5) =================
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;            // tile row == TMEM lane
    const int half = r >> 6;                   // 0: block A, 1: block B
    const bool live = (half == 0) || hasB;
    const uint32_t lane_base = uint32_t(quad * 32) << 16;
    const float scale32 = P.scale;
    const float sm_scale = scale32 * kLog2e;
    const int64_t last_len = P.T - (NT - 1) * kBlock;
    float m_true = -INFINITY, m_used = -INFINITY, l1 = 0.f, gl = 0.f;
    uint32_t qpk[D / 2];  // this row of Q as packed bf16 pairs (phase 2)
    bool ok = mbar_wait_bounded(q_full, 0, kPollLimit);

    auto rescale_o = [&](int64_t n, float alpha) -> bool {
      // O is consistent once the MMAs of step n-1 have completed
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

    for (int64_t n = 0; n < total && ok; ++n) {
      const int b = int(n & 1);
      if (!mbar_wait_bounded(&s_full[b], uint32_t((n >> 1) & 1), kPollLimit)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + C::kColS0 + 64u * b;
      if (n < nU) {
        // ---------------- Phase 1: exact block ----------------
        const uint32_t e = ulist[n];
        const int64_t j = e >> 2;
        const bool active = live && ((e >> half) & 1u);
        uint32_t pk[32];
        if (active) {
          uint32_t sv[64];
          tmem_ld16(tS + 0, *reinterpret_cast<uint32_t(*)[16]>(&sv[0]));
          tmem_ld16(tS + 16, *reinterpret_cast<uint32_t(*)[16]>(&sv[16]));
          tmem_ld16(tS + 32, *reinterpret_cast<uint32_t(*)[16]>(&sv[32]));
          tmem_ld16(tS + 48, *reinterpret_cast<uint32_t(*)[16]>(&sv[48]));
          tmem_wait_ld();
          const int nvalid = (j == NT - 1) ? int(last_len) : kBlock;  // key rows >= T masked (:178)
          float s[64];
          float mx = -INFINITY;
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            s[c] = (c < nvalid) ? __uint_as_float(sv[c]) * sm_scale : -INFINITY;
            mx = fmaxf(mx, s[c]);
          }
          m_true = fmaxf(m_true, mx);
          const bool grow = mx > m_used + kRescaleThresh;
          const bool need = grow && (m_used != -INFINITY);
          const float alpha = need ? fast_exp2(m_used - mx) : 1.0f;
          if (__any_sync(0xffffffffu, need)) {  // tcgen05.ld/st are warp-collective
            if (!rescale_o(n, alpha)) ok = false;
          }
          l1 *= alpha;
          if (grow) m_used = mx;
          float sum = 0.f;
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const float p0 = fast_exp2(s[c] - m_used), p1 = fast_exp2(s[c + 1] - m_used);
            sum += p0 + p1;
            pk[c / 2] = pack_bf16x2(p0, p1);
          }
          l1 += sum;
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) pk[c] = 0u;
        }
        tmem_st16(tS + 0, *reinterpret_cast<uint32_t(*)[16]>(&pk[0]));
        tmem_st16(tS + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[16]));
        tmem_wait_st();
      } else {
        // ---------------- Phase 2: group g ----------------
        const int64_t g = n - nU;
        if (g == 0) {  // this row of Q, read once from the swizzled tile
          const unsigned char* qrow = sm + C::kOffQ;
#pragma unroll
          for (int bx = 0; bx < C::kBoxes; ++bx)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 v = *reinterpret_cast<const uint4*>(qrow + bx * (kRowsPerTile * 128) + r * 128 +
                                                             ((c ^ (r & 7)) << 4));
              qpk[bx * 32 + c * 4 + 0] = v.x;
              qpk[bx * 32 + c * 4 + 1] = v.y;
              qpk[bx * 32 + c * 4 + 2] = v.z;
              qpk[bx * 32 + c * 4 + 3] = v.w;
            }
        }
        uint32_t pk[16];
        uint32_t upk[D / 2];
        if (live) {
          uint32_t sv[32];
          tmem_ld16(tS + 0, *reinterpret_cast<uint32_t(*)[16]>(&sv[0]));
          tmem_ld16(tS + 16, *reinterpret_cast<uint32_t(*)[16]>(&sv[16]));
          tmem_wait_ld();
          const uint32_t word = maskw[half * kMaxNG + g];
          float a[32];
          float mx = -INFINITY;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int64_t jb = g * kGroup + c;
            const bool valid = (jb < NT) && !((word >> c) & 1u);  // :228
            a[c] = valid ? __uint_as_float(sv[c]) * sm_scale : -INFINITY;
            mx = fmaxf(mx, a[c]);
          }
          const float m_true_new = fmaxf(m_true, mx);
          const bool grow = mx > m_used + kRescaleThresh;  // m_used is finite for live rows here
          const float alpha = grow ? fast_exp2(m_used - mx) : 1.0f;
          if (__any_sync(0xffffffffu, grow)) {
            if (!rescale_o(n, alpha)) ok = false;
          }
          l1 *= alpha;
          if (grow) m_used = mx;
          float psum = 0.f, wsum = 0.f;
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float p0 = fast_exp2(a[c] - m_used), p1 = fast_exp2(a[c + 1] - m_used);
            const int64_t jb = g * kGroup + c;
            const float len0 = (jb == NT - 1) ? float(last_len) : float(kBlock);
            const float len1 = (jb + 1 == NT - 1) ? float(last_len) : float(kBlock);
            psum += p0 + p1;
            wsum += p0 * len0 + p1 * len1;
            pk[c / 2] = pack_bf16x2(p0, p1);
          }
          // the reference's probabilities use the exact running max (:237, :243)
          gl += wsum * fast_exp2(m_used - m_true_new);
          m_true = m_true_new;
          const float w = psum * scale32;  // :253
#pragma unroll
          for (int x = 0; x < D / 2; ++x) {
            __nv_bfloat162 q2 = *reinterpret_cast<const __nv_bfloat162*>(&qpk[x]);
            const float2 qf = __bfloat1622float2(q2);
            upk[x] = pack_bf16x2(qf.x * w, qf.y * w);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) pk[c] = 0u;
#pragma unroll
          for (int x = 0; x < D / 2; ++x) upk[x] = 0u;
        }
        tmem_st16(tS + 0, pk);
        const uint32_t tU = tmem + lane_base + C::kColU0 + 64u * b;
#pragma unroll
        for (int c0 = 0; c0 < D / 2; c0 += 16)
          tmem_st16(tU + c0, *reinterpret_cast<uint32_t(*)[16]>(&upk[c0]));
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[b]);
    }

    // ---------------- Final: o = O / (l + g_l) ----------------
    if (ok && total >= 1) {
      const int64_t m = total - 1;
      ok = mbar_wait_bounded(&o_done[m & 1], uint32_t((m >> 1) & 1), kPollLimit);
      tc_fence_after();
    }
    const int64_t blk = (half == 0) ? blkA : blkB;
    const int64_t t = blk * kBlock + (r & 63);
    if (__all_sync(0xffffffffu, ok) && live) {  // warp-uniform: tcgen05.ld is warp-collective
      const bool store = t < P.T;
      const float denom = l1 + gl * fast_exp2(m_true - m_used);
      const float inv = 1.0f / denom;
      __nv_bfloat16* orow = P.o + (bh * P.T + t) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_base + C::kColO + c0, v);
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
    if (!ok) report(P.err);
  }

  tc_fence_before();
  __syncthreads();
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
