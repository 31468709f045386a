// Shared helpers of the pasa_b200 CUDA library: element conversion, sizes,
// and thin inline-PTX wrappers for mbarriers, TMA and tcgen05 (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/pasa_b200.h"

namespace pasa {

// Scatter of the attention output to the ranks that own its tokens (the
// fused head-to-sequence exchange); npeer = 0 means a plain store.
struct OutScatter {
  void* const* peer = nullptr;  // device table of npeer token-major buffers
  int npeer = 0;
  int64_t tokens = 0, heads_total = 0, head0 = 0;
};

constexpr int kBlock = 64;   // tokens per block (BT of the reference)
constexpr int kGroup = 32;   // blocks per correction group (GROUP_SIZE)
constexpr float kLog2e = 1.44269504f;  // group_pisa_attention.py:162

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// element access: values are computed in fp32; bf16 stores round to nearest
// even, as the reference's `.to(dtype)` does.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ float round(float x) { return x; }
  static __device__ __forceinline__ void store(float* p, float x) { *p = x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
};

// 2^x with the hardware approximation (ex2.approx.f32), the instruction the
// reference's tl.math.exp2 lowers to.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The same approximation with subnormal inputs and results flushed to zero
// (ex2.approx.ftz.f32, one MUFU instruction; the non-flushing form needs
// extra instructions around it).  For the softmax probabilities a result
// below 2^-126 is irrelevant: it rounds into a bf16 P that contributes
// nothing next to the row maximum's 2^0.
__device__ __forceinline__ float exp2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// workspace layout used by pasa_forward (all offsets 256-byte aligned)
// ---------------------------------------------------------------------------
struct Layout {
  int64_t BH, T, NT, NG, NTP, NS;  // NTP = NG * kGroup (padded block rows)
  int D, esize;
  size_t off_qc, off_kc, off_vc, off_hnorm, off_hgroup, off_idx, off_mask, off_err, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

inline Layout make_layout(int64_t BH, int64_t T, int D, int esize, int64_t NS) {
  Layout L{};
  L.BH = BH; L.T = T; L.D = D; L.esize = esize; L.NS = NS;
  L.NT = cdiv(T, kBlock);
  L.NG = cdiv(L.NT, kGroup);
  L.NTP = L.NG * kGroup;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align256(o + bytes); return at; };
  L.off_qc = take(size_t(BH) * L.NTP * D * esize);
  L.off_kc = take(size_t(BH) * L.NTP * D * esize);
  L.off_vc = take(size_t(BH) * L.NTP * D * esize);
  L.off_hnorm = take(size_t(BH) * L.NT * sizeof(float));
  L.off_hgroup = take(size_t(BH) * L.NG * D * D * esize);
  L.off_idx = take(size_t(BH) * L.NT * NS * sizeof(int32_t));
  L.off_mask = take(size_t(BH) * L.NT * L.NG * sizeof(uint32_t));
  L.off_err = take(sizeof(uint32_t) * 4);
  L.total = o;
  return L;
}

// ---------------------------------------------------------------------------
// PTX wrappers (sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// SM clock cycles (cheap to read; compared only within one thread).
__device__ __forceinline__ uint64_t sm_cycles() { return clock64(); }

// Bound on any single barrier wait: 4e9 SM cycles (about 2 s at B200 clocks,
// against kernels of milliseconds).
constexpr uint64_t kWaitLimitCycles = 4000000000ull;

// Bounded wait: returns false (the phase still incomplete) once `limit`
// SM cycles have passed without the phase completing.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit = kWaitLimitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = sm_cycles();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (sm_cycles() - t0 > limit) return false;
  }
}

// TMA: 3-D tiled load global -> shared, completion on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      :: "r"(smem_u32(smem_dst)), "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(tmap) : "memory");
}

// tcgen05 --------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(smem_slot)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
         "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// UMMA shared-memory descriptor, 128-byte swizzle (sm_100 version field = 1).
// lbo/sbo in bytes.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFF);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;   // version
  d |= uint64_t(2) << 61;   // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and an fp32 accumulator.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                       // D format f32
       | (1u << 7)                       // A bf16
       | (1u << 10)                      // B bf16
       | ((a_mn_major ? 1u : 0u) << 15)
       | ((b_mn_major ? 1u : 0u) << 16)
       | (uint32_t(N >> 3) << 17)
       | (uint32_t(M >> 4) << 24);
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
         "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
         "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
         "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Named barrier over `nthreads` threads (multiple of 32); id 0 is __syncthreads.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}
// Arrive on a named barrier without waiting (the producer side of a
// producer/consumer hand-off; the consumer uses named_bar_sync).
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Maximum of 32 fp32 values held as raw bits (shallow tree of 3-input max).
__device__ __forceinline__ float max_tree32(const uint32_t (&v)[32]) {
  float m[12];
#pragma unroll
  for (int i = 0; i < 10; ++i)
    m[i] = fmax3(__uint_as_float(v[3 * i]), __uint_as_float(v[3 * i + 1]), __uint_as_float(v[3 * i + 2]));
  m[10] = __uint_as_float(v[30]);
  m[11] = __uint_as_float(v[31]);
  const float a = fmax3(m[0], m[1], m[2]), b = fmax3(m[3], m[4], m[5]);
  const float c = fmax3(m[6], m[7], m[8]), d = fmax3(m[9], m[10], m[11]);
  return fmaxf(fmax3(a, b, c), d);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi);

// p_c = 2^(s_c * scale + negm) for N (a multiple of 4) raw fp32 scores;
// packs bf16 pairs into pk and returns the fp32 sum of the p_c.  The
// scale/shift and the sums use the sm_100 packed fp32 pair instructions.
template <int N>
__device__ __forceinline__ float exp2_pack(const uint32_t (&sv)[N], float scale, float negm,
                                           uint32_t (&pk)[N / 2]) {
  static_assert(N % 4 == 0, "exp2_pack width");
  const float2 sc = make_float2(scale, scale), nm = make_float2(negm, negm);
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < N; c += 4) {
    float2 x01 = __ffma2_rn(make_float2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])), sc, nm);
    float2 x23 = __ffma2_rn(make_float2(__uint_as_float(sv[c + 2]), __uint_as_float(sv[c + 3])), sc, nm);
    x01.x = exp2_ftz(x01.x); x01.y = exp2_ftz(x01.y);
    x23.x = exp2_ftz(x23.x); x23.y = exp2_ftz(x23.y);
    pk[c / 2] = pack_bf16x2(x01.x, x01.y);
    pk[c / 2 + 1] = pack_bf16x2(x23.x, x23.y);
    acc0 = __fadd2_rn(acc0, x01);
    acc1 = __fadd2_rn(acc1, x23);
  }
  return (acc0.x + acc0.y) + (acc1.x + acc1.y);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace pasa
