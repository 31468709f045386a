// pasa_forward_host: the whole PASA forward on host-resident q, k, v and o,
// pipelined over chunks of heads so that the PCIe copies overlap the GPU
// work: while chunk i is computed, chunk i+1 is copied in and chunk i-1 is
// copied out (copy-in, compute and copy-out run on three streams of their
// own, with two device slots per buffer).  Heads are independent, so every
// chunk is a complete pasa_forward call on its heads and the result is the
// same as one pasa_forward over all of them.
//
// The call is synchronous: it returns when o is in host memory.  The copies
// overlap only when the host buffers are page-locked (cudaHostAlloc or
// cudaHostRegister); pageable buffers still give the right result.
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace {

using pasa::cdiv;

constexpr int kSlots = 2;
constexpr int kMaxDevices = 64;

struct Pipe {
  cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
  cudaEvent_t start = nullptr;
  cudaEvent_t in_done[kSlots] = {}, comp_done[kSlots] = {}, out_done[kSlots] = {};
};

std::mutex g_pipe_mu;
Pipe g_pipe[kMaxDevices];

// The three streams and their events of the current device, created on first use.
int get_pipe(Pipe** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PASA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return PASA_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  Pipe& p = g_pipe[dev];
  if (!p.in) {
    Pipe n;
    bool ok = cudaStreamCreateWithFlags(&n.in, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&n.comp, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&n.out, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&n.start, cudaEventDisableTiming) == cudaSuccess;
    for (int s = 0; s < kSlots && ok; ++s)
      ok = cudaEventCreateWithFlags(&n.in_done[s], cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&n.comp_done[s], cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&n.out_done[s], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) return PASA_ERR_CUDA;
    p = n;
  }
  *out = &p;
  return PASA_OK;
}

// Device workspace of pasa_forward_host: per slot the q, k, v, o chunk
// buffers, the pasa_forward workspace of one chunk and its noise rows; then
// one error word per chunk.  Offsets are 256-byte aligned.
struct HostLayout {
  int64_t c = 0, nchunks = 0, ns = 0;
  size_t chunk_bytes = 0, fwd_bytes = 0, noise_bytes = 0;
  size_t off_q[kSlots] = {}, off_k[kSlots] = {}, off_v[kSlots] = {}, off_o[kSlots] = {};
  size_t off_fwd[kSlots] = {}, off_noise[kSlots] = {};
  size_t off_err = 0, total = 0;
};

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

int host_layout(int64_t B, int64_t H, int64_t T, int D, int dtype, double density, int64_t heads_per_chunk,
                HostLayout* L) {
  if (B < 1 || H < 1 || T < 1) return PASA_ERR_SHAPE;
  if (dtype != PASA_BF16 && dtype != PASA_F32) return PASA_ERR_DTYPE;
  if (heads_per_chunk < 1) return PASA_ERR_SHAPE;
  if (!std::isfinite(density)) return PASA_ERR_DENSITY;
  const int64_t BH = B * H;
  HostLayout l;
  l.c = heads_per_chunk < BH ? heads_per_chunk : BH;
  l.nchunks = cdiv(BH, l.c);
  int64_t nt = 0, ng = 0, ns = 0;
  int st = pasa_derive(T, pasa::kBlock, pasa::kGroup, density, &nt, &ng, &ns);
  if (st) return st;
  l.ns = ns;
  st = pasa_workspace_size(1, l.c, T, D, dtype, pasa::kBlock, pasa::kGroup, ns, &l.fwd_bytes);
  if (st) return st;
  const size_t esize = dtype == PASA_BF16 ? 2 : 4;
  l.chunk_bytes = up256(size_t(l.c) * size_t(T) * size_t(D) * esize);
  l.noise_bytes = up256(size_t(l.c) * size_t(nt) * sizeof(float));
  size_t o = 0;
  for (int s = 0; s < kSlots; ++s) {
    l.off_q[s] = o; o += l.chunk_bytes;
    l.off_k[s] = o; o += l.chunk_bytes;
    l.off_v[s] = o; o += l.chunk_bytes;
    l.off_o[s] = o; o += l.chunk_bytes;
    l.off_fwd[s] = o; o += up256(l.fwd_bytes);
    l.off_noise[s] = o; o += l.noise_bytes;
  }
  l.off_err = o; o += up256(size_t(l.nchunks) * sizeof(uint32_t));
  l.total = o;
  *L = l;
  return PASA_OK;
}

}  // namespace

extern "C" PASA_API int pasa_forward_host_workspace_size(int64_t B, int64_t H, int64_t T, int D, int dtype,
                                                         double density, int64_t heads_per_chunk, size_t* bytes) {
  if (!bytes) return PASA_ERR_NULL;
  HostLayout L;
  const int st = host_layout(B, H, T, D, dtype, density, heads_per_chunk, &L);
  if (st) return st;
  *bytes = L.total;
  return PASA_OK;
}

extern "C" PASA_API int pasa_forward_host(void* stream, const void* q_h, const void* k_h, const void* v_h, int64_t B,
                                          int64_t H, int64_t T, int D, int dtype, double density, float scale,
                                          int use_cov_bias, const float* noise_h, void* workspace,
                                          size_t workspace_bytes, int64_t heads_per_chunk, void* o_h,
                                          uint32_t* err_bits, int kernel) {
  HostLayout L;
  int st = host_layout(B, H, T, D, dtype, density, heads_per_chunk, &L);
  if (st) return st;
  if (!q_h || !k_h || !v_h || !o_h) return PASA_ERR_NULL;
  if (!workspace || workspace_bytes < L.total) return PASA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PASA_ERR_ALIGN;
  Pipe* p = nullptr;
  if ((st = get_pipe(&p))) return st;

  const int64_t BH = B * H, NT = cdiv(T, pasa::kBlock);
  const size_t esize = dtype == PASA_BF16 ? 2 : 4;
  const size_t head_bytes = size_t(T) * size_t(D) * esize;
  char* w = static_cast<char*>(workspace);
  uint32_t* err_dev = reinterpret_cast<uint32_t*>(w + L.off_err);
  const char* qh = static_cast<const char*>(q_h);
  const char* kh = static_cast<const char*>(k_h);
  const char* vh = static_cast<const char*>(v_h);
  char* oh = static_cast<char*>(o_h);

  // everything already queued on the caller's stream (workspace, inputs) comes first
  if (cudaEventRecord(p->start, static_cast<cudaStream_t>(stream)) != cudaSuccess ||
      cudaStreamWaitEvent(p->in, p->start, 0) != cudaSuccess)
    return PASA_ERR_CUDA;
  bool ok = true;
  for (int64_t i = 0; i < L.nchunks && ok && st == PASA_OK; ++i) {
    const int s = int(i % kSlots);
    const int64_t h0 = i * L.c, nh = (h0 + L.c <= BH) ? L.c : BH - h0;
    const size_t bytes = size_t(nh) * head_bytes, off = size_t(h0) * head_bytes;
    // copy in: the slot is free once chunk i - kSlots has been copied out
    if (i >= kSlots) ok = ok && cudaStreamWaitEvent(p->in, p->out_done[s], 0) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(w + L.off_q[s], qh + off, bytes, cudaMemcpyHostToDevice, p->in) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(w + L.off_k[s], kh + off, bytes, cudaMemcpyHostToDevice, p->in) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(w + L.off_v[s], vh + off, bytes, cudaMemcpyHostToDevice, p->in) == cudaSuccess;
    if (noise_h)
      ok = ok && cudaMemcpyAsync(w + L.off_noise[s], noise_h + size_t(h0) * size_t(NT), size_t(nh) * size_t(NT) * 4,
                                 cudaMemcpyHostToDevice, p->in) == cudaSuccess;
    ok = ok && cudaEventRecord(p->in_done[s], p->in) == cudaSuccess;
    // compute: the whole op on this chunk's heads; keep its error word
    ok = ok && cudaStreamWaitEvent(p->comp, p->in_done[s], 0) == cudaSuccess;
    if (!ok) break;
    st = pasa_forward(p->comp, w + L.off_q[s], w + L.off_k[s], w + L.off_v[s], 1, nh, T, D, dtype, density, scale,
                      use_cov_bias, noise_h ? reinterpret_cast<const float*>(w + L.off_noise[s]) : nullptr,
                      w + L.off_fwd[s], L.fwd_bytes, w + L.off_o[s], kernel);
    if (st) break;
    // the chunk's device error word, at its place in pasa_forward's workspace layout
    const pasa::Layout FL = pasa::make_layout(nh, T, D, int(esize), L.ns);
    ok = ok && cudaMemcpyAsync(err_dev + i, w + L.off_fwd[s] + FL.off_err, sizeof(uint32_t),
                               cudaMemcpyDeviceToDevice, p->comp) == cudaSuccess;
    ok = ok && cudaEventRecord(p->comp_done[s], p->comp) == cudaSuccess;
    // copy out
    ok = ok && cudaStreamWaitEvent(p->out, p->comp_done[s], 0) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(oh + off, w + L.off_o[s], bytes, cudaMemcpyDeviceToHost, p->out) == cudaSuccess;
    ok = ok && cudaEventRecord(p->out_done[s], p->out) == cudaSuccess;
  }
  // drain every stream before returning (also after a failure: nothing may
  // still be reading the caller's buffers)
  const bool drained = cudaStreamSynchronize(p->in) == cudaSuccess &&
                       cudaStreamSynchronize(p->comp) == cudaSuccess &&
                       cudaStreamSynchronize(p->out) == cudaSuccess;
  if (st) return st;
  if (!ok || !drained) return PASA_ERR_CUDA;
  if (err_bits) {
    std::vector<uint32_t> e(size_t(L.nchunks), 0u);
    if (cudaMemcpy(e.data(), err_dev, e.size() * sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
      return PASA_ERR_CUDA;
    uint32_t acc = 0;
    for (uint32_t x : e) acc |= x;
    *err_bits = acc;
  }
  return PASA_OK;
}
