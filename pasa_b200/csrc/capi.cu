// extern "C" entry points of libpasa_b200.so: argument validation, the
// workspace layout, and kernel dispatch.  Declarations and the reference
// interface each entry point replaces are in include/pasa_b200.h.
#include <cmath>
#include <cstring>

#include "common.cuh"

namespace pasa {
cudaError_t launch_prep(cudaStream_t, int, int, const void*, const void*, const void*, int64_t, int64_t, void*,
                        void*, void*, float*, void*, uint32_t*);
cudaError_t launch_select(cudaStream_t, int, int, const void*, const void*, const float*, const float*, int64_t,
                          int64_t, int64_t, float, int, int32_t*, uint32_t*);
size_t select_smem_bytes(int D, int64_t NT, int64_t NG, int64_t NS);
cudaError_t launch_attn_simt(cudaStream_t, int, int, const void*, const void*, const void*, const void*,
                             const void*, const void*, const int32_t*, const uint32_t*, int64_t, int64_t,
                             int64_t, float, void*);
cudaError_t launch_attn_tc(cudaStream_t, int, const void*, const void*, const void*, const void*, const void*,
                           const void*, const uint32_t*, int64_t, int64_t, int64_t, float, void*, uint32_t*, int,
                           int64_t, const OutScatter&, int64_t blk_lo, int64_t blk_hi);
cudaError_t launch_place(cudaStream_t, const void*, void*, const int32_t*, int64_t, int64_t, int64_t, int, int,
                         int64_t, int64_t, int64_t, int);
size_t sample_mse_workspace(int64_t BH, int64_t T, int D);
cudaError_t launch_sample_mse(cudaStream_t, int, int, const void*, const void*, const void*, int64_t, int64_t,
                              const int64_t*, int, int, int64_t, int64_t, int64_t, void*, void*, int32_t*);
int dit_max_cols();
cudaError_t launch_row_norm(cudaStream_t, const void*, const void*, const float*, void*, const float*, const float*,
                            const float*, const float*, int64_t, int64_t, int, float, int, int, void*);
cudaError_t launch_qkv_rope(cudaStream_t, const void*, const void*, const void*, const float*, const float*,
                            const double*, const double*, int64_t, int64_t, int, int, float, int, void*, void*,
                            void*, void* const*, int, int);
}  // namespace pasa

using namespace pasa;

namespace {

constexpr size_t kMaxSmem = 227 * 1024;

int esize_of(int dtype) { return dtype == PASA_BF16 ? 2 : 4; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int64_t BH, int64_t T, int D, int dtype) {
  if (dtype != PASA_BF16 && dtype != PASA_F32) return PASA_ERR_DTYPE;
  if (D != 64 && D != 128) return PASA_ERR_UNSUPPORTED;
  if (BH < 1 || T < 1) return PASA_ERR_SHAPE;
  if (BH > 65535) return PASA_ERR_SHAPE;                     // grid.y
  const int64_t NT = cdiv(T, kBlock);
  if (NT > (int64_t(1) << 24)) return PASA_ERR_SHAPE;
  return PASA_OK;
}

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PASA_ERR_CUDA;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return PASA_ERR_CUDA;
  return major == 10 ? PASA_OK : PASA_ERR_DEVICE;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? PASA_OK : PASA_ERR_CUDA; }

int64_t top_k_of(double density, int64_t NT) {
  // min(max(1, int(density * NT)), NT)   (group_pisa_attention.py:373)
  const double prod = density * double(NT);
  int64_t t = (prod >= 9.0e18) ? NT : (prod <= -9.0e18 ? 0 : int64_t(prod));  // int() truncates toward 0
  if (t < 1) t = 1;
  if (t > NT) t = NT;
  return t;
}

// cols rounded up to a power of two (the reference's Triton row programs)
int padded_cols(int cols) {
  int p = 1;
  while (p < cols) p <<= 1;
  return p;
}

int check_select_fit(int D, int64_t NT, int64_t NS) {
  const int64_t NG = cdiv(NT, kGroup);
  return select_smem_bytes(D, NT, NG, NS) <= kMaxSmem ? PASA_OK : PASA_ERR_SHAPE;
}

}  // namespace

extern "C" {

int pasa_abi_version(void) { return PASA_ABI_VERSION; }

const char* pasa_status_string(int status) {
  switch (status) {
    case PASA_OK: return "ok";
    case PASA_ERR_SHAPE: return "invalid shape or size";
    case PASA_ERR_DTYPE: return "unsupported dtype (bf16 or fp32 expected)";
    case PASA_ERR_ALIGN: return "pointer not 16-byte aligned";
    case PASA_ERR_DENSITY: return "density is not a finite number";
    case PASA_ERR_UNSUPPORTED: return "unsupported configuration (head_dim 64/128, block 64, group 32)";
    case PASA_ERR_WORKSPACE: return "workspace missing or too small";
    case PASA_ERR_NULL: return "required pointer is NULL";
    case PASA_ERR_CUDA: return "CUDA runtime error";
    case PASA_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    default: return "unknown status";
  }
}

int pasa_derive(int64_t T, int block, int group, double density, int64_t* nt, int64_t* ng, int64_t* ns) {
  if (block != kBlock || group != kGroup) return PASA_ERR_UNSUPPORTED;
  if (T < 1) return PASA_ERR_SHAPE;
  if (!std::isfinite(density)) return PASA_ERR_DENSITY;
  const int64_t NT = cdiv(T, kBlock);
  if (nt) *nt = NT;
  if (ng) *ng = cdiv(NT, kGroup);
  if (ns) *ns = top_k_of(density, NT);
  return PASA_OK;
}

int pasa_workspace_size(int64_t B, int64_t H, int64_t T, int D, int dtype, int block, int group, int64_t ns,
                        size_t* bytes) {
  if (!bytes) return PASA_ERR_NULL;
  if (block != kBlock || group != kGroup) return PASA_ERR_UNSUPPORTED;
  if (B < 1 || H < 1) return PASA_ERR_SHAPE;
  int st = check_common(B * H, T, D, dtype);
  if (st) return st;
  const int64_t NT = cdiv(T, kBlock);
  if (ns < 1 || ns > NT) return PASA_ERR_SHAPE;
  *bytes = make_layout(B * H, T, D, esize_of(dtype), ns).total;
  return PASA_OK;
}

namespace {
// pasa_prep with an error word (nullable, device) for the kernel's bounded waits
int prep_impl(void* stream, const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t T, int D,
              int dtype, int block, int group, void* qc, void* kc, void* vc, float* h_norm, void* h_group,
              uint32_t* err) {
  if (block != kBlock || group != kGroup) return PASA_ERR_UNSUPPORTED;
  if (B < 1 || H < 1) return PASA_ERR_SHAPE;
  int st = check_common(B * H, T, D, dtype);
  if (st) return st;
  if (!q || !k || !v || !qc || !kc || !vc || !h_norm || !h_group) return PASA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(qc) || !aligned16(kc) || !aligned16(vc) ||
      !aligned16(h_group))
    return PASA_ERR_ALIGN;
  if ((st = check_device())) return st;
  return cuda_status(launch_prep(static_cast<cudaStream_t>(stream), dtype, D, q, k, v, B * H, T, qc, kc, vc,
                                 h_norm, h_group, err));
}
}  // namespace

int pasa_prep(void* stream, const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t T, int D,
              int dtype, int block, int group, void* qc, void* kc, void* vc, float* h_norm, void* h_group) {
  return prep_impl(stream, q, k, v, B, H, T, D, dtype, block, group, qc, kc, vc, h_norm, h_group, nullptr);
}

int pasa_select(void* stream, const void* qc, const void* kc, const float* h_norm, const float* noise, int64_t BH,
                int64_t NT, int D, int dtype, float scale, int use_cov_bias, int64_t ns, int32_t* indices,
                uint32_t* sel_mask) {
  if (dtype != PASA_BF16 && dtype != PASA_F32) return PASA_ERR_DTYPE;
  if (D != 64 && D != 128) return PASA_ERR_UNSUPPORTED;
  if (BH < 1 || BH > 65535 || NT < 1) return PASA_ERR_SHAPE;
  if (ns < 1 || ns > NT) return PASA_ERR_SHAPE;
  if (!qc || !kc || !indices || (use_cov_bias && !h_norm)) return PASA_ERR_NULL;
  if (!std::isfinite(scale)) return PASA_ERR_SHAPE;
  int st = check_select_fit(D, NT, ns);
  if (st) return st;
  if ((st = check_device())) return st;
  return cuda_status(launch_select(static_cast<cudaStream_t>(stream), dtype, D, qc, kc, h_norm,
                                   use_cov_bias ? noise : nullptr, BH, NT, ns, scale, use_cov_bias, indices,
                                   sel_mask));
}

namespace {

// pasa_attn with the output layout: o_heads = 0 writes [B*H, T, D], o_heads =
// H > 0 writes [B, T, H, D]; sc.npeer > 0 scatters the rows to the token
// owners' buffers instead of o (tensor-core kernel only for both).
int attn_dispatch(void* stream, const void* q, const void* k, const void* v, const void* kc, const void* vc,
                  const void* h_group, const int32_t* indices, const uint32_t* sel_mask, int64_t BH, int64_t T,
                  int D, int dtype, float scale, int64_t ns, void* o, uint32_t* err_word, int kernel,
                  int64_t o_heads, const OutScatter& sc = OutScatter{}) {
  int st = check_common(BH, T, D, dtype);
  if (st) return st;
  const int64_t NT = cdiv(T, kBlock), NG = cdiv(NT, kGroup);
  if (ns < 1 || ns > NT) return PASA_ERR_SHAPE;
  const bool scatter = sc.npeer > 0;
  if (!q || !k || !v || !kc || !vc || !h_group || !sel_mask || (!o && !scatter)) return PASA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(kc) || !aligned16(vc) ||
      !aligned16(h_group) || (!scatter && !aligned16(o)))
    return PASA_ERR_ALIGN;
  if (!std::isfinite(scale)) return PASA_ERR_SHAPE;
  if (kernel == PASA_ATTN_AUTO) kernel = (dtype == PASA_BF16) ? PASA_ATTN_TCGEN05 : PASA_ATTN_SIMT;
  if (o_heads < 0 || (o_heads > 0 && BH % o_heads != 0)) return PASA_ERR_SHAPE;
  if ((st = check_device())) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kernel == PASA_ATTN_TCGEN05) {
    if (dtype != PASA_BF16) return PASA_ERR_DTYPE;
    return cuda_status(launch_attn_tc(s, D, q, k, v, kc, vc, h_group, sel_mask, BH, T, ns, scale, o, err_word, 0,
                                      o_heads, sc, 0, -1));
  }
  if (kernel != PASA_ATTN_SIMT) return PASA_ERR_UNSUPPORTED;
  if (o_heads > 0 || scatter) return PASA_ERR_UNSUPPORTED;  // the CUDA-core kernel writes [B*H, T, D] only
  if (!indices) return PASA_ERR_NULL;
  if (NG > 64) return PASA_ERR_SHAPE;  // the CUDA-core kernel keeps one word per group in shared memory
  return cuda_status(launch_attn_simt(s, dtype, D, q, k, v, kc, vc, h_group, indices, sel_mask, BH, T, ns, scale,
                                      o));
}

}  // namespace

int pasa_attn(void* stream, const void* q, const void* k, const void* v, const void* kc, const void* vc,
              const void* h_group, const int32_t* indices, const uint32_t* sel_mask, int64_t BH, int64_t T, int D,
              int dtype, float scale, int64_t ns, void* o, uint32_t* err_word, int kernel) {
  return attn_dispatch(stream, q, k, v, kc, vc, h_group, indices, sel_mask, BH, T, D, dtype, scale, ns, o,
                       err_word, kernel, 0);
}

int pasa_forward(void* stream, const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t T, int D,
                 int dtype, double density, float scale, int use_cov_bias, const float* noise, void* workspace,
                 size_t workspace_bytes, void* o, int kernel) {
  return pasa_forward_ex(stream, q, k, v, B, H, T, D, dtype, density, scale, use_cov_bias, noise, workspace,
                         workspace_bytes, o, kernel, PASA_O_BHTD);
}

namespace {

// prep -> select -> attention on one workspace (pasa_forward_ex, pasa_forward_scatter).
int forward_impl(void* stream, const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t T, int D,
                 int dtype, double density, float scale, int use_cov_bias, const float* noise, void* workspace,
                 size_t workspace_bytes, void* o, int kernel, int64_t o_heads, const OutScatter& sc) {
  if (B < 1 || H < 1) return PASA_ERR_SHAPE;
  int st = check_common(B * H, T, D, dtype);
  if (st) return st;
  if (!std::isfinite(density)) return PASA_ERR_DENSITY;
  if (!q || !k || !v || (!o && sc.npeer == 0)) return PASA_ERR_NULL;
  const int64_t BH = B * H, NT = cdiv(T, kBlock);
  const int64_t NS = top_k_of(density, NT);
  const Layout L = make_layout(BH, T, D, esize_of(dtype), NS);
  if (!workspace || workspace_bytes < L.total) return PASA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PASA_ERR_ALIGN;
  if ((st = check_select_fit(D, NT, NS))) return st;
  if ((st = check_device())) return st;
  char* w = static_cast<char*>(workspace);
  void* qc = w + L.off_qc;
  void* kc = w + L.off_kc;
  void* vc = w + L.off_vc;
  float* hn = reinterpret_cast<float*>(w + L.off_hnorm);
  void* hg = w + L.off_hgroup;
  int32_t* idx = reinterpret_cast<int32_t*>(w + L.off_idx);
  uint32_t* mask = reinterpret_cast<uint32_t*>(w + L.off_mask);
  uint32_t* err = reinterpret_cast<uint32_t*>(w + L.off_err);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(err, 0, sizeof(uint32_t), s) != cudaSuccess) return PASA_ERR_CUDA;
  if ((st = prep_impl(stream, q, k, v, B, H, T, D, dtype, kBlock, kGroup, qc, kc, vc, hn, hg, err))) return st;
  if ((st = pasa_select(stream, qc, kc, hn, noise, BH, NT, D, dtype, scale, use_cov_bias, NS, idx, mask)))
    return st;
  return attn_dispatch(stream, q, k, v, kc, vc, hg, idx, mask, BH, T, D, dtype, scale, NS, o, err, kernel, o_heads,
                       sc);
}

}  // namespace

int pasa_forward_ex(void* stream, const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t T,
                    int D, int dtype, double density, float scale, int use_cov_bias, const float* noise,
                    void* workspace, size_t workspace_bytes, void* o, int kernel, int o_layout) {
  if (o_layout != PASA_O_BHTD && o_layout != PASA_O_BTHD) return PASA_ERR_UNSUPPORTED;
  if (!o) return PASA_ERR_NULL;
  return forward_impl(stream, q, k, v, B, H, T, D, dtype, density, scale, use_cov_bias, noise, workspace,
                      workspace_bytes, o, kernel, o_layout == PASA_O_BTHD ? H : 0, OutScatter{});
}

int pasa_forward_scatter(void* stream, const void* q, const void* k, const void* v, int64_t H_local, int64_t T,
                         int D, double density, float scale, int use_cov_bias, const float* noise, void* workspace,
                         size_t workspace_bytes, void* const* o_peer_table, int n_ranks, int64_t head0,
                         int64_t heads_total, int kernel) {
  if (n_ranks < 1 || n_ranks > 64 || T < 1 || T % n_ranks != 0) return PASA_ERR_SHAPE;
  if (H_local < 1 || head0 < 0 || heads_total < head0 + H_local) return PASA_ERR_SHAPE;
  if (!o_peer_table) return PASA_ERR_NULL;
  if (kernel != PASA_ATTN_AUTO && kernel != PASA_ATTN_TCGEN05) return PASA_ERR_UNSUPPORTED;
  OutScatter sc;
  sc.peer = o_peer_table;
  sc.npeer = n_ranks;
  sc.tokens = T / n_ranks;
  sc.heads_total = heads_total;
  sc.head0 = head0;
  return forward_impl(stream, q, k, v, 1, H_local, T, D, PASA_BF16, density, scale, use_cov_bias, noise, workspace,
                      workspace_bytes, nullptr, PASA_ATTN_TCGEN05, 0, sc);
}

namespace {

// heads [h0, h1) that hold the query blocks [block_begin, block_end) of the
// B*H*NT blocks in (head, block) order
int range_heads(int64_t B, int64_t H, int64_t T, int64_t block_begin, int64_t block_end, int64_t* h0,
                int64_t* h1) {
  const int64_t NT = cdiv(T, kBlock);
  if (block_begin < 0 || block_end <= block_begin || block_end > B * H * NT) return PASA_ERR_SHAPE;
  *h0 = block_begin / NT;
  *h1 = cdiv(block_end, NT);
  return PASA_OK;
}

}  // namespace

int pasa_forward_range_workspace_size(int64_t B, int64_t H, int64_t T, int D, int dtype, double density,
                                      int64_t block_begin, int64_t block_end, size_t* bytes) {
  if (!bytes) return PASA_ERR_NULL;
  if (B < 1 || H < 1) return PASA_ERR_SHAPE;
  int st = check_common(B * H, T, D, dtype);
  if (st) return st;
  if (!std::isfinite(density)) return PASA_ERR_DENSITY;
  int64_t h0 = 0, h1 = 0;
  if ((st = range_heads(B, H, T, block_begin, block_end, &h0, &h1))) return st;
  *bytes = make_layout(h1 - h0, T, D, esize_of(dtype), top_k_of(density, cdiv(T, kBlock))).total;
  return PASA_OK;
}

int pasa_forward_range(void* stream, const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t T,
                       int D, int dtype, double density, float scale, int use_cov_bias, const float* noise,
                       void* workspace, size_t workspace_bytes, void* o, int kernel, int64_t block_begin,
                       int64_t block_end) {
  if (B < 1 || H < 1) return PASA_ERR_SHAPE;
  int st = check_common(B * H, T, D, dtype);
  if (st) return st;
  if (!std::isfinite(density)) return PASA_ERR_DENSITY;
  if (kernel != PASA_ATTN_AUTO && kernel != PASA_ATTN_TCGEN05) return PASA_ERR_UNSUPPORTED;
  if (dtype != PASA_BF16) return PASA_ERR_DTYPE;  // the tensor-core kernel runs bf16
  if (!q || !k || !v || !o) return PASA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return PASA_ERR_ALIGN;
  if (!std::isfinite(scale)) return PASA_ERR_SHAPE;
  int64_t h0 = 0, h1 = 0;
  if ((st = range_heads(B, H, T, block_begin, block_end, &h0, &h1))) return st;
  const int64_t NT = cdiv(T, kBlock), NS = top_k_of(density, NT), BHt = h1 - h0;
  const Layout L = make_layout(BHt, T, D, esize_of(dtype), NS);
  if (!workspace || workspace_bytes < L.total) return PASA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PASA_ERR_ALIGN;
  if ((st = check_select_fit(D, NT, NS))) return st;
  if ((st = check_device())) return st;
  const size_t head_bytes = size_t(T) * D * esize_of(dtype);
  auto at = [&](const void* base, int64_t h) { return static_cast<const char*>(base) + size_t(h) * head_bytes; };
  char* w = static_cast<char*>(workspace);
  char* qc = w + L.off_qc;
  char* kc = w + L.off_kc;
  char* vc = w + L.off_vc;
  float* hn = reinterpret_cast<float*>(w + L.off_hnorm);
  char* hg = w + L.off_hgroup;
  int32_t* idx = reinterpret_cast<int32_t*>(w + L.off_idx);
  uint32_t* mask = reinterpret_cast<uint32_t*>(w + L.off_mask);
  uint32_t* err = reinterpret_cast<uint32_t*>(w + L.off_err);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the block statistics and the selection cover the touched heads whole
  // (a head shared with another caller's range is prepared by both)
  if (cudaMemsetAsync(err, 0, sizeof(uint32_t), s) != cudaSuccess) return PASA_ERR_CUDA;
  if ((st = prep_impl(stream, at(q, h0), at(k, h0), at(v, h0), 1, BHt, T, D, dtype, kBlock, kGroup, qc, kc, vc, hn,
                      hg, err)))
    return st;
  if ((st = pasa_select(stream, qc, kc, hn, noise ? noise + h0 * NT : nullptr, BHt, NT, D, dtype, scale,
                        use_cov_bias, NS, idx, mask)))
    return st;
  const size_t stat_bytes = size_t(L.NTP) * D * esize_of(dtype), hg_bytes = size_t(L.NG) * D * D * esize_of(dtype);
  // attention: the first and the last head may be partial, the heads between are whole
  int64_t h = h0;
  while (h < h1) {
    const int64_t lo = (h == h0) ? block_begin - h0 * NT : 0;
    const int64_t hi = (h == h1 - 1) ? block_end - (h1 - 1) * NT : NT;
    int64_t n = 1;  // whole heads go in one launch
    if (lo == 0 && hi == NT)
      while (h + n < h1 && !(h + n == h1 - 1 && block_end - (h1 - 1) * NT != NT)) ++n;
    const int64_t j = h - h0;
    cudaError_t e = launch_attn_tc(s, D, at(q, h), at(k, h), at(v, h), kc + j * stat_bytes, vc + j * stat_bytes,
                                   hg + j * hg_bytes, mask + j * NT * L.NG, n, T, NS, scale,
                                   static_cast<char*>(o) + size_t(h) * head_bytes, err, 0, 0, OutScatter{}, lo, hi);
    if (e != cudaSuccess) return PASA_ERR_CUDA;
    h += n;
  }
  return PASA_OK;
}

int pasa_dense_attn(void* stream, const void* q, const void* k, const void* v, int64_t BH, int64_t T, int D,
                    int dtype, float scale, void* o, uint32_t* err_word) {
  int st = check_common(BH, T, D, dtype);
  if (st) return st;
  if (dtype != PASA_BF16) return PASA_ERR_DTYPE;  // the tensor-core kernel runs bf16
  if (!q || !k || !v || !o) return PASA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return PASA_ERR_ALIGN;
  if (!std::isfinite(scale)) return PASA_ERR_SHAPE;
  if ((st = check_device())) return st;
  // the block statistics are not read in dense mode; q stands in for their (unused) tensor maps
  return cuda_status(launch_attn_tc(static_cast<cudaStream_t>(stream), D, q, k, v, q, q, q, nullptr, BH, T,
                                    cdiv(T, kBlock), scale, o, err_word, 1, 0, OutScatter{}, 0, -1));
}

int pasa_sample_mse_workspace_size(int64_t BH, int64_t T, int D, size_t* bytes) {
  if (!bytes) return PASA_ERR_NULL;
  if (BH < 1 || BH > 65535 || T < 1) return PASA_ERR_SHAPE;
  if (D != 64 && D != 128) return PASA_ERR_UNSUPPORTED;
  *bytes = sample_mse_workspace(BH, T, D);
  return PASA_OK;
}

int pasa_sample_mse(void* stream, const void* q, const void* k, const void* v, int64_t cfg, int64_t H, int64_t T,
                    int D, int dtype, const int64_t* rows, int64_t n_rows, int model, int64_t context_length,
                    int64_t num_frame, int64_t frame_size, void* workspace, size_t workspace_bytes, void* mse,
                    int32_t* best_mask_idx) {
  if (dtype != PASA_BF16 && dtype != PASA_F32) return PASA_ERR_DTYPE;
  if (D != 64 && D != 128) return PASA_ERR_UNSUPPORTED;
  if (model != PASA_MODEL_HUNYUAN && model != PASA_MODEL_WAN) return PASA_ERR_UNSUPPORTED;
  if (cfg < 1 || H < 1 || cfg * H > 65535 || T < 1) return PASA_ERR_SHAPE;
  if (n_rows < 1 || n_rows > 32) return PASA_ERR_SHAPE;
  if (context_length < 0 || num_frame < 1 || frame_size < 1) return PASA_ERR_SHAPE;
  // the sequence is the video (plus the text tail for HunyuanVideo), as the
  // processors assert (hyvideo/attention.py:491-494, wan/attention.py:359-362)
  // (Wan's mask has no text tail: its temporal reshape needs T = num_frame *
  // frame_size, wan/utils.py:99-103)
  if (model == PASA_MODEL_WAN && context_length != 0) return PASA_ERR_UNSUPPORTED;
  if (context_length + num_frame * frame_size != T) return PASA_ERR_SHAPE;
  if (!q || !k || !v || !rows || !workspace || (!mse && !best_mask_idx)) return PASA_ERR_NULL;
  for (int64_t r = 0; r < n_rows; ++r)
    if (rows[r] < 0 || rows[r] >= T) return PASA_ERR_SHAPE;  // the reference's indexing would fail too
  if (workspace_bytes < sample_mse_workspace(cfg * H, T, D)) return PASA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PASA_ERR_ALIGN;
  int st = check_device();
  if (st) return st;
  return cuda_status(launch_sample_mse(static_cast<cudaStream_t>(stream), dtype, D, q, k, v, cfg * H, T, rows,
                                       int(n_rows), model, context_length, num_frame, frame_size, workspace, mse,
                                       best_mask_idx));
}

int pasa_place(void* stream, const void* src, void* dst, const int32_t* head_is_temporal, int64_t cfg, int64_t H,
               int64_t T, int D, int dtype, int64_t context_length, int64_t num_frame, int64_t frame_size,
               int inverse) {
  if (dtype != PASA_BF16 && dtype != PASA_F32) return PASA_ERR_DTYPE;
  if (D < 8 || (D * esize_of(dtype)) % 16 != 0 || D * esize_of(dtype) > 4096) return PASA_ERR_UNSUPPORTED;
  if (cfg < 1 || H < 1 || T < 1 || context_length < 0 || num_frame < 1 || frame_size < 1) return PASA_ERR_SHAPE;
  if (context_length + num_frame * frame_size != T) return PASA_ERR_SHAPE;  // placement.py:128
  if (!src || !dst || !head_is_temporal) return PASA_ERR_NULL;
  if (!aligned16(src) || !aligned16(dst)) return PASA_ERR_ALIGN;
  int st = check_device();
  if (st) return st;
  return cuda_status(launch_place(static_cast<cudaStream_t>(stream), src, dst, head_is_temporal, cfg, H, T, D,
                                  esize_of(dtype), context_length, num_frame, frame_size, inverse));
}

int pasa_dit_row_norm(void* stream, const void* x, const void* add, const float* gate, void* x_out,
                      const float* weight, const float* bias, const float* scale, const float* shift, int64_t rows,
                      int64_t batch_rows, int cols, float eps, int norm, void* y) {
  if (norm != PASA_DIT_RMSNORM && norm != PASA_DIT_LAYERNORM && norm != PASA_DIT_LAYERNORM_PADDED)
    return PASA_ERR_UNSUPPORTED;
  if (rows < 1 || rows > INT32_MAX || cols < 8 || cols % 8 != 0 || cols > dit_max_cols()) return PASA_ERR_SHAPE;
  if (batch_rows < 1 || rows % batch_rows != 0) return PASA_ERR_SHAPE;
  if (!std::isfinite(eps) || eps < 0.f) return PASA_ERR_SHAPE;
  if (!x || !y || (scale == nullptr) != (shift == nullptr)) return PASA_ERR_NULL;
  if (gate && !add) return PASA_ERR_NULL;
  const void* ptrs[] = {x, add, gate, x_out, weight, bias, scale, shift, y};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return PASA_ERR_ALIGN;
  int st = check_device();
  if (st) return st;
  return cuda_status(launch_row_norm(static_cast<cudaStream_t>(stream), x, add, gate, add ? x_out : nullptr, weight,
                                     bias, scale, shift, rows, batch_rows, cols, eps, norm != PASA_DIT_RMSNORM,
                                     norm == PASA_DIT_LAYERNORM_PADDED ? padded_cols(cols) - cols : 0, y));
}

int pasa_dit_qkv_rope(void* stream, const void* xq, const void* xk, const void* xv, const float* wq, const float* wk,
                      const double* cos, const double* sin, int64_t batch, int64_t tokens, int heads, int head_dim,
                      float eps, int head_major, void* q, void* k, void* v) {
  if (batch < 1 || tokens < 1 || heads < 1 || head_dim < 8 || head_dim % 8 != 0) return PASA_ERR_SHAPE;
  const int64_t cols = int64_t(heads) * head_dim;
  if (cols > dit_max_cols() || batch * tokens > INT32_MAX) return PASA_ERR_SHAPE;
  if (!std::isfinite(eps) || eps < 0.f) return PASA_ERR_SHAPE;
  if (!xq || !wq || !q || (cos == nullptr) != (sin == nullptr)) return PASA_ERR_NULL;
  if (xk && (!wk || !k)) return PASA_ERR_NULL;
  if (xv && !v) return PASA_ERR_NULL;
  const void* ptrs[] = {xq, xk, xv, wq, wk, cos, sin, q, k, v};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return PASA_ERR_ALIGN;
  int st = check_device();
  if (st) return st;
  return cuda_status(launch_qkv_rope(static_cast<cudaStream_t>(stream), xq, xk, xv, wq, wk, cos, sin, batch, tokens,
                                     int(cols), head_dim, eps, head_major ? 1 : 0, q, xk ? k : nullptr,
                                     xv ? v : nullptr, nullptr, 0, 0));
}

int pasa_dit_qkv_rope_scatter(void* stream, const void* xq, const void* xk, const void* xv, const float* wq,
                              const float* wk, const double* cos, const double* sin, int64_t tokens, int heads,
                              int head_dim, float eps, void* const* peer_table, int n_ranks, int rank) {
  if (tokens < 1 || heads < 1 || head_dim < 8 || head_dim % 8 != 0) return PASA_ERR_SHAPE;
  const int64_t cols = int64_t(heads) * head_dim;
  if (cols > dit_max_cols() || tokens * n_ranks > INT32_MAX) return PASA_ERR_SHAPE;
  if (n_ranks < 1 || n_ranks > 64 || heads % n_ranks != 0 || rank < 0 || rank >= n_ranks) return PASA_ERR_SHAPE;
  if (!std::isfinite(eps) || eps < 0.f) return PASA_ERR_SHAPE;
  if (!xq || !xk || !xv || !wq || !wk || !peer_table || (cos == nullptr) != (sin == nullptr)) return PASA_ERR_NULL;
  const void* ptrs[] = {xq, xk, xv, wq, wk, cos, sin};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return PASA_ERR_ALIGN;
  int st = check_device();
  if (st) return st;
  return cuda_status(launch_qkv_rope(static_cast<cudaStream_t>(stream), xq, xk, xv, wq, wk, cos, sin, 1, tokens,
                                     int(cols), head_dim, eps, 1, nullptr, nullptr, nullptr, peer_table, n_ranks,
                                     rank));
}

}  // extern "C"
