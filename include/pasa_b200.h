/*
 * pasa_b200 — C ABI of the B200 (sm_100a) precision-allocated sparse
 * attention forward.
 *
 * The reference implementation is ZHANGWENTAI/PASA
 * svg/kernels/triton/group_pisa_attention.py.  Each entry point below names
 * the reference interface it replaces.  Conventions shared by all entry
 * points:
 *
 *   - every pointer is a device pointer owned by the caller, except where a
 *     parameter says "host";
 *   - tensors are dense and row-major; q, k, v, o are [B*H, T, D];
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); nothing
 *     synchronises the stream and nothing allocates device memory;
 *   - the return value is a pasa_status (0 = success); a non-zero status
 *     means no kernel was launched, except PASA_ERR_CUDA, which reports a
 *     launch failure of the CUDA runtime.
 *
 * Supported: dtype bf16 or fp32, head_dim 64 or 128, block 64, group 32.
 */
#ifndef PASA_B200_H
#define PASA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PASA_ABI_VERSION 1

#if defined(__GNUC__)
#define PASA_API __attribute__((visibility("default")))
#else
#define PASA_API
#endif

typedef enum pasa_status {
  PASA_OK = 0,
  PASA_ERR_SHAPE = 1,      /* a size or count is out of range            */
  PASA_ERR_DTYPE = 2,      /* unsupported element type                   */
  PASA_ERR_ALIGN = 3,      /* a pointer is not 16-byte aligned           */
  PASA_ERR_DENSITY = 4,    /* density outside (0, 1] or not finite       */
  PASA_ERR_UNSUPPORTED = 5,/* head_dim / block / group not supported     */
  PASA_ERR_WORKSPACE = 6,  /* workspace missing or too small             */
  PASA_ERR_NULL = 7,       /* a required pointer is NULL                 */
  PASA_ERR_CUDA = 8,       /* the CUDA runtime reported an error         */
  PASA_ERR_DEVICE = 9      /* the device is not an sm_100 GPU            */
} pasa_status;

typedef enum pasa_dtype {
  PASA_BF16 = 0,
  PASA_F32 = 1
} pasa_dtype;

/* Attention kernel selection for pasa_attn / pasa_forward. */
typedef enum pasa_attn_kernel {
  PASA_ATTN_AUTO = 0,     /* tcgen05 kernel for bf16, CUDA-core kernel for fp32 */
  PASA_ATTN_TCGEN05 = 1,  /* bf16 only: TMA + tcgen05/TMEM pair-tile kernel     */
  PASA_ATTN_SIMT = 2      /* CUDA-core kernel, one 64-query block per CTA       */
} pasa_attn_kernel;

/* Bits a kernel may set in the caller's error word (see pasa_attn). */
#define PASA_DEVERR_WAIT_TIMEOUT 0x1u  /* a bounded barrier wait gave up */

/* ABI version of the loaded library (PASA_ABI_VERSION). */
PASA_API int pasa_abi_version(void);

/* Static text for a status code. */
PASA_API const char* pasa_status_string(int status);

/*
 * Derived sizes: NT = ceil(T / block), NG = ceil(NT / group) and the number
 * of exactly attended blocks per query block
 * NS = min(max(1, (int)(density * NT)), NT).
 * Replaces the host arithmetic of group_pisa_attention.py:345, :294-299, :373.
 * All outputs are host pointers; any may be NULL.
 */
PASA_API int pasa_derive(int64_t T, int block, int group, double density,
                int64_t* nt, int64_t* ng, int64_t* ns);

/* Bytes of device workspace pasa_forward needs (host output). */
PASA_API int pasa_workspace_size(int64_t B, int64_t H, int64_t T, int D, int dtype,
                        int block, int group, int64_t ns, size_t* bytes);

/*
 * Block statistics.  Replaces fused_chunk_reduce + compute_h_group
 * (group_pisa_attention.py:268-301, kernel :75-129):
 *   qc, kc  [B*H, NG*group, D]  block means (rows >= NT written as zero)
 *   vc      [B*H, NG*group, D]  block sums  (rows >= NT written as zero)
 *   h_norm  [B*H, NT]           fp32 Frobenius norm of k^T v - kc (x) vc
 *   h_group [B*H, NG, D, D]     per-group mean of the per-block matrices
 * qc, kc, vc, h_group have the input dtype.  The per-block matrices
 * themselves are never written to memory.  The bf16 D = 128 kernel waits
 * on its pipeline barriers with a bound; a wait that gives up (a GPU that
 * stopped answering) ends the kernel with its outputs incomplete.  The
 * pasa_forward* entry points report that as PASA_DEVERR_WAIT_TIMEOUT in
 * their error word, like the attention kernel's own waits.
 */
PASA_API int pasa_prep(void* stream, const void* q, const void* k, const void* v,
              int64_t B, int64_t H, int64_t T, int D, int dtype, int block, int group,
              void* qc, void* kc, void* vc, float* h_norm, void* h_group);

/*
 * Covariance-aware top-k block selection.  Replaces
 * group_pisa_attention.py:365-375 (einsum score, log(h_norm + 1e-6) bias,
 * optional noise, torch.topk):
 *   indices  [B*H, NT, ns] int32, best first; equal scores by lower index
 *   sel_mask [B*H, NT, NG] uint32; bit b of word g set when block 32g+b is
 *            among the row's indices (may be NULL)
 * qc, kc are as written by pasa_prep (row stride NG*group).  noise
 * [B*H, NT] fp32 is added to the bias when non-NULL (the reference's
 * use_random draw).  use_cov_bias = 0 ranks by the dot product alone.
 */
PASA_API int pasa_select(void* stream, const void* qc, const void* kc, const float* h_norm,
                const float* noise, int64_t BH, int64_t NT, int D, int dtype,
                float scale, int use_cov_bias, int64_t ns,
                int32_t* indices, uint32_t* sel_mask);

/*
 * Exact attention over the selected blocks plus the zero-order and per-group
 * first-order correction over all other blocks, one online-softmax pass.
 * Replaces pisa_pg_fwd_kernel (group_pisa_attention.py:136-262) and its
 * launch (:380-396).  o is [B*H, T, D] in the input dtype.  err_word
 * (nullable, device uint32) receives PASA_DEVERR_* bits.
 */
PASA_API int pasa_attn(void* stream, const void* q, const void* k, const void* v,
              const void* kc, const void* vc, const void* h_group,
              const int32_t* indices, const uint32_t* sel_mask,
              int64_t BH, int64_t T, int D, int dtype, float scale, int64_t ns,
              void* o, uint32_t* err_word, int kernel);

/*
 * Dense attention o = softmax(q k^T scale) v on the tensor-core kernel, for
 * the layers and timesteps the models run dense (the `full_attention_flag`
 * branch of attention_core_logic, svg/models/wan/attention.py:364-383 and
 * svg/models/hyvideo/attention.py:666-672, which calls SDPA / FlashInfer).
 * It is pisa_pg_attention with every block selected (density 1) without the
 * block statistics, the selection and the correction, whose terms are then
 * exactly zero.  q, k, v, o: [BH, T, D] bf16.
 */
PASA_API int pasa_dense_attn(void* stream, const void* q, const void* k, const void* v,
              int64_t BH, int64_t T, int D, int dtype, float scale,
              void* o, uint32_t* err_word);

/*
 * The whole op, pisa_pg_attention(q, k, v, density, ..., scale,
 * use_cov_bias) (group_pisa_attention.py:307-398) on caller memory:
 * prep -> select -> attention on `stream`.  workspace must hold
 * pasa_workspace_size() bytes, 256-byte aligned.  noise as in pasa_select.
 */
PASA_API int pasa_forward(void* stream, const void* q, const void* k, const void* v,
                 int64_t B, int64_t H, int64_t T, int D, int dtype,
                 double density, float scale, int use_cov_bias, const float* noise,
                 void* workspace, size_t workspace_bytes, void* o, int kernel);

/*
 * pasa_forward restricted to a range of query blocks, for callers that
 * split one call over several GPUs finer than by heads (12 heads over 8
 * GPUs, say).  No counterpart in the reference, which runs the whole op on
 * one device.  The B*H*NT query blocks are numbered head by head
 * (bh * NT + block); [block_begin, block_end) selects some of them.  The
 * heads they touch are prepared and selected whole (a head shared with
 * another range is prepared by both), and only the rows of the selected
 * blocks of o ([B*H, T, D], bf16, tensor-core kernel) are written; every
 * other row of o is left as it was.  The union of disjoint ranges that
 * cover all blocks gives pasa_forward's output bit for bit.
 *   workspace: pasa_forward_range_workspace_size() bytes (256-byte aligned)
 */
PASA_API int pasa_forward_range_workspace_size(int64_t B, int64_t H, int64_t T, int D, int dtype,
                 double density, int64_t block_begin, int64_t block_end, size_t* bytes);
PASA_API int pasa_forward_range(void* stream, const void* q, const void* k, const void* v,
                 int64_t B, int64_t H, int64_t T, int D, int dtype, double density, float scale,
                 int use_cov_bias, const float* noise, void* workspace, size_t workspace_bytes,
                 void* o, int kernel, int64_t block_begin, int64_t block_end);

/* Output layouts of pasa_forward_ex. */
typedef enum pasa_o_layout {
  PASA_O_BHTD = 0,  /* o [B*H, T, D] (head-major), as pasa_forward           */
  PASA_O_BTHD = 1   /* o [B, T, H, D] (token-major): the layout the output
                       projection after the attention reads, so the
                       transpose the reference's processors run after it
                       (attention.py:154, get_o) is not a copy; tcgen05
                       kernel only                                          */
} pasa_o_layout;

/* pasa_forward with the output layout chosen by o_layout (same arguments
 * otherwise; pasa_forward is o_layout = PASA_O_BHTD). */
PASA_API int pasa_forward_ex(void* stream, const void* q, const void* k, const void* v,
                int64_t B, int64_t H, int64_t T, int D, int dtype, double density, float scale,
                int use_cov_bias, const float* noise, void* workspace, size_t workspace_bytes,
                void* o, int kernel, int o_layout);

/*
 * The whole op like pasa_forward, but with no workspace argument and no
 * allocation anywhere: the scratch (block statistics, top-k indices,
 * selection bitmask, error word) is a 32 MiB array built into this library,
 * which every GPU that loads the library holds until the process exits.
 * This entry point has no counterpart in the reference.  It is meant for
 * callers that cannot call cudaMalloc: hosts that own all device memory
 * through their own pool, plugin interfaces that pass no allocator, and
 * latency-critical paths where an allocation's implicit synchronisation is
 * not acceptable.
 *   - Problems whose scratch (pasa_workspace_size) exceeds 32 MiB return
 *     PASA_ERR_WORKSPACE without launching anything.  At D=128, bf16 and
 *     density 0.1 that allows about 11 heads of 75600 tokens per call.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress) and caches it per CUDA context; a call from
 *     another context (one the caller created, or the primary context
 *     again after cudaDeviceReset) resolves it anew.  Make the first call
 *     in each context before any stream capture.
 *   - Every call on a device shares the one array, which keeps the last
 *     call's contents.  Calls whose work overlaps on the GPU (for example on
 *     two streams at once) race on it and must be serialised by the caller.
 * Arguments and results are those of pasa_forward.
 */
PASA_API int pasa_forward_noalloc(void* stream, const void* q, const void* k, const void* v,
                 int64_t B, int64_t H, int64_t T, int D, int dtype,
                 double density, float scale, int use_cov_bias, const float* noise,
                 void* o, int kernel);

/*
 * The whole op on HOST memory: q, k, v and o are [B, H, T, D] host buffers.
 * This entry point has no counterpart in the reference (whose op takes
 * device tensors); it serves callers whose activations live on the host.
 * The heads are split into chunks of heads_per_chunk; chunk i is computed
 * (a pasa_forward call on its heads) while chunk i+1 is copied in and chunk
 * i-1 copied out, on three streams owned by the library.  The result is the
 * one pasa_forward gives on the same heads.
 *   - The call is synchronous: it returns when o holds the result.  Work
 *     queued on `stream` before the call is ordered before it.
 *   - The copies overlap the compute only when the host buffers are
 *     page-locked (cudaHostAlloc / cudaHostRegister).
 *   - workspace: device memory of pasa_forward_host_workspace_size() bytes,
 *     256-byte aligned, not used by anything else during the call.
 *   - noise_h: NULL, or host [B*H, NT] floats as in pasa_select.
 *   - err_bits (nullable, host): the OR of the chunks' PASA_DEVERR_* bits.
 *   - The three streams and their events belong to the library, one set
 *     per device, created on the first call and kept until the process
 *     exits (they do not survive cudaDeviceReset).  Concurrent calls on
 *     one device from several host threads are correct but share these
 *     streams, so they run one after the other on the GPU and each call's
 *     final wait also waits for the others' queued work.
 */
PASA_API int pasa_forward_host_workspace_size(int64_t B, int64_t H, int64_t T, int D, int dtype,
                 double density, int64_t heads_per_chunk, size_t* bytes);
PASA_API int pasa_forward_host(void* stream, const void* q_h, const void* k_h, const void* v_h,
                 int64_t B, int64_t H, int64_t T, int D, int dtype,
                 double density, float scale, int use_cov_bias, const float* noise_h,
                 void* workspace, size_t workspace_bytes, int64_t heads_per_chunk,
                 void* o_h, uint32_t* err_bits, int kernel);

/* Emulated-mask layouts of the head classification (pasa_sample_mse). */
typedef enum pasa_model {
  PASA_MODEL_HUNYUAN = 0,  /* band of floor(1.5 * frame_size / 128) blocks of 128
                              tokens; the context_length text tokens at the tail
                              attend and are attended by everything
                              (svg/models/hyvideo/utils.py:48-94)              */
  PASA_MODEL_WAN = 1       /* band of floor(2 * frame_size / 128) blocks plus the
                              first frame as a sink; no text tokens
                              (svg/models/wan/utils.py:63-110)                 */
} pasa_model;

/*
 * Spatial / temporal head classification.  Replaces sample_mse
 * (svg/models/hyvideo/attention.py:381-405; Wan twin
 * svg/models/wan/attention.py:264-288) and the emulated masks it indexes
 * (get_attention_mask, evaluated in closed form instead of as dense T x T
 * tensors).  For each of the n_rows sampled query positions `rows` (host
 * int64, 1 <= n_rows <= 32, each in [0, T) -- the reference's
 * torch.randint draw), the attention output under the spatial mask, the
 * temporal mask (the spatial band in token-major order) and no mask, with
 * the reference's roundings in the input dtype; then per head the mean
 * squared difference of each masked output from the unmasked one.
 *   q, k, v        [cfg, H, T, D] device, T = context_length +
 *                  num_frame * frame_size (context_length 0 for Wan)
 *   mse            [2, cfg, H] in the input dtype (spatial, temporal), or NULL
 *   best_mask_idx  [cfg, H] int32 argmin (0 spatial, 1 temporal; ties 0), or NULL
 *   workspace      device, pasa_sample_mse_workspace_size() bytes, 256-byte aligned
 */
PASA_API int pasa_sample_mse_workspace_size(int64_t BH, int64_t T, int D, size_t* bytes);
PASA_API int pasa_sample_mse(void* stream, const void* q, const void* k, const void* v,
                 int64_t cfg, int64_t H, int64_t T, int D, int dtype,
                 const int64_t* rows, int64_t n_rows, int model,
                 int64_t context_length, int64_t num_frame, int64_t frame_size,
                 void* workspace, size_t workspace_bytes, void* mse, int32_t* best_mask_idx);

/*
 * Token-layout permutation of the temporal heads (frame-major <-> token-
 * major), text tail untouched.  Replaces hunyuan_sparse_head_placement
 * (svg/models/hyvideo/placement.py:34-153) when inverse = 0 and
 * hunyuan_hidden_states_placement (:285-387) when inverse = 1.
 *   src, dst          [cfg, H, T, D], T = context_length + num_frame*frame_size
 *   head_is_temporal  [cfg, H] int32 (the best_mask_idx of the reference)
 * Spatial heads (0) are copied unchanged.  src and dst must not overlap.
 * Rows of D elements are 16-byte multiples of at most 4096 bytes.
 */
PASA_API int pasa_place(void* stream, const void* src, void* dst, const int32_t* head_is_temporal,
               int64_t cfg, int64_t H, int64_t T, int D, int dtype,
               int64_t context_length, int64_t num_frame, int64_t frame_size, int inverse);

/*
 * DiT row kernels around the attention op (bf16 activations, fp32 per-channel
 * vectors, one 16-byte vector per element group: cols % 8 == 0, cols <= 8192,
 * every pointer 16-byte aligned).
 *
 * Gated residual + LayerNorm / RMSNorm + affine + modulation in one pass.
 * Replaces, for one row of cols elements, the reference's
 * triton_modulate_gate_residual_forward (svg/kernels/triton/modulate.py:90-164),
 * triton_layernorm_forward (layernorm.py:13-218), triton_modulate_shift_forward
 * (modulate.py:12-85) and triton_rmsnorm_forward (rmsnorm.py:8-100), as the
 * Wan block chains them (svg/models/wan/custom_models.py:38-111):
 *   x' = add ? bf16(x + add * gate) : x        (gate NULL: plain add)
 *   x_out = x'                                  (when add and x_out are given; may alias x)
 *   y  = bf16(((x' - mean) * rstd) [* weight] [+ bias] [* (1 + scale) + shift])
 * with rstd = 1 / sqrt(ssq / cols + eps) and, by `norm`:
 *   PASA_DIT_RMSNORM           mean = 0, ssq = sum(x'^2)                (rmsnorm.py:31-35)
 *   PASA_DIT_LAYERNORM         mean = sum(x') / cols, ssq = sum((x' - mean)^2)
 *                              (the torch FP32LayerNorm the block runs without
 *                              the fast kernels, custom_models.py:45)
 *   PASA_DIT_LAYERNORM_PADDED  as LAYERNORM plus (P - cols) * mean^2, P = cols
 *                              rounded up to a power of two: the reference's
 *                              Triton LayerNorm sums its zero padding into the
 *                              variance (layernorm.py:40-42, :138-140)
 *   x, add, x_out, y  [rows, cols] bf16
 *   gate, scale, shift [rows / batch_rows, cols] fp32 (row r uses entry r / batch_rows)
 *   weight, bias      [cols] fp32 (NULL: omitted)
 * scale and shift are given together or not at all.
 */
typedef enum pasa_dit_norm {
  PASA_DIT_RMSNORM = 0,
  PASA_DIT_LAYERNORM = 1,
  PASA_DIT_LAYERNORM_PADDED = 2
} pasa_dit_norm;

PASA_API int pasa_dit_row_norm(void* stream, const void* x, const void* add, const float* gate, void* x_out,
              const float* weight, const float* bias, const float* scale, const float* shift,
              int64_t rows, int64_t batch_rows, int cols, float eps, int norm, void* y);

/*
 * Self-attention producer: RMSNorm of the q and k rows over cols = heads *
 * head_dim, the rotary embedding of every head's (2i, 2i+1) pairs as an fp64
 * complex multiply, and the transpose to head-major.  Replaces get_qk_norm,
 * get_transpose_qkv and apply_rotary_emb of the Wan processor
 * (svg/models/wan/attention.py:122-149 and its torch rotary path :49-57):
 *   xq, xk, xv  [batch, tokens, cols] bf16 (xk / xv may be NULL: skipped)
 *   wq, wk      [cols] fp32 RMSNorm weights
 *   cos, sin    [tokens, head_dim / 2] fp64, or both NULL (no rotation)
 *   q, k, v     head_major ? [batch, heads, tokens, head_dim] : [batch, tokens, cols]
 * q = bf16(rotate(bf16(xq * rstd * wq))), rotate in fp64 and rounded to bf16
 * through fp32; v is copied.  Outputs must not overlap the inputs.
 */
PASA_API int pasa_dit_qkv_rope(void* stream, const void* xq, const void* xk, const void* xv,
              const float* wq, const float* wk, const double* cos, const double* sin,
              int64_t batch, int64_t tokens, int heads, int head_dim, float eps, int head_major,
              void* q, void* k, void* v);

/*
 * Fused Ulysses exchange of the DiT step (no reference counterpart: the
 * reference has no collectives).  With P ranks, rank r holds tokens
 * [r*L, (r+1)*L) of the sequence (L = tokens per rank) and attends heads
 * [r*H/P, (r+1)*H/P).  Peer buffers are allocated by the library and shared
 * through CUDA IPC handles (PASA_PEER_HANDLE_BYTES each, exchanged by the
 * caller, e.g. an all-gather); kernels store into them over NVLink with plain
 * peer stores.  The caller orders the kernels across ranks (a stream-ordered
 * barrier collective after each scatter, before the buffers are read).
 */
#define PASA_PEER_HANDLE_BYTES 64

/* cudaMalloc `bytes` and export its IPC handle (host buffer of
 * PASA_PEER_HANDLE_BYTES). */
PASA_API int pasa_peer_alloc(size_t bytes, void** ptr, void* handle);
PASA_API int pasa_peer_free(void* ptr);
/* Map another process's buffer from its handle (same node); pasa_peer_close
 * unmaps it. */
PASA_API int pasa_peer_open(const void* handle, void** ptr);
PASA_API int pasa_peer_close(void* ptr);

/*
 * pasa_dit_qkv_rope for one batch entry, with the head-major outputs
 * scattered to the ranks that attend them: the row of head h and local
 * token t goes to rank h / (H/P), whose buffer peer_table[rank] holds
 * [3][H/P][P*tokens][D] (q, k, v), at token rank*tokens + t.  peer_table is
 * a DEVICE array of P pointers (this rank's own buffer included).
 * Replaces the producer + sequence-to-head all-to-all.
 */
PASA_API int pasa_dit_qkv_rope_scatter(void* stream, const void* xq, const void* xk, const void* xv,
              const float* wq, const float* wk, const double* cos, const double* sin,
              int64_t tokens, int heads, int head_dim, float eps,
              void* const* peer_table, int n_ranks, int rank);

/*
 * pasa_forward (B = 1, bf16, tcgen05) on this rank's H_local heads over all T
 * tokens, with every output row stored at its token's owner: token t goes to
 * rank t / (T/P), whose buffer o_peer_table[rank] holds [T/P][heads_total][D]
 * (token-major, the output projection's layout), at head head0 + h.
 * Replaces the attention + head-to-sequence all-to-all.
 */
PASA_API int pasa_forward_scatter(void* stream, const void* q, const void* k, const void* v,
              int64_t H_local, int64_t T, int D, double density, float scale, int use_cov_bias,
              const float* noise, void* workspace, size_t workspace_bytes,
              void* const* o_peer_table, int n_ranks, int64_t head0, int64_t heads_total, int kernel);

#ifdef __cplusplus
}
#endif

#endif /* PASA_B200_H */
