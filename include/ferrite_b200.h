/*
 * ferrite_b200.h -- C ABI of the B200 (sm_100a) kernels behind ferrite's three
 * hot-path operators: causal flash attention (forward, delta prep, dK/dV, dQ),
 * fused residual-add + RMSNorm (forward and backward) and the blocked matmul.
 *
 * Conventions shared by every entry point
 *   - All tensor arguments are DEVICE pointers, row-major, densely packed unless a
 *     leading-dimension argument says otherwise.  Nothing is allocated, freed or
 *     synchronised: work is enqueued on `stream` (a cudaStream_t passed as void*,
 *     NULL = legacy default stream) and the call returns.
 *   - Return value: FERRITE_OK (0) or one of the ferrite_status codes below.  On a
 *     non-zero return nothing was launched and ferrite_last_error() describes why
 *     (thread-local string).
 *   - dtype codes: FERRITE_F32, FERRITE_BF16, FERRITE_F16 (storage types; all
 *     statistics and accumulators are f32).
 *   - Kernels that wait on an mbarrier bound every wait; a wait that runs out sets
 *     a device-side status word that ferrite_device_status() reads back as
 *     FERRITE_DEVICE_TIMEOUT.
 *
 * Each declaration names the reference interface it replaces (file:line inside
 * anxnd2211/ferrite-tpu).  In the reference every one of these is a
 * `pl.pallas_call` (or an XLA fusion) inside a `jax.custom_vjp`.
 */
#ifndef FERRITE_B200_H_
#define FERRITE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(FERRITE_BUILD) && defined(__GNUC__)
#define FERRITE_API __attribute__((visibility("default")))
#else
#define FERRITE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  FERRITE_OK = 0,
  FERRITE_BAD_SHAPE = 1,         /* a size, stride or block argument is invalid   */
  FERRITE_UNSUPPORTED_DTYPE = 2, /* dtype combination not implemented            */
  FERRITE_LAUNCH_FAILED = 3,     /* cudaGetLastError() after the launch           */
  FERRITE_DEVICE_TIMEOUT = 4,    /* a bounded device-side wait expired            */
  FERRITE_BAD_ALIGNMENT = 5,     /* a pointer/stride breaks a TMA or vector rule  */
  FERRITE_WORKSPACE_TOO_SMALL = 6,
  FERRITE_INJECTED_FAULT = 7     /* host-side fault injection (FERRITE_FAULT_INJECT) */
} ferrite_status;

typedef enum { FERRITE_F32 = 0, FERRITE_BF16 = 1, FERRITE_F16 = 2 } ferrite_dtype;

/* ---- library / error plumbing ------------------------------------------------ */

/* Human-readable description of the last non-zero status on this host thread. */
FERRITE_API const char* ferrite_last_error(void);
/* Library version string, e.g. "ferrite_b200 0.1.0 sm_100a". */
FERRITE_API const char* ferrite_version(void);
/* Synchronises `stream`, then returns the device status word of the current device
 * (FERRITE_OK or FERRITE_DEVICE_TIMEOUT) and, if `clear` != 0, resets it. */
FERRITE_API int ferrite_device_status(void* stream, int clear);

/* Exercises the bounded-wait failure path of the tensor-core kernels: one CTA holds
 * a TMEM allocation and waits on an mbarrier that nothing arrives on, for at most
 * `limit_ns` (0 < limit_ns <= the library's 2 s bound).  The wait expires, the
 * status word reads FERRITE_DEVICE_TIMEOUT, the other waiters leave through the
 * CTA's abort flag and TMEM is freed before the CTA exits.  `out` is 4 u64 on the
 * device: ns waited, 1 if the wait reported a timeout, waiters that left (4),
 * 1 once TMEM was freed.  No counterpart kernel in the reference: its stand-in is
 * the interpret-mode data-race detector run over the kernels
 * (tests/test_flash_attention.py:79-85); Mosaic kernels have no device waits. */
FERRITE_API int ferrite_wait_probe(void* stream, uint64_t limit_ns, void* out);

/* ---- fused residual-add + RMSNorm ------------------------------------------- */

/* y = x * rsqrt(mean(x^2) + eps) * w over the last axis of x[rows, dim].
 * x, y: dtype `dtype`; w: dtype `w_dtype` (f32 or bf16); statistics in f32.
 * Replaces ferrite_rmsnorm: rmsnorm.py:46-49 (_rmsnorm_kernel) via _call
 * rmsnorm.py:77-110 with n_out=1. */
FERRITE_API int ferrite_rmsnorm_fwd(void* stream, const void* x, const void* w, void* y,
                        int64_t rows, int64_t dim, float eps, int dtype,
                        int w_dtype);

/* h = x + r (f32, stored rounded to dtype); y = h * rsqrt(mean(h^2)+eps) * w,
 * computed from the UNROUNDED f32 h.  Replaces ferrite_add_rmsnorm:
 * rmsnorm.py:52-56 (_add_rmsnorm_kernel) via _call rmsnorm.py:77-110, n_out=2. */
FERRITE_API int ferrite_add_rmsnorm_fwd(void* stream, const void* x, const void* r,
                            const void* w, void* h, void* y, int64_t rows,
                            int64_t dim, float eps, int dtype, int w_dtype);

/* Bytes of scratch ferrite_rmsnorm_bwd needs for (rows, dim): per-CTA f32
 * partial sums of dw, reduced deterministically by a second kernel. */
FERRITE_API size_t ferrite_rmsnorm_bwd_workspace_size(int64_t rows, int64_t dim);

/* RMSNorm backward from the saved (rounded) input h:
 *   inv = rsqrt(mean(h^2)+eps), xhat = h*inv, g = dy*w,
 *   dh  = inv * (g - xhat * mean(g*xhat)) [+ dh_direct],   dw = sum_rows dy*xhat.
 * dh_direct may be NULL (plain rmsnorm).  dh has dtype `dtype`, dw has `w_dtype`.
 * Replaces the XLA backward of the reference: rmsnorm.py:159-166
 * (_rmsnorm_bwd_math), rmsnorm.py:148-153 (_add_norm_bwd: returns dh twice) and
 * rmsnorm.py:128-131 (_norm_bwd). */
FERRITE_API int ferrite_rmsnorm_bwd(void* stream, const void* h, const void* w,
                        const void* dy, const void* dh_direct, void* dh,
                        void* dw, void* workspace, size_t workspace_bytes,
                        int64_t rows, int64_t dim, float eps, int dtype,
                        int w_dtype);

/* Allocation-free variant of ferrite_rmsnorm_bwd (same arguments minus the
 * workspace).  No counterpart in the reference: it exists for callers that cannot
 * allocate device memory -- a host framework that owns all device memory and
 * gives its kernels no scratch allocator, or a runtime that sizes its device
 * arena once and allows no allocation afterwards (cudaMalloc/cudaFree can
 * synchronise the device and are not stream-ordered).  The dw partial sums live
 * in a library-owned device array of 2^20 floats (4 MiB, held on every GPU that
 * loads the library until the process exits); dim above 131072 is rejected with
 * FERRITE_BAD_SHAPE.  The first call on a device looks the array's address up
 * (that device must be current); make it before any stream capture.  All calls
 * share the array, so calls that overlap on the GPU (e.g. on two streams) race;
 * nothing in it needs clearing between calls. */
FERRITE_API int ferrite_rmsnorm_bwd_noalloc(void* stream, const void* h, const void* w,
                        const void* dy, const void* dh_direct, void* dh,
                        void* dw, int64_t rows, int64_t dim, float eps,
                        int dtype, int w_dtype);

/* ---- matmul ---------------------------------------------------------------- */

/* C[M,N] = op(A)[M,K] @ op(B)[K,N] with an f32 accumulator, cast to c_dtype.
 *   trans_a = 0: A stored [M,K] (row stride lda);  1: A stored [K,M] (stride lda)
 *   trans_b = 0: B stored [K,N] (row stride ldb);  1: B stored [N,K] (stride ldb)
 * C stored [M,N] with row stride ldc.  ab_dtype is the operand dtype (both the
 * same); bf16/f16 run on tcgen05 tensor cores (kind::f16, f32 accumulator in
 * TMEM); f32 runs an exact-f32 CUDA-core path (the Precision.HIGHEST contract).
 * Any M, N, K >= 1 is accepted (ragged edges are zero-filled by TMA, no padding
 * copies).  Replaces ferrite_matmul: matmul.py:27-38 (_matmul_kernel) via
 * _matmul_impl matmul.py:52-86; the transposed forms serve the VJP
 * matmul.py:99-104 without materialised transposes. */
FERRITE_API int ferrite_gemm(void* stream, const void* a, const void* b, void* c,
                 int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                 int64_t ldc, int trans_a, int trans_b, int ab_dtype,
                 int c_dtype);

/* bf16 GEMM with the GPT MLP's activation fused into the epilogue (no
 * reference kernel counterpart: the reference applies jax.nn.gelu(approximate=
 * True) between two ferrite_matmul calls, gpt.py:141):
 *   epilogue 1 (GELU):     c = u = A B rounded, aux = gelu_tanh(u) rounded
 *                          (A [M][K], B [K][N]: trans_a = trans_b = 0);
 *   epilogue 2 (GELU_BWD): c = round(round(A B^T) * gelu_tanh'(aux)), aux = u
 *                          (dU from dA = dP W2^T: trans_a = 0, trans_b = 1).
 * Both run on the tensor-core path (16-byte aligned operands and strides, m, n >=
 * 128, k >= 64); epilogue 1 also runs for decode-sized products (m <= 16, B 16-byte
 * aligned with n and ldb multiples of 8) on the skinny CUDA path.  Other shapes
 * return FERRITE_UNSUPPORTED_DTYPE. */
FERRITE_API int ferrite_gemm_epilogue(void* stream, const void* a, const void* b, void* c,
                          int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                          int64_t ldc, int trans_a, int trans_b, int epilogue,
                          void* aux, int64_t ld_aux);

/* Residual-add + RMSNorm folded in front of a skinny product, one launch (the
 * decode step's norm feeding its next linear; no reference kernel counterpart: the
 * reference runs ferrite_rmsnorm -- rmsnorm.py:52-56, add_rmsnorm -- then a matmul,
 * engine.py:107-131 / gpt.py:131-143):
 *   h = x + r (f32; x alone when r is null), y = round(h * rsqrt(mean(h^2) + eps) * w),
 *   c = y op(B) with an f32 accumulator (op as ferrite_gemm's trans_b), and h_out =
 *   round(h) when given (it needs r, and must not overlap x or r).
 * x, r, h_out: [m][k] with row stride ldx (a multiple of 8), 16-byte aligned; w_norm: f32
 * [k], 16-byte aligned; m <= 16, k a multiple of 8; ab_dtype bf16 or f16, c_dtype the
 * same or f32.  epilogue 1 (GELU, bf16, B stored [K][N]): c = u rounded, aux =
 * gelu_tanh(u) rounded, as ferrite_gemm_epilogue. */
FERRITE_API int ferrite_gemm_rmsnorm(void* stream, const void* x, const void* r, const float* w_norm, float eps,
                          void* h_out, const void* b, void* c, int64_t m, int64_t n, int64_t k,
                          int64_t ldx, int64_t ldb, int64_t ldc, int trans_b, int epilogue, void* aux,
                          int64_t ld_aux, int ab_dtype, int c_dtype);

/* Bytes of f32 scratch ferrite_gemm_ws can use for a split-K launch of this
 * shape on the current device (0: the shape gets no split).  Splitting K helps
 * when the output has fewer tiles than the GPU has SMs -- the weight gradients
 * dW = X^T G of the reference's VJP (matmul.py:99-104) at transformer shapes
 * (M x N = d_model x d_ff, K = tokens). */
FERRITE_API size_t ferrite_gemm_workspace_size(int64_t m, int64_t n, int64_t k,
                                   int64_t lda, int64_t ldb, int trans_a,
                                   int trans_b, int ab_dtype);

/* ferrite_gemm with caller-provided scratch (256-byte aligned): with at least
 * ferrite_gemm_workspace_size() bytes the K range of each output tile is split
 * over several SMs, the f32 partials are summed in a fixed order (results are
 * run-to-run deterministic) and rounded once; with less, it behaves exactly
 * like ferrite_gemm.  Replaces the same reference kernel as ferrite_gemm. */
FERRITE_API int ferrite_gemm_ws(void* stream, const void* a, const void* b, void* c,
                    int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                    int64_t ldc, int trans_a, int trans_b, int ab_dtype,
                    int c_dtype, void* workspace, size_t workspace_bytes);

/* ---- causal flash attention ------------------------------------------------ */

/* Shapes: q [b, h, sq, d], k/v [b, h, sk, d], all of dtype `dtype`, densely
 * packed (the *_strided forms below take other layouts).  lse/delta are f32 [b, h, sq] (the reference keeps them
 * lane-replicated as [b, h, sq, 128]; that layout is internal to its custom_vjp
 * residuals, so the compact one is a drop-in).  block_q/block_k are the caller's
 * BlockSizes; the kernels validate them exactly like _validate
 * (flash_attention.py:336-353) and tile internally. */

/* o = softmax(scale * q k^T [causal mask]) v, lse = m + log(l).
 * Replaces ferrite_flash_attention_fwd: flash_attention.py:91-127
 * (_fwd_kernel) via _flash_forward flash_attention.py:130-175. */
FERRITE_API int ferrite_attn_fwd(void* stream, const void* q, const void* k, const void* v,
                     void* o, float* lse, int64_t b, int64_t h, int64_t sq,
                     int64_t sk, int64_t d, float scale, int causal,
                     int block_q, int block_k, int dtype);

/* delta[b,h,s] = sum_d dO*O in f32.  Replaces the XLA fusion at
 * flash_attention.py:328-329 (_flash_bwd). */
FERRITE_API int ferrite_attn_bwd_prep(void* stream, const void* dout, const void* out,
                          float* delta, int64_t b, int64_t h, int64_t s,
                          int64_t d, int dtype);

/* dK = scale * sum_q dS^T Q, dV = sum_q P^T dO (no atomics; one CTA per key
 * tile).  Replaces ferrite_flash_attention_bwd_dkv: flash_attention.py:197-221
 * with the grid of flash_attention.py:253-279. */
FERRITE_API int ferrite_attn_bwd_dkv(void* stream, const void* q, const void* k,
                         const void* v, const void* dout, const float* lse,
                         const float* delta, void* dk, void* dv, int64_t b,
                         int64_t h, int64_t sq, int64_t sk, int64_t d,
                         float scale, int causal, int block_q, int block_k,
                         int dtype);

/* dQ = scale * sum_k dS K (no atomics; one CTA per query tile).  Replaces
 * ferrite_flash_attention_bwd_dq: flash_attention.py:224-243 with the grid of
 * flash_attention.py:281-306. */
FERRITE_API int ferrite_attn_bwd_dq(void* stream, const void* q, const void* k,
                        const void* v, const void* dout, const float* lse,
                        const float* delta, void* dq, int64_t b, int64_t h,
                        int64_t sq, int64_t sk, int64_t d, float scale,
                        int causal, int block_q, int block_k, int dtype);

/* ---- softmax cross-entropy (the GPT loss) --------------------------------- */

/* lse[r] = log sum_c exp(logits[r, c]) and nll[r] = lse[r] - logits[r, t[r]] over
 * f32 logits [rows, vocab] (row stride ld elements); targets int32
 * (target_dtype 0) or int64 (1).  A target outside [0, vocab) gives nll = NaN.
 * Replaces the loss of the reference's training step: jax.nn.log_softmax and
 * the target gather in loss_fn, model/gpt.py:147-152 (the mean of nll is left
 * to the caller).  No reference kernel counterpart: the reference runs this in
 * XLA. */
FERRITE_API int ferrite_xent_fwd(void* stream, const float* logits, const void* targets,
                     float* lse, float* nll, int64_t rows, int64_t vocab, int64_t ld,
                     int target_dtype);

/* dlogits[r, c] = g * (exp(logits[r, c] - lse[r]) - [c == t[r]]) with
 * g = (*dloss) * scale (dloss a device scalar, NULL meaning 1; scale = 1/rows
 * for a mean), written as out_dtype (FERRITE_BF16 for the LM-head GEMMs) with
 * row stride ld_out.  The backward of loss_fn (gpt.py:147-152) in one pass. */
FERRITE_API int ferrite_xent_bwd(void* stream, const float* logits, const void* targets,
                     const float* lse, const float* dloss, float scale, void* dlogits,
                     int64_t rows, int64_t vocab, int64_t ld, int64_t ld_out,
                     int target_dtype, int out_dtype);

/* ---- AdamW over flat parameters --------------------------------------------- */

/* Bytes of scratch ferrite_adamw_step needs for n elements (the grad-norm
 * partials). */
FERRITE_API size_t ferrite_adamw_workspace_size(int64_t n);

/* One AdamW step with global-norm clipping over flat f32 buffers of n elements
 * (params, grads, m, v; 16-byte aligned), the reference's adamw_update
 * (model/train.py:59-74) on the gradients g = grad_scale * grads (grad_scale =
 * 1 / ranks turns a summed all-reduce into the mean): gnorm = ||g||_2,
 * g' = g * min(1, clip / (gnorm + 1e-6)), m = b1 m + (1-b1) g', v = b2 v + (1-b2) g'^2,
 * p -= lr ((m / (1-b1^step)) / (sqrt(v / (1-b2^step)) + eps) + wd p), with the
 * decay term on elements [0, n_decay) only (the caller lays out the ndim >= 2
 * parameters first).  gnorm is written to *gnorm_out (device, may be NULL).
 * Deterministic (fixed-order norm reduction, no atomics). */
FERRITE_API int ferrite_adamw_step(void* stream, float* params, const float* grads, float* m,
                       float* v, int64_t n, int64_t n_decay, float lr, float b1, float b2,
                       float eps, float weight_decay, int64_t step, float clip,
                       float grad_scale, float* gnorm_out, void* workspace,
                       size_t workspace_bytes);

/* ---- strided flash attention ----------------------------------------------- */

/* Element strides (batch, head, sequence) of each [b, h, s, d] operand; d is
 * unit-stride.  Each call reads the fields of the operands it takes:
 * fwd q,k,v,o; bwd_prep dout,o; bwd_dkv q,k,v,dout,dk,dv; bwd_dq q,k,v,dout,dq.
 * Contiguous [b, h, s, d] is {h*s*d, s*d, d}.  The packed projection of a
 * transformer block, [b, s, 3, h, d] (q, k, v slots), is read in place with
 * {3*s*h*d, d, 3*h*d} at base + slot*h*d, and an output written as [b, s, h, d]
 * (ready for the output projection) has {s*h*d, d, h*d}.  The tensor-core path
 * needs 16-byte aligned bases and strides that are multiples of 8 elements;
 * other layouts run the CUDA-core path.  Strides must be non-negative. */
typedef struct ferrite_attn_strides {
  int64_t q[3], k[3], v[3], o[3], dout[3], dq[3], dk[3], dv[3];
} ferrite_attn_strides;

/* The four entry points above on strided operands.  They replace the same
 * reference kernels; the strided forms fold the head split and q/k/v
 * transposes of the reference's attention caller (gpt.py:136-138, which
 * transposes [b, s, h, d] to [b, h, s, d] before flash_attention) into the
 * kernels' tensor maps. */
FERRITE_API int ferrite_attn_fwd_strided(void* stream, const void* q, const void* k,
                             const void* v, void* o, float* lse,
                             const ferrite_attn_strides* strides, int64_t b, int64_t h,
                             int64_t sq, int64_t sk, int64_t d, float scale, int causal,
                             int block_q, int block_k, int dtype);
FERRITE_API int ferrite_attn_bwd_prep_strided(void* stream, const void* dout, const void* out,
                                  float* delta, const ferrite_attn_strides* strides,
                                  int64_t b, int64_t h, int64_t s, int64_t d, int dtype);
FERRITE_API int ferrite_attn_bwd_dkv_strided(void* stream, const void* q, const void* k,
                                 const void* v, const void* dout, const float* lse,
                                 const float* delta, void* dk, void* dv,
                                 const ferrite_attn_strides* strides, int64_t b, int64_t h,
                                 int64_t sq, int64_t sk, int64_t d, float scale, int causal,
                                 int block_q, int block_k, int dtype);
FERRITE_API int ferrite_attn_bwd_dq_strided(void* stream, const void* q, const void* k,
                                const void* v, const void* dout, const float* lse,
                                const float* delta, void* dq,
                                const ferrite_attn_strides* strides, int64_t b, int64_t h,
                                int64_t sq, int64_t sk, int64_t d, float scale, int causal,
                                int block_q, int block_k, int dtype);

/* ---- attention backward with a materialised dS ------------------------------ */

/* Bytes of scratch that lets ferrite_attn_bwd_ds process all b*h slices in one
 * pass: the bf16/f16 dS^T of every slice, [sk][sq rounded up to 64] (0 when the
 * shape cannot take the tensor-core path). */
FERRITE_API size_t ferrite_attn_bwd_ds_workspace_size(int64_t b, int64_t h, int64_t sq,
                                          int64_t sk, int64_t d, int dtype);

/* The whole attention backward after delta prep: dK, dV and dQ.  The dK/dV
 * kernel also writes the dS it forms (rounded to the input dtype, the values the
 * reference feeds its dQ product, flash_attention.py:234) into the workspace, and
 * dQ = scale * dS K is then one tensor-core GEMM per slice instead of a second
 * recomputation of S, P, dP and dS (flash_attention.py:224-243) -- still without
 * atomics.  Slices are processed in chunks of as many as fit in workspace_bytes
 * (256-byte aligned); with less than one slice, or layouts/dtypes the tensor
 * cores cannot read, it runs ferrite_attn_bwd_dkv_strided +
 * ferrite_attn_bwd_dq_strided.  Replaces the pair of backward pallas_calls of
 * _flash_bwd, flash_attention.py:253-306. */
FERRITE_API int ferrite_attn_bwd_ds(void* stream, const void* q, const void* k, const void* v,
                        const void* dout, const float* lse, const float* delta, void* dq,
                        void* dk, void* dv, const ferrite_attn_strides* strides,
                        void* workspace, size_t workspace_bytes, int64_t b, int64_t h,
                        int64_t sq, int64_t sk, int64_t d, float scale, int causal,
                        int block_q, int block_k, int dtype);

/* The two halves of ferrite_attn_bwd_ds, for callers that schedule them (or
 * time them) separately, on the slice range [bh_begin, bh_begin + bh_count) of
 * the flattened batch*head index.  ds is [bh_count][sk][sq rounded up to 64]
 * (256-byte aligned); both need the tensor-core path and return
 * FERRITE_UNSUPPORTED_DTYPE otherwise.  dkv_ds: dK, dV as ferrite_attn_bwd_dkv
 * (flash_attention.py:197-221) plus dS^T; dq_ds: dQ = scale * dS K
 * (replaces flash_attention.py:224-243). */
FERRITE_API int ferrite_attn_bwd_dkv_ds(void* stream, const void* q, const void* k,
                            const void* v, const void* dout, const float* lse,
                            const float* delta, void* dk, void* dv, void* ds,
                            const ferrite_attn_strides* strides, int64_t bh_begin,
                            int64_t bh_count, int64_t b, int64_t h, int64_t sq,
                            int64_t sk, int64_t d, float scale, int causal,
                            int block_q, int block_k, int dtype);
FERRITE_API int ferrite_attn_bwd_dq_ds(void* stream, const void* ds, const void* k, void* dq,
                           const ferrite_attn_strides* strides, int64_t bh_begin,
                           int64_t bh_count, int64_t b, int64_t h, int64_t sq,
                           int64_t sk, int64_t d, float scale, int causal, int block_q,
                           int block_k, int dtype);

/* ---- decode attention against a static KV cache ------------------------------ */

/* One greedy-decode step of attention for a new token per batch row:
 *   k_cache[b, h, pos[b], :] = k_new[b, h, :];  v_cache likewise      (if k_new != NULL)
 *   o[b, h, :] = softmax_j(scale * q[b, h] . k_cache[b, h, j]) v_cache[b, h, j], j <= pos[b]
 * in f32, cast to dtype.  q, k_new, v_new: row (b, h) at element b * ld_new + h * d (the
 * [b, 3, h, d] qkv projection is read in place with ld_new = 3 * h * d); k_cache and
 * v_cache: one layer of the cache, [b, h, max_len, d], densely packed; pos: int64
 * [b] on the device; o: [b, h, d], densely packed.  k_new and v_new are both given
 * or both NULL (NULL: the cache is only read).  dtype bf16 or f16 with d in {32, 64,
 * 128, 256}, or f32 with d in {32, 64, 128}; all pointers 16-byte aligned and ld_new *
 * element size a multiple of 16.  A pos[b] outside [0, max_len) writes nothing and
 * gives o = NaN for that row.  Positions after pos[b] are never read (the reference
 * masks them to -1e30, a softmax weight of exactly 0).  Replaces the reference's
 * decode step attention, which runs in XLA: _write_cache (serving/engine.py:98-104)
 * followed by _cache_attention (serving/engine.py:89-95). */
FERRITE_API int ferrite_attn_decode(void* stream, const void* q, const void* k_new,
                        const void* v_new, void* k_cache, void* v_cache, const int64_t* pos,
                        void* o, int64_t b, int64_t h, int64_t max_len, int64_t d,
                        int64_t ld_new, float scale, int dtype);

/* The thread-block cluster size (1, 2, 4 or 8 CTAs per (batch, head) slice) that
 * ferrite_attn_decode launches for `bh` = b * h slices of a `max_len`-row cache of
 * head_dim `d` and dtype `dtype` on a GPU with `slots` resident CTAs (SMs x CTAs per
 * SM): the largest C whose grid of bh * C CTAs fits in one wave while every CTA keeps
 * at least one row per lane group.  Host-only (launches nothing); returns -1 with
 * the error set for invalid arguments.  No counterpart in the reference, whose
 * decode attention is an XLA fusion (serving/engine.py:89-95). */
FERRITE_API int ferrite_attn_decode_cluster(int64_t bh, int64_t max_len, int64_t d, int dtype,
                                            int64_t slots);

#ifdef __cplusplus
}
#endif
#endif /* FERRITE_B200_H_ */
