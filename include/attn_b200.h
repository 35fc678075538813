/*
 * attn_b200.h — C ABI of the B200 (sm_100a) causal multi-head attention library.
 *
 * Replaces the kernels and host NumPy that llm-gpu-5's MultiHeadAttention runs today:
 *   - fused_attention_forward_kernel   core/mha_kernels.py:404-521  (launched at model/gpt.py:587-592)
 *   - the NumPy attention backward     model/gpt.py:652-689
 *   - matmul_2d_kernel projections     core/kernels.py:119-140      (model/gpt.py:558, :629)
 *   - split_heads_kernel / merge_heads_kernel  core/mha_kernels.py:534-584 (model/gpt.py:578-598)
 *   - the unwired GPU grad kernels     core/mha_kernels.py:195-236, 592-680
 *
 * Conventions shared by every entry point:
 *   - All pointers are raw device addresses; buffers are allocated by the caller.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Return value: ATTN_OK (0) or a negative ATTN_ERR_* code.  On a bad argument nothing is
 *     launched.  attn_last_error_string() describes the last failure of the calling thread.
 *   - Attention tensors are addressed by element strides: element (b, t, h, d) of Q/K/V/dQ/dK/dV
 *     lives at ptr[b*sb + t*st + h*sh + d] (d contiguous).  Both the reference's split layout
 *     [B*NH, T, D] (sb = NH*T*D, st = D, sh = T*D) and the token layout of the fused projection
 *     [B*T, 3C] (sb = T*3C, st = 3C, sh = D, K at +C, V at +2C) are expressible, so the head
 *     split/merge of the reference can be folded into addressing.
 *   - lse is float32 [B, NH, T] (natural-log log-sum-exp of the scaled causal scores per row);
 *     the backward recomputes P = exp(scale*q.k - lse) instead of storing the T x T matrix.
 *
 * Environment variables, read once at the library's first launch of the kind concerned:
 *   ATTN_NO_PDL=1      launch every kernel without programmatic stream serialization (by default
 *                      a kernel's CTAs may do their set-up while its predecessor on the stream
 *                      drains; each waits for the predecessor before touching memory)
 *   ATTN_GEMM_PAIRS=1  run the bf16 tensor-core GEMMs with at least 256 rows on pairs of SMs
 *                      (256x256 tiles per cluster of two CTAs) instead of one 128x256 tile per SM
 */
#ifndef ATTN_B200_H
#define ATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ATTN_OK 0
#define ATTN_ERR_ARG (-1)         /* invalid argument: null pointer, bad shape, bad stride   */
#define ATTN_ERR_UNSUPPORTED (-2) /* valid but not implemented (e.g. head_dim > 128)          */
#define ATTN_ERR_CUDA (-3)        /* a CUDA runtime/driver call failed                        */
#define ATTN_ERR_WORKSPACE (-4)   /* workspace missing or smaller than *_workspace_size()     */

#define ATTN_F32 0  /* float32                       */
#define ATTN_BF16 1 /* bfloat16 (stored as uint16_t) */
#define ATTN_TF32 2 /* float32 storage, multiplied on the tensor cores as tf32 (10-bit mantissa)
                       with float32 accumulation; shapes the tensor-core kernels do not take run
                       the exact float32 CUDA-core path */

/*
 * Data-parallel gradient all-reduce (SUM) over NVSwitch multicast.  No counterpart in the
 * reference, which trains on one GPU (its scaling is gradient accumulation, auto_train.py:
 * 1591-1615); it sums the flat float32 gradient buffer [dWqkv | dbqkv | dWo | dbo] (or the
 * FeedForward's) over the ranks, so every rank holds the full-batch gradient of
 * model/gpt.py:687-694.  One launch per rank, on `stream`, after the kernels that wrote the
 * gradients; every rank of the group must call it with the same n and world.
 *   multicast    the buffer's multicast address (symmetric memory bound to an NVLink multicast
 *                object, n float32 per rank, 16-byte aligned); the sum is written back to every
 *                rank's buffer through it
 *   signal_pads  device address of an array of `world` pointers, rank p's uint32 signal pad at
 *                [p]; each pad holds at least attn_grad_allreduce_signal_bytes(n, world) bytes, zero
 *                before the first call (the kernel leaves them zero)
 *   max_blocks   CTAs of 256 threads to use (0: the default of 16); at most 128, the same on every
 *                rank.  To overlap the reduction with a GEMM on another stream, give the GEMM
 *                that many fewer SMs (attn_gemm_ex): sharing an SM slows the persistent GEMM.
 * world 2 .. 8.  The kernel meets the other ranks in cross-GPU barriers before and after the
 * reduction; a barrier wait that gives up (after 2 s) records site 400 or 401 in the status word
 * (attn_device_error) and the kernel returns.
 */
size_t attn_grad_allreduce_signal_bytes(int64_t n, int world);
int attn_grad_allreduce(void* multicast, const void* signal_pads, int rank, int world, int64_t n,
                        size_t signal_pad_bytes, int max_blocks, void* stream);

/* Epilogue activations of attn_gemm_act (the feed-forward block, model/gpt.py:327-456). */
#define ATTN_ACT_NONE 0
#define ATTN_ACT_GELU 1     /* C = gelu(acc + bias); aux (optional) = acc + bias          */
#define ATTN_ACT_GELU_BWD 2 /* C = acc * gelu'(aux)                                       */

/* Library version (major*10000 + minor*100 + patch). */
int attn_version(void);

/* Text of the last error raised on the calling thread ("" if none). */
const char* attn_last_error_string(void);

/* Number of kernels this library has launched in this process (all entry points). */
uint64_t attn_launch_count(void);

/*
 * Status word of the tensor-core kernels on the current device: 0, or the code of a bounded
 * wait inside a kernel that gave up (that launch then skipped its remaining work and returned
 * instead of hanging, so its outputs are incomplete).  Codes are grouped by kernel: 1xx the GEMM
 * (106: its dynamic shared memory did not start 1024-byte aligned, checked before any work),
 * 2xx the attention forward, 3xx the attention backward (300: its dynamic shared memory did not
 * start 1024-byte aligned, checked before any work), 4xx the barriers of attn_grad_allreduce, 900
 * the self-test below.  The word keeps the first code until it is cleared; a set word does not
 * affect later launches (each launch only stops early for a wait of its own that gave up).
 * Synchronises with the device.
 * clear != 0 resets it to 0.  Has no counterpart in the reference, whose kernels cannot give up.
 * (Replaces the launch-failure exceptions PyCUDA raises, model/gpt.py:649-650 for the module.)
 */
int attn_device_error(int clear);

/*
 * Enqueue on `stream` a copy of the status word into *host_dst (pinned host memory, so that the
 * copy is asynchronous), without synchronising.  Once the stream has passed the copy, *host_dst
 * holds the word as it stood after every kernel enqueued before it.  The Python modules use it to
 * raise AttnError at their next call without a per-call synchronisation.
 */
int attn_device_error_async(int* host_dst, void* stream);

/* The code attn_wait_selftest leaves in the device error word. */
#define ATTN_SELFTEST_SITE 900

/*
 * Failure-detection self-test, with no counterpart in the reference (whose kernels have no
 * bounded waits): launches a one-warp kernel whose mbarrier wait can never complete, with a limit
 * of limit_us microseconds (1 .. 1000000).  The wait gives up after that limit, sets the device
 * error word to ATTN_SELFTEST_SITE (if it was 0) and the kernel returns, the same path a real
 * wait inside the tensor-core kernels takes; the context stays usable.  Read the word with
 * attn_device_error(1), which also clears it.
 */
int attn_wait_selftest(int limit_us, void* stream);

/*
 * Causal attention forward: O = softmax(scale * Q K^T + causal mask) V, plus lse.
 * Replaces fused_attention_forward_kernel (core/mha_kernels.py:404-521); instead of writing the
 * normalised probabilities Scores[B*NH,T,T] it writes lse[B,NH,T].
 * dtype ATTN_F32: CUDA-core fp32 path (any D <= 128, D % 4 == 0).
 * dtype ATTN_BF16: tcgen05 tensor-core path for D a multiple of 8 up to 64 (TMA-staged K/V, TMEM
 *                  accumulators; heads narrower than 64 are zero-padded to 64 by TMA) when the
 *                  tensors are 16-byte aligned with strides in 8-element steps, CUDA-core path
 *                  otherwise; fp32 softmax statistics and accumulation.
 * dtype ATTN_TF32: float32 tensors; tcgen05 kind::tf32 path for D a multiple of 4 up to 32 (the
 *                  same kernel with 32-float rows) under the same layout conditions, the float32
 *                  CUDA-core path otherwise.  attn_bwd then recomputes the scores from q and k
 *                  truncated to tf32, so that they match the lse this forward wrote.
 * Q/K/V share the input strides; O uses the output strides.
 */
int attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
             int B, int NH, int T, int D,
             int64_t in_sb, int64_t in_st, int64_t in_sh,
             int64_t out_sb, int64_t out_st, int64_t out_sh,
             float scale, int dtype, void* stream);

/* Bytes of workspace attn_bwd needs for this problem (row dots dO.O, dQ accumulators). */
size_t attn_bwd_workspace_size(int B, int NH, int T, int D, int dtype);

/*
 * Causal attention backward (the softmax VJP with the scale applied to dS, then dQ/dK/dV).
 * Replaces the NumPy steps of model/gpt.py:669-680 and the unwired kernels
 * softmax_fused_backward / matmul_grad_{q,k,v} (core/mha_kernels.py:195-236, 592-680).
 * q, k, v, dq, dk, dv use the input strides; o and dout use the output strides.
 * workspace: device buffer of at least attn_bwd_workspace_size() bytes.
 * The tensor-core path takes T up to 2,097,024; longer rows run the CUDA-core backward, whose
 * workspace attn_bwd_workspace_size() then sizes.
 */
int attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
             const float* lse, void* dq, void* dk, void* dv,
             void* workspace, size_t workspace_bytes,
             int B, int NH, int T, int D,
             int64_t in_sb, int64_t in_st, int64_t in_sh,
             int64_t out_sb, int64_t out_st, int64_t out_sh,
             float scale, int dtype, void* stream);

/*
 * Debug/test accessor: rebuild the normalised causal probabilities from lse,
 * P[b, h, i, j] = exp(scale * q_i . k_j - lse[b, h, i]) for j <= i, else 0, into a float32
 * [B, NH, T, T] buffer.  This is the cache_attn_weights matrix the reference forward writes
 * (core/mha_kernels.py:492-498, downloaded at model/gpt.py:612-614); the training path never
 * materialises it.  q/k use the input strides of attn_fwd.
 */
int attn_probs(const void* q, const void* k, const float* lse, float* probs,
               int B, int NH, int T, int D, int64_t in_sb, int64_t in_st, int64_t in_sh,
               float scale, int dtype, void* stream);

/* Bytes of workspace attn_decode needs (per-split partial softmax states). */
size_t attn_decode_workspace_size(int B, int NH, int L, int D);

/*
 * Single-query decode: one new query row per (b, h) attending over an L-token K/V prefix
 * (every cached key is visible).  Equals the last row of the causal forward that
 * GenerationSession.generate re-runs per token (generate.py:611-628).
 * q, o: element (b, h, d) at ptr[b*q_sb + h*q_sh + d].  K/V cache: element (b, l, h, d) at
 * ptr[b*kv_sb + l*kv_sl + h*kv_sh + d].  lse may be NULL.  Split over L, then combined.
 * B*NH (one grid row per sequence and head) is at most 65535; beyond it the call returns
 * ATTN_ERR_UNSUPPORTED without launching.
 */
int attn_decode(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse,
                int B, int NH, int L, int D,
                int64_t q_sb, int64_t q_sh,
                int64_t kv_sb, int64_t kv_sl, int64_t kv_sh,
                float scale, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/*
 * attn_decode without a workspace argument: it allocates nothing.  No counterpart in the
 * reference (which has no decode kernel at all); it exists for callers that cannot allocate a
 * per-call device workspace: callers whose device memory is owned by another allocator (a pool
 * that reserved the free HBM up front, as a serving process sizing its KV cache does) and thin
 * FFI callers that hold only the q/K/V/o pointers.
 * The split partial states go to one fixed file-scope device array of 4 MiB (1,048,576 floats),
 * held on every GPU that loads the library until the process exits.  Problems needing more,
 * B*NH*ceil(L/256)*(D+2) > 1,048,576 (e.g. B=64, NH=8, L=2048, D=64 needs 270,336), are rejected
 * with ATTN_ERR_UNSUPPORTED and a message; nothing is launched.
 * The first call on each device resolves the array's device address (cudaGetSymbolAddress, with
 * that device current); make that first call before any stream capture.  The address is resolved
 * again when the device's CUDA context changes (after a cudaDeviceReset the module reloads and the
 * array may move); that call too must come before any capture.  B*NH is at most 65535, as for
 * attn_decode.  Every call shares the array and it keeps the last call's contents (each call
 * writes every partial state before reading it, so nothing needs zeroing); calls that overlap on
 * the GPU (concurrent streams or threads) race on the array and must be serialised by the caller.
 * Arguments otherwise as attn_decode.
 */
int attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse,
                        int B, int NH, int L, int D,
                        int64_t q_sb, int64_t q_sh,
                        int64_t kv_sb, int64_t kv_sl, int64_t kv_sh,
                        float scale, int dtype, void* stream);

/*
 * Projection GEMM: C[M,N] = op(A)[M,K] . op(B)[K,N] (+ bias[N]) ; with accumulate, C += ...
 * Replaces matmul_2d_kernel (core/kernels.py:119-140) and the projection-gradient GEMMs of
 * model/gpt.py:666-689 (dWo = ctx^T dY, dCtx = dY Wo^T, dWqkv = x^T dQKV, dX = dQKV Wqkv^T).
 *   a_trans = 0: A stored row-major [M][lda] (K contiguous);  1: stored [K][lda] (A = X^T).
 *   b_trans = 0: B stored row-major [K][ldb] (N contiguous);  1: stored [N][ldb] (B = W^T).
 * a_dtype == b_dtype.  ATTN_BF16 operands run on tcgen05 tensor cores (kind::f16, fp32
 * accumulate); ATTN_TF32 operands (float32 storage, 16-byte aligned rows) on tcgen05 as tf32
 * (kind::tf32, fp32 accumulate); ATTN_F32 operands on the CUDA-core fp32 path.  C is ATTN_F32
 * or ATTN_BF16; accumulate requires ATTN_F32 C.  bias is float32 or NULL.
 */
int attn_gemm(const void* A, int64_t lda, int a_trans,
              const void* B, int64_t ldb, int b_trans, int ab_dtype,
              void* C, int64_t ldc, int c_dtype, const float* bias,
              int M, int N, int K, int accumulate, void* stream);

/*
 * attn_gemm on at most max_ctas SMs (0: all of them).  The tensor-core GEMM is persistent, one CTA
 * per SM; a caller that overlaps it with a kernel on another stream (the gradient all-reduce beside
 * the dX GEMM) leaves that kernel whole SMs this way.  The CUDA-core path ignores max_ctas.
 */
int attn_gemm_ex(const void* A, int64_t lda, int a_trans,
                 const void* B, int64_t ldb, int b_trans, int ab_dtype,
                 void* C, int64_t ldc, int c_dtype, const float* bias,
                 int M, int N, int K, int accumulate, int max_ctas, void* stream);

/*
 * attn_gemm with the feed-forward activation in the epilogue (no accumulate), replacing the FFN's
 * kernel sequences (model/gpt.py:345-365 and :428-449):
 *   ATTN_ACT_GELU:     C = gelu(op(A) op(B) + bias), gelu the tanh form of activation_kernel
 *                      (core/kernels.py:237-250); if aux is non-NULL it receives the pre-activation
 *                      op(A) op(B) + bias (FeedForward's cache_pre_act), in C's dtype on the
 *                      tensor cores.  Replaces matmul_2d_kernel + the cache copy + activation_kernel.
 *   ATTN_ACT_GELU_BWD: C = (op(A) op(B)) * gelu'(aux), aux the cached pre-activation [M][ldaux]
 *                      (gelu_backward_kernel, core/kernels.py:424-447).  With A = dOut and
 *                      B = W_proj^T this is dHidden followed by the GELU backward.
 * aux_dtype is ATTN_F32 or ATTN_BF16.  ATTN_BF16 operands run on tcgen05 (tanh.approx in the
 * epilogue); ATTN_F32 operands on CUDA cores with tanhf.  ATTN_ACT_NONE behaves as attn_gemm.
 */
int attn_gemm_act(const void* A, int64_t lda, int a_trans,
                  const void* B, int64_t ldb, int b_trans, int ab_dtype,
                  void* C, int64_t ldc, int c_dtype, const float* bias,
                  int M, int N, int K, int act, void* aux, int64_t ldaux, int aux_dtype,
                  void* stream);

/* Bytes of workspace attn_colsum needs. */
size_t attn_colsum_workspace_size(int M, int N);

/*
 * Column sum out[n] = sum_m X[m, n] (accumulate: out[n] += ...), X row-major [M][ldx] of
 * ATTN_F32 or ATTN_BF16; out float32.  The bias gradients of model/gpt.py:667 and :688.
 * Deterministic (fixed split of rows, fixed combine order).
 */
int attn_colsum(const void* X, int x_dtype, int64_t ldx, int M, int N, float* out,
                int accumulate, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Y = bf16(X) and out[n] (+)= sum_m X[m, n] in one pass over X (float32 [M][ldx]; Y bf16 [M][ldy]).
 * The upstream-gradient cast of the bf16 path fused with the output-projection bias gradient
 * (model/gpt.py:667).  Workspace: attn_colsum_workspace_size(M, N).
 */
int attn_cast_colsum_f32(const float* X, int64_t ldx, int M, int N, void* Y, int64_t ldy,
                         float* out, int accumulate, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * Y[m, n] = bf16(X[m, n]) for n < N, Y[m, N] = 1, Y[m, n] = 0 for N < n < ldy (X float32 [M][ldx],
 * Y bf16 [M][ldy], ldy > N and a multiple of 8).  The bf16 input of the QKV projection with a ones
 * column: the weight-gradient GEMM Y^T dQKV over N+1 rows then yields dWqkv and, as its last row,
 * dbqkv = sum over tokens of dQKV (model/gpt.py:687-688) without a separate column-sum pass.
 */
int attn_cast_rows_ones_bf16(const float* x, int64_t ldx, int M, int N, void* y, int64_t ldy,
                             void* stream);

/*
 * LayerNorm of the rows of X (float32 [M][ldx]): Y = (X - mean) * rsqrt(var + eps) * gamma + beta
 * with the biased variance, as layernorm_kernel (core/kernels.py:75-110; the reference uses
 * eps = 1e-5).  Y is float32 or bf16 [M][ldy]; with ones_col, Y[m, C] = 1 and the columns after it
 * are 0 (the bf16 QKV-projection input of attn_cast_rows_ones_bf16).  Replaces the pre-attention
 * LayerNorm of TransformerBlock.forward (model/gpt.py:778) and the cast that would follow it.
 */
int attn_layernorm(const float* x, int64_t ldx, const float* gamma, const float* beta, int M, int C,
                   float eps, void* y, int64_t ldy, int y_dtype, int ones_col, void* stream);

/*
 * LayerNorm backward (layernorm_backward_kernel, core/kernels.py:361-416): for rows of dy and the
 * forward input x (float32 [M][C], contiguous), dx = rstd/C * (C*g - sum(g) - x_hat*sum(g*x_hat))
 * with g = dy*gamma, written or, with accumulate_dx, added to dx (the residual branch of
 * TransformerBlock.backward, model/gpt.py:826-838, in place); dgamma = sum over rows of dy*x_hat
 * and dbeta = sum of dy, set or (accumulate_params) added.  dx must not alias x or dy.
 */
int attn_layernorm_bwd(const float* dy, const float* x, const float* gamma, int M, int C, float eps,
                       float* dx, int accumulate_dx, float* dgamma, float* dbeta,
                       int accumulate_params, void* stream);

/* y[i] = bf16(x[i]) (round to nearest even), n elements. */
int attn_cast_f32_to_bf16(const float* x, void* y, int64_t n, void* stream);

/*
 * Layout adapters with the reference's semantics (float32):
 * split_heads_kernel (core/mha_kernels.py:534-558): QKV[B*T, 3C] -> Q/K/V[B*NH, T, HD];
 * merge_heads_kernel (core/mha_kernels.py:567-584): ContextHeads[B*NH, T, HD] -> Context[B*T, C].
 */
int attn_split_heads(const float* qkv, float* q, float* k, float* v,
                     int B, int T, int NH, int HD, void* stream);
int attn_merge_heads(const float* ctx_heads, float* ctx, int B, int T, int NH, int HD,
                     void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ATTN_B200_H */
