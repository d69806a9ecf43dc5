/* spar_b200 — B200 (sm_100a) training backend for Spar's Transformer hot path.
 *
 * New C ABI entry points. They keep the conventions of Spar's backend ABI
 * (src/backend/cuda_kernels.hpp:41-44 status struct, int dtype tags, raw caller-owned device
 * pointers, a device index per call) and add one thing: every call takes a CUDA stream
 * (`stream`, a cudaStream_t passed as void*; NULL = the legacy default stream) and is
 * asynchronous. A returned status reports argument and launch errors; errors that happen while
 * the kernel runs surface at the caller's next synchronisation, and device-side data errors
 * (bad class ids, non-finite gradient norms) are reported through caller-provided int32 flags.
 *
 * All tensors are row-major fp32 unless stated otherwise; index tensors are int32.
 */
#ifndef SPAR_B200_H
#define SPAR_B200_H

#include <stdint.h>

#include "spar_cuda_kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------ */
/* LayerNorm over the last axis of x[rows, cols] (cols % 4 == 0).                              */
/* y = (x - mean) * rstd * gamma + beta with mean, rstd = 1/sqrt(var + epsilon), var biased.    */
/* Spar has no LayerNorm op; this is the composition mean/subtract/square/mean/add_scalar/     */
/* sqrt/divide/multiply/add of src/ops (pattern of src/nn/rmsnorm.cpp:50-52) fused into one.   */
/* mean/rstd ([rows] each) are saved for the backward pass.                                     */
struct SparCudaStatus spar_b200_layernorm_forward(float* y, float* mean, float* rstd,
                                                  const float* x, const float* gamma,
                                                  const float* beta, uint64_t rows, uint64_t cols,
                                                  double epsilon, int device, void* stream);

/* dX, dgamma, dbeta of the LayerNorm above in one pass over (x, dy). dgamma/dbeta are reduced */
/* deterministically (fixed per-block partial order); accumulate != 0 adds them to the existing */
/* contents (gradient accumulation across micro-steps, Spar autograd.cpp:240-246). dx may be   */
/* accumulated into with accumulate_dx != 0 (residual-stream gradients).                       */
struct SparCudaStatus spar_b200_layernorm_backward(float* dx, float* dgamma, float* dbeta,
                                                   const float* dy, const float* x,
                                                   const float* gamma, const float* mean,
                                                   const float* rstd, uint64_t rows, uint64_t cols,
                                                   int accumulate_params, int accumulate_dx,
                                                   int device, void* stream);

/* Allocation-free LayerNorm backward: same arguments and results as                            */
/* spar_b200_layernorm_backward, for callers that cannot allocate device memory at call time.   */
/* No counterpart in the reference (Spar's ops allocate their outputs and scratch per call).    */
/* Scratch is a static device array shared by all calls: cols <= 2048, at most 296 partial rows */
/* (4.85 MB per GPU, held until exit); rejects larger sizes with code 1. The first call on a    */
/* device looks up the array's address (make it before any stream capture); calls that overlap */
/* on the GPU race and must be serialised by the caller. The looked-up address is cached for   */
/* the process's life and does not survive cudaDeviceReset (or another teardown of the device's */
/* primary context): do not call this entry point again after one. x, dy, dx and gamma must be   */
/* 16-byte aligned (code 1 otherwise), as for spar_b200_layernorm_backward.                     */
struct SparCudaStatus spar_b200_layernorm_backward_noalloc(
    float* dx, float* dgamma, float* dbeta, const float* dy, const float* x, const float* gamma,
    const float* mean, const float* rstd, uint64_t rows, uint64_t cols, int accumulate_params,
    int accumulate_dx, int device, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* RMSNorm over the last axis of x[rows, cols] (cols % 4 == 0, cols <= 2048):                   */
/* y = x / sqrt(mean(x^2) + epsilon) * weight, replacing nn::RMSNorm::forward                   */
/* (src/nn/rmsnorm.cpp:40-53: mean(square), add_scalar, sqrt, divide, multiply(weight)); the    */
/* divide is taken as a multiply by rstd. rstd [rows] = 1 / sqrt(mean(x^2) + epsilon) is saved.  */
struct SparCudaStatus spar_b200_rmsnorm_forward(float* y, float* rstd, const float* x,
                                                const float* weight, uint64_t rows, uint64_t cols,
                                                double epsilon, int device, void* stream);
/* dx and dweight of the RMSNorm above in one pass over (x, dy) (the autograd sweep of that      */
/* chain): dx = rstd * (g - xhat * mean(g * xhat)), g = dy * weight, xhat = x * rstd;           */
/* dweight = sum over rows of dy * xhat, reduced deterministically. accumulate_params /         */
/* accumulate_dx add to the existing dweight / dx as in spar_b200_layernorm_backward.           */
struct SparCudaStatus spar_b200_rmsnorm_backward(float* dx, float* dweight, const float* dy,
                                                 const float* x, const float* weight,
                                                 const float* rstd, uint64_t rows, uint64_t cols,
                                                 int accumulate_params, int accumulate_dx,
                                                 int device, void* stream);

/* qk-norm, replacing the q_norm / k_norm RMSNorm(head_dim) of nn::SelfAttention               */
/* (src/nn/attention.cpp:183-186, 212-213) on the head-major view of the projections: RMSNorm   */
/* over each head's head_dim features where x[tokens, ld] holds `heads` consecutive heads from   */
/* column 0 of each row (pass the packed projection output + the q or k part's column offset). */
/* y and x share the layout and may be the same buffer (each head row is read before it is     */
/* written); rstd [tokens * heads] (token-major). head_dim % 4 == 0, ld % 4 == 0, 16-byte       */
/* aligned pointers.                                                                            */
struct SparCudaStatus spar_b200_head_rmsnorm_forward(float* y, const float* x, uint64_t ld,
                                                     uint64_t tokens, uint64_t heads,
                                                     uint64_t head_dim, const float* weight,
                                                     float* rstd, double epsilon, int device,
                                                     void* stream);
/* dx (same layout; may be dy's buffer) and dweight of the qk-norm above.                       */
struct SparCudaStatus spar_b200_head_rmsnorm_backward(float* dx, float* dweight, const float* dy,
                                                      const float* x, uint64_t ld,
                                                      uint64_t tokens, uint64_t heads,
                                                      uint64_t head_dim, const float* weight,
                                                      const float* rstd, int accumulate_params,
                                                      int device, void* stream);

/* SwiGLU gate, replacing nn::swiglu (src/nn/functional.cpp:9-11) as used by SwiGLUMLP          */
/* (src/nn/mlp.cpp:33-46): h = silu(gate) * value, silu(x) = x * sigmoid(x) with Spar's stable   */
/* sigmoid (src/ops/unary.cpp:55-61, 150-152), over rows x cols with row strides (ld*, in        */
/* floats), so gate and value may be the two column halves of one fused projection output.      */
struct SparCudaStatus spar_b200_swiglu_forward(float* h, uint64_t ldh, const float* gate,
                                               uint64_t ldg, const float* value, uint64_t ldv,
                                               uint64_t rows, uint64_t cols, int device,
                                               void* stream);
/* d gate = (dh * value) * (s + gate * (s * (1 - s))), d value = dh * silu(gate), s = sigmoid(gate) */
/* (silu's local derivative, src/ops/unary.cpp:155-160, through multiply's backward).             */
struct SparCudaStatus spar_b200_swiglu_backward(float* dgate, uint64_t lddg, float* dvalue,
                                                uint64_t lddv, const float* dh, uint64_t lddh,
                                                const float* gate, uint64_t ldg,
                                                const float* value, uint64_t ldv, uint64_t rows,
                                                uint64_t cols, int device, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* GELU, tanh form: gelu(x) = x * sigmoid(2*sqrt(2/pi)*(x + 0.044715 x^3)), the identity that  */
/* writes the tanh form with Spar's stable sigmoid (src/ops/unary.cpp:137-148).                 */
struct SparCudaStatus spar_b200_gelu_forward(float* y, const float* x, uint64_t count, int device,
                                             void* stream);
/* dx = gelu'(x) * dy                                                                           */
struct SparCudaStatus spar_b200_gelu_backward(float* dx, const float* dy, const float* x,
                                              uint64_t count, int device, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Causal softmax over the last axis of `batch` square [T, T] score matrices (row stride ld).  */
/* P[i, j] = softmax_j(scale * S[i, j] + mask) with mask = 0 for j <= i, -inf otherwise; this  */
/* is Spar's scaled_dot_product_attention scale + causal_mask + softmax(axis 3) chain          */
/* (src/nn/attention.cpp:128-134). Entries above the diagonal are never read; they are written */
/* as 0 for j < zero_fill_to(i) = min(T, round_up(i + 1, zero_fill_block)), zero_fill_block == 0 */
/* meaning the whole row.                                                                       */
struct SparCudaStatus spar_b200_causal_softmax_forward(float* p, const float* s, uint64_t batch,
                                                       uint64_t t, uint64_t ld, float scale,
                                                       uint64_t zero_fill_block, int device,
                                                       void* stream);
/* dS[i, j] = scale * P[i, j] * (dP[i, j] - sum_k dP[i, k] P[i, k]) for j <= i (Spar softmax   */
/* backward, src/ops/softmax.cpp:110-150, times the score scale of attention.cpp:128-129);      */
/* zero fill above the diagonal as in the forward call. ds may alias dp.                        */
struct SparCudaStatus spar_b200_causal_softmax_backward(float* ds, const float* dp, const float* p,
                                                        uint64_t batch, uint64_t t, uint64_t ld,
                                                        float scale, uint64_t zero_fill_block,
                                                        int device, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Fused softmax cross-entropy forward + backward over logits[rows, classes] (row stride ld).   */
/* For every row r with a target: loss[r] = logsumexp(z_r) - z_r[target] and                  */
/* dlogits[r, :] = grad_scale * (softmax(z_r) - onehot(target)); rows without a target get     */
/* loss 0 and dlogits 0. dlogits may alias logits (in-place).                                   */
/* sequence_length == 0: target of row r is targets[r] (Spar loss::cross_entropy,              */
/*   src/loss/cross_entropy.cpp:146-174).                                                       */
/* sequence_length == T > 1: language-model shift (cross_entropy.cpp:176-214): row r = b*T + t */
/*   has target targets[b*T + t + 1] for t < T-1 and no target for t = T-1.                     */
/* grad_scale is the upstream gradient of the mean, 1/(number of targets) for Spar's mean      */
/* reduction. Targets outside [0, classes) set *invalid_target = 1 (never cleared here) and the */
/* row gets loss NaN and dlogits 0.                                                              */
struct SparCudaStatus spar_b200_cross_entropy_forward_backward(
    float* loss, float* dlogits, const float* logits, const int32_t* targets, uint64_t rows,
    uint64_t classes, uint64_t ld, uint64_t sequence_length, float grad_scale,
    int32_t* invalid_target, int device, void* stream);

/* Deterministic sum of `count` floats into *out (double accumulation, fixed order).          */
struct SparCudaStatus spar_b200_sum(float* out, const float* values, uint64_t count, int device,
                                    void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Gradient clipping + AdamW over flat fp32 arrays.                                            */
/* Step 1 (spar_b200_grad_norm_squared): norm_state[0] = sum of g^2 (double), norm_state[1] =   */
/*   non-finite flag, over every (grad, count) pair in the list. Equivalent to Spar's          */
/*   global_grad_norm (src/training/gradients.cpp:28-137) up to double rounding.               */
/* Step 2 (spar_b200_adamw_clipped): clip factor = max_norm / norm when norm > max_norm        */
/*   (clip_grad_norm, gradients.cpp:176-190), computed on the device from norm_state; then     */
/*   Spar's AdamW update (src/optim/adamw.cpp:37-63) in double with moments rounded to fp32.   */
/*   A non-finite norm sets *nonfinite_flag = 1 and leaves every tensor untouched (Spar throws */
/*   "Cannot clip nonfinite gradients" before any update). max_norm < 0 disables clipping.     */
struct SparB200TensorSlice {
  float* parameter;
  float* gradient;
  float* first_moment;
  float* second_moment;
  uint64_t count;
};
struct SparCudaStatus spar_b200_grad_norm_squared(double* norm_state,
                                                  const struct SparB200TensorSlice* slices,
                                                  uint64_t slice_count, int device, void* stream);
struct SparCudaStatus spar_b200_adamw_clipped(const struct SparB200TensorSlice* slices,
                                              uint64_t slice_count, const double* norm_state,
                                              double max_norm, double learning_rate, double beta1,
                                              double beta2, double epsilon, double weight_decay,
                                              uint64_t step, int32_t* nonfinite_flag,
                                              int device, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Embedding gather out[i, :] = weight[ids[i], :] (src/ops/embedding.cpp:89-121, 55-67).             */
/* Ids outside [0, vocab) set *invalid_index = 1 and produce a zero row.                        */
struct SparCudaStatus spar_b200_embedding_forward(float* out, const float* weight,
                                                  const int32_t* ids, uint64_t count,
                                                  uint64_t vocab, uint64_t dim,
                                                  int32_t* invalid_index, int device,
                                                  void* stream);
/* grad_weight[v, :] += sum_{i: ids[i] == v} grad_out[i, :], deterministic (no atomics): the   */
/* ids are counting-sorted on the device and every vocabulary row is reduced in index order.   */
/* Needs scratch of spar_b200_embedding_backward_scratch_bytes(count, vocab) bytes.            */
uint64_t spar_b200_embedding_backward_scratch_bytes(uint64_t count, uint64_t vocab);
struct SparCudaStatus spar_b200_embedding_backward(float* grad_weight, const float* grad_out,
                                                   const int32_t* ids, uint64_t count,
                                                   uint64_t vocab, uint64_t dim, void* scratch,
                                                   int device, void* stream);

/* Column sums: out[c] (+)= sum_r x[r, c] over x[rows, cols] (row stride ld): the bias gradient */
/* db = reduce_gradient_to_shape(dY, [out]) (src/core/tensor.cpp:597-632), deterministic.      */
struct SparCudaStatus spar_b200_column_sum(float* out, const float* x, uint64_t rows,
                                           uint64_t cols, uint64_t ld, int accumulate, int device,
                                           void* stream);

/* Rotary embedding on interleaved pairs, in place on q/k heads laid out [B, T, H, D] with row */
/* stride ld (elements between consecutive tokens). Angle table as Spar's apply_rope           */
/* (src/nn/rope.cpp:35-66): angle = pos * theta^(-2i/D) in double, cos/sin rounded to fp32.    */
/* `table` is [T, D/2] float2 (cos, sin) from spar_b200_rope_table; inverse != 0 rotates back  */
/* (the backward pass).                                                                         */
struct SparCudaStatus spar_b200_rope_table(float* table, uint64_t t, uint64_t d, double theta,
                                           uint64_t start_position, int device, void* stream);
struct SparCudaStatus spar_b200_rope_apply(float* x, const float* table, uint64_t batch,
                                           uint64_t t, uint64_t heads, uint64_t d, uint64_t ld,
                                           int inverse, int device, void* stream);

/* ------------------------------------------------------------------------------------------ */
/* Dense contraction on the tcgen05 tensor cores (TMA-fed, TMEM accumulators, fp32 accumulate). */
/* Replaces Spar's cuBLAS seam spar::detail::cuda_blas::matmul (src/backend/cuda_blas.cppm:    */
/* 122-194) and the transposed-operand copies of the matmul backward (src/ops/matmul.cpp:      */
/* 140-153).                                                                                    */
/*   C[b0,b1] = epilogue(alpha * opA(A[b0,b1]) * opB(B[b0,b1]))                                */
/* A is logical [m, k]: stored row-major [m, k] (a_transposed = 0) or [k, m] (= 1).             */
/* B is logical [k, n]: stored row-major [k, n] (b_transposed = 0) or [n, k] (= 1).             */
/* Leading dimensions and batch strides are in elements and must be multiples of 4 (16 bytes); */
/* base pointers 16-byte aligned.                                                               */
enum SparB200Precision {
  SPAR_B200_TF32 = 0,   /* operands rounded to TF32 (10-bit mantissa), fp32 accumulate */
  SPAR_B200_TF32X3 = 1, /* split a = hi + lo, three TF32 products: fp32-faithful; no      */
                        /* tensor-core accumulator sums more than 512 K elements (the      */
                        /* sums move to fp32 registers or split-K partials beyond that)    */
};
enum SparB200Epilogue {
  SPAR_B200_EPI_NONE = 0,      /* C = alpha*acc                                            */
  SPAR_B200_EPI_BIAS = 1,      /* C = alpha*acc + bias[n]                                  */
  SPAR_B200_EPI_BIAS_GELU = 2, /* aux = alpha*acc + bias[n] (pre-activation); C = gelu(aux) */
  SPAR_B200_EPI_GELU_BWD = 3,  /* C = alpha*acc * gelu'(aux)  (aux = saved pre-activation)  */
  SPAR_B200_EPI_BIAS_ADD = 4,  /* C = alpha*acc (+ bias[n] if bias) + aux  (residual add)    */
};
enum SparB200Causal {
  SPAR_B200_CAUSAL_NONE = 0,
  SPAR_B200_CAUSAL_LOWER = 1,  /* m == n: output tiles strictly above the diagonal skipped  */
  SPAR_B200_CAUSAL_K_UPTO = 2, /* reduction limited to k <= row index (P*V, dS*K)          */
  SPAR_B200_CAUSAL_K_FROM = 3, /* reduction limited to k >= row index (P^T*dO, dS^T*Q)     */
};
struct SparB200Gemm {
  uint64_t m, n, k;
  uint64_t batch[2];
  const float* a;
  uint64_t lda;
  uint64_t a_batch_stride[2];
  int a_transposed;
  const float* b;
  uint64_t ldb;
  uint64_t b_batch_stride[2];
  int b_transposed;
  float* c;
  uint64_t ldc; /* multiple of 4, like every leading dimension and batch stride here. Rows of C */
                /* are stored in whole 16-byte chunks: when n is not a multiple of 4, the up to  */
                /* 3 floats after column n - 1 of a row (inside ldc) may be overwritten.        */
  uint64_t c_batch_stride[2];
  float alpha;
  int accumulate; /* 1: C += result (beta = 1) */
  int epilogue;   /* SparB200Epilogue */
  const float* bias;
  float* aux; /* same shape/strides as C, leading dimension ldaux */
  uint64_t ldaux;
  int precision; /* SparB200Precision */
  int causal;    /* SparB200Causal */
  int round_output; /* 1: store C rounded to nearest TF32 (for results that only feed TF32
                       products, which otherwise drop the low mantissa bits by truncation) */
  /* Optional RoPE rotation in the epilogue (after bias, before rounding / storing), as           */
  /* spar_b200_rope_apply on the result: for columns c < rope_cols, pairs (c, c+1) with c even    */
  /* rotate by table[(row % rope_seq) * rope_dim/2 + (c % rope_dim)/2] (cos, sin). The fused      */
  /* QKV projection uses it for its q and k thirds. Unbatched, non-accumulating GEMMs only.      */
  const float* rope_table; /* [rope_seq, rope_dim/2] float2 from spar_b200_rope_table, or NULL */
  uint64_t rope_seq;
  uint64_t rope_dim;  /* even */
  uint64_t rope_cols; /* multiple of rope_dim */
  /* Optional, unbatched GEMMs only: per 32-row block column sums of this product's epilogue     */
  /* output (before accumulation into C and before output rounding; rows past m count as zero),  */
  /* written to column_partials[(row / 32) * n + col], a [ceil(m / 32), n] array. Summing its    */
  /* rows gives the column sums of the result (a bias gradient) without re-reading C. With a K   */
  /* split the split-K reduction writes them (summed row by row, same values to fp32 rounding).  */
  float* column_partials;
};
struct SparCudaStatus spar_b200_gemm(const struct SparB200Gemm* gemm, int device, void* stream);

/* Contiguous batched matmul of any shape: C[b] = A[b] B[b] for b < batch, row-major            */
/* [batch, m, k] x [batch, k, n] -> [batch, m, n], dtype SPAR_CUDA_FLOAT32 (tcgen05, precision  */
/* SparB200Precision; shapes or pointers the tensor-core GEMM cannot address directly are staged */
/* through zero-padded copies) or SPAR_CUDA_FLOAT64 (SIMT, precision ignored). The body of the   */
/* replacement for Spar's cuBLAS seam spar::detail::cuda_blas::matmul (reference                 */
/* src/backend/cuda_blas.cppm:122-194, which loops cublasSgemm / cublasDgemm over the batch).    */
/* k == 0 writes zeros; asynchronous on `stream`.                                               */
struct SparCudaStatus spar_b200_matmul(const void* a, const void* b, void* c, uint64_t batch,
                                       uint64_t m, uint64_t k, uint64_t n, int dtype,
                                       int precision, int device, void* stream);

/* Returns 1 if a GEMM on `device` gave up on a bounded pipeline wait (the kernel records the    */
/* event and exits instead of hanging), 0 otherwise, -1 on a CUDA error; clear != 0 resets it.  */
int spar_b200_gemm_error(int device, int clear);

/* ------------------------------------------------------------------------------------------ */
/* Fused causal self-attention (tensor cores, TF32 products, fp32 softmax and accumulation).    */
/* Replaces scaled_dot_product_attention (reference src/nn/attention.cpp:121-135: scores =     */
/* Q K^T / sqrt(head_dim), causal -inf mask, softmax over keys, P V) and the backward of that   */
/* chain, without materialising the [seq, seq] scores or probabilities.                         */
/* qkv: [batch, seq, 3 * heads * head_dim] row-major, Q | K | V thirds, head h at columns       */
/* h * head_dim of each third (the fused projection output). ctx: [batch, seq, heads*head_dim]. */
/* row_max / row_inv: [batch, heads, seq] softmax statistics written by the forward (row max of */
/* scores * scale * log2(e), 1 / sum of exponentials) and read by the backward.                 */
/* Backward: dctx in, dqkv [batch, seq, 3 * heads * head_dim] out (every column of every row     */
/* overwritten); delta [batch, heads, seq] is scratch. head_dim must be 32 or 64; pointers      */
/* 16-byte aligned. Asynchronous on `stream`; deterministic (no atomics). With a RoPE table     */
/* ([seq, head_dim/2] float2 from spar_b200_rope_table, else NULL) the q and k thirds of dqkv    */
/* are returned rotated back (the gradient of the projection before RoPE).                      */
struct SparCudaStatus spar_b200_attention_forward(const float* qkv, float* ctx, float* row_max,
                                                  float* row_inv, uint64_t batch, uint64_t seq,
                                                  uint64_t heads, uint64_t head_dim, int device,
                                                  void* stream);
struct SparCudaStatus spar_b200_attention_backward(const float* qkv, const float* ctx,
                                                   const float* dctx, const float* row_max,
                                                   const float* row_inv, float* delta, float* dqkv,
                                                   uint64_t batch, uint64_t seq, uint64_t heads,
                                                   uint64_t head_dim, const float* rope_table,
                                                   int device, void* stream);
/* Grouped-query attention (SelfAttention with num_kv_heads < num_query_heads,                  */
/* src/nn/attention.cpp:168-186; repeat_kv_heads :77-94): query head h attends with key / value  */
/* head h / (heads / kv_heads), without materialising the repeated heads. qkv and dqkv rows are  */
/* [Q (heads) | K (kv_heads) | V (kv_heads)] x head_dim; dK / dV sum over each head's group      */
/* (deterministic). kv_heads must divide heads; kv_heads == heads is the call above.            */
struct SparCudaStatus spar_b200_attention_forward_gqa(const float* qkv, float* ctx, float* row_max,
                                                      float* row_inv, uint64_t batch, uint64_t seq,
                                                      uint64_t heads, uint64_t kv_heads,
                                                      uint64_t head_dim, int device, void* stream);
struct SparCudaStatus spar_b200_attention_backward_gqa(
    const float* qkv, const float* ctx, const float* dctx, const float* row_max,
    const float* row_inv, float* delta, float* dqkv, uint64_t batch, uint64_t seq, uint64_t heads,
    uint64_t kv_heads, uint64_t head_dim, const float* rope_table, int device, void* stream);
/* As spar_b200_gemm_error, for the attention kernels' bounded waits. */
int spar_b200_attention_error(int device, int clear);
/* Host-side fault injection for tests of the error path (no counterpart in the reference): sets  */
/* (value != 0) or clears the bounded-wait flag of the GEMM (kernel 0) or attention (kernel 1)    */
/* kernels on `device` without running a kernel. A training step that finds either flag set      */
/* updates nothing and returns {2, cudaErrorTimeout}. Returns 0, or -1 on a bad argument / CUDA   */
/* error.                                                                                         */
int spar_b200_set_wait_error(int device, int kernel, int value);

/* ------------------------------------------------------------------------------------------ */
/* Training-step runtime for the pre-LN / GELU decoder LM (BASELINE's model family): tied token */
/* embedding, `num_layers` blocks of LayerNorm -> causal self-attention with RoPE (fused QKV     */
/* projection, biases) -> residual -> LayerNorm -> Linear/GELU/Linear MLP -> residual, final     */
/* LayerNorm, logits = h E^T, language-model cross-entropy, global-norm clip and AdamW. This is  */
/* the work one Spar training step does through DecoderLM::forward (src/nn/decoder.cpp:73-90),  */
/* loss::language_model_cross_entropy (src/loss/cross_entropy.cpp:176-214), Tensor::backward     */
/* (src/autograd/autograd.cpp:201-265), training::clip_grad_norm (gradients.cpp:176-190) and    */
/* optim::AdamW::step (src/optim/adamw.cpp:83-170), scheduled on one CUDA stream.               */
/* Parameters are exposed under Spar's named_parameters names (src/nn/parameters.cpp:51-132).   */
/* family (the fields after max_grad_norm; a zero-initialised tail is family 0):                */
/*   SPAR_B200_FAMILY_LN_GELU (0): the benchmark decoder above.                                  */
/*   SPAR_B200_FAMILY_SPAR (1): Spar's own nn::DecoderLM (src/nn/decoder.cpp, transformer.cpp:   */
/*   53-69, attention.cpp:168-225, mlp.cpp:33-46): RMSNorm pre-norms and final norm, no biases,  */
/*   num_kv_heads key/value heads (grouped-query attention), optional RMSNorm of each q / k head */
/*   before RoPE (qk_norm, qk_norm_epsilon), SwiGLU MLP (gate, up, down), tied logits. Names as */
/*   nn::named_parameters (src/nn/parameters.cpp:51-132); TF32 only, head_dim 32 or 64.         */
enum { SPAR_B200_FAMILY_LN_GELU = 0, SPAR_B200_FAMILY_SPAR = 1 };
struct SparB200LMConfig {
  uint64_t vocab_size, model_dim, hidden_dim, num_layers, num_heads, sequence_length;
  uint64_t micro_batch; /* sequences per micro-step */
  double norm_epsilon;  /* LayerNorm / RMSNorm epsilon (Spar's norm default 1e-5) */
  double rope_theta;    /* 10000 in Spar */
  int use_rope;
  int precision; /* SparB200Precision of every GEMM */
  double beta1, beta2, adam_epsilon, weight_decay;
  double max_grad_norm; /* < 0: no clipping */
  int family;           /* SPAR_B200_FAMILY_* */
  int qk_norm;          /* family 1 */
  uint64_t num_kv_heads; /* family 1; 0 = num_heads */
  double qk_norm_epsilon; /* family 1 (Spar's default 1e-6) */
};
struct SparCudaStatus spar_b200_lm_create(const struct SparB200LMConfig* config, int device,
                                          void** handle);
void spar_b200_lm_destroy(void* handle);
uint64_t spar_b200_lm_parameter_count(void* handle);
uint64_t spar_b200_lm_flat_size(void* handle);
/* which: 0 parameters, 1 gradients, 2 first moments, 3 second moments (flat device arrays). */
float* spar_b200_lm_flat_buffer(void* handle, int which);
struct SparCudaStatus spar_b200_lm_parameter_info(void* handle, uint64_t index, char* name,
                                                  uint64_t name_capacity, uint64_t* rows,
                                                  uint64_t* cols);
struct SparCudaStatus spar_b200_lm_parameter_copy(void* handle, uint64_t index, int which,
                                                  int to_device, float* host);
struct SparCudaStatus spar_b200_lm_init_normal(void* handle, uint64_t seed, double std,
                                               void* stream);
struct SparCudaStatus spar_b200_lm_zero_grad(void* handle, void* stream);
struct SparCudaStatus spar_b200_lm_forward_backward(void* handle, const int32_t* ids,
                                                    uint64_t micro_index, float grad_scale,
                                                    int last_micro, void* stream);
struct SparCudaStatus spar_b200_lm_optimizer_step(void* handle, double learning_rate,
                                                  uint64_t step, void* stream);
/* One whole optimiser step (zero grads, micro-steps, reduction, clip + AdamW); synchronises      */
/* `stream` and reads back the mean loss, the pre-clip norm and flags [invalid id, non-finite      */
/* norm]. If a GEMM or attention kernel of the step gave up a bounded wait (on any rank), nothing  */
/* is updated and the call returns {2, cudaErrorTimeout}; see spar_b200_gemm_error.                */
struct SparCudaStatus spar_b200_lm_train_step(void* handle, const int32_t* ids, int ids_on_host,
                                              uint64_t micro_steps, double learning_rate,
                                              uint64_t step, float* loss_out,
                                              double* grad_norm_out, int32_t* flags_out,
                                              void* stream);
struct SparCudaStatus spar_b200_lm_set_comm(void* handle, void* comm, int world_size);
/* Sharded optimiser (data parallel, on by default when world_size > 1): after a train step each */
/* rank's arenas hold only its own pieces of the reduced gradients, the updated moments and (until */
/* the next step's start) the updated parameters. spar_b200_lm_gather, called by EVERY rank in   */
/* the same order, all-gathers one arena (which as in flat_buffer) ordered on `stream`; until     */
/* then spar_b200_lm_parameter_copy refuses reads of it (code 1, cuda_error cudaErrorNotReady).   */
struct SparCudaStatus spar_b200_lm_gather(void* handle, int which, void* stream);
/* Input pipeline, replacing data::LMBatchIterator (src/data/batch_iterator.cpp:56-143) over    */
/* data::WindowDataset (src/data/tokenized_corpus.cpp:49-80): window i = tokens [i * stride,     */
/* i * stride + sequence_length) of a packed corpus held in device memory; each epoch visits the  */
/* windows in Spar's (optionally Fisher-Yates shuffled, derive_epoch_seed) order, batch_size at a */
/* time (the last batch shorter unless drop_last). For data parallelism rank r of world receives */
/* rows [r n / world, (r + 1) n / world) of every n-row batch. next gathers this rank's rows as   */
/* int32 ids [rows, sequence_length] into `ids` (device) on `stream`; global_rows = 0 means the  */
/* epoch is finished (rows alone can be 0 for a rank whose share of a short last batch is empty). */
struct SparCudaStatus spar_b200_batches_create(const int32_t* tokens, uint64_t token_count,
                                               uint64_t sequence_length, uint64_t stride,
                                               uint64_t batch_size, int shuffle,
                                               uint64_t shuffle_seed, int drop_last, int rank,
                                               int world, int device, void** handle);
struct SparCudaStatus spar_b200_batches_next(void* handle, int32_t* ids, uint64_t* rows,
                                             uint64_t* global_rows, void* stream);
struct SparCudaStatus spar_b200_batches_next_epoch(void* handle);
/* BatchIteratorState: epoch and windows of its order consumed (set_state rebuilds the order). */
struct SparCudaStatus spar_b200_batches_state(void* handle, uint64_t* epoch, uint64_t* cursor,
                                              uint64_t* windows);
struct SparCudaStatus spar_b200_batches_set_state(void* handle, uint64_t epoch, uint64_t cursor);
void spar_b200_batches_destroy(void* handle);
/* Host-only, no GPU: this rank's window start offsets (token index) of the batch at (epoch,     */
/* cursor), its row counts and the cursor after it.                                              */
struct SparCudaStatus spar_b200_batch_windows(uint64_t token_count, uint64_t sequence_length,
                                              uint64_t stride, uint64_t batch_size, int shuffle,
                                              uint64_t shuffle_seed, int drop_last, uint64_t epoch,
                                              uint64_t cursor, int rank, int world,
                                              uint64_t* starts, uint64_t* rows,
                                              uint64_t* global_rows, uint64_t* next_cursor);

/* data::split_documents (src/data/batch_iterator.cpp:144-162), host-only: `order` receives the  */
/* document_count indices in Spar's shuffled order; the first validation_count are validation.   */
struct SparCudaStatus spar_b200_split_documents(uint64_t document_count, uint64_t validation_count,
                                                uint64_t seed, uint64_t* order);

/* Training checkpoints in Spar's SPARCKPT v1 format (src/checkpoint/checkpoint.cpp:18-475:    */
/* save_training_checkpoint / load_training_checkpoint), family 1 only (the format stores a      */
/* DecoderConfig): model parameters and AdamW moments by name, progress, RNG state, optimiser    */
/* hyper-parameters. adam_step: completed AdamW steps (0: no optimiser state; the next          */
/* train_step is then step adam_step + 1). The writer writes `path`.tmp, then renames it.        */
struct SparB200Checkpoint {
  uint64_t global_step, tokens_seen; /* TrainingProgress */
  uint64_t rng_state;                /* Random::state() of the caller's data RNG */
  double learning_rate;              /* the optimiser's current learning rate */
  uint64_t adam_step;
};
/* Device state -> file (synchronises the device). With a sharded optimiser this is collective:  */
/* every rank calls it (path NULL on ranks that only take part in the gather).                   */
struct SparCudaStatus spar_b200_lm_save_checkpoint(void* handle, const char* path,
                                                   const struct SparB200Checkpoint* meta);
/* File -> device state (parameters and moments; gradients untouched). Code 1 when the file does */
/* not match the handle's config (dimensions, norms, AdamW hyper-parameters) or is malformed.   */
struct SparCudaStatus spar_b200_lm_load_checkpoint(void* handle, const char* path,
                                                   struct SparB200Checkpoint* meta);
/* The same format from / to host arrays, without a GPU: one contiguous row-major float array    */
/* per named tensor of `config` (spar_b200_lm_layout_tensor order and shapes).                  */
struct SparCudaStatus spar_b200_checkpoint_write(const char* path,
                                                 const struct SparB200LMConfig* config,
                                                 const struct SparB200Checkpoint* meta,
                                                 const float* const* values,
                                                 const float* const* first_moments,
                                                 const float* const* second_moments);
struct SparCudaStatus spar_b200_checkpoint_read(const char* path,
                                                const struct SparB200LMConfig* config,
                                                struct SparB200Checkpoint* meta,
                                                float* const* values, float* const* first_moments,
                                                float* const* second_moments);
/* Host-only queries of the parameter-arena layout a config produces (no device work, usable   */
/* without a GPU): flat size in floats, the named tensors (Spar's names, offset into the arena, */
/* rows x cols with row stride ld; cols == 0 for vectors) and the gradient all-reduce buckets    */
/* (offset, count) in the order a data-parallel step issues them (last block first, then the    */
/* tied embedding and the final norm). The buckets tile [0, flat).                              */
struct SparCudaStatus spar_b200_lm_layout(const struct SparB200LMConfig* config, uint64_t* flat_size,
                                          uint64_t* num_tensors, uint64_t* num_buckets);
struct SparCudaStatus spar_b200_lm_layout_tensor(const struct SparB200LMConfig* config,
                                                 uint64_t index, char* name, uint64_t name_capacity,
                                                 uint64_t* offset, uint64_t* rows, uint64_t* cols,
                                                 uint64_t* ld);
struct SparCudaStatus spar_b200_lm_layout_bucket(const struct SparB200LMConfig* config,
                                                 uint64_t index, uint64_t* offset, uint64_t* count);
/* Rank `rank` of `world` under the sharded optimiser: of bucket `index`, the reduce-scattered    */
/* piece [own_offset, own_offset + shard) it updates (shard a multiple of 64 floats) and the      */
/* uneven tail [tail_offset, tail_offset + tail_count) all-reduced and updated on every rank.     */
struct SparCudaStatus spar_b200_lm_layout_shard(const struct SparB200LMConfig* config,
                                                uint64_t index, int world, int rank,
                                                uint64_t* own_offset, uint64_t* shard,
                                                uint64_t* tail_offset, uint64_t* tail_count);
struct SparCudaStatus spar_b200_lm_read_losses(void* handle, float* host, uint64_t count);
/* Event timing of every tensor-core GEMM launch (for roofline accounting) and a kernel-launch */
/* counter; profile_read synchronises the device.                                              */
struct SparCudaStatus spar_b200_lm_profile(void* handle, int enable);
struct SparCudaStatus spar_b200_lm_profile_read(void* handle, double* gemm_ms, double* gemm_flops,
                                                uint64_t* gemm_launches,
                                                uint64_t* kernel_launches);
double spar_b200_warmup_cosine(double peak, double minimum, uint64_t warmup_steps,
                               uint64_t decay_steps, uint64_t completed_steps);

/* ------------------------------------------------------------------------------------------ */
/* Data-parallel communicator (NCCL). Status code 3 = communication error (ncclResult_t in      */
/* cuda_error). Spar has no distributed backend; this is the new gradient exchange.             */
struct SparCudaStatus spar_b200_comm_unique_id(char* out, uint64_t capacity);
struct SparCudaStatus spar_b200_comm_init(const char* unique_id, int rank, int world_size,
                                          int device, void** comm);
struct SparCudaStatus spar_b200_comm_allreduce_sum(void* comm, float* data, uint64_t count,
                                                   void* stream);
struct SparCudaStatus spar_b200_comm_check(void* comm);
struct SparCudaStatus spar_b200_comm_destroy(void* comm, int abort);
/* Failure path (no counterpart in the reference, which has no collectives; its error contract   */
/* is the status code, src/backend/cuda_ops.cppm:194-206). spar_b200_comm_wait waits for         */
/* `stream` with a deadline, polling the stream and NCCL's asynchronous error state; after an    */
/* asynchronous error or at the deadline it aborts the communicator (ncclCommAbort) and returns  */
/* {3, ncclResult}. spar_b200_lm_train_step uses it for its final wait when a communicator is    */
/* attached, so a rank whose peer left gets code 3 instead of hanging. The deadline is           */
/* $SPAR_B200_COMM_TIMEOUT_S (default 600 s) or set per communicator. The bound covers device   */
/* work: the step's results are read into pinned host memory so no copy holds the host first.  */
/* NCCL's host-side connection setup with the peers (inside the enqueue of a collective's first */
/* use) is not covered; a peer lost before then is found between steps                          */
/* (spar_b200.dp.Heartbeat). After code 3 the communicator is aborted (destroy it with abort =  */
/* 1, which then only frees the handle), the trainer's captured steps are dropped without being */
/* destroyed, and its sharded state holds only this rank's pieces: resume from a checkpoint.    */
/* ncclCommAbort does not return while CUDA graphs holding the communicator's collectives are   */
/* in flight or alive (seen on this build's NCCL 2.28): the bounded wait therefore runs it on a */
/* detached thread and waits at most 20 s (then cuda_error = ncclInProgress: the step's streams */
/* may still hold the aborted work; end the process), and a rank tearing down normally destroys */
/* the trainer (spar_b200_lm_destroy, which releases its graphs) before the communicator.       */
struct SparCudaStatus spar_b200_comm_set_timeout(void* comm, double seconds);
struct SparCudaStatus spar_b200_comm_wait(void* comm, void* stream);

/* Library version string. */
const char* spar_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif
