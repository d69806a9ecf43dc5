// Internal launchers shared by the C ABI wrappers and the training-step runtime, plus the
// element functions that several kernels (and GEMM epilogues) evaluate.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace spar_b200 {

// 4-D fp32 TMA tensor map: element (x, r) of batch (q1, q0) at base + q0*bs0 + q1*bs1 + r*ld + x
// (x contiguous, extents inner x rows x b1 x b0), boxes of 32 x box_rows elements; 128-byte
// swizzle of 16-byte chunks (K-major operands, staging boxes) or of 32-byte chunks (mn_major:
// MN-major tf32 operands). Bytes outside the extents read as zero and are not written.
bool make_map(CUtensorMap* map, const float* base, uint64_t inner, uint64_t rows, uint64_t b1,
              uint64_t b0, uint64_t ld, uint64_t bs1, uint64_t bs0, uint32_t box_rows,
              bool mn_major);

// Fused causal attention over the packed qkv buffer [batch, seq, 3 * heads * head_dim]
// (head_dim 32 or 64): ctx [batch, seq, heads * head_dim]; per (batch, head, row) statistics
// row_max (max of scores * scale * log2 e) and row_inv (1 / sum of exponentials).
bool attention_supported(uint64_t head_dim);
cudaError_t attention_forward_launch(const float* qkv, float* ctx, float* row_max, float* row_inv,
                                     uint64_t batch, uint64_t seq, uint64_t heads,
                                     uint64_t head_dim, int device, cudaStream_t stream,
                                     uint64_t kv_heads = 0,  // 0: heads (no grouping)
                                     bool round_out = false);  // ctx rounded to nearest TF32
// dqkv (every column of the rows < seq written) from dctx; delta [batch * heads * seq] scratch.
cudaError_t attention_backward_launch(const float* qkv, const float* ctx, const float* dctx,
                                      const float* row_max, const float* row_inv, float* delta,
                                      float* dqkv, uint64_t batch, uint64_t seq, uint64_t heads,
                                      uint64_t head_dim, int device, cudaStream_t stream,
                                      const float* rope_table = nullptr,
                                      cudaStream_t key_stream = nullptr, cudaEvent_t fork = nullptr,
                                      cudaEvent_t join = nullptr, uint64_t kv_heads = 0,
                                      bool round_out = false,  // dqkv rounded to nearest TF32
                                      // optional [batch * seq / 32, packed width] per-32-row
                                      // column sums of dqkv (seq % 32 == 0)
                                      float* column_partials = nullptr);

// Spar's stable sigmoid (src/ops/unary.cpp:55-61 / cuda_kernels.cu:105-111), in fp32.
__device__ __forceinline__ float stable_sigmoid(float v) {
  if (v >= 0.f) return 1.f / (1.f + expf(-v));
  const float e = expf(v);
  return e / (1.f + e);
}

// GELU (tanh form) written through the sigmoid: x * sigmoid(2*sqrt(2/pi)*(x + 0.044715 x^3)).
// Constants are fp32, as Spar's scalar ops round their scalar to the tensor dtype
// (src/ops/scalar.cpp:40).
constexpr float kGeluA = 1.5957691216057308f;  // 2*sqrt(2/pi)
constexpr float kGeluB = 0.044715f;

// Round-to-nearest to a TF32-representable fp32 (10 explicit mantissa bits): add half an ulp
// of the 13 dropped bits, then clear them. The tensor cores read an fp32 operand as TF32 by
// dropping those bits (truncation, biased toward zero); values stored pre-rounded by this enter
// the products unbiased.
__device__ __forceinline__ float round_tf32(float v) {
  const uint32_t b = __float_as_uint(v);
  if ((b & 0x7f800000u) == 0x7f800000u) return v;  // inf / nan unchanged
  return __uint_as_float((b + 0x1000u) & 0xFFFFE000u);
}

// Column sums of a warp's 32 x 32 register box (lane = row, v[c] = column c; rows with
// live == false count as zero): a transposing butterfly over the warp, after which lane l holds
// the sum of column l over the 32 rows. 31 shuffles and adds per lane, no shared memory.
__device__ __forceinline__ float box_column_sum(const float (&v)[32], bool live) {
  const uint32_t lane = threadIdx.x & 31;
  float a[16];
  {
    const bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float lo = live ? v[i] : 0.f, hi = live ? v[i + 16] : 0.f;
      a[i] = (up ? hi : lo) + __shfl_xor_sync(0xffffffffu, up ? lo : hi, 16);
    }
  }
  float b[8];
  {
    const bool up = lane & 8;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      b[i] = (up ? a[i + 8] : a[i]) + __shfl_xor_sync(0xffffffffu, up ? a[i] : a[i + 8], 8);
  }
  float c[4];
  {
    const bool up = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      c[i] = (up ? b[i + 4] : b[i]) + __shfl_xor_sync(0xffffffffu, up ? b[i] : b[i + 4], 4);
  }
  float d[2];
  {
    const bool up = lane & 2;
#pragma unroll
    for (int i = 0; i < 2; ++i)
      d[i] = (up ? c[i + 2] : c[i]) + __shfl_xor_sync(0xffffffffu, up ? c[i] : c[i + 2], 2);
  }
  const bool up = lane & 1;
  return (up ? d[1] : d[0]) + __shfl_xor_sync(0xffffffffu, up ? d[0] : d[1], 1);
}

__device__ __forceinline__ float gelu_value(float x) {
  const float x3 = (x * x) * x;
  const float u = (x + x3 * kGeluB) * kGeluA;
  return x * stable_sigmoid(u);
}

__device__ __forceinline__ float gelu_derivative(float x) {
  const float x2 = x * x;
  const float u = (x + (x2 * x) * kGeluB) * kGeluA;
  const float s = stable_sigmoid(u);
  const float du = kGeluA * (1.f + 3.f * kGeluB * x2);
  return s + x * (s * (1.f - s)) * du;
}

// The same sigmoid / GELU / GELU' through the hardware exponential and an approximate divide
// (__expf, __fdividef: a few ulp from the correctly rounded forms), for GEMM epilogues, where
// the accurate library calls made the epilogue, not the tensor cores, the bound.
__device__ __forceinline__ float fast_sigmoid(float v) {
  const float e = __expf(-fabsf(v));
  const float r = __fdividef(1.f, 1.f + e);
  return v >= 0.f ? r : e * r;
}

__device__ __forceinline__ float gelu_value_fast(float x) {
  const float x3 = (x * x) * x;
  const float u = (x + x3 * kGeluB) * kGeluA;
  return x * fast_sigmoid(u);
}

__device__ __forceinline__ float gelu_derivative_fast(float x) {
  const float x2 = x * x;
  const float u = (x + (x2 * x) * kGeluB) * kGeluA;
  const float s = fast_sigmoid(u);
  const float du = kGeluA * (1.f + 3.f * kGeluB * x2);
  return s + x * (s * (1.f - s)) * du;
}

// ---------------------------------------------------------------- launchers (async, on stream)
// round_out: store y rounded to nearest TF32 (for outputs that only feed TF32 products, which
// would otherwise truncate them: a systematic shrink of about 2^-11 per operand).
cudaError_t layernorm_forward_launch(float* y, float* mean, float* rstd, const float* x,
                                     const float* gamma, const float* beta, uint64_t rows,
                                     uint64_t cols, float eps, int device, cudaStream_t stream,
                                     bool round_out = false);
int layernorm_backward_parts(uint64_t rows, int device);
cudaError_t layernorm_backward_launch(float* dx, float* dgamma, float* dbeta, const float* dy,
                                      const float* x, const float* gamma, const float* mean,
                                      const float* rstd, uint64_t rows, uint64_t cols,
                                      int accumulate_params, int accumulate_dx, float* workspace,
                                      int device, cudaStream_t stream, float* dsum = nullptr);
// RMSNorm (the LayerNorm kernels without centring / bias). Rows of `cols` floats, `group`
// consecutive rows per `ld` floats (ld 0: cols; group = heads for qk-norm inside a projection).
// Backward workspace: layernorm_backward_parts(rows) * cols floats.
cudaError_t rmsnorm_forward_launch(float* y, float* rstd, const float* x, const float* weight,
                                   uint64_t rows, uint64_t cols, float eps, int device,
                                   cudaStream_t stream, uint64_t ld = 0, uint32_t group = 1,
                                   bool round_out = false);
cudaError_t rmsnorm_backward_launch(float* dx, float* dweight, const float* dy, const float* x,
                                    const float* weight, const float* rstd, uint64_t rows,
                                    uint64_t cols, int accumulate_params, int accumulate_dx,
                                    float* workspace, int device, cudaStream_t stream,
                                    uint64_t ld = 0, uint32_t group = 1);
// qk-norm + RoPE of the Spar-family projection (qknorm.cu): out (q | k | v rows of ld floats,
// TF32-rounded) from raw; rstd [tokens * heads] then [tokens * kv_heads]; rope_table may be null.
cudaError_t qk_norm_rope_launch(float* out, const float* raw, uint64_t tokens, uint64_t seq,
                                uint64_t heads, uint64_t kv_heads, uint64_t head_dim, uint64_t ld,
                                const float* wq, const float* wk, float* rstd,
                                const float* rope_table, float eps, int device,
                                cudaStream_t stream, bool round_out = true);
// Backward in place over the dq | dk part of dqk; dwq / dwk (+)= the weight gradients; workspace
// qk_norm_backward_parts(tokens) * 2 * head_dim floats.
int qk_norm_backward_parts(uint64_t tokens, int device);
cudaError_t qk_norm_backward_launch(float* dqk, const float* raw, uint64_t tokens, uint64_t heads,
                                    uint64_t kv_heads, uint64_t head_dim, uint64_t ld,
                                    const float* wq, const float* wk, const float* rstd,
                                    float* dwq, float* dwk, int accumulate, float* workspace,
                                    int device, cudaStream_t stream);
// SwiGLU h = silu(gate) * value and its backward over rows x cols with row strides (floats).
cudaError_t swiglu_forward_launch(float* h, uint64_t ldh, const float* gate, uint64_t ldg,
                                  const float* value, uint64_t ldv, uint64_t rows, uint64_t cols,
                                  int device, cudaStream_t stream);
cudaError_t swiglu_backward_launch(float* dgate, uint64_t lddg, float* dvalue, uint64_t lddv,
                                   const float* dh, uint64_t lddh, const float* gate, uint64_t ldg,
                                   const float* value, uint64_t ldv, uint64_t rows, uint64_t cols,
                                   int device, cudaStream_t stream);

cudaError_t gelu_launch(float* y, const float* dy, const float* x, uint64_t n, int backward,
                        int device, cudaStream_t stream);
cudaError_t rope_table_launch(float* table, uint64_t t, uint64_t d, double theta, uint64_t start,
                              cudaStream_t stream);
// round != 0: results stored rounded to nearest TF32 (rotated q / k that only feed TF32 products).
cudaError_t rope_apply_launch(float* x, const float* table, uint64_t tokens, uint64_t t,
                              uint64_t heads, uint64_t d, uint64_t ld, int inverse, int device,
                              cudaStream_t stream, int round = 0);
int column_sum_parts(uint64_t rows, uint64_t cols, int device);
cudaError_t column_sum_launch(float* out, const float* x, uint64_t rows, uint64_t cols,
                              uint64_t ld, int accumulate, float* workspace, int device,
                              cudaStream_t stream);
cudaError_t sum_launch(float* out, const float* v, uint64_t n, cudaStream_t stream);

cudaError_t causal_softmax_launch(float* out, const float* in, const float* p, uint64_t batch,
                                  uint64_t t, uint64_t ld, float scale, uint64_t zero_fill_block,
                                  int backward, cudaStream_t stream);

// round_out: dlogits stored rounded to nearest TF32 (they only feed TF32 products).
cudaError_t cross_entropy_launch(float* loss, float* dlogits, const float* logits,
                                 const int32_t* targets, uint64_t rows, uint64_t classes,
                                 uint64_t ld, uint64_t sequence_length, float grad_scale,
                                 int32_t* invalid_target, int device, cudaStream_t stream,
                                 bool round_out = false);

// Multi-slice gradient norm + clipped AdamW. `norm_state` holds kNormStateDoubles doubles.
constexpr int kNormStateDoubles = 1024;
struct Slice {
  float* parameter;
  float* gradient;
  float* first_moment;
  float* second_moment;
  uint64_t count;
};
// Device addresses of the flags a GEMM / attention kernel sets when one of its bounded waits
// expires (looked up once per device with that device current); nullptr if the lookup failed.
int* gemm_wait_flag(int device);
int* attention_wait_flag(int device);
// Added to norm_state[1] by the norm pass when a wait flag given to it is set: AdamW then updates
// nothing (as for a non-finite norm) and the step reports cudaErrorTimeout. A non-finite gradient
// adds at most 1 per rank, so the mark stays recognisable after the flags are summed over ranks.
constexpr double kWaitErrorMark = 1024.0;
cudaError_t grad_norm_launch(double* norm_state, const Slice* slices, uint64_t slice_count,
                             int device, cudaStream_t stream, const int* wait_flag_a = nullptr,
                             const int* wait_flag_b = nullptr);
// AdamW scalars for one step (bias corrections c1 = 1 - beta1^step, c2 = 1 - beta2^step).
struct AdamWArgs {
  double lr, beta1, beta2, eps, decay_factor, c1, c2, max_norm;
};
AdamWArgs adamw_args(double max_norm, double lr, double beta1, double beta2, double eps,
                     double weight_decay, uint64_t step);
// args_dev != nullptr: the kernels read the scalars from that device struct instead of the
// values given (so a captured launch can be replayed for later steps).
// rounded_base != nullptr: each updated parameter is also written, rounded to nearest TF32, at the
// same offset from rounded_base as it has from param_base (the copy the TF32 GEMMs read).
cudaError_t adamw_launch(const Slice* slices, uint64_t slice_count, const double* norm_state,
                         double max_norm, double lr, double beta1, double beta2, double eps,
                         double weight_decay, uint64_t step, int32_t* nonfinite_flag, int device,
                         cudaStream_t stream, const AdamWArgs* args_dev = nullptr,
                         const float* param_base = nullptr, float* rounded_base = nullptr);
// dst[i] = src[i] rounded to nearest TF32, i < count.
cudaError_t round_copy_launch(float* dst, const float* src, uint64_t count, int device,
                              cudaStream_t stream);

cudaError_t embedding_forward_launch(float* out, const float* weight, const int32_t* ids,
                                     uint64_t count, uint64_t vocab, uint64_t dim,
                                     int32_t* invalid_index, int device, cudaStream_t stream);
uint64_t embedding_backward_scratch(uint64_t count, uint64_t vocab);
cudaError_t embedding_backward_launch(float* grad_weight, const float* grad_out,
                                      const int32_t* ids, uint64_t count, uint64_t vocab,
                                      uint64_t dim, void* scratch, int device,
                                      cudaStream_t stream);

// Grouped-query attention on the unfused path: k | v (kv_heads heads at column kcol of the
// packed [tokens, ld] projection) expanded to `heads` heads in out [tokens, 2 * heads * dh], and
// the reverse group sum of d(expanded) into dqkv's k | v columns.
cudaError_t repeat_kv_launch(float* out, const float* qkv, uint64_t tokens, uint64_t heads,
                             uint64_t kv_heads, uint64_t dh, uint64_t ld, uint64_t kcol,
                             int device, cudaStream_t stream);
cudaError_t group_sum_launch(float* dqkv, const float* drep, uint64_t tokens, uint64_t heads,
                             uint64_t kv_heads, uint64_t dh, uint64_t ld, uint64_t kcol,
                             int device, cudaStream_t stream);

}  // namespace spar_b200
