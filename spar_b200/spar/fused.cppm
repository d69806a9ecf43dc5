// Spar module `spar.b200`: differentiable fused operations on libspar_b200 for Spar models whose
// tensors live on a CUDA device, recorded on Spar's own autograd tape through its operator
// extension point (detail::record_operation, src/core/tensor.cppm:209-213; raw device pointers
// through detail::CudaTensorAccess, :184-187). Spar itself is unchanged: these are new
// operations a model calls in place of their composed equivalents.
//
//   layer_norm(x, gamma, beta, eps)      one kernel forward, one backward (dx, dgamma, dbeta)
//                                        instead of nine composed ops (mean, subtract, square,
//                                        mean, add_scalar, sqrt, divide, multiply, add)
//   linear_gelu(x, weight, bias)         gelu(x W + b) with the bias and GELU in the GEMM
//                                        epilogue (tanh form, as x * sigmoid(2u)); backward
//                                        dX = dU W^T, dW = X^T dU, db = column sums of dU
//   language_model_cross_entropy(...)    mean NLL of log_softmax over targets = ids shifted by
//                                        one (src/loss/cross_entropy.cpp:176-214), one pass
//                                        writing dlogits; full-vocabulary probabilities are never
//                                        materialised
//   grad_ready(parameter, hook)          identity whose backward receives the parameter's final,
//                                        summed gradient exactly once (Spar sums every
//                                        contribution before a node's backward runs,
//                                        src/autograd/autograd.cpp:231-263): the point where a
//                                        data-parallel bucket can be marked ready
//
// Contract as Spar's backend: float32, contiguous CUDA tensors on one device; calls return after
// the device finished; a failure throws std::runtime_error (std::out_of_range for a class id
// outside the vocabulary). Products run in 3xTF32 unless SPAR_B200_MATMUL_PRECISION is "tf32".
module;

#if SPAR_ENABLE_CUDA
#include <cuda_runtime_api.h>

#include "spar_b200.h"
#endif

export module spar.b200;

import std;
import spar.device;
import spar.dtype;
import spar.shape;
import spar.tensor;
import spar.ops;

export namespace spar::b200 {

[[nodiscard]] Tensor layer_norm(const Tensor& x, const Tensor& gamma, const Tensor& beta,
                                double epsilon = 1e-5);
[[nodiscard]] Tensor linear_gelu(const Tensor& x, const Tensor& weight, const Tensor& bias);
[[nodiscard]] Tensor language_model_cross_entropy(const Tensor& logits, const Tensor& token_ids);
[[nodiscard]] Tensor grad_ready(const Tensor& parameter,
                                std::function<void(const Tensor& gradient)> hook);

} // namespace spar::b200

namespace spar::b200 {
namespace {

#if SPAR_ENABLE_CUDA

void check(SparCudaStatus status, std::string_view operation) {
  if (status.code == 0) {
    return;
  }
  throw std::runtime_error{std::string{operation} + " failed: " +
                           (status.code == 1 ? std::string{"invalid argument"}
                                             : std::string{cudaGetErrorString(
                                                   static_cast<cudaError_t>(status.cuda_error))})};
}

// Synchronous like the rest of Spar's CUDA backend: the device finished before the call returns.
void finish(const Device& device, std::string_view operation) {
  int previous{0};
  cudaError_t e{cudaGetDevice(&previous)};
  if (e == cudaSuccess && previous != device.index()) {
    e = cudaSetDevice(device.index());
  }
  if (e == cudaSuccess) {
    e = cudaDeviceSynchronize();
  }
  if (previous != device.index()) {
    static_cast<void>(cudaSetDevice(previous));
  }
  if (e != cudaSuccess) {
    check(SparCudaStatus{2, static_cast<int>(e)}, operation);
  }
}

void require(const Tensor& t, const Device& device, std::string_view operation) {
  if (!t.device().is_cuda() || t.device() != device || t.dtype() != DType::Float32) {
    throw std::invalid_argument{std::string{operation} +
                                " requires float32 tensors on one CUDA device"};
  }
}

float* data(Tensor& t) { return static_cast<float*>(detail::CudaTensorAccess::mutable_data(t)); }
const float* data(const Tensor& t) {
  return static_cast<const float*>(detail::CudaTensorAccess::data(t));
}

int precision() {
  const char* v = std::getenv("SPAR_B200_MATMUL_PRECISION");
  return (v != nullptr && std::string_view{v} == "tf32") ? SPAR_B200_TF32 : SPAR_B200_TF32X3;
}

std::size_t rows_of(const Tensor& t) {
  std::size_t rows{1};
  for (std::size_t i{0}; i + 1 < t.rank(); ++i) {
    rows *= static_cast<std::size_t>(t.shape()[i]);
  }
  return rows;
}

// C [m, n] = op(A) op(B) with Spar's row-major layouts (op = transpose read in place).
void gemm(std::size_t m, std::size_t n, std::size_t k, const float* a, bool at, const float* b,
          bool bt, float* c, int epilogue, const float* bias, float* aux, const Device& device) {
  SparB200Gemm g{};
  g.m = m;
  g.n = n;
  g.k = k;
  g.batch[0] = 1;
  g.batch[1] = 1;
  g.a = a;
  g.lda = at ? m : k;
  g.a_transposed = at ? 1 : 0;
  g.b = b;
  g.ldb = bt ? k : n;
  g.b_transposed = bt ? 1 : 0;
  g.c = c;
  g.ldc = n;
  g.alpha = 1.0F;
  g.epilogue = epilogue;
  g.bias = bias;
  g.aux = aux;
  g.ldaux = aux != nullptr ? n : 0;
  g.precision = precision();
  check(spar_b200_gemm(&g, device.index(), nullptr), "spar_b200_gemm");
}

#else

[[noreturn]] void unavailable() {
  throw std::runtime_error{"Spar was built without CUDA support"};
}

#endif

} // namespace

Tensor layer_norm(const Tensor& x, const Tensor& gamma, const Tensor& beta, double epsilon) {
#if SPAR_ENABLE_CUDA
  const Device device{x.device()};
  for (const Tensor* t : {&x, &gamma, &beta}) {
    require(*t, device, "b200::layer_norm");
  }
  const std::size_t cols{static_cast<std::size_t>(x.shape()[x.rank() - 1])};
  const std::size_t rows{rows_of(x)};
  if (gamma.numel() != cols || beta.numel() != cols) {
    throw std::invalid_argument{"b200::layer_norm: gamma and beta must have the last extent"};
  }
  const Tensor xc{x.contiguous()};
  const Tensor gc{gamma.contiguous()};
  const Tensor bc{beta.contiguous()};
  Tensor y{x.shape(), DType::Float32, device};
  Tensor mean{Shape{static_cast<Shape::dimension_type>(rows)}, DType::Float32, device};
  Tensor rstd{Shape{static_cast<Shape::dimension_type>(rows)}, DType::Float32, device};
  check(spar_b200_layernorm_forward(data(y), data(mean), data(rstd), data(xc), data(gc), data(bc),
                                    rows, cols, static_cast<float>(epsilon), device.index(),
                                    nullptr),
        "spar_b200_layernorm_forward");
  finish(device, "b200::layer_norm");
  std::vector<Tensor> parents;
  const bool gx{x.requires_grad()}, gg{gamma.requires_grad()}, gb{beta.requires_grad()};
  if (gx) parents.push_back(x);
  if (gg) parents.push_back(gamma);
  if (gb) parents.push_back(beta);
  if (!parents.empty()) {
    const Tensor sx{xc.detach()}, sg{gc.detach()};
    detail::record_operation(
        y, std::move(parents),
        [sx, sg, mean, rstd, rows, cols, gx, gg, gb, device](const Tensor& gradient) {
          const Tensor dy{gradient.contiguous()};
          Tensor dx{sx.shape(), DType::Float32, device};
          Tensor dgamma{sg.shape(), DType::Float32, device};
          Tensor dbeta{sg.shape(), DType::Float32, device};
          check(spar_b200_layernorm_backward(data(dx), data(dgamma), data(dbeta), data(dy),
                                             data(sx), data(sg), data(mean), data(rstd), rows,
                                             cols, 0, 0, device.index(), nullptr),
                "spar_b200_layernorm_backward");
          finish(device, "b200::layer_norm backward");
          std::vector<Tensor> out;
          if (gx) out.push_back(dx);
          if (gg) out.push_back(dgamma);
          if (gb) out.push_back(dbeta);
          return out;
        });
  }
  return y;
#else
  static_cast<void>(x);
  static_cast<void>(gamma);
  static_cast<void>(beta);
  static_cast<void>(epsilon);
  unavailable();
#endif
}

Tensor linear_gelu(const Tensor& x, const Tensor& weight, const Tensor& bias) {
#if SPAR_ENABLE_CUDA
  const Device device{x.device()};
  for (const Tensor* t : {&x, &weight, &bias}) {
    require(*t, device, "b200::linear_gelu");
  }
  if (weight.rank() != 2 || x.shape()[x.rank() - 1] != weight.shape()[0] ||
      bias.numel() != static_cast<std::size_t>(weight.shape()[1])) {
    throw std::invalid_argument{"b200::linear_gelu: x [..., in], weight [in, out], bias [out]"};
  }
  const std::size_t in{static_cast<std::size_t>(weight.shape()[0])};
  const std::size_t outf{static_cast<std::size_t>(weight.shape()[1])};
  const std::size_t rows{rows_of(x)};
  const Tensor xc{x.contiguous()};
  const Tensor wc{weight.contiguous()};
  const Tensor bc{bias.contiguous()};
  std::vector<Shape::dimension_type> dims(x.shape().dimensions().begin(),
                                          x.shape().dimensions().end());
  dims.back() = static_cast<Shape::dimension_type>(outf);
  Tensor y{Shape{dims}, DType::Float32, device};
  Tensor pre{Shape{dims}, DType::Float32, device};  // pre-activation, kept for the backward
  gemm(rows, outf, in, data(xc), false, data(wc), false, data(y), SPAR_B200_EPI_BIAS_GELU,
       data(bc), data(pre), device);
  finish(device, "b200::linear_gelu");
  std::vector<Tensor> parents;
  const bool gx{x.requires_grad()}, gw{weight.requires_grad()}, gb{bias.requires_grad()};
  if (gx) parents.push_back(x);
  if (gw) parents.push_back(weight);
  if (gb) parents.push_back(bias);
  if (!parents.empty()) {
    const Tensor sx{xc.detach()}, sw{wc.detach()};
    detail::record_operation(
        y, std::move(parents),
        [sx, sw, pre, rows, in, outf, gx, gw, gb, device](const Tensor& gradient) {
          const Tensor dy{gradient.contiguous()};
          Tensor du{pre.shape(), DType::Float32, device};  // dy o gelu'(pre)
          check(spar_b200_gelu_backward(data(du), data(dy), data(pre), rows * outf,
                                        device.index(), nullptr),
                "spar_b200_gelu_backward");
          std::vector<Tensor> out;
          if (gx) {
            Tensor dx{sx.shape(), DType::Float32, device};
            gemm(rows, in, outf, data(du), false, data(sw), true, data(dx), SPAR_B200_EPI_NONE,
                 nullptr, nullptr, device);
            out.push_back(dx);
          }
          if (gw) {
            Tensor dw{sw.shape(), DType::Float32, device};
            gemm(in, outf, rows, data(sx), true, data(du), false, data(dw), SPAR_B200_EPI_NONE,
                 nullptr, nullptr, device);
            out.push_back(dw);
          }
          if (gb) {
            Tensor db{Shape{static_cast<Shape::dimension_type>(outf)}, DType::Float32, device};
            check(spar_b200_column_sum(data(db), data(du), rows, outf, outf, 0, device.index(),
                                       nullptr),
                  "spar_b200_column_sum");
            out.push_back(db);
          }
          finish(device, "b200::linear_gelu backward");
          return out;
        });
  }
  return y;
#else
  static_cast<void>(x);
  static_cast<void>(weight);
  static_cast<void>(bias);
  unavailable();
#endif
}

Tensor language_model_cross_entropy(const Tensor& logits, const Tensor& token_ids) {
#if SPAR_ENABLE_CUDA
  const Device device{logits.device()};
  require(logits, device, "b200::language_model_cross_entropy");
  if (logits.rank() != 3 || token_ids.rank() != 2 || token_ids.device() != device ||
      token_ids.dtype() != DType::Int32 || token_ids.shape()[0] != logits.shape()[0] ||
      token_ids.shape()[1] != logits.shape()[1] || logits.shape()[1] < 2) {
    throw std::invalid_argument{
        "b200::language_model_cross_entropy requires logits [B,T,V] and int32 IDs [B,T]"};
  }
  const std::size_t batch{static_cast<std::size_t>(logits.shape()[0])};
  const std::size_t seq{static_cast<std::size_t>(logits.shape()[1])};
  const std::size_t classes{static_cast<std::size_t>(logits.shape()[2])};
  const std::size_t rows{batch * seq};
  const double predictions{static_cast<double>(batch * (seq - 1))};
  const Tensor z{logits.contiguous()};
  const Tensor ids{token_ids.contiguous()};
  Tensor row_loss{Shape{static_cast<Shape::dimension_type>(rows)}, DType::Float32, device};
  Tensor dlogits{logits.shape(), DType::Float32, device};  // d(mean loss) / d logits
  Tensor invalid{Shape{1}, DType::Int32, device};
  check(spar_b200_cross_entropy_forward_backward(
            data(row_loss), data(dlogits), data(z),
            static_cast<const int32_t*>(detail::CudaTensorAccess::data(ids)), rows, classes,
            classes, seq, static_cast<float>(1.0 / predictions),
            static_cast<int32_t*>(detail::CudaTensorAccess::mutable_data(invalid)),
            device.index(), nullptr),
        "spar_b200_cross_entropy_forward_backward");
  finish(device, "b200::language_model_cross_entropy");
  const Tensor flag{invalid.to(Device::cpu())};
  if (flag.span<std::int32_t>()[0] != 0) {
    throw std::out_of_range{"b200::language_model_cross_entropy: class ID outside the vocabulary"};
  }
  // Rows without a target (each sequence's last position) hold 0: the mean is sum / (B (T - 1)).
  Tensor loss{multiply_scalar(sum(row_loss), 1.0 / predictions)};
  if (logits.requires_grad()) {
    detail::record_operation(loss, {logits}, [dlogits](const Tensor& gradient) {
      return std::vector<Tensor>{multiply(dlogits, gradient)};
    });
  }
  return loss;
#else
  static_cast<void>(logits);
  static_cast<void>(token_ids);
  unavailable();
#endif
}

Tensor grad_ready(const Tensor& parameter, std::function<void(const Tensor& gradient)> hook) {
  Tensor view{parameter.detach()};
  if (parameter.requires_grad()) {
    detail::record_operation(view, {parameter},
                             [hook = std::move(hook)](const Tensor& gradient) {
                               if (hook) {
                                 hook(gradient);
                               }
                               return std::vector<Tensor>{gradient};
                             });
  }
  return view;
}

} // namespace spar::b200
