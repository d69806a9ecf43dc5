// Spar module `spar.cuda_blas` for a Spar build on libspar_b200: replaces the reference's
// src/backend/cuda_blas.cppm (same module name, same exported function, same contract) so that
// every Spar matmul on a CUDA tensor runs on the B200 tensor cores instead of a cublasSgemm /
// cublasDgemm loop per batch matrix (reference cuda_blas.cppm:122-194).
//
// Contract kept from the reference: both operands contiguous, same device, same floating dtype;
// output [output_shape] = batch x [m, n] of A [m, k] x B [k, n]; k == 0 gives zeros; errors
// throw std::runtime_error naming the operation and device; the call returns after the device
// finished (Spar's backend is synchronous). Float32 runs in 3xTF32 (fp32-faithful) unless the
// environment variable SPAR_B200_MATMUL_PRECISION is "tf32"; Float64 runs on a SIMT kernel.
module;

#if SPAR_ENABLE_CUDA
#include <cuda_runtime_api.h>

#include "spar_b200.h"
#endif

export module spar.cuda_blas;

import std;
import spar.dtype;
import spar.shape;
import spar.tensor;

export namespace spar::detail::cuda_blas {

[[nodiscard]] Tensor matmul(const Tensor& a, const Tensor& b, Shape output_shape, std::size_t m,
                            std::size_t k, std::size_t n);

} // namespace spar::detail::cuda_blas

namespace spar::detail::cuda_blas {
namespace {

#if SPAR_ENABLE_CUDA

// Read on every call (next to a synchronous matmul the lookup costs nothing), so a process can
// switch modes between steps.
int float32_precision() {
  const char* v = std::getenv("SPAR_B200_MATMUL_PRECISION");
  return (v != nullptr && std::string_view{v} == "tf32") ? SPAR_B200_TF32 : SPAR_B200_TF32X3;
}

[[noreturn]] void fail(std::string_view operation, Device device, SparCudaStatus status) {
  std::string what{std::string{operation} + " failed on cuda:" + std::to_string(device.index()) +
                   ": "};
  what += status.code == 1 ? std::string{"invalid argument"}
                           : std::string{cudaGetErrorString(static_cast<cudaError_t>(status.cuda_error))};
  throw std::runtime_error{what};
}

#else

[[noreturn]] void unavailable() {
  throw std::runtime_error{"Spar was built without CUDA support"};
}

#endif

} // namespace

Tensor matmul(const Tensor& a, const Tensor& b, Shape output_shape, std::size_t m, std::size_t k,
              std::size_t n) {
#if SPAR_ENABLE_CUDA
  if (!a.device().is_cuda() || a.device() != b.device() || !a.is_contiguous() ||
      !b.is_contiguous() || a.dtype() != b.dtype() ||
      (a.dtype() != DType::Float32 && a.dtype() != DType::Float64)) {
    throw std::logic_error{"Internal CUDA matmul received invalid tensors"};
  }
  Tensor output{std::move(output_shape), a.dtype(), a.device()};
  if (output.numel() == 0) {
    return output;
  }
  if (m == 0 || n == 0) {
    throw std::logic_error{"Internal CUDA matmul received invalid geometry"};
  }
  const std::size_t matrix{m * n};
  if (output.numel() % matrix != 0) {
    throw std::logic_error{"Internal CUDA matmul output geometry is inconsistent"};
  }
  const std::size_t batch{output.numel() / matrix};
  if (a.numel() != batch * m * k || b.numel() != batch * k * n) {
    throw std::logic_error{"Internal CUDA matmul input geometry is inconsistent"};
  }
  const Device device{output.device()};
  const int dtype{a.dtype() == DType::Float32 ? SPAR_CUDA_FLOAT32 : SPAR_CUDA_FLOAT64};
  SparCudaStatus status{spar_b200_matmul(CudaTensorAccess::data(a), CudaTensorAccess::data(b),
                                         CudaTensorAccess::mutable_data(output), batch, m, k, n,
                                         dtype, float32_precision(),
                                         static_cast<int>(device.index()), nullptr)};
  if (status.code != 0) {
    fail("spar_b200_matmul", device, status);
  }
  int previous{0};
  cudaError_t synced{cudaGetDevice(&previous)};
  if (synced == cudaSuccess) {
    const bool switched{previous != static_cast<int>(device.index())};
    if (switched) {
      synced = cudaSetDevice(static_cast<int>(device.index()));
    }
    if (synced == cudaSuccess) {
      synced = cudaDeviceSynchronize();
    }
    if (switched) {
      static_cast<void>(cudaSetDevice(previous));
    }
  }
  if (synced != cudaSuccess) {
    fail("CUDA matmul synchronization", device, SparCudaStatus{2, static_cast<int>(synced)});
  }
  return output;
#else
  static_cast<void>(a);
  static_cast<void>(b);
  static_cast<void>(output_shape);
  static_cast<void>(m);
  static_cast<void>(k);
  static_cast<void>(n);
  unavailable();
#endif
}

} // namespace spar::detail::cuda_blas
