// Contiguous batched matmul of any shape: the body behind Spar's cuBLAS seam
// spar::detail::cuda_blas::matmul (src/backend/cuda_blas.cppm:122-194).
//
// The reference loops cublasSgemm / cublasDgemm over the batch (FP32 SIMT math, since it never
// enables TF32). Here:
//   - Float32 runs on the tcgen05 GEMM (spar_b200_gemm) in the requested precision (3xTF32 is
//     fp32-faithful, TF32 is the fast mode), the whole batch in one launch. The tensor-core GEMM
//     needs 16-byte aligned rows; shapes whose k or n is not a multiple of 4 (or whose tensors start
//     off a 16-byte boundary) are staged through zero-padded copies (pitched 2-D copies, no kernel)
//     and the result copied back.
//   - Float64 runs on a shared-memory-tiled SIMT kernel (no FP64 tensor-core path is used).
#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

constexpr int kTile = 64;   // output tile per block (kTile x kTile)
constexpr int kDepth = 16;  // k slice staged per iteration

// C[b] = A[b] · B[b], row-major contiguous [m, k] · [k, n] -> [m, n], double precision.
// 256 threads, each owns a 4 x 4 block of the 64 x 64 tile; A and B slices staged in shared memory.
__global__ void __launch_bounds__(256)
gemm_f64_kernel(const double* __restrict__ a, const double* __restrict__ b, double* __restrict__ c,
                uint64_t m, uint64_t n, uint64_t k) {
  __shared__ double as[kDepth][kTile + 1];
  __shared__ double bs[kDepth][kTile + 1];
  const uint64_t batch = blockIdx.z;
  a += batch * m * k;
  b += batch * k * n;
  c += batch * m * n;
  const uint64_t row0 = static_cast<uint64_t>(blockIdx.y) * kTile;
  const uint64_t col0 = static_cast<uint64_t>(blockIdx.x) * kTile;
  const int tr = threadIdx.x / 16, tc = threadIdx.x % 16;  // 16 x 16 threads, 4 x 4 each
  double acc[4][4] = {};
  for (uint64_t k0 = 0; k0 < k; k0 += kDepth) {
    for (int i = threadIdx.x; i < kDepth * kTile; i += blockDim.x) {
      const int kk = i % kDepth, r = i / kDepth;  // A tile: rows r, k slice kk
      const uint64_t gr = row0 + r, gk = k0 + kk;
      as[kk][r] = (gr < m && gk < k) ? a[gr * k + gk] : 0.0;
      const int cc = i % kTile, kb = i / kTile;   // B tile: k slice kb, columns cc
      const uint64_t gkb = k0 + kb, gc = col0 + cc;
      bs[kb][cc] = (gkb < k && gc < n) ? b[gkb * n + gc] : 0.0;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kDepth; ++kk) {
      double av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = as[kk][tr * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tc * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t gr = row0 + tr * 4 + i;
    if (gr >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t gc = col0 + tc * 4 + j;
      if (gc < n) c[gr * n + gc] = acc[i][j];
    }
  }
}

uint64_t round4(uint64_t x) { return (x + 3) & ~3ull; }

bool aligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

SparB200Gemm contiguous_desc(const float* a, const float* b, float* c, uint64_t batch, uint64_t m,
                             uint64_t k, uint64_t n, uint64_t lda, uint64_t ldb, uint64_t ldc,
                             int precision) {
  SparB200Gemm g{};
  g.m = m;
  g.n = n;
  g.k = k;
  g.batch[0] = batch;
  g.batch[1] = 1;
  g.a = a;
  g.lda = lda;
  g.a_batch_stride[0] = m * lda;
  g.b = b;
  g.ldb = ldb;
  g.b_batch_stride[0] = k * ldb;
  g.c = c;
  g.ldc = ldc;
  g.c_batch_stride[0] = m * ldc;
  g.alpha = 1.0f;
  g.precision = precision;
  return g;
}

}  // namespace
}  // namespace spar_b200

using namespace spar_b200;

// C[b] = A[b] · B[b] for b < batch, all three row-major and contiguous ([batch, m, k],
// [batch, k, n], [batch, m, n]); dtype SPAR_CUDA_FLOAT32 (precision SparB200Precision) or
// SPAR_CUDA_FLOAT64 (precision ignored). Asynchronous on `stream`.
extern "C" SparCudaStatus spar_b200_matmul(const void* a, const void* b, void* c, uint64_t batch,
                                           uint64_t m, uint64_t k, uint64_t n, int dtype,
                                           int precision, int device, void* stream) {
  if (dtype != SPAR_CUDA_FLOAT32 && dtype != SPAR_CUDA_FLOAT64) return invalid();
  if (dtype == SPAR_CUDA_FLOAT32 && precision != SPAR_B200_TF32 && precision != SPAR_B200_TF32X3)
    return invalid();
  if (batch == 0 || m == 0 || n == 0) return ok();
  if (!a || !b || !c) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t esize = dtype == SPAR_CUDA_FLOAT32 ? sizeof(float) : sizeof(double);
  if (k == 0) {  // empty reduction: zeros
    const cudaError_t e = cudaMemsetAsync(c, 0, batch * m * n * esize, s);
    return e == cudaSuccess ? ok() : runtime(e);
  }
  if (dtype == SPAR_CUDA_FLOAT64) {
    if (batch > 65535 || (n + kTile - 1) / kTile > 0x7fffffffull || (m + kTile - 1) / kTile > 65535)
      return invalid();
    dim3 grid(static_cast<unsigned>((n + kTile - 1) / kTile),
              static_cast<unsigned>((m + kTile - 1) / kTile), static_cast<unsigned>(batch));
    gemm_f64_kernel<<<grid, 256, 0, s>>>(static_cast<const double*>(a),
                                         static_cast<const double*>(b), static_cast<double*>(c), m,
                                         n, k);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : runtime(e);
  }
  const float* af = static_cast<const float*>(a);
  const float* bf = static_cast<const float*>(b);
  float* cf = static_cast<float*>(c);
  if (k % 4 == 0 && n % 4 == 0 && aligned(af) && aligned(bf) && aligned(cf)) {
    const SparB200Gemm g = contiguous_desc(af, bf, cf, batch, m, k, n, k, n, n, precision);
    return spar_b200_gemm(&g, device, stream);
  }
  // Staged: A' [batch*m, k4], B' [batch, k4, n4] and C' [batch*m, n4], zero padded.
  const uint64_t k4 = round4(k), n4 = round4(n);
  float* pa = nullptr;
  float* pb = nullptr;
  float* pc = nullptr;
  const uint64_t fa = batch * m * k4, fb = batch * k4 * n4, fc = batch * m * n4;
  cudaError_t e = stream_alloc(reinterpret_cast<void**>(&pa), (fa + fb + fc) * sizeof(float), s);
  if (e != cudaSuccess) return runtime(e);
  pb = pa + fa;
  pc = pb + fb;
  e = cudaMemsetAsync(pa, 0, (fa + fb) * sizeof(float), s);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(pa, k4 * sizeof(float), af, k * sizeof(float), k * sizeof(float),
                          batch * m, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess && k4 == k) {  // B' rows line up across the batch: one pitched copy
    e = cudaMemcpy2DAsync(pb, n4 * sizeof(float), bf, n * sizeof(float), n * sizeof(float),
                          batch * k, cudaMemcpyDeviceToDevice, s);
  } else {
    for (uint64_t i = 0; i < batch && e == cudaSuccess; ++i)
      e = cudaMemcpy2DAsync(pb + i * k4 * n4, n4 * sizeof(float), bf + i * k * n, n * sizeof(float),
                            n * sizeof(float), k, cudaMemcpyDeviceToDevice, s);
  }
  SparCudaStatus st = ok();
  if (e == cudaSuccess) {
    const SparB200Gemm g = contiguous_desc(pa, pb, pc, batch, m, k4, n4, k4, n4, n4, precision);
    st = spar_b200_gemm(&g, device, stream);
  }
  if (e == cudaSuccess && st.code == 0)
    e = cudaMemcpy2DAsync(cf, n * sizeof(float), pc, n4 * sizeof(float), n * sizeof(float),
                          batch * m, cudaMemcpyDeviceToDevice, s);
  const cudaError_t f = cudaFreeAsync(pa, s);
  if (st.code != 0) return st;
  if (e != cudaSuccess) return runtime(e);
  return f == cudaSuccess ? ok() : runtime(f);
}
