// LayerNorm forward/backward over the last axis, fp32.
//
// Spar has no LayerNorm op. The harness composes it from Spar ops in the order
//   mean(x) -> subtract -> square -> mean -> add_scalar(eps) -> sqrt -> divide -> multiply(gamma)
//   -> add(beta)
// which is the RMSNorm pattern of src/nn/rmsnorm.cpp:50-52 with a centring step; the forward here
// evaluates that chain per element with the division by sqrt(var + eps) taken as a multiply by
// rstd = 1 / sqrt(var + eps) (within an ulp of the divide). The backward is the closed form of
// that chain's autograd:
//   xhat = (x - mean) * rstd, g = dy * gamma
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), dgamma = sum_rows dy * xhat, dbeta = sum dy
// RMSNorm itself (nn::RMSNorm, src/nn/rmsnorm.cpp:40-53: mean(square(x)), add_scalar(eps), sqrt,
// divide, multiply(weight)) is the same kernels without the centring and the bias (kRms):
//   y = x * rstd * w, rstd = 1 / sqrt(mean(x^2) + eps)
//   dx = rstd * (g - xhat * mean(g * xhat)) with xhat = x * rstd, dw = sum_rows dy * xhat
//
// Layout: one warp per row, the row held in registers as float4 (lane l owns float4 columns
// l, l + 32, ...), so x and dy are read from HBM exactly once per pass. dgamma/dbeta are
// accumulated per warp in shared memory, reduced over the block's warps in a fixed order and
// written as one partial row per block; a second kernel sums the partials in a fixed order
// (deterministic, no atomics).
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

constexpr int kWarps = 8;  // rows in flight per block

// Where row r of x / y / dy / dx starts: rows of `cols` floats, `group` consecutive rows per
// stride of `ld` floats (group 1, ld = cols: a plain [rows, cols] matrix; group = heads,
// ld = the projection's row stride: the heads of one token inside a packed q / k projection).
struct RowMap {
  uint64_t ld;
  uint32_t group;
  __device__ __forceinline__ uint64_t operator()(uint64_t row, int cols) const {
    return group == 1 ? row * ld : (row / group) * ld + (row % group) * static_cast<uint64_t>(cols);
  }
};

// One warp per row, the row in registers (VPL float4 per lane); gamma and beta are read per use
// (L1-resident, the same for every row) rather than held, which keeps the registers low enough
// for three blocks (24 rows in flight) per SM.
template <int VPL, bool kRms>
__global__ void __launch_bounds__(kWarps * 32, 3)
layernorm_forward_kernel(float* __restrict__ y, float* __restrict__ mean_out,
                         float* __restrict__ rstd_out, const float* __restrict__ x,
                         const float* __restrict__ gamma, const float* __restrict__ beta,
                         uint64_t rows, int cols, float eps, RowMap rm, int round_out) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int vec_cols = cols >> 2;
  const float inv_cols = 1.0f / static_cast<float>(cols);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  const uint64_t warp_global = (static_cast<uint64_t>(blockIdx.x) * kWarps) + (threadIdx.x >> 5);
  const uint64_t warp_stride = static_cast<uint64_t>(gridDim.x) * kWarps;
  for (uint64_t row = warp_global; row < rows; row += warp_stride) {
    const float4* xr = reinterpret_cast<const float4*>(x + rm(row, cols));
    float4 v[VPL];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int f = lane + 32 * j;
      if (f < vec_cols) {
        v[j] = ld_stream(xr + f);
        if constexpr (!kRms) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
      }
    }
    float mean = 0.f;
    if constexpr (!kRms) mean = warp_sum(s) * inv_cols;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int f = lane + 32 * j;
      if (f < vec_cols) {
        const float a = v[j].x - mean, c = v[j].y - mean, d = v[j].z - mean, e = v[j].w - mean;
        q += (a * a + c * c) + (d * d + e * e);
      }
    }
    const float var = warp_sum(q) * inv_cols;
    const float rstd = 1.0f / sqrtf(var + eps);
    float4* yr = reinterpret_cast<float4*>(y + rm(row, cols));
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int f = lane + 32 * j;
      if (f < vec_cols) {
        const float4 g = __ldg(g4 + f);
        float4 o;
        if constexpr (kRms) {
          o = make_float4(v[j].x * rstd * g.x, v[j].y * rstd * g.y, v[j].z * rstd * g.z,
                          v[j].w * rstd * g.w);
        } else {
          const float4 b = __ldg(b4 + f);
          o.x = (v[j].x - mean) * rstd * g.x + b.x;
          o.y = (v[j].y - mean) * rstd * g.y + b.y;
          o.z = (v[j].z - mean) * rstd * g.z + b.z;
          o.w = (v[j].w - mean) * rstd * g.w + b.w;
        }
        if (round_out) {  // the output only feeds TF32 products: round to nearest once here
          o.x = round_tf32(o.x);
          o.y = round_tf32(o.y);
          o.z = round_tf32(o.z);
          o.w = round_tf32(o.w);
        }
        yr[f] = o;  // read next by the projection GEMM: left in L2
      }
    }
    if (lane == 0) {
      if constexpr (!kRms) mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

template <int VPL, bool kRms>
__global__ void __launch_bounds__(kWarps * 32, VPL <= 8 ? 2 : 1)
layernorm_backward_kernel(float* __restrict__ dx, float* __restrict__ partial_dgamma,
                          float* __restrict__ partial_dbeta, float* __restrict__ partial_dsum,
                          const float* __restrict__ dy, const float* __restrict__ x,
                          const float* __restrict__ gamma, const float* __restrict__ mean_in,
                          const float* __restrict__ rstd_in, uint64_t rows, int cols,
                          uint64_t rows_per_block, int accumulate_dx, RowMap rm) {
  pdl_begin();
  // Per-warp dgamma / dbeta accumulators live in shared memory ([kWarps][cols] twice; lane l
  // owns float4 columns l, l + 32, ... of its warp's slice), which keeps the registers for the
  // row in flight and lets two blocks share an SM. With partial_dsum, a third slice sums the
  // stored dx rows: the column sums of dx (the bias gradient of the layer whose output dx is).
  extern __shared__ float smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vec_cols = cols >> 2;
  const float inv_cols = 1.0f / static_cast<float>(cols);
  const bool with_sum = partial_dsum != nullptr;
  constexpr int kSumSlice = kRms ? 1 : 2;  // RMSNorm has no dbeta slice
  float4* acc_g = reinterpret_cast<float4*>(smem + warp * cols);
  float4* acc_b = reinterpret_cast<float4*>(smem + (kWarps + warp) * cols);
  float4* acc_s = reinterpret_cast<float4*>(smem + (kSumSlice * kWarps + warp) * cols);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int f = lane + 32 * j;
    if (f < vec_cols) {
      acc_g[f] = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (!kRms) acc_b[f] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (with_sum) acc_s[f] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const uint64_t row_begin = static_cast<uint64_t>(blockIdx.x) * rows_per_block;
  uint64_t row_end = row_begin + rows_per_block;
  if (row_end > rows) row_end = rows;
  for (uint64_t row = row_begin + warp; row < row_end; row += kWarps) {
    const uint64_t off = rm(row, cols);
    const float4* xr = reinterpret_cast<const float4*>(x + off);
    const float4* dyr = reinterpret_cast<const float4*>(dy + off);
    float4* dxr = reinterpret_cast<float4*>(dx + off);
    const float mean = kRms ? 0.f : mean_in[row], rstd = rstd_in[row];
    float4 xh[VPL], d[VPL], prev[VPL];
    // Issue every load of the row (x, dy and the dx being accumulated into) before any use.
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int f = lane + 32 * j;
      if (f < vec_cols) {
        xh[j] = ld_stream(xr + f);
        d[j] = ld_stream(dyr + f);
        if (accumulate_dx) prev[j] = dxr[f];
      }
    }
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int f = lane + 32 * j;
      if (f < vec_cols) {
        xh[j] = make_float4((xh[j].x - mean) * rstd, (xh[j].y - mean) * rstd,
                            (xh[j].z - mean) * rstd, (xh[j].w - mean) * rstd);
        const float4 g = __ldg(g4 + f);
        const float g0 = d[j].x * g.x, g1 = d[j].y * g.y, g2 = d[j].z * g.z, g3 = d[j].w * g.w;
        if constexpr (!kRms) sg += (g0 + g1) + (g2 + g3);
        sgx += (g0 * xh[j].x + g1 * xh[j].y) + (g2 * xh[j].z + g3 * xh[j].w);
        float4 ag = acc_g[f];
        ag.x += d[j].x * xh[j].x;
        ag.y += d[j].y * xh[j].y;
        ag.z += d[j].z * xh[j].z;
        ag.w += d[j].w * xh[j].w;
        acc_g[f] = ag;
        if constexpr (!kRms) {
          float4 ab = acc_b[f];
          ab.x += d[j].x;
          ab.y += d[j].y;
          ab.z += d[j].z;
          ab.w += d[j].w;
          acc_b[f] = ab;
        }
      }
    }
    float mg = 0.f;
    if constexpr (!kRms) mg = warp_sum(sg) * inv_cols;
    const float mgx = warp_sum(sgx) * inv_cols;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int f = lane + 32 * j;
      if (f < vec_cols) {
        const float4 g = __ldg(g4 + f);
        float4 o;
        o.x = rstd * (d[j].x * g.x - mg - xh[j].x * mgx);
        o.y = rstd * (d[j].y * g.y - mg - xh[j].y * mgx);
        o.z = rstd * (d[j].z * g.z - mg - xh[j].z * mgx);
        o.w = rstd * (d[j].w * g.w - mg - xh[j].w * mgx);
        if (accumulate_dx) {
          o.x += prev[j].x;
          o.y += prev[j].y;
          o.z += prev[j].z;
          o.w += prev[j].w;
        }
        dxr[f] = o;
        if (with_sum) {
          float4 as = acc_s[f];
          as.x += o.x;
          as.y += o.y;
          as.z += o.z;
          as.w += o.w;
          acc_s[f] = as;
        }
      }
    }
  }
  // Reduce the per-warp partials over the block (fixed warp order).
  __syncthreads();
  const float* sg_ = smem;
  const float* sb_ = smem + kWarps * cols;
  const float* ss_ = smem + kSumSlice * kWarps * cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float a = 0.f, bsum = 0.f, ssum = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      a += sg_[w * cols + c];
      if constexpr (!kRms) bsum += sb_[w * cols + c];
      if (with_sum) ssum += ss_[w * cols + c];
    }
    partial_dgamma[static_cast<uint64_t>(blockIdx.x) * cols + c] = a;
    if constexpr (!kRms) partial_dbeta[static_cast<uint64_t>(blockIdx.x) * cols + c] = bsum;
    if (with_sum) partial_dsum[static_cast<uint64_t>(blockIdx.x) * cols + c] = ssum;
  }
}

// Sums `parts` partial rows of length cols in a fixed order; out (+)= result. blockIdx.y picks
// the array (0: dgamma, 1: dbeta, 2: dx column sums). Block = 32 columns x 16 warps: warp w
// sums parts w, w + 16, ... into four interleaved accumulators (independent loads in flight),
// combined in a fixed order; warp 0 then adds the 16 warp sums in warp order (deterministic).
struct PartialJobs {
  float* out[3];
  const float* part[3];
  int accumulate[3];
};

constexpr int kReduceWarps = 16;

__global__ void __launch_bounds__(kReduceWarps * 32)
reduce_partials_kernel(const __grid_constant__ PartialJobs jobs, int parts, int cols) {
  pdl_begin();
  __shared__ float sums[kReduceWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const float* part = jobs.part[blockIdx.y];
  float* out = jobs.out[blockIdx.y];
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (c < cols) {
    int p = warp;
    for (; p + 3 * kReduceWarps < parts; p += 4 * kReduceWarps) {
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += part[static_cast<uint64_t>(p + u * kReduceWarps) * cols + c];
    }
    for (int u = 0; p < parts; p += kReduceWarps, ++u) acc[u] += part[static_cast<uint64_t>(p) * cols + c];
  }
  sums[warp][lane] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  __syncthreads();
  if (warp == 0 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kReduceWarps; ++w) t += sums[w][lane];
    if (jobs.accumulate[blockIdx.y]) t += out[c];
    out[c] = t;
  }
}

int vectors_per_lane(uint64_t cols) {
  const uint64_t v = (cols / 4 + 31) / 32;
  if (v <= 1) return 1;
  if (v <= 2) return 2;
  if (v <= 4) return 4;
  if (v <= 6) return 6;
  if (v <= 8) return 8;
  if (v <= 12) return 12;
  if (v <= 16) return 16;
  return 0;
}

}  // namespace

// Number of partial rows the backward writes for `rows` (workspace = 3 * parts * cols floats
// with the dx column sums, 2 * parts * cols without).
int layernorm_backward_parts(uint64_t rows, int device) {
  uint64_t parts = static_cast<uint64_t>(sm_count(device)) * 2;
  const uint64_t by_rows = (rows + kWarps - 1) / kWarps;
  if (parts > by_rows) parts = by_rows;
  if (parts < 1) parts = 1;
  return static_cast<int>(parts);
}

cudaError_t layernorm_forward_launch(float* y, float* mean, float* rstd, const float* x,
                                     const float* gamma, const float* beta, uint64_t rows,
                                     uint64_t cols, float eps, int device, cudaStream_t stream,
                                     bool round_out) {
  const unsigned grid = grid_for(rows, kWarps, sm_count(device) * 8);
  const int c = static_cast<int>(cols);
  switch (vectors_per_lane(cols)) {
#define SPAR_LN_FWD(V) \
  case V:              \
    launch(layernorm_forward_kernel<V, false>, dim3(grid), dim3(kWarps * 32), 0, stream, y, mean, rstd, x, gamma, beta, rows, c, eps, RowMap{cols, 1}, round_out ? 1 : 0); \
    break;
    SPAR_LN_FWD(1) SPAR_LN_FWD(2) SPAR_LN_FWD(4) SPAR_LN_FWD(6) SPAR_LN_FWD(8) SPAR_LN_FWD(12)
    SPAR_LN_FWD(16)
#undef SPAR_LN_FWD
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t layernorm_backward_launch(float* dx, float* dgamma, float* dbeta, const float* dy,
                                      const float* x, const float* gamma, const float* mean,
                                      const float* rstd, uint64_t rows, uint64_t cols,
                                      int accumulate_params, int accumulate_dx, float* workspace,
                                      int device, cudaStream_t stream, float* dsum) {
  const int parts = layernorm_backward_parts(rows, device);
  const uint64_t rows_per_block = (rows + parts - 1) / parts;
  const int c = static_cast<int>(cols);
  const int arrays = dsum ? 3 : 2;
  const size_t smem = arrays * kWarps * cols * sizeof(float);
  float* pa = workspace;
  float* pb = workspace + static_cast<uint64_t>(parts) * cols;
  float* ps = dsum ? workspace + 2 * static_cast<uint64_t>(parts) * cols : nullptr;
  switch (vectors_per_lane(cols)) {
#define SPAR_LN_BWD(V)                                                                          \
  case V: {                                                                                    \
    auto k = layernorm_backward_kernel<V, false>;                                              \
    const cudaError_t se = raise_dynamic_smem(reinterpret_cast<const void*>(k), device, smem);  \
    if (se != cudaSuccess) return se;                                                          \
    launch(k, dim3(parts), dim3(kWarps * 32), smem, stream, dx, pa, pb, ps, dy, x, gamma, mean, \
           rstd, rows, c, rows_per_block, accumulate_dx, RowMap{cols, 1});                      \
    break;                                                                                     \
  }
    SPAR_LN_BWD(1) SPAR_LN_BWD(2) SPAR_LN_BWD(4) SPAR_LN_BWD(6) SPAR_LN_BWD(8) SPAR_LN_BWD(12)
    SPAR_LN_BWD(16)
#undef SPAR_LN_BWD
    default:
      return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PartialJobs jobs = {{dgamma, dbeta, dsum}, {pa, pb, ps}, {accumulate_params, accumulate_params, 1}};
  return launch(reduce_partials_kernel, dim3((c + 31) / 32, arrays), dim3(kReduceWarps * 32), 0,
                stream, jobs, parts, c);
}

cudaError_t rmsnorm_forward_launch(float* y, float* rstd, const float* x, const float* weight,
                                   uint64_t rows, uint64_t cols, float eps, int device,
                                   cudaStream_t stream, uint64_t ld, uint32_t group,
                                   bool round_out) {
  const RowMap rm{ld ? ld : cols, group};
  const unsigned grid = grid_for(rows, kWarps, sm_count(device) * 8);
  const int c = static_cast<int>(cols);
  switch (vectors_per_lane(cols)) {
#define SPAR_RMS_FWD(V) \
  case V:               \
    launch(layernorm_forward_kernel<V, true>, dim3(grid), dim3(kWarps * 32), 0, stream, y, nullptr, rstd, x, weight, nullptr, rows, c, eps, rm, round_out ? 1 : 0); \
    break;
    SPAR_RMS_FWD(1) SPAR_RMS_FWD(2) SPAR_RMS_FWD(4) SPAR_RMS_FWD(6) SPAR_RMS_FWD(8) SPAR_RMS_FWD(12)
    SPAR_RMS_FWD(16)
#undef SPAR_RMS_FWD
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// workspace: layernorm_backward_parts(rows) x cols floats (the per-block dweight partial rows).
cudaError_t rmsnorm_backward_launch(float* dx, float* dweight, const float* dy, const float* x,
                                    const float* weight, const float* rstd, uint64_t rows,
                                    uint64_t cols, int accumulate_params, int accumulate_dx,
                                    float* workspace, int device, cudaStream_t stream,
                                    uint64_t ld, uint32_t group) {
  const RowMap rm{ld ? ld : cols, group};
  const int parts = layernorm_backward_parts(rows, device);
  const uint64_t rows_per_block = (rows + parts - 1) / parts;
  const int c = static_cast<int>(cols);
  const size_t smem = kWarps * cols * sizeof(float);
  switch (vectors_per_lane(cols)) {
#define SPAR_RMS_BWD(V)                                                                         \
  case V: {                                                                                    \
    auto k = layernorm_backward_kernel<V, true>;                                               \
    const cudaError_t se = raise_dynamic_smem(reinterpret_cast<const void*>(k), device, smem);  \
    if (se != cudaSuccess) return se;                                                          \
    launch(k, dim3(parts), dim3(kWarps * 32), smem, stream, dx, workspace, nullptr, nullptr, dy, \
           x, weight, nullptr, rstd, rows, c, rows_per_block, accumulate_dx, rm);               \
    break;                                                                                     \
  }
    SPAR_RMS_BWD(1) SPAR_RMS_BWD(2) SPAR_RMS_BWD(4) SPAR_RMS_BWD(6) SPAR_RMS_BWD(8)
    SPAR_RMS_BWD(12) SPAR_RMS_BWD(16)
#undef SPAR_RMS_BWD
    default:
      return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PartialJobs jobs = {{dweight, nullptr, nullptr}, {workspace, nullptr, nullptr}, {accumulate_params, 0, 0}};
  return launch(reduce_partials_kernel, dim3((c + 31) / 32, 1), dim3(kReduceWarps * 32), 0,
                stream, jobs, parts, c);
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_layernorm_forward(float* y, float* mean, float* rstd,
                                                      const float* x, const float* gamma,
                                                      const float* beta, uint64_t rows,
                                                      uint64_t cols, double epsilon, int device,
                                                      void* stream) {
  if (rows == 0) return ok();
  if (cols == 0 || cols % 4 != 0 || vectors_per_lane(cols) == 0 || !y || !mean || !rstd || !x ||
      !gamma || !beta || !(epsilon > 0.0))
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = layernorm_forward_launch(y, mean, rstd, x, gamma, beta, rows, cols,
                                                 static_cast<float>(epsilon), device,
                                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : runtime(e);
}

namespace {
// The backward kernel reads x, dy and gamma and writes dx as float4 (rows are cols floats apart,
// cols a multiple of 4), so those base pointers must be 16-byte aligned.
bool backward_pointers_aligned(const float* dx, const float* dy, const float* x,
                               const float* gamma) {
  return ((reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dy) |
           reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gamma)) & 15) == 0;
}
}  // namespace

extern "C" SparCudaStatus spar_b200_layernorm_backward(float* dx, float* dgamma, float* dbeta,
                                                       const float* dy, const float* x,
                                                       const float* gamma, const float* mean,
                                                       const float* rstd, uint64_t rows,
                                                       uint64_t cols, int accumulate_params,
                                                       int accumulate_dx, int device,
                                                       void* stream) {
  if (cols == 0 || cols % 4 != 0 || vectors_per_lane(cols) == 0 || !dgamma || !dbeta || !gamma)
    return invalid();
  if (rows != 0 && (!dx || !dy || !x || !mean || !rstd)) return invalid();
  if (!backward_pointers_aligned(dx, dy, x, gamma)) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (accumulate_params) return ok();
    cudaError_t e = cudaMemsetAsync(dgamma, 0, cols * sizeof(float), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(dbeta, 0, cols * sizeof(float), s);
    return e == cudaSuccess ? ok() : runtime(e);
  }
  const int parts = layernorm_backward_parts(rows, device);
  float* workspace = nullptr;
  cudaError_t e = stream_alloc(reinterpret_cast<void**>(&workspace),
                                  2ull * parts * cols * sizeof(float), s);
  if (e != cudaSuccess) return runtime(e);
  e = layernorm_backward_launch(dx, dgamma, dbeta, dy, x, gamma, mean, rstd, rows, cols,
                                accumulate_params, accumulate_dx, workspace, device, s, nullptr);
  const cudaError_t f = cudaFreeAsync(workspace, s);
  if (e != cudaSuccess) return runtime(e);
  return f == cudaSuccess ? ok() : runtime(f);
}

// RMSNorm (nn::RMSNorm, src/nn/rmsnorm.cpp:40-53): the LayerNorm kernels without centring/bias.
extern "C" SparCudaStatus spar_b200_rmsnorm_forward(float* y, float* rstd, const float* x,
                                                    const float* weight, uint64_t rows,
                                                    uint64_t cols, double epsilon, int device,
                                                    void* stream) {
  if (rows == 0) return ok();
  // RMSNorm's constructor checks (rmsnorm.cpp:17-28): positive size, finite positive epsilon.
  if (cols == 0 || cols % 4 != 0 || vectors_per_lane(cols) == 0 || !y || !rstd || !x || !weight ||
      !(epsilon > 0.0) || !std::isfinite(epsilon))
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = rmsnorm_forward_launch(y, rstd, x, weight, rows, cols,
                                               static_cast<float>(epsilon), device,
                                               static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_rmsnorm_backward(float* dx, float* dweight, const float* dy,
                                                     const float* x, const float* weight,
                                                     const float* rstd, uint64_t rows,
                                                     uint64_t cols, int accumulate_params,
                                                     int accumulate_dx, int device, void* stream) {
  if (cols == 0 || cols % 4 != 0 || vectors_per_lane(cols) == 0 || !dweight || !weight)
    return invalid();
  if (rows != 0 && (!dx || !dy || !x || !rstd)) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (accumulate_params) return ok();
    const cudaError_t e = cudaMemsetAsync(dweight, 0, cols * sizeof(float), s);
    return e == cudaSuccess ? ok() : runtime(e);
  }
  const int parts = layernorm_backward_parts(rows, device);
  float* workspace = nullptr;
  cudaError_t e = stream_alloc(reinterpret_cast<void**>(&workspace),
                                  static_cast<uint64_t>(parts) * cols * sizeof(float), s);
  if (e != cudaSuccess) return runtime(e);
  e = rmsnorm_backward_launch(dx, dweight, dy, x, weight, rstd, rows, cols, accumulate_params,
                              accumulate_dx, workspace, device, s);
  const cudaError_t f = cudaFreeAsync(workspace, s);
  if (e != cudaSuccess) return runtime(e);
  return f == cudaSuccess ? ok() : runtime(f);
}

// qk-norm: RMSNorm(head_dim) over each head of the q or k part of a packed projection output,
// addressed in place in the [tokens, ld] layout (head h of token t at t * ld + h * head_dim).
extern "C" SparCudaStatus spar_b200_head_rmsnorm_forward(float* y, const float* x, uint64_t ld,
                                                         uint64_t tokens, uint64_t heads,
                                                         uint64_t head_dim, const float* weight,
                                                         float* rstd, double epsilon, int device,
                                                         void* stream) {
  if (tokens == 0) return ok();
  if (head_dim == 0 || head_dim % 4 != 0 || vectors_per_lane(head_dim) == 0 || heads == 0 ||
      heads > 0xFFFFFFFFull || ld % 4 != 0 || ld < heads * head_dim || !y || !x || !weight ||
      !rstd || !(epsilon > 0.0) || !std::isfinite(epsilon) ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15))
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = rmsnorm_forward_launch(y, rstd, x, weight, tokens * heads, head_dim,
                                               static_cast<float>(epsilon), device,
                                               static_cast<cudaStream_t>(stream), ld,
                                               static_cast<uint32_t>(heads));
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_head_rmsnorm_backward(float* dx, float* dweight,
                                                          const float* dy, const float* x,
                                                          uint64_t ld, uint64_t tokens,
                                                          uint64_t heads, uint64_t head_dim,
                                                          const float* weight, const float* rstd,
                                                          int accumulate_params, int device,
                                                          void* stream) {
  if (head_dim == 0 || head_dim % 4 != 0 || vectors_per_lane(head_dim) == 0 || heads == 0 ||
      heads > 0xFFFFFFFFull || ld % 4 != 0 || ld < heads * head_dim || !dweight || !weight)
    return invalid();
  if (tokens != 0 && (!dx || !dy || !x || !rstd ||
                      ((reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dy) |
                        reinterpret_cast<uintptr_t>(x)) & 15)))
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (tokens == 0) {
    if (accumulate_params) return ok();
    const cudaError_t e = cudaMemsetAsync(dweight, 0, head_dim * sizeof(float), s);
    return e == cudaSuccess ? ok() : runtime(e);
  }
  const uint64_t rows = tokens * heads;
  const int parts = layernorm_backward_parts(rows, device);
  float* workspace = nullptr;
  cudaError_t e = stream_alloc(reinterpret_cast<void**>(&workspace),
                                  static_cast<uint64_t>(parts) * head_dim * sizeof(float), s);
  if (e != cudaSuccess) return runtime(e);
  e = rmsnorm_backward_launch(dx, dweight, dy, x, weight, rstd, rows, head_dim, accumulate_params,
                              0, workspace, device, s, ld, static_cast<uint32_t>(heads));
  const cudaError_t f = cudaFreeAsync(workspace, s);
  if (e != cudaSuccess) return runtime(e);
  return f == cudaSuccess ? ok() : runtime(f);
}

// ============================================================== allocation-free backward
// Variant of spar_b200_layernorm_backward for callers that cannot allocate device memory at call
// time (for example a host whose device memory is reserved up front by its own allocator, or a
// step loop that must not allocate because an allocation can fail or stall in the middle of a
// step). The per-block dgamma/dbeta partial rows live in the file-scope array below instead of a
// stream-ordered allocation. Limits: cols <= 2048 (the kernel's own limit) and at most 296
// partial rows (two per SM on a 148-SM B200), i.e. 2 * 296 * 2048 floats = 4.85 MB that every GPU
// which loads this library holds until the process exits.
namespace spar_b200 {
namespace {

constexpr uint64_t kNoAllocMaxCols = 2048;
constexpr int kNoAllocMaxParts = 296;
static __device__ __align__(256) float g_ln_backward_scratch[2ull * kNoAllocMaxParts * kNoAllocMaxCols];

std::mutex g_scratch_mutex;
float* g_scratch_address[64] = {};  // device address of g_ln_backward_scratch, per device

// Host code cannot pass &g_ln_backward_scratch to a kernel (on the host that name is only a
// stand-in); the device address is looked up once per device, with that device current.
cudaError_t scratch_address(int device, float** out) {
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_address[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_ln_backward_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_address[device] = static_cast<float*>(p);
  }
  *out = g_scratch_address[device];
  return cudaSuccess;
}

}  // namespace
}  // namespace spar_b200

// Same arguments and results as spar_b200_layernorm_backward; allocates nothing.
// The first call on a device looks up the scratch address (make that first call before any
// stream capture). The address is cached for the life of the process: it does not survive
// cudaDeviceReset (or any other teardown of the device's primary context), after which this entry
// point must not be called again in that process. All calls share one scratch array, so calls that overlap on the GPU (two
// streams, or two host threads on one device) race; serialise them. The array keeps the previous
// call's partials, which is harmless: every partial row a call reads is written earlier in the
// same call, so nothing has to start at zero.
extern "C" SparCudaStatus spar_b200_layernorm_backward_noalloc(
    float* dx, float* dgamma, float* dbeta, const float* dy, const float* x, const float* gamma,
    const float* mean, const float* rstd, uint64_t rows, uint64_t cols, int accumulate_params,
    int accumulate_dx, int device, void* stream) {
  if (cols == 0 || cols % 4 != 0 || !dgamma || !dbeta || !gamma) return invalid();
  if (cols > kNoAllocMaxCols) return invalid();  // beyond the static scratch size
  if (rows != 0 && (!dx || !dy || !x || !mean || !rstd)) return invalid();
  if (!backward_pointers_aligned(dx, dy, x, gamma)) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (accumulate_params) return ok();
    cudaError_t e = cudaMemsetAsync(dgamma, 0, cols * sizeof(float), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(dbeta, 0, cols * sizeof(float), s);
    return e == cudaSuccess ? ok() : runtime(e);
  }
  if (layernorm_backward_parts(rows, device) > kNoAllocMaxParts) return invalid();
  float* scratch = nullptr;
  cudaError_t e = scratch_address(device, &scratch);
  if (e != cudaSuccess) return runtime(e);
  e = layernorm_backward_launch(dx, dgamma, dbeta, dy, x, gamma, mean, rstd, rows, cols,
                                accumulate_params, accumulate_dx, scratch, device, s, nullptr);
  return e == cudaSuccess ? ok() : runtime(e);
}
