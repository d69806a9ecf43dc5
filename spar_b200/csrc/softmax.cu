// Causal softmax forward/backward over square [T, T] score blocks (attention probabilities).
//
// Forward follows Spar's attention chain (src/nn/attention.cpp:128-134): scores are scaled by
// 1/sqrt(d_head) (multiply_scalar), the causal mask adds -inf above the diagonal
// (causal_mask, attention.cpp:96-118) and softmax runs over the last axis
// (src/ops/softmax.cpp:42-108: max, exp(x - max), sum, divide). Masked entries are never read, so
// the GEMM producing the scores may skip tiles above the diagonal.
// Backward is softmax.cpp:110-150 (P * (g - sum(g * P))) followed by the scalar-multiply backward.
// Causal rows always contain their diagonal entry, so the NaN/inf special cases of the reference
// (softmax.cpp:75-92) cannot arise from finite scores; non-finite scores propagate as NaN.
//
// One warp per row; for T <= 1024 the row lives in registers (lane l owns float4 columns
// l, l + 32, ...), so each row is read once. Larger T uses a two-pass loop.
#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ uint64_t fill_end(uint64_t i, uint64_t t, uint64_t block) {
  if (block == 0) return t;
  const uint64_t e = ((i + block) / block) * block;
  return e < t ? e : t;
}

template <int VPL>
__global__ void __launch_bounds__(kWarps * 32)
causal_softmax_forward_kernel(float* __restrict__ p, const float* __restrict__ s, uint64_t rows,
                              uint64_t t, uint64_t ld, float scale, uint64_t zblock) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kWarps;
  for (uint64_t r = static_cast<uint64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); r < rows;
       r += stride) {
    const uint64_t i = r % t;
    const uint64_t nvalid = i + 1;
    const uint64_t nfill = fill_end(i, t, zblock);
    const float* sr = s + r * ld;  // row r of the flattened [batch*T, ld] view
    float* pr = p + r * ld;
    if constexpr (VPL > 0) {
      float4 v[VPL];
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const uint64_t c = 4ull * (lane + 32 * j);
        v[j] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        if (c < nvalid) {
          const float4 x = reinterpret_cast<const float4*>(sr)[lane + 32 * j];
          v[j].x = x.x * scale;
          if (c + 1 < nvalid) v[j].y = x.y * scale;
          if (c + 2 < nvalid) v[j].z = x.z * scale;
          if (c + 3 < nvalid) v[j].w = x.w * scale;
          m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
        }
      }
      m = warp_max(m);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const uint64_t c = 4ull * (lane + 32 * j);
        if (c < nvalid) {
          v[j].x = expf(v[j].x - m);
          v[j].y = expf(v[j].y - m);
          v[j].z = expf(v[j].z - m);
          v[j].w = expf(v[j].w - m);
          sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        } else {
          v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      sum = warp_sum(sum);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const uint64_t c = 4ull * (lane + 32 * j);
        if (c < nfill) {
          const float4 o = make_float4(v[j].x / sum, v[j].y / sum, v[j].z / sum, v[j].w / sum);
          reinterpret_cast<float4*>(pr)[lane + 32 * j] = o;
        }
      }
    } else {
      float m = -INFINITY;
      for (uint64_t c = lane; c < nvalid; c += 32) m = fmaxf(m, sr[c] * scale);
      m = warp_max(m);
      float sum = 0.f;
      for (uint64_t c = lane; c < nvalid; c += 32) sum += expf(sr[c] * scale - m);
      sum = warp_sum(sum);
      for (uint64_t c = lane; c < nfill; c += 32)
        pr[c] = c < nvalid ? expf(sr[c] * scale - m) / sum : 0.f;
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(kWarps * 32)
causal_softmax_backward_kernel(float* ds, const float* dp, const float* __restrict__ p,
                               uint64_t rows, uint64_t t, uint64_t ld, float scale,
                               uint64_t zblock) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kWarps;
  for (uint64_t r = static_cast<uint64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); r < rows;
       r += stride) {
    const uint64_t i = r % t;
    const uint64_t nvalid = i + 1;
    const uint64_t nfill = fill_end(i, t, zblock);
    const float* dpr = dp + r * ld;
    const float* pr = p + r * ld;
    float* dsr = ds + r * ld;
    if constexpr (VPL > 0) {
      float4 g[VPL], q[VPL];
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const uint64_t c = 4ull * (lane + 32 * j);
        g[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        q[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < nvalid) {
          const float4 a = reinterpret_cast<const float4*>(dpr)[lane + 32 * j];
          const float4 b = reinterpret_cast<const float4*>(pr)[lane + 32 * j];
          g[j].x = a.x;
          q[j].x = b.x;
          if (c + 1 < nvalid) { g[j].y = a.y; q[j].y = b.y; }
          if (c + 2 < nvalid) { g[j].z = a.z; q[j].z = b.z; }
          if (c + 3 < nvalid) { g[j].w = a.w; q[j].w = b.w; }
          dot += (g[j].x * q[j].x + g[j].y * q[j].y) + (g[j].z * q[j].z + g[j].w * q[j].w);
        }
      }
      dot = warp_sum(dot);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const uint64_t c = 4ull * (lane + 32 * j);
        if (c < nfill) {
          float4 o;
          o.x = (q[j].x * (g[j].x - dot)) * scale;
          o.y = (q[j].y * (g[j].y - dot)) * scale;
          o.z = (q[j].z * (g[j].z - dot)) * scale;
          o.w = (q[j].w * (g[j].w - dot)) * scale;
          reinterpret_cast<float4*>(dsr)[lane + 32 * j] = o;
        }
      }
    } else {
      float dot = 0.f;
      for (uint64_t c = lane; c < nvalid; c += 32) dot += dpr[c] * pr[c];
      dot = warp_sum(dot);
      for (uint64_t c = lane; c < nfill; c += 32)
        dsr[c] = c < nvalid ? (pr[c] * (dpr[c] - dot)) * scale : 0.f;
    }
  }
}

}  // namespace

cudaError_t causal_softmax_launch(float* out, const float* in, const float* p, uint64_t batch,
                                  uint64_t t, uint64_t ld, float scale, uint64_t zero_fill_block,
                                  int backward, cudaStream_t stream) {
  const uint64_t rows = batch * t;
  const unsigned grid = grid_for(rows, kWarps, 148 * 16);
  const uint64_t v = (t / 4 + 31) / 32;
  const int vpl = (t % 4 != 0 || ld % 4 != 0) ? 0 : v <= 1 ? 1 : v <= 2 ? 2 : v <= 4 ? 4 : v <= 8 ? 8 : 0;
#define SPAR_SMX(V)                                                                              \
  case V:                                                                                       \
    if (backward)                                                                               \
      launch(causal_softmax_backward_kernel<V>, dim3(grid), dim3(kWarps * 32), 0, stream, out, in, p, rows, t,  \
                                                                          ld, scale,            \
                                                                          zero_fill_block);     \
    else                                                                                        \
      launch(causal_softmax_forward_kernel<V>, dim3(grid), dim3(kWarps * 32), 0, stream, out, in, rows, t, ld, \
                                                                         scale,                 \
                                                                         zero_fill_block);      \
    break;
  switch (vpl) {
    SPAR_SMX(0) SPAR_SMX(1) SPAR_SMX(2) SPAR_SMX(4) SPAR_SMX(8)
    default:
      return cudaErrorInvalidValue;
  }
#undef SPAR_SMX
  return cudaGetLastError();
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_causal_softmax_forward(float* p, const float* s,
                                                           uint64_t batch, uint64_t t, uint64_t ld,
                                                           float scale, uint64_t zero_fill_block,
                                                           int device, void* stream) {
  if (batch == 0 || t == 0) return ok();
  if (!p || !s || ld < t) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = causal_softmax_launch(p, s, nullptr, batch, t, ld, scale, zero_fill_block,
                                              0, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_causal_softmax_backward(float* ds, const float* dp,
                                                            const float* p, uint64_t batch,
                                                            uint64_t t, uint64_t ld, float scale,
                                                            uint64_t zero_fill_block, int device,
                                                            void* stream) {
  if (batch == 0 || t == 0) return ok();
  if (!ds || !dp || !p || ld < t) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = causal_softmax_launch(ds, dp, p, batch, t, ld, scale, zero_fill_block, 1,
                                              (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}
