// Fused softmax cross-entropy forward + backward.
//
// Spar computes the loss as log_softmax over the class axis (src/ops/softmax.cpp:342-398:
// max, sum exp(x - max), (x - max) - log(sum)), gathers -logp[target] (select_nll,
// src/loss/cross_entropy.cpp:52-100) and takes the mean; the backward of that chain is
// dlogits = g * (exp(logp) - onehot(target)) (softmax.cpp:406-444 with the one-hot upstream of
// nll_gradient), g = 1/N. This kernel evaluates exactly that per row, without materialising
// logp or a zeroed [rows, V] gradient: one read of the logits row, one write of dlogits.
//
// Large vocabularies: one 1024-thread block per row with the row held in registers
// (EPT float4 per thread). Small vocabularies: one warp per row.
#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

__device__ __forceinline__ int row_target(const int32_t* targets, uint64_t r, uint64_t seq,
                                          bool* has_target) {
  if (seq == 0) {
    *has_target = true;
    return targets[r];
  }
  const uint64_t t = r % seq;
  *has_target = t + 1 < seq;
  return *has_target ? targets[r + 1] : 0;
}

template <int EPT>
__global__ void __launch_bounds__(1024)
ce_block_kernel(float* __restrict__ loss, float* dlogits, const float* logits,
                const int32_t* __restrict__ targets, uint64_t rows, uint64_t classes, uint64_t ld,
                uint64_t seq, float grad_scale, int32_t* invalid) {
  pdl_begin();
  __shared__ float scratch[32];
  const uint64_t vec = classes / 4;
  for (uint64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    bool has_target;
    const int target = row_target(targets, r, seq, &has_target);
    const bool bad = has_target && (target < 0 || static_cast<uint64_t>(target) >= classes);
    const float4* zr = reinterpret_cast<const float4*>(logits + r * ld);
    float4* dr = reinterpret_cast<float4*>(dlogits + r * ld);
    if (!has_target || bad) {
      for (uint64_t f = threadIdx.x; f < vec; f += blockDim.x) dr[f] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (threadIdx.x == 0) {
        loss[r] = bad ? NAN : 0.f;
        if (bad) atomicExch(invalid, 1);
      }
      continue;
    }
    float4 v[EPT];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const uint64_t f = threadIdx.x + 1024ull * j;
      if (f < vec) {
        v[j] = ld_stream(zr + f);
        m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
      }
    }
    m = block_max(m, scratch);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const uint64_t f = threadIdx.x + 1024ull * j;
      if (f < vec)
        s += (expf(v[j].x - m) + expf(v[j].y - m)) + (expf(v[j].z - m) + expf(v[j].w - m));
    }
    s = block_sum(s, scratch);
    const float log_sum = logf(s);
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const uint64_t f = threadIdx.x + 1024ull * j;
      if (f < vec) {
        const uint64_t c = 4 * f;
        float4 o;
        o.x = grad_scale * (expf((v[j].x - m) - log_sum) - (c == (uint64_t)target ? 1.f : 0.f));
        o.y = grad_scale * (expf((v[j].y - m) - log_sum) - (c + 1 == (uint64_t)target ? 1.f : 0.f));
        o.z = grad_scale * (expf((v[j].z - m) - log_sum) - (c + 2 == (uint64_t)target ? 1.f : 0.f));
        o.w = grad_scale * (expf((v[j].w - m) - log_sum) - (c + 3 == (uint64_t)target ? 1.f : 0.f));
        if (c <= (uint64_t)target && (uint64_t)target < c + 4) {
          const float zt = target == c ? v[j].x : target == c + 1 ? v[j].y
                         : target == c + 2 ? v[j].z : v[j].w;
          loss[r] = -((zt - m) - log_sum);
        }
        st_stream(dr + f, o);
      }
    }
    __syncthreads();  // scratch reuse in the next row
  }
}

template <int VPL>
__global__ void __launch_bounds__(256)
ce_warp_kernel(float* __restrict__ loss, float* dlogits, const float* logits,
               const int32_t* __restrict__ targets, uint64_t rows, uint64_t classes, uint64_t ld,
               uint64_t seq, float grad_scale, int32_t* invalid) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const uint64_t vec = classes / 4;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * 8;
  for (uint64_t r = static_cast<uint64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); r < rows;
       r += stride) {
    bool has_target;
    const int target = row_target(targets, r, seq, &has_target);
    const bool bad = has_target && (target < 0 || static_cast<uint64_t>(target) >= classes);
    const float4* zr = reinterpret_cast<const float4*>(logits + r * ld);
    float4* dr = reinterpret_cast<float4*>(dlogits + r * ld);
    if (!has_target || bad) {
      for (uint64_t f = lane; f < vec; f += 32) dr[f] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (lane == 0) {
        loss[r] = bad ? NAN : 0.f;
        if (bad) atomicExch(invalid, 1);
      }
      continue;
    }
    float4 v[VPL];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint64_t f = lane + 32 * j;
      if (f < vec) {
        v[j] = zr[f];
        m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
      }
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint64_t f = lane + 32 * j;
      if (f < vec)
        s += (expf(v[j].x - m) + expf(v[j].y - m)) + (expf(v[j].z - m) + expf(v[j].w - m));
    }
    s = warp_sum(s);
    const float log_sum = logf(s);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint64_t f = lane + 32 * j;
      if (f < vec) {
        const uint64_t c = 4 * f;
        float4 o;
        o.x = grad_scale * (expf((v[j].x - m) - log_sum) - (c == (uint64_t)target ? 1.f : 0.f));
        o.y = grad_scale * (expf((v[j].y - m) - log_sum) - (c + 1 == (uint64_t)target ? 1.f : 0.f));
        o.z = grad_scale * (expf((v[j].z - m) - log_sum) - (c + 2 == (uint64_t)target ? 1.f : 0.f));
        o.w = grad_scale * (expf((v[j].w - m) - log_sum) - (c + 3 == (uint64_t)target ? 1.f : 0.f));
        if (c <= (uint64_t)target && (uint64_t)target < c + 4) {
          const float zt = target == c ? v[j].x : target == c + 1 ? v[j].y
                         : target == c + 2 ? v[j].z : v[j].w;
          loss[r] = -((zt - m) - log_sum);
        }
        dr[f] = o;
      }
    }
  }
}

// Generic two-pass path for any class count (and ld/classes not multiples of 4).
__global__ void __launch_bounds__(256)
ce_generic_kernel(float* __restrict__ loss, float* dlogits, const float* logits,
                  const int32_t* __restrict__ targets, uint64_t rows, uint64_t classes,
                  uint64_t ld, uint64_t seq, float grad_scale, int32_t* invalid) {
  pdl_begin();
  __shared__ float scratch[32];
  for (uint64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    bool has_target;
    const int target = row_target(targets, r, seq, &has_target);
    const bool bad = has_target && (target < 0 || static_cast<uint64_t>(target) >= classes);
    const float* zr = logits + r * ld;
    float* dr = dlogits + r * ld;
    if (!has_target || bad) {
      for (uint64_t c = threadIdx.x; c < classes; c += blockDim.x) dr[c] = 0.f;
      if (threadIdx.x == 0) {
        loss[r] = bad ? NAN : 0.f;
        if (bad) atomicExch(invalid, 1);
      }
      continue;
    }
    float m = -INFINITY;
    for (uint64_t c = threadIdx.x; c < classes; c += blockDim.x) m = fmaxf(m, zr[c]);
    m = block_max(m, scratch);
    float s = 0.f;
    for (uint64_t c = threadIdx.x; c < classes; c += blockDim.x) s += expf(zr[c] - m);
    s = block_sum(s, scratch);
    const float log_sum = logf(s);
    const float zt = zr[target];
    __syncthreads();
    for (uint64_t c = threadIdx.x; c < classes; c += blockDim.x)
      dr[c] = grad_scale * (expf((zr[c] - m) - log_sum) - (c == (uint64_t)target ? 1.f : 0.f));
    if (threadIdx.x == 0) loss[r] = -((zt - m) - log_sum);
    __syncthreads();
  }
}

}  // namespace

cudaError_t cross_entropy_launch(float* loss, float* dlogits, const float* logits,
                                 const int32_t* targets, uint64_t rows, uint64_t classes,
                                 uint64_t ld, uint64_t seq, float grad_scale,
                                 int32_t* invalid, int device, cudaStream_t stream) {
  const bool vec_ok = classes % 4 == 0 && ld % 4 == 0;
  const uint64_t vec = classes / 4;
  const int sms = sm_count(device);
  if (vec_ok && vec <= 32 * 16) {
    const uint64_t v = (vec + 31) / 32;
    const unsigned grid = grid_for(rows, 8, sms * 16);
    switch (v <= 1 ? 1 : v <= 2 ? 2 : v <= 4 ? 4 : v <= 8 ? 8 : 16) {
#define SPAR_CE_W(V) case V: launch(ce_warp_kernel<V>, dim3(grid), dim3(256), 0, stream, loss, dlogits, logits, targets, rows, classes, ld, seq, grad_scale, invalid); break;
      SPAR_CE_W(1) SPAR_CE_W(2) SPAR_CE_W(4) SPAR_CE_W(8) SPAR_CE_W(16)
#undef SPAR_CE_W
    }
  } else if (vec_ok && vec <= 1024ull * 16) {
    const uint64_t e = (vec + 1023) / 1024;
    const unsigned grid = grid_for(rows, 1, sms * 2);
    switch (e <= 4 ? 4 : e <= 8 ? 8 : e <= 12 ? 12 : 16) {
#define SPAR_CE_B(E) case E: launch(ce_block_kernel<E>, dim3(grid), dim3(1024), 0, stream, loss, dlogits, logits, targets, rows, classes, ld, seq, grad_scale, invalid); break;
      SPAR_CE_B(4) SPAR_CE_B(8) SPAR_CE_B(12) SPAR_CE_B(16)
#undef SPAR_CE_B
    }
  } else {
    const unsigned grid = grid_for(rows, 1, sms * 8);
    launch(ce_generic_kernel, dim3(grid), dim3(256), 0, stream, loss, dlogits, logits, targets, rows, classes, ld,
                                                seq, grad_scale, invalid);
  }
  return cudaGetLastError();
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_cross_entropy_forward_backward(
    float* loss, float* dlogits, const float* logits, const int32_t* targets, uint64_t rows,
    uint64_t classes, uint64_t ld, uint64_t sequence_length, float grad_scale,
    int32_t* invalid_target, int device, void* stream) {
  if (rows == 0) return ok();
  if (!loss || !dlogits || !logits || !targets || !invalid_target || classes == 0 ||
      ld < classes || sequence_length == 1 ||
      (sequence_length != 0 && rows % sequence_length != 0) || classes > 0x7fffffffull)
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = cross_entropy_launch(loss, dlogits, logits, targets, rows, classes, ld,
                                             sequence_length, grad_scale, invalid_target, device,
                                             (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}
