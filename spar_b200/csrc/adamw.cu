// Global gradient norm, clipping and AdamW as two streaming passes over flat fp32 arrays.
//
// Reference semantics:
//   norm  = ||g||_2 over all unique parameters, accumulated in double
//           (training::global_grad_norm, src/training/gradients.cpp:28-137; the scaled
//           sum-of-squares there only guards double overflow, which fp32 squares cannot reach)
//   clip  = if norm is non-finite: error, nothing updated; if norm > max_norm (and != 0):
//           g <- fp32(double(g) * max_norm / norm)       (clip_grad_norm :176-190,
//           scale_gradients :139-174)
//   AdamW = per element in double, moments rounded to fp32 (src/optim/adamw.cpp:37-63):
//           m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2
//           p = p (1 - lr wd) - lr (m / c1) / (sqrt(v / c2) + eps), c = 1 - b^step
// Here the clip factor is derived on the device from the norm pass, so no host round trip sits
// between the two passes, and the clipped gradient is consumed in registers instead of being
// written back.
#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

constexpr int kPartialBase = 8;

int norm_blocks(int device) {
  int g = sm_count(device) * 2;
  if (g > (kNormStateDoubles - kPartialBase) / 2) g = (kNormStateDoubles - kPartialBase) / 2;
  return g;
}

__global__ void __launch_bounds__(512)
norm_partial_kernel(double* __restrict__ state, const float* __restrict__ g, uint64_t count,
                    int first) {
  pdl_begin();
  __shared__ double red[16];
  __shared__ int bad_any;
  if (threadIdx.x == 0) bad_any = 0;
  __syncthreads();
  const uint64_t per_block = ((count + gridDim.x - 1) / gridDim.x + 3) & ~3ull;
  const uint64_t begin = per_block * blockIdx.x;
  uint64_t end = begin + per_block;
  if (end > count) end = count;
  double s = 0.0;
  int bad = 0;
  if (begin < end) {
    const uint64_t n4 = (end - begin) / 4;
    const float4* g4 = reinterpret_cast<const float4*>(g + begin);
    const bool aligned = (reinterpret_cast<uintptr_t>(g + begin) & 15) == 0;
    if (aligned) {
      for (uint64_t i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = ld_stream(g4 + i);
        bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
        s += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y +
             static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
      }
    }
    for (uint64_t i = begin + (aligned ? n4 * 4 : 0) + threadIdx.x; i < end; i += blockDim.x) {
      const float v = g[i];
      bad |= !isfinite(v);
      s += static_cast<double>(v) * v;
    }
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  if (bad) bad_any = 1;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    t = warp_sum(t);
    if (threadIdx.x == 0) {
      double* partial = state + kPartialBase;
      double* flags = partial + gridDim.x;
      partial[blockIdx.x] = first ? t : partial[blockIdx.x] + t;
      flags[blockIdx.x] = first ? (double)bad_any : fmax(flags[blockIdx.x], (double)bad_any);
    }
  }
}

__global__ void norm_final_kernel(double* state, int parts, const int* wait_a, const int* wait_b) {
  pdl_begin();
  if (threadIdx.x != 0) return;
  double s = 0.0, bad = 0.0;
  const double* partial = state + kPartialBase;
  for (int p = 0; p < parts; ++p) {
    s += partial[p];
    bad = fmax(bad, partial[parts + p]);
  }
  // A kernel of this step gave up a bounded wait: its outputs are not trustworthy.
  if ((wait_a && *reinterpret_cast<const volatile int*>(wait_a)) ||
      (wait_b && *reinterpret_cast<const volatile int*>(wait_b)))
    bad += kWaitErrorMark;
  state[0] = s;
  state[1] = bad;
}


__device__ __forceinline__ void adamw_element(float& p, float g, float& m, float& v,
                                              const AdamWArgs& a, double clip) {
  double gd = static_cast<double>(g);
  if (clip != 1.0) gd = static_cast<double>(static_cast<float>(gd * clip));
  m = static_cast<float>(a.beta1 * static_cast<double>(m) + (1.0 - a.beta1) * gd);
  v = static_cast<float>(a.beta2 * static_cast<double>(v) + (1.0 - a.beta2) * gd * gd);
  const double mc = static_cast<double>(m) / a.c1;
  const double vc = static_cast<double>(v) / a.c2;
  const double decayed = static_cast<double>(p) * a.decay_factor;
  p = static_cast<float>(decayed - a.lr * mc / (sqrt(vc) + a.eps));
}

__global__ void __launch_bounds__(256)
adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
             float* __restrict__ v, uint64_t count, const double* __restrict__ state,
             AdamWArgs args, const AdamWArgs* __restrict__ args_dev, int32_t* nonfinite_flag,
             float* __restrict__ rounded) {
  pdl_begin();
  // Scalars by value, or (args_dev != nullptr) from device memory, which a replayed CUDA graph
  // reads afresh every step.
  const AdamWArgs a = args_dev ? *args_dev : args;
  const double ssq = state[0];
  const bool bad = state[1] != 0.0 || !isfinite(ssq);
  if (bad) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *nonfinite_flag = 1;
    return;
  }
  const double norm = sqrt(ssq);
  const double clip = (a.max_norm >= 0.0 && norm != 0.0 && norm > a.max_norm) ? a.max_norm / norm : 1.0;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  const uint64_t start = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool aligned = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                         reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v) |
                         reinterpret_cast<uintptr_t>(rounded)) & 15) == 0;
  const uint64_t n4 = aligned ? count / 4 : 0;
  for (uint64_t i = start; i < n4; i += stride) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    const float4 gv = ld_stream(reinterpret_cast<const float4*>(g) + i);
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    adamw_element(pv.x, gv.x, mv.x, vv.x, a, clip);
    adamw_element(pv.y, gv.y, mv.y, vv.y, a, clip);
    adamw_element(pv.z, gv.z, mv.z, vv.z, a, clip);
    adamw_element(pv.w, gv.w, mv.w, vv.w, a, clip);
    reinterpret_cast<float4*>(p)[i] = pv;
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (rounded)
      reinterpret_cast<float4*>(rounded)[i] =
          make_float4(round_tf32(pv.x), round_tf32(pv.y), round_tf32(pv.z), round_tf32(pv.w));
  }
  for (uint64_t i = n4 * 4 + start; i < count; i += stride) {
    float pv = p[i], mv = m[i], vv = v[i];
    adamw_element(pv, g[i], mv, vv, a, clip);
    p[i] = pv;
    m[i] = mv;
    v[i] = vv;
    if (rounded) rounded[i] = round_tf32(pv);
  }
}

}  // namespace

cudaError_t grad_norm_launch(double* norm_state, const Slice* slices, uint64_t slice_count,
                             int device, cudaStream_t stream, const int* wait_flag_a,
                             const int* wait_flag_b) {
  const int parts = norm_blocks(device);
  bool first = true;
  for (uint64_t i = 0; i < slice_count; ++i) {
    if (slices[i].count == 0) continue;
    launch(norm_partial_kernel, dim3(parts), dim3(512), 0, stream, norm_state, slices[i].gradient,
                                                   slices[i].count, first ? 1 : 0);
    first = false;
  }
  // Nothing to reduce: norm 0 (the final pass still reads the wait flags).
  launch(norm_final_kernel, dim3(1), dim3(32), 0, stream, norm_state, first ? 0 : parts,
         wait_flag_a, wait_flag_b);
  return cudaGetLastError();
}

AdamWArgs adamw_args(double max_norm, double lr, double beta1, double beta2, double eps,
                     double weight_decay, uint64_t step) {
  AdamWArgs a;
  a.lr = lr;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.decay_factor = 1.0 - lr * weight_decay;
  a.c1 = 1.0 - pow(beta1, static_cast<double>(step));
  a.c2 = 1.0 - pow(beta2, static_cast<double>(step));
  a.max_norm = max_norm;
  return a;
}

cudaError_t adamw_launch(const Slice* slices, uint64_t slice_count, const double* norm_state,
                         double max_norm, double lr, double beta1, double beta2, double eps,
                         double weight_decay, uint64_t step, int32_t* nonfinite_flag, int device,
                         cudaStream_t stream, const AdamWArgs* args_dev,
                         const float* param_base, float* rounded_base) {
  const AdamWArgs a = adamw_args(max_norm, lr, beta1, beta2, eps, weight_decay, step);
  const int sms = sm_count(device);
  for (uint64_t i = 0; i < slice_count; ++i) {
    const Slice& s = slices[i];
    if (s.count == 0) continue;
    const unsigned grid = grid_for((s.count + 3) / 4, 256, sms * 8);
    float* rounded = rounded_base ? rounded_base + (s.parameter - param_base) : nullptr;
    launch(adamw_kernel, dim3(grid), dim3(256), 0, stream, s.parameter, s.gradient, s.first_moment,
                                           s.second_moment, s.count, norm_state, a, args_dev,
                                           nonfinite_flag, rounded);
  }
  return cudaGetLastError();
}

namespace {
__global__ void round_copy_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                  uint64_t count) {
  pdl_begin();
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride)
    dst[i] = round_tf32(src[i]);
}
}  // namespace

cudaError_t round_copy_launch(float* dst, const float* src, uint64_t count, int device,
                              cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  launch(round_copy_kernel, dim3(grid_for(count, 256, sm_count(device) * 16)), dim3(256), 0,
         stream, dst, src, count);
  return cudaGetLastError();
}

}  // namespace spar_b200

using namespace spar_b200;

static_assert(sizeof(SparB200TensorSlice) == sizeof(Slice), "slice layout");

extern "C" SparCudaStatus spar_b200_grad_norm_squared(double* norm_state,
                                                      const SparB200TensorSlice* slices,
                                                      uint64_t slice_count, int device,
                                                      void* stream) {
  if (!norm_state || (slice_count != 0 && !slices)) return invalid();
  for (uint64_t i = 0; i < slice_count; ++i)
    if (slices[i].count != 0 && !slices[i].gradient) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = grad_norm_launch(norm_state, reinterpret_cast<const Slice*>(slices),
                                         slice_count, device, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_adamw_clipped(const SparB200TensorSlice* slices,
                                                  uint64_t slice_count, const double* norm_state,
                                                  double max_norm, double learning_rate,
                                                  double beta1, double beta2, double epsilon,
                                                  double weight_decay, uint64_t step,
                                                  int32_t* nonfinite_flag, int device,
                                                  void* stream) {
  // Hyper-parameter validation of AdamW's constructor (src/optim/adamw.cpp:14-35).
  if (!norm_state || !nonfinite_flag || (slice_count != 0 && !slices) || step == 0 ||
      !(learning_rate >= 0.0) || !(beta1 >= 0.0 && beta1 < 1.0) || !(beta2 >= 0.0 && beta2 < 1.0) ||
      !(epsilon > 0.0) || !(weight_decay >= 0.0))
    return invalid();
  for (uint64_t i = 0; i < slice_count; ++i) {
    const SparB200TensorSlice& s = slices[i];
    if (s.count != 0 && (!s.parameter || !s.gradient || !s.first_moment || !s.second_moment))
      return invalid();
  }
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = adamw_launch(reinterpret_cast<const Slice*>(slices), slice_count,
                                     norm_state, max_norm, learning_rate, beta1, beta2, epsilon,
                                     weight_decay, step, nonfinite_flag, device,
                                     (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}
