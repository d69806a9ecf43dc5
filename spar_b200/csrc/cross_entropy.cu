// Fused softmax cross-entropy forward + backward.
//
// Spar computes the loss as log_softmax over the class axis (src/ops/softmax.cpp:342-398:
// max, sum exp(x - max), (x - max) - log(sum)), gathers -logp[target] (select_nll,
// src/loss/cross_entropy.cpp:52-100) and takes the mean; the backward of that chain is
// dlogits = g * (exp(logp) - onehot(target)) (softmax.cpp:406-444 with the one-hot upstream of
// nll_gradient), g = 1/N. This kernel evaluates exactly that per row, without materialising
// logp or a zeroed [rows, V] gradient: one read of the logits row, one write of dlogits.
//
// Large vocabularies: one block per row streaming the row twice (the second read from L2).
// Small vocabularies: one warp per row with the row in registers.
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

// Large vocabularies: one 256-thread block per row, two passes over the row. Pass 1 keeps a
// running (max, sum of exponentials) per thread over batches of eight float4 (one rescale per
// batch); the block combines the pairs in a fixed order. Pass 2 reads the row again (an L2 hit:
// only a few rows per SM are in flight) and writes dlogits. With several rows per SM, one row's
// loads overlap another's arithmetic; a row held in registers (128 KB at 32K classes, half the
// register file) would allow one row per SM and leave its memory idle during the reductions.
constexpr int kCeThreads = 256;
constexpr int kCeBatch = 8;

// (m, s) <- the pair for the union of two sets, s relative to the larger maximum.
__device__ __forceinline__ void ms_combine(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - mn));
  m = mn;
}

__device__ __forceinline__ float4 round4(float4 v) {
  return make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
}

__global__ void __launch_bounds__(kCeThreads, 3)
ce_stream_kernel(float* __restrict__ loss, float* dlogits, const float* logits,
                 const int32_t* __restrict__ targets, uint64_t rows, uint64_t classes, uint64_t ld,
                 uint64_t seq, float grad_scale, int32_t* invalid, int round_out) {
  pdl_begin();
  __shared__ float part_m[kCeThreads / 32], part_s[kCeThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t vec = classes / 4;
  for (uint64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    bool has_target;
    const int target = row_target(targets, r, seq, &has_target);
    const bool bad = has_target && (target < 0 || static_cast<uint64_t>(target) >= classes);
    const float4* zr = reinterpret_cast<const float4*>(logits + r * ld);
    float4* dr = reinterpret_cast<float4*>(dlogits + r * ld);
    if (!has_target || bad) {
      for (uint64_t f = threadIdx.x; f < vec; f += kCeThreads) dr[f] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (threadIdx.x == 0) {
        loss[r] = bad ? NAN : 0.f;
        if (bad) atomicExch(invalid, 1);
      }
      continue;
    }
    // Pass 1: running maximum and sum of exponentials relative to it.
    float m = -INFINITY, s = 0.f;
    for (uint64_t f0 = threadIdx.x; f0 < vec; f0 += kCeThreads * kCeBatch) {
      float4 x[kCeBatch];
      float bm = -INFINITY;
#pragma unroll
      for (int u = 0; u < kCeBatch; ++u) {
        const uint64_t f = f0 + static_cast<uint64_t>(u) * kCeThreads;
        x[u] = f < vec ? __ldcg(zr + f) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        bm = fmaxf(bm, fmaxf(fmaxf(x[u].x, x[u].y), fmaxf(x[u].z, x[u].w)));
      }
      const float mn = fmaxf(m, bm);
      if (mn == -INFINITY) continue;
      float bs = 0.f;
#pragma unroll
      for (int u = 0; u < kCeBatch; ++u)
        bs += (expf(x[u].x - mn) + expf(x[u].y - mn)) + (expf(x[u].z - mn) + expf(x[u].w - mn));
      s = (m == -INFINITY ? 0.f : s * expf(m - mn)) + bs;
      m = mn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      ms_combine(m, s, m2, s2);
    }
    if (lane == 0) {
      part_m[warp] = m;
      part_s[warp] = s;
    }
    __syncthreads();
    float M = part_m[0], S = part_s[0];
#pragma unroll
    for (int w = 1; w < kCeThreads / 32; ++w) ms_combine(M, S, part_m[w], part_s[w]);
    const float log_sum = logf(S);
    // Pass 2: dlogits = g * (softmax - onehot), the row's last read.
    for (uint64_t f0 = threadIdx.x; f0 < vec; f0 += kCeThreads * kCeBatch) {
      float4 x[kCeBatch];
#pragma unroll
      for (int u = 0; u < kCeBatch; ++u) {
        const uint64_t f = f0 + static_cast<uint64_t>(u) * kCeThreads;
        if (f < vec) x[u] = ld_stream(zr + f);
      }
#pragma unroll
      for (int u = 0; u < kCeBatch; ++u) {
        const uint64_t f = f0 + static_cast<uint64_t>(u) * kCeThreads;
        if (f < vec) {
          const uint64_t c = 4 * f;
          float4 o;
          o.x = grad_scale * (expf((x[u].x - M) - log_sum) - (c == (uint64_t)target ? 1.f : 0.f));
          o.y = grad_scale * (expf((x[u].y - M) - log_sum) - (c + 1 == (uint64_t)target ? 1.f : 0.f));
          o.z = grad_scale * (expf((x[u].z - M) - log_sum) - (c + 2 == (uint64_t)target ? 1.f : 0.f));
          o.w = grad_scale * (expf((x[u].w - M) - log_sum) - (c + 3 == (uint64_t)target ? 1.f : 0.f));
          if (c <= (uint64_t)target && (uint64_t)target < c + 4) {
            const float zt = target == c ? x[u].x : target == c + 1 ? x[u].y
                           : target == c + 2 ? x[u].z : x[u].w;
            loss[r] = -((zt - M) - log_sum);
          }
          if (round_out) o = round4(o);
          st_stream(dr + f, o);
        }
      }
    }
    __syncthreads();  // part_m / part_s reuse in the next row
  }
}

template <int VPL>
__global__ void __launch_bounds__(256)
ce_warp_kernel(float* __restrict__ loss, float* dlogits, const float* logits,
               const int32_t* __restrict__ targets, uint64_t rows, uint64_t classes, uint64_t ld,
               uint64_t seq, float grad_scale, int32_t* invalid, int round_out) {
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
        if (round_out) o = round4(o);
        dr[f] = o;
      }
    }
  }
}

// Generic two-pass path for any class count (and ld/classes not multiples of 4).
__global__ void __launch_bounds__(256)
ce_generic_kernel(float* __restrict__ loss, float* dlogits, const float* logits,
                  const int32_t* __restrict__ targets, uint64_t rows, uint64_t classes,
                  uint64_t ld, uint64_t seq, float grad_scale, int32_t* invalid, int round_out) {
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
    for (uint64_t c = threadIdx.x; c < classes; c += blockDim.x) {
      const float d = grad_scale * (expf((zr[c] - m) - log_sum) - (c == (uint64_t)target ? 1.f : 0.f));
      dr[c] = round_out ? round_tf32(d) : d;
    }
    if (threadIdx.x == 0) loss[r] = -((zt - m) - log_sum);
    __syncthreads();
  }
}

}  // namespace

cudaError_t cross_entropy_launch(float* loss, float* dlogits, const float* logits,
                                 const int32_t* targets, uint64_t rows, uint64_t classes,
                                 uint64_t ld, uint64_t seq, float grad_scale,
                                 int32_t* invalid, int device, cudaStream_t stream,
                                 bool round_out) {
  const bool vec_ok = classes % 4 == 0 && ld % 4 == 0;
  const int rnd = round_out ? 1 : 0;
  const uint64_t vec = classes / 4;
  const int sms = sm_count(device);
  if (vec_ok && vec <= 32 * 16) {
    const uint64_t v = (vec + 31) / 32;
    const unsigned grid = grid_for(rows, 8, sms * 16);
    switch (v <= 1 ? 1 : v <= 2 ? 2 : v <= 4 ? 4 : v <= 8 ? 8 : 16) {
#define SPAR_CE_W(V) case V: launch(ce_warp_kernel<V>, dim3(grid), dim3(256), 0, stream, loss, dlogits, logits, targets, rows, classes, ld, seq, grad_scale, invalid, rnd); break;
      SPAR_CE_W(1) SPAR_CE_W(2) SPAR_CE_W(4) SPAR_CE_W(8) SPAR_CE_W(16)
#undef SPAR_CE_W
    }
  } else if (vec_ok) {
    const unsigned grid = grid_for(rows, 1, sms * 3);
    launch(ce_stream_kernel, dim3(grid), dim3(kCeThreads), 0, stream, loss, dlogits, logits,
           targets, rows, classes, ld, seq, grad_scale, invalid, rnd);
  } else {
    const unsigned grid = grid_for(rows, 1, sms * 8);
    launch(ce_generic_kernel, dim3(grid), dim3(256), 0, stream, loss, dlogits, logits, targets, rows, classes, ld,
                                                seq, grad_scale, invalid, rnd);
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
