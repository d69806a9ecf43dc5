// Token embedding gather and its deterministic scatter-add backward.
//
// Forward is Spar's embedding_lookup (src/ops/embedding.cpp:89-121, 55-67): out[i, :] = E[ids[i], :].
// The reference backward scatters with atomicAdd (cuda_kernels.cu:650-661), whose summation order
// changes run to run. Here the ids are counting-sorted on the device (count, exclusive scan,
// bucket fill, then a rank sort inside every bucket so each bucket lists its positions in
// increasing order), and one warp per vocabulary row sums its positions' gradients in position
// order: the same bits on every run, and the same order as the reference's CPU scatter loop
// (embedding_gradient, src/ops/embedding.cpp:70-85).
#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

__global__ void embedding_forward_kernel(float4* __restrict__ out, const float4* __restrict__ w,
                                         const int32_t* __restrict__ ids, uint64_t count,
                                         uint64_t vocab, uint64_t dim4, int32_t* invalid) {
  pdl_begin();
  const uint64_t total = count * dim4;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += stride) {
    const uint64_t pos = idx / dim4, f = idx % dim4;
    const int32_t id = ids[pos];
    if (id < 0 || static_cast<uint64_t>(id) >= vocab) {
      if (f == 0) atomicExch(invalid, 1);
      out[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    out[idx] = w[static_cast<uint64_t>(id) * dim4 + f];
  }
}

__global__ void count_kernel(int32_t* counts, const int32_t* __restrict__ ids, uint64_t n,
                             uint64_t vocab) {
  pdl_begin();
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t id = ids[i];
  if (id >= 0 && static_cast<uint64_t>(id) < vocab) atomicAdd(counts + id, 1);
}

// Exclusive scan of counts[0, vocab) into offsets[0, vocab], single block.
__global__ void __launch_bounds__(1024) scan_kernel(int32_t* offsets, const int32_t* counts,
                                                    uint64_t vocab) {
  pdl_begin();
  __shared__ int32_t sums[1024];
  const uint64_t per = (vocab + blockDim.x - 1) / blockDim.x;
  const uint64_t b = per * threadIdx.x;
  uint64_t e = b + per;
  if (e > vocab) e = vocab;
  int32_t local = 0;
  for (uint64_t i = b; i < e; ++i) local += counts[i];
  sums[threadIdx.x] = local;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int32_t v = threadIdx.x >= off ? sums[threadIdx.x - off] : 0;
    __syncthreads();
    sums[threadIdx.x] += v;
    __syncthreads();
  }
  int32_t run = sums[threadIdx.x] - local;  // exclusive prefix of this chunk
  for (uint64_t i = b; i < e; ++i) {
    offsets[i] = run;
    run += counts[i];
  }
  if (threadIdx.x == blockDim.x - 1) offsets[vocab] = sums[threadIdx.x];
}

__global__ void fill_kernel(int32_t* slots, int32_t* cursor, const int32_t* __restrict__ offsets,
                            const int32_t* __restrict__ ids, uint64_t n, uint64_t vocab) {
  pdl_begin();
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t id = ids[i];
  if (id < 0 || static_cast<uint64_t>(id) >= vocab) return;
  slots[offsets[id] + atomicAdd(cursor + id, 1)] = static_cast<int32_t>(i);
}

// Rank sort inside each bucket: sorted[offset + rank] = position.
__global__ void rank_kernel(int32_t* sorted, const int32_t* __restrict__ slots,
                            const int32_t* __restrict__ offsets, const int32_t* __restrict__ ids,
                            uint64_t vocab) {
  pdl_begin();
  const uint64_t s = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // offsets[vocab] = number of valid ids = number of filled slots.
  if (s >= static_cast<uint64_t>(offsets[vocab])) return;
  const int32_t pos = slots[s];
  const int32_t id = ids[pos];
  const int32_t b = offsets[id], e = offsets[id + 1];
  int32_t rank = 0;
  for (int32_t k = b; k < e; ++k) rank += slots[k] < pos;
  sorted[b + rank] = pos;
}

// One warp per vocabulary row; rows without occurrences are left untouched.
__global__ void __launch_bounds__(256)
segment_reduce_kernel(float* __restrict__ gw, const float* __restrict__ go,
                      const int32_t* __restrict__ sorted, const int32_t* __restrict__ offsets,
                      uint64_t vocab, uint64_t dim) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * 8;
  const uint64_t dim4 = dim / 4;
  for (uint64_t v = static_cast<uint64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); v < vocab;
       v += stride) {
    const int32_t b = offsets[v], e = offsets[v + 1];
    if (b == e) continue;
    for (uint64_t f = lane; f < dim4; f += 32) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int32_t k = b; k < e; ++k) {
        const float4 g = reinterpret_cast<const float4*>(go + static_cast<uint64_t>(sorted[k]) * dim)[f];
        acc.x += g.x;
        acc.y += g.y;
        acc.z += g.z;
        acc.w += g.w;
      }
      float4* dst = reinterpret_cast<float4*>(gw + v * dim) + f;
      const float4 prev = *dst;
      *dst = make_float4(prev.x + acc.x, prev.y + acc.y, prev.z + acc.z, prev.w + acc.w);
    }
  }
}

uint64_t align16(uint64_t b) { return (b + 15) & ~15ull; }

}  // namespace

cudaError_t embedding_forward_launch(float* out, const float* weight, const int32_t* ids,
                                     uint64_t count, uint64_t vocab, uint64_t dim,
                                     int32_t* invalid, int device, cudaStream_t stream) {
  const uint64_t dim4 = dim / 4;
  const unsigned grid = grid_for(count * dim4, 256, sm_count(device) * 16);
  launch(embedding_forward_kernel, dim3(grid), dim3(256), 0, stream, reinterpret_cast<float4*>(out),
                                                     reinterpret_cast<const float4*>(weight), ids,
                                                     count, vocab, dim4, invalid);
  return cudaGetLastError();
}

uint64_t embedding_backward_scratch(uint64_t count, uint64_t vocab) {
  return align16(4 * vocab) + align16(4 * (vocab + 1)) + align16(4 * vocab) +
         align16(4 * count) * 2;
}

cudaError_t embedding_backward_launch(float* grad_weight, const float* grad_out,
                                      const int32_t* ids, uint64_t count, uint64_t vocab,
                                      uint64_t dim, void* scratch, int device,
                                      cudaStream_t stream) {
  char* p = static_cast<char*>(scratch);
  int32_t* counts = reinterpret_cast<int32_t*>(p);
  p += align16(4 * vocab);
  int32_t* offsets = reinterpret_cast<int32_t*>(p);
  p += align16(4 * (vocab + 1));
  int32_t* cursor = reinterpret_cast<int32_t*>(p);
  p += align16(4 * vocab);
  int32_t* slots = reinterpret_cast<int32_t*>(p);
  p += align16(4 * count);
  int32_t* sorted = reinterpret_cast<int32_t*>(p);
  cudaError_t e = cudaMemsetAsync(counts, 0, 4 * vocab, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(cursor, 0, 4 * vocab, stream);
  if (e != cudaSuccess) return e;
  const unsigned gn = static_cast<unsigned>((count + 255) / 256);
  launch(count_kernel, dim3(gn), dim3(256), 0, stream, counts, ids, count, vocab);
  launch(scan_kernel, dim3(1), dim3(1024), 0, stream, offsets, counts, vocab);
  launch(fill_kernel, dim3(gn), dim3(256), 0, stream, slots, cursor, offsets, ids, count, vocab);
  // Invalid ids are skipped, so only offsets[vocab] <= count slots are filled; the rank kernel
  // reads that bound on the device.
  launch(rank_kernel, dim3(gn), dim3(256), 0, stream, sorted, slots, offsets, ids, vocab);
  const unsigned gv = grid_for(vocab, 8, sm_count(device) * 16);
  launch(segment_reduce_kernel, dim3(gv), dim3(256), 0, stream, grad_weight, grad_out, sorted, offsets, vocab,
                                                dim);
  return cudaGetLastError();
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_embedding_forward(float* out, const float* weight,
                                                      const int32_t* ids, uint64_t count,
                                                      uint64_t vocab, uint64_t dim,
                                                      int32_t* invalid_index, int device,
                                                      void* stream) {
  if (count == 0) return ok();
  if (!out || !weight || !ids || !invalid_index || vocab == 0 || dim == 0 || dim % 4 != 0)
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = embedding_forward_launch(out, weight, ids, count, vocab, dim,
                                                 invalid_index, device, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" uint64_t spar_b200_embedding_backward_scratch_bytes(uint64_t count, uint64_t vocab) {
  return embedding_backward_scratch(count, vocab);
}

extern "C" SparCudaStatus spar_b200_embedding_backward(float* grad_weight, const float* grad_out,
                                                       const int32_t* ids, uint64_t count,
                                                       uint64_t vocab, uint64_t dim,
                                                       void* scratch, int device, void* stream) {
  if (count == 0) return ok();
  if (!grad_weight || !grad_out || !ids || !scratch || vocab == 0 || dim == 0 || dim % 4 != 0 ||
      count > 0x7fffffffull || vocab > 0x7fffffffull)
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = embedding_backward_launch(grad_weight, grad_out, ids, count, vocab, dim,
                                                  scratch, device, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}
