// Shared host/device helpers for the spar_b200 kernel library.
//
// Status convention follows the reference C ABI (src/backend/cuda_kernels.cu:12-22):
//   code 0 = success, 1 = invalid argument, 2 = CUDA runtime error (cuda_error filled in).
// Unlike the reference, launches here are asynchronous on a caller-supplied stream; only
// launch/configuration errors are reported by the call itself.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <map>
#include <mutex>
#include <utility>

#include "spar_b200.h"

namespace spar_b200 {

inline SparCudaStatus ok() { return {0, static_cast<int>(cudaSuccess)}; }
inline SparCudaStatus invalid() { return {1, static_cast<int>(cudaErrorInvalidValue)}; }
inline SparCudaStatus runtime(cudaError_t e) { return {2, static_cast<int>(e)}; }

// Selects `device` for the duration of a call and restores the caller's device afterwards,
// mirroring the reference's select_device/finish_launch pair (cuda_kernels.cu:24-49).
class DeviceScope {
 public:
  explicit DeviceScope(int device) {
    error_ = cudaGetDevice(&previous_);
    if (error_ == cudaSuccess && previous_ != device) {
      error_ = cudaSetDevice(device);
      changed_ = error_ == cudaSuccess;
    }
  }
  ~DeviceScope() {
    if (changed_) cudaSetDevice(previous_);
  }
  cudaError_t error() const { return error_; }

 private:
  int previous_ = 0;
  bool changed_ = false;
  cudaError_t error_ = cudaSuccess;
};

inline SparCudaStatus launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ok() : runtime(e);
}

constexpr int kNumSMs = 148;

inline int sm_count(int device) {
  static int cached[64] = {0};
  if (device >= 0 && device < 64 && cached[device] != 0) return cached[device];
  int n = kNumSMs;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  if (device >= 0 && device < 64) cached[device] = n;
  return n;
}

inline unsigned grid_for(uint64_t work, unsigned per_block, unsigned cap) {
  uint64_t b = (work + per_block - 1) / per_block;
  if (b < 1) b = 1;
  if (b > cap) b = cap;
  return static_cast<unsigned>(b);
}

// ------------------------------------------------------ programmatic dependent launches
// Every kernel of the library is launched with programmatic stream serialization: its CTAs may
// be scheduled while the previous kernel on the stream is still finishing, run their set-up
// (barrier init, TMEM allocation), then block in pdl_wait() until that kernel has completed and
// its memory is visible. pdl_wait() therefore comes before a kernel's first global-memory
// access (read or write). pdl_trigger() lets the next kernel's launch begin once every CTA of
// this one has passed its wait. Outside such a launch both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Both, in that order: the usual first statement of a kernel.
__device__ __forceinline__ void pdl_begin() {
  pdl_wait();
  pdl_trigger();
}

// SPAR_B200_PDL=0 in the environment launches without the attribute (plain stream order).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("SPAR_B200_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// cudaMallocAsync from the current device's memory pool, which is first told (once per device)
// to keep freed memory reserved instead of returning it to the driver at every synchronisation:
// with the default release threshold of 0, each synchronous call that takes a large workspace
// (the 3xTF32 operand splits: 1.6 GB for an 8192 x 16384 x 4096 product) would map and unmap it
// again, which measured slower than the product itself. Memory stays with the pool up to its peak.
inline cudaError_t stream_alloc(void** ptr, size_t bytes, cudaStream_t stream) {
  static std::mutex mu;
  static bool done[64] = {};
  int device = 0;
  if (cudaGetDevice(&device) == cudaSuccess && device >= 0 && device < 64) {
    std::lock_guard<std::mutex> lock(mu);
    if (!done[device]) {
      cudaMemPool_t pool = nullptr;
      if (cudaDeviceGetMemPool(&pool, device) == cudaSuccess) {
        uint64_t keep = ~0ull;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
      }
      cudaGetLastError();
      done[device] = true;
    }
  }
  return cudaMallocAsync(ptr, bytes, stream);
}

// Raises (never lowers) the dynamic shared memory `kernel` may be launched with on `device`.
// A kernel launched with different sizes must never have its limit lowered by a smaller launch:
// a CUDA graph captured earlier with the larger size re-issues that launch later (and a profiler
// replaying the graph's nodes re-launches them one by one) under the limit in force at that time,
// and a launch above the limit fails.
inline cudaError_t raise_dynamic_smem(const void* kernel, int device, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> limit;
  std::lock_guard<std::mutex> lock(mu);
  size_t& current = limit[{kernel, device}];
  if (current >= bytes) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) current = bytes;
  return e;
}

// ---------------------------------------------------------------- device reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum of one float per thread; every thread receives the total. `scratch` holds
// at least 32 floats. Threads per block must be a multiple of 32.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < warps ? scratch[lane] : 0.f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < warps ? scratch[lane] : -INFINITY;
  return warp_max(t);
}

// Streaming 128-bit global accesses (data touched once per kernel).
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }

}  // namespace spar_b200
