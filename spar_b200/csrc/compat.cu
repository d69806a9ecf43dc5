// Drop-in implementation of Spar's backend C ABI (src/backend/cuda_kernels.hpp:46-129).
//
// Same names, signatures, argument validation, special-value semantics and status convention as
// the reference launchers (src/backend/cuda_kernels.cu:711-1477), so Spar's tensor-level
// wrappers (src/backend/cuda_ops.cppm) work unchanged on top of this library. Differences are
// internal:
//   - grids sized from the SM count, 128-bit accesses where the layout allows;
//   - strided_copy / broadcast_reduce take their shape metadata as kernel parameters instead of a
//     cudaMalloc + cudaMemcpy + cudaFree per call (rank <= 16);
//   - broadcast_reduce is deterministic (one thread owns each destination element and sums its
//     reduced coordinates in order) instead of atomicAdd; embedding_backward keeps the
//     reference's atomic scatter (the hot path uses the sorted, deterministic
//     spar_b200_embedding_backward instead);
//   - the norm summary is a grid-wide two-pass reduction (max |g|, then sum (g/max)^2 in
//     double) instead of one 256-thread block.
// Like the reference, every call returns after the device finished (cudaDeviceSynchronize), so
// runtime errors are reported by the call that caused them.
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

constexpr int kMaxRank = 16;

bool valid_dtype(int d) { return d == SPAR_CUDA_FLOAT32 || d == SPAR_CUDA_FLOAT64; }
bool valid_index(int d) { return d == SPAR_CUDA_INT32 || d == SPAR_CUDA_INT64; }

SparCudaStatus finish() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e == cudaSuccess ? ok() : runtime(e);
}

unsigned blocks_for(uint64_t n, int device) { return grid_for(n, 256, sm_count(device) * 16); }

#define GRID_LOOP(i, n)                                                                   \
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (n); \
       i += static_cast<uint64_t>(blockDim.x) * gridDim.x)

template <typename T>
__device__ __forceinline__ T sigmoid_t(T v) {
  if (v >= T{0}) return T{1} / (T{1} + exp(-v));
  const T e = exp(v);
  return e / (T{1} + e);
}

template <typename T>
__global__ void binary_k(T* o, const T* a, const T* b, uint64_t n, int op) {
  GRID_LOOP(i, n) {
    const T x = a[i], y = b[i];
    o[i] = op == SPAR_CUDA_ADD ? x + y : op == SPAR_CUDA_SUBTRACT ? x - y
         : op == SPAR_CUDA_MULTIPLY ? x * y : x / y;
  }
}

template <typename T>
__global__ void scalar_k(T* o, const T* a, uint64_t n, int op, T s) {
  GRID_LOOP(i, n) {
    const T x = a[i];
    o[i] = op == SPAR_CUDA_ADD ? x + s : op == SPAR_CUDA_SUBTRACT ? x - s
         : op == SPAR_CUDA_MULTIPLY ? x * s : x / s;
  }
}

template <typename T>
__global__ void unary_k(T* o, const T* a, uint64_t n, int op) {
  GRID_LOOP(i, n) {
    const T v = a[i];
    T r;
    switch (op) {
      case SPAR_CUDA_NEGATE: r = -v; break;
      case SPAR_CUDA_SQUARE: r = v * v; break;
      case SPAR_CUDA_RECIPROCAL: r = T{1} / v; break;
      case SPAR_CUDA_EXP: r = exp(v); break;
      case SPAR_CUDA_LOG: r = log(v); break;
      case SPAR_CUDA_SQRT: r = sqrt(v); break;
      case SPAR_CUDA_SIGMOID: r = sigmoid_t(v); break;
      default: r = v * sigmoid_t(v); break;
    }
    o[i] = r;
  }
}

// Full sum/mean/max with one block (the result is a single scalar; NaN propagates for max).
template <typename T>
__global__ void full_reduce_k(T* out, const T* a, uint64_t n, int op) {
  __shared__ T part[1024];
  __shared__ int nan_part[1024];
  T v = op == SPAR_CUDA_MAX ? -static_cast<T>(INFINITY) : T{0};
  int has_nan = 0;
  for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const T x = a[i];
    if (op == SPAR_CUDA_MAX) {
      if (isnan(x)) has_nan = 1;
      else if (x > v) v = x;
    } else {
      v += x;
    }
  }
  part[threadIdx.x] = v;
  nan_part[threadIdx.x] = has_nan;
  __syncthreads();
  for (unsigned w = blockDim.x / 2; w; w >>= 1) {
    if (threadIdx.x < w) {
      if (op == SPAR_CUDA_MAX) {
        nan_part[threadIdx.x] |= nan_part[threadIdx.x + w];
        if (part[threadIdx.x + w] > part[threadIdx.x]) part[threadIdx.x] = part[threadIdx.x + w];
      } else {
        part[threadIdx.x] += part[threadIdx.x + w];
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (op == SPAR_CUDA_MAX) out[0] = nan_part[0] ? static_cast<T>(NAN) : part[0];
    else out[0] = op == SPAR_CUDA_MEAN ? part[0] / static_cast<T>(n) : part[0];
  }
}

// One warp per row.
template <typename T>
__global__ void row_reduce_k(T* out, const T* a, uint64_t rows, uint64_t cols, int mean) {
  const int lane = threadIdx.x & 31;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
  for (uint64_t r = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += stride) {
    T s = T{0};
    for (uint64_t c = lane; c < cols; c += 32) s += a[r * cols + c];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[r] = mean ? s / static_cast<T>(cols) : s;
  }
}

// Softmax / log-softmax along an axis of an (outer, axis, inner) view; one warp per slice with
// the reference's special cases (NaN or all -inf -> NaN slice; +inf entries share the mass).
template <typename T>
__global__ void probability_forward_k(T* out, int32_t* undefined, const T* in, uint64_t outer,
                                      uint64_t axis, uint64_t inner, int logarithmic) {
  const int lane = threadIdx.x & 31;
  const uint64_t slices = outer * inner;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
  const T inf = static_cast<T>(INFINITY);
  for (uint64_t s = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       s < slices; s += stride) {
    const uint64_t o = s / inner, in_i = s % inner;
    auto at = [&](uint64_t a) { return (o * axis + a) * inner + in_i; };
    T m = -inf;
    int has_nan = 0;
    unsigned long long pinf = 0;
    for (uint64_t a = lane; a < axis; a += 32) {
      const T v = in[at(a)];
      has_nan |= isnan(v);
      pinf += v == inf;
      if (v > m) m = v;
    }
#pragma unroll
    for (int d = 16; d; d >>= 1) {
      const T mo = __shfl_xor_sync(0xffffffffu, m, d);
      m = mo > m ? mo : m;
      has_nan |= __shfl_xor_sync(0xffffffffu, has_nan, d);
      pinf += __shfl_xor_sync(0xffffffffu, pinf, d);
    }
    const bool bad = has_nan || m == -inf;
    if (lane == 0) undefined[s] = (bad || pinf != 0) ? 1 : 0;
    if (bad) {
      for (uint64_t a = lane; a < axis; a += 32) out[at(a)] = static_cast<T>(NAN);
      continue;
    }
    if (pinf != 0) {
      const T hit = logarithmic ? -log(static_cast<T>(pinf)) : T{1} / static_cast<T>(pinf);
      const T miss = logarithmic ? -inf : T{0};
      for (uint64_t a = lane; a < axis; a += 32) out[at(a)] = in[at(a)] == inf ? hit : miss;
      continue;
    }
    T sum = T{0};
    for (uint64_t a = lane; a < axis; a += 32) sum += exp(in[at(a)] - m);
#pragma unroll
    for (int d = 16; d; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
    const T norm = logarithmic ? log(sum) : sum;
    for (uint64_t a = lane; a < axis; a += 32) {
      const T v = in[at(a)];
      out[at(a)] = logarithmic ? (v - m) - norm : exp(v - m) / norm;
    }
  }
}

template <typename T>
__global__ void probability_backward_k(T* out, const T* g, const T* y, const int32_t* undefined,
                                       uint64_t outer, uint64_t axis, uint64_t inner,
                                       int logarithmic) {
  const int lane = threadIdx.x & 31;
  const uint64_t slices = outer * inner;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
  for (uint64_t s = static_cast<uint64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       s < slices; s += stride) {
    const uint64_t o = s / inner, in_i = s % inner;
    auto at = [&](uint64_t a) { return (o * axis + a) * inner + in_i; };
    if (undefined[s]) {
      for (uint64_t a = lane; a < axis; a += 32) out[at(a)] = static_cast<T>(NAN);
      continue;
    }
    T acc = T{0};
    for (uint64_t a = lane; a < axis; a += 32) acc += logarithmic ? g[at(a)] : g[at(a)] * y[at(a)];
#pragma unroll
    for (int d = 16; d; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
    for (uint64_t a = lane; a < axis; a += 32) {
      const uint64_t k = at(a);
      out[k] = logarithmic ? g[k] - exp(y[k]) * acc : y[k] * (g[k] - acc);
    }
  }
}

template <typename I>
__global__ void validate_indices_k(int32_t* bad, const I* idx, uint64_t n, uint64_t bound) {
  GRID_LOOP(i, n) {
    const I v = idx[i];
    if (v < 0 || static_cast<uint64_t>(v) >= bound) atomicExch(bad, 1);
  }
}

template <typename T, typename I>
__global__ void embedding_fwd_k(T* o, int32_t* bad, const T* w, const I* idx, uint64_t n,
                                uint64_t vocab, uint64_t dim) {
  GRID_LOOP(i, n * dim) {
    const I id = idx[i / dim];
    if (id < 0 || static_cast<uint64_t>(id) >= vocab) {
      atomicExch(bad, 1);
      continue;
    }
    o[i] = w[static_cast<uint64_t>(id) * dim + i % dim];
  }
}

template <typename T, typename I>
__global__ void embedding_bwd_atomic_k(T* o, const T* g, const I* idx, uint64_t n, uint64_t dim) {
  GRID_LOOP(i, n * dim) {
    atomicAdd(o + static_cast<uint64_t>(idx[i / dim]) * dim + i % dim, g[i]);
  }
}

template <typename T>
__global__ void rope_k(T* o, const T* x, uint64_t pairs, uint64_t seq, uint64_t feat,
                       uint64_t start, double theta, int inverse) {
  const uint64_t per_token = feat / 2;
  GRID_LOOP(p, pairs) {
    const uint64_t pair = p % per_token;
    const uint64_t token = (p / per_token) % seq;
    const uint64_t idx = (p / per_token) * feat + 2 * pair;
    const double ang = static_cast<double>(start + token) *
                       pow(theta, -2.0 * static_cast<double>(pair) / static_cast<double>(feat));
    const T c = static_cast<T>(cos(ang));
    T s = static_cast<T>(sin(ang));
    if (inverse) s = -s;
    const T a = x[idx], b = x[idx + 1];
    o[idx] = a * c - b * s;
    o[idx + 1] = a * s + b * c;
  }
}

template <typename T>
__global__ void causal_mask_k(T* o, uint64_t seq) {
  GRID_LOOP(i, seq * seq) o[i] = (i % seq) <= (i / seq) ? T{0} : -static_cast<T>(INFINITY);
}

template <typename T>
__global__ void fill_k(T* o, const T* s, uint64_t n, T scale) {
  const T v = s[0] * scale;
  GRID_LOOP(i, n) o[i] = v;
}

template <typename T>
__global__ void add_in_place_k(T* d, const T* s, uint64_t n) {
  GRID_LOOP(i, n) d[i] += s[i];
}

struct Shape16 {
  uint64_t extent[kMaxRank];
  uint64_t stride[kMaxRank];
  uint64_t orig_extent[kMaxRank];
};

template <typename P>
__global__ void strided_copy_k(P* d, const P* s, Shape16 sh, uint64_t rank, uint64_t offset,
                               uint64_t n) {
  GRID_LOOP(i, n) {
    uint64_t rem = i, src = offset;
    for (uint64_t a = rank; a-- > 0;) {
      src += (rem % sh.extent[a]) * sh.stride[a];
      rem /= sh.extent[a];
    }
    d[i] = s[src];
  }
}

// Deterministic broadcast reduction: one thread per kept-coordinate tuple sums every reduced
// coordinate in increasing logical order, then adds into the destination.
template <typename T>
__global__ void broadcast_reduce_k(T* dst, const T* g, Shape16 sh, uint64_t grank, uint64_t orank,
                                   uint64_t kept_count, uint64_t red_count) {
  const uint64_t leading = grank - orank;
  GRID_LOOP(kidx, kept_count) {
    // Decompose kidx over kept axes and build the destination index + gradient base offset.
    uint64_t rem = kidx, dest = 0, base = 0, gstride = 1;
    uint64_t gstrides[kMaxRank];
    for (uint64_t a = grank; a-- > 0;) {
      gstrides[a] = gstride;
      gstride *= sh.extent[a];
    }
    for (uint64_t a = grank; a-- > 0;) {
      const bool kept = a >= leading && sh.orig_extent[a - leading] != 1;
      if (!kept) continue;
      const uint64_t c = rem % sh.extent[a];
      rem /= sh.extent[a];
      dest += c * sh.stride[a - leading];
      base += c * gstrides[a];
    }
    T acc = T{0};
    for (uint64_t r = 0; r < red_count; ++r) {
      uint64_t rr = r, off = base;
      for (uint64_t a = grank; a-- > 0;) {
        const bool kept = a >= leading && sh.orig_extent[a - leading] != 1;
        if (kept) continue;
        off += (rr % sh.extent[a]) * gstrides[a];
        rr /= sh.extent[a];
      }
      acc += g[off];
    }
    dst[dest] += acc;
  }
}

template <typename T, typename I>
__global__ void nll_k(T* o, const T* src, const I* tg, uint64_t n, uint64_t classes, uint64_t seq,
                      int lm, int backward) {
  GRID_LOOP(i, n) {
    uint64_t t_idx = i, row = i;
    if (lm) {
      const uint64_t pl = seq - 1, b = i / pl, t = i % pl;
      t_idx = b * seq + t + 1;
      row = b * seq + t;
    }
    const uint64_t k = row * classes + static_cast<uint64_t>(tg[t_idx]);
    if (backward) o[k] = -src[i];
    else o[i] = -src[k];
  }
}

// Norm summary, pass 1: per-block max |g| over finite values and non-finite flags.
template <typename T>
__global__ void norm_max_k(double* part_max, int* part_flags, const T* g, uint64_t n) {
  __shared__ double smax[32];
  __shared__ int sflag[32];
  double m = 0.0;
  int flags = 0;  // bit0 inf, bit1 nan
  GRID_LOOP(i, n) {
    const double v = fabs(static_cast<double>(g[i]));
    if (isnan(v)) flags |= 2;
    else if (isinf(v)) flags |= 1;
    else m = fmax(m, v);
  }
#pragma unroll
  for (int d = 16; d; d >>= 1) {
    m = fmax(m, __shfl_xor_sync(0xffffffffu, m, d));
    flags |= __shfl_xor_sync(0xffffffffu, flags, d);
  }
  if ((threadIdx.x & 31) == 0) {
    smax[threadIdx.x >> 5] = m;
    sflag[threadIdx.x >> 5] = flags;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
      m = fmax(smax[0], smax[w]);
      smax[0] = m;
      sflag[0] |= sflag[w];
    }
    part_max[blockIdx.x] = smax[0];
    part_flags[blockIdx.x] = sflag[0];
  }
}

// Pass 2: per-block sum of (g / scale)^2 over finite values, scale = global max |g|.
template <typename T>
__global__ void norm_ssq_k(double* part_ssq, const double* part_max, int parts, const T* g,
                           uint64_t n) {
  __shared__ double s[32];
  double scale = 0.0;
  for (int p = 0; p < parts; ++p) scale = fmax(scale, part_max[p]);
  double acc = 0.0;
  if (scale > 0.0) {
    GRID_LOOP(i, n) {
      const double v = fabs(static_cast<double>(g[i]));
      if (isfinite(v)) {
        const double r = v / scale;
        acc += r * r;
      }
    }
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) s[0] += s[w];
    part_ssq[blockIdx.x] = s[0];
  }
}

__global__ void norm_final_k(SparCudaNormSummary* out, const double* part_max,
                             const int* part_flags, const double* part_ssq, int parts) {
  double scale = 0.0, ssq = 0.0;
  int flags = 0;
  for (int p = 0; p < parts; ++p) {
    scale = fmax(scale, part_max[p]);
    flags |= part_flags[p];
  }
  for (int p = 0; p < parts; ++p) ssq += part_ssq[p];
  out->scale = scale;
  out->scaled_sum_squares = scale == 0.0 ? 1.0 : ssq;
  out->has_infinity = (flags & 1) ? 1 : 0;
  out->has_nan = (flags & 2) ? 1 : 0;
}

template <typename T>
__global__ void scale_k(T* v, uint64_t n, double f) {
  GRID_LOOP(i, n) v[i] = static_cast<T>(static_cast<double>(v[i]) * f);
}

template <typename T>
__global__ void adamw_k(T* p, const T* g, T* m, T* v, uint64_t n, double lr, double b1, double b2,
                        double eps, double wd, double c1, double c2) {
  // The decay factor is formed on the device, as the reference does: a host-side 1 - lr * wd
  // rounds twice where the device's contracted multiply-add rounds once, which moves float64
  // parameters by an ulp.
  const double decay = 1.0 - lr * wd;
  GRID_LOOP(i, n) {
    const double gd = static_cast<double>(g[i]);
    m[i] = static_cast<T>(b1 * static_cast<double>(m[i]) + (1.0 - b1) * gd);
    v[i] = static_cast<T>(b2 * static_cast<double>(v[i]) + (1.0 - b2) * gd * gd);
    const double mc = static_cast<double>(m[i]) / c1;
    const double vc = static_cast<double>(v[i]) / c2;
    p[i] = static_cast<T>(static_cast<double>(p[i]) * decay - lr * mc / (sqrt(vc) + eps));
  }
}

}  // namespace
}  // namespace spar_b200

using namespace spar_b200;

#define SPAR_SCOPE(device)                                        \
  DeviceScope scope_(device);                                     \
  if (scope_.error() != cudaSuccess) return runtime(scope_.error())

#define SPAR_DISPATCH_T(dtype, KERNEL, grid, ...)                                              \
  do {                                                                                        \
    if ((dtype) == SPAR_CUDA_FLOAT32) KERNEL<float><<<grid, 256>>>(__VA_ARGS__);               \
    else KERNEL<double><<<grid, 256>>>(__VA_ARGS__);                                           \
  } while (0)

template <typename T>
static T* tp(void* p) { return static_cast<T*>(p); }
template <typename T>
static const T* ctp(const void* p) { return static_cast<const T*>(p); }

extern "C" SparCudaStatus spar_cuda_launch_binary(void* output, const void* left, const void* right,
                                                  uint64_t count, int dtype, int operation,
                                                  int device) {
  if (!valid_dtype(dtype) || operation < SPAR_CUDA_ADD || operation > SPAR_CUDA_DIVIDE ||
      (count != 0 && (!output || !left || !right)))
    return invalid();
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    binary_k<float><<<g, 256>>>(tp<float>(output), ctp<float>(left), ctp<float>(right), count, operation);
  else
    binary_k<double><<<g, 256>>>(tp<double>(output), ctp<double>(left), ctp<double>(right), count, operation);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_scalar(void* output, const void* input, uint64_t count,
                                                  int dtype, int operation, double scalar,
                                                  int device) {
  if (!valid_dtype(dtype) || operation < SPAR_CUDA_ADD || operation > SPAR_CUDA_DIVIDE ||
      (count != 0 && (!output || !input)))
    return invalid();
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    scalar_k<float><<<g, 256>>>(tp<float>(output), ctp<float>(input), count, operation, static_cast<float>(scalar));
  else
    scalar_k<double><<<g, 256>>>(tp<double>(output), ctp<double>(input), count, operation, scalar);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_unary(void* output, const void* input, uint64_t count,
                                                 int dtype, int operation, int device) {
  if (!valid_dtype(dtype) || operation < SPAR_CUDA_NEGATE || operation > SPAR_CUDA_SILU ||
      (count != 0 && (!output || !input)))
    return invalid();
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    unary_k<float><<<g, 256>>>(tp<float>(output), ctp<float>(input), count, operation);
  else
    unary_k<double><<<g, 256>>>(tp<double>(output), ctp<double>(input), count, operation);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_reduction(void* output, const void* input,
                                                     uint64_t count, int dtype, int operation,
                                                     int device) {
  if (!valid_dtype(dtype) || operation < SPAR_CUDA_SUM || operation > SPAR_CUDA_MAX || !output ||
      (count != 0 && !input) ||
      ((operation == SPAR_CUDA_MEAN || operation == SPAR_CUDA_MAX) && count == 0))
    return invalid();
  SPAR_SCOPE(device);
  if (dtype == SPAR_CUDA_FLOAT32)
    full_reduce_k<float><<<1, 1024>>>(tp<float>(output), ctp<float>(input), count, operation);
  else
    full_reduce_k<double><<<1, 1024>>>(tp<double>(output), ctp<double>(input), count, operation);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_row_reduction(void* output, const void* input,
                                                         uint64_t row_count,
                                                         uint64_t reduction_count, int dtype,
                                                         int operation, int device) {
  if (!valid_dtype(dtype) || (operation != SPAR_CUDA_SUM && operation != SPAR_CUDA_MEAN) ||
      (row_count != 0 && !output) || (row_count != 0 && reduction_count != 0 && !input) ||
      (operation == SPAR_CUDA_MEAN && reduction_count == 0))
    return invalid();
  if (row_count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = grid_for(row_count, 8, sm_count(device) * 16);
  const int mean = operation == SPAR_CUDA_MEAN;
  if (dtype == SPAR_CUDA_FLOAT32)
    row_reduce_k<float><<<g, 256>>>(tp<float>(output), ctp<float>(input), row_count, reduction_count, mean);
  else
    row_reduce_k<double><<<g, 256>>>(tp<double>(output), ctp<double>(input), row_count, reduction_count, mean);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_probability_forward(void* output,
                                                               int32_t* undefined_slices,
                                                               const void* input, uint64_t outer,
                                                               uint64_t axis_extent, uint64_t inner,
                                                               int dtype, int logarithmic,
                                                               int device) {
  if (inner == 0 || outer > UINT64_MAX / inner) return invalid();
  const uint64_t slices = outer * inner;
  if (!valid_dtype(dtype) || axis_extent == 0 || (logarithmic != 0 && logarithmic != 1) ||
      slices == 0 || !output || !undefined_slices || !input)
    return invalid();
  SPAR_SCOPE(device);
  const unsigned g = grid_for(slices, 8, sm_count(device) * 16);
  if (dtype == SPAR_CUDA_FLOAT32)
    probability_forward_k<float><<<g, 256>>>(tp<float>(output), undefined_slices, ctp<float>(input), outer, axis_extent, inner, logarithmic);
  else
    probability_forward_k<double><<<g, 256>>>(tp<double>(output), undefined_slices, ctp<double>(input), outer, axis_extent, inner, logarithmic);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_probability_backward(
    void* output, const void* gradient, const void* saved_output, const int32_t* undefined_slices,
    uint64_t outer, uint64_t axis_extent, uint64_t inner, int dtype, int logarithmic, int device) {
  if (inner == 0 || outer > UINT64_MAX / inner) return invalid();
  const uint64_t slices = outer * inner;
  if (!valid_dtype(dtype) || axis_extent == 0 || (logarithmic != 0 && logarithmic != 1) ||
      slices == 0 || !output || !gradient || !saved_output || !undefined_slices)
    return invalid();
  SPAR_SCOPE(device);
  const unsigned g = grid_for(slices, 8, sm_count(device) * 16);
  if (dtype == SPAR_CUDA_FLOAT32)
    probability_backward_k<float><<<g, 256>>>(tp<float>(output), ctp<float>(gradient), ctp<float>(saved_output), undefined_slices, outer, axis_extent, inner, logarithmic);
  else
    probability_backward_k<double><<<g, 256>>>(tp<double>(output), ctp<double>(gradient), ctp<double>(saved_output), undefined_slices, outer, axis_extent, inner, logarithmic);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_validate_embedding_indices(int32_t* invalid_index,
                                                                      const void* indices,
                                                                      uint64_t index_count,
                                                                      uint64_t vocabulary_size,
                                                                      int index_dtype, int device) {
  if (!valid_index(index_dtype) || index_count == 0 || !invalid_index || !indices) return invalid();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(index_count, device);
  if (index_dtype == SPAR_CUDA_INT32)
    validate_indices_k<int32_t><<<g, 256>>>(invalid_index, ctp<int32_t>(indices), index_count, vocabulary_size);
  else
    validate_indices_k<int64_t><<<g, 256>>>(invalid_index, ctp<int64_t>(indices), index_count, vocabulary_size);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_embedding_forward(void* output, int32_t* invalid_index,
                                                             const void* weight,
                                                             const void* indices,
                                                             uint64_t index_count,
                                                             uint64_t vocabulary_size,
                                                             uint64_t embedding_dimension,
                                                             int weight_dtype, int index_dtype,
                                                             int device) {
  if (!valid_dtype(weight_dtype) || !valid_index(index_dtype) || vocabulary_size == 0 ||
      embedding_dimension == 0 || !invalid_index || index_count > UINT64_MAX / embedding_dimension)
    return invalid();
  if (index_count * embedding_dimension == 0) return ok();
  if (!output || !weight || !indices) return invalid();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(index_count * embedding_dimension, device);
  const uint64_t n = index_count, v = vocabulary_size, d = embedding_dimension;
  if (weight_dtype == SPAR_CUDA_FLOAT32 && index_dtype == SPAR_CUDA_INT32)
    embedding_fwd_k<float, int32_t><<<g, 256>>>(tp<float>(output), invalid_index, ctp<float>(weight), ctp<int32_t>(indices), n, v, d);
  else if (weight_dtype == SPAR_CUDA_FLOAT32)
    embedding_fwd_k<float, int64_t><<<g, 256>>>(tp<float>(output), invalid_index, ctp<float>(weight), ctp<int64_t>(indices), n, v, d);
  else if (index_dtype == SPAR_CUDA_INT32)
    embedding_fwd_k<double, int32_t><<<g, 256>>>(tp<double>(output), invalid_index, ctp<double>(weight), ctp<int32_t>(indices), n, v, d);
  else
    embedding_fwd_k<double, int64_t><<<g, 256>>>(tp<double>(output), invalid_index, ctp<double>(weight), ctp<int64_t>(indices), n, v, d);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_embedding_backward(void* output, const void* gradient,
                                                              const void* indices,
                                                              uint64_t index_count,
                                                              uint64_t embedding_dimension,
                                                              int weight_dtype, int index_dtype,
                                                              int device) {
  if (!valid_dtype(weight_dtype) || !valid_index(index_dtype) || embedding_dimension == 0 ||
      index_count > UINT64_MAX / embedding_dimension)
    return invalid();
  if (index_count * embedding_dimension == 0) return ok();
  if (!output || !gradient || !indices) return invalid();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(index_count * embedding_dimension, device);
  const uint64_t n = index_count, d = embedding_dimension;
  if (weight_dtype == SPAR_CUDA_FLOAT32 && index_dtype == SPAR_CUDA_INT32)
    embedding_bwd_atomic_k<float, int32_t><<<g, 256>>>(tp<float>(output), ctp<float>(gradient), ctp<int32_t>(indices), n, d);
  else if (weight_dtype == SPAR_CUDA_FLOAT32)
    embedding_bwd_atomic_k<float, int64_t><<<g, 256>>>(tp<float>(output), ctp<float>(gradient), ctp<int64_t>(indices), n, d);
  else if (index_dtype == SPAR_CUDA_INT32)
    embedding_bwd_atomic_k<double, int32_t><<<g, 256>>>(tp<double>(output), ctp<double>(gradient), ctp<int32_t>(indices), n, d);
  else
    embedding_bwd_atomic_k<double, int64_t><<<g, 256>>>(tp<double>(output), ctp<double>(gradient), ctp<int64_t>(indices), n, d);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_rope(void* output, const void* input, uint64_t pair_count,
                                                uint64_t sequence_length, uint64_t feature_count,
                                                uint64_t start_position, double theta, int dtype,
                                                int inverse, int device) {
  if (!valid_dtype(dtype) || feature_count == 0 || feature_count % 2 != 0 ||
      (inverse != 0 && inverse != 1) || !(theta > 0.0) || !std::isfinite(theta))
    return invalid();
  if (pair_count == 0) return ok();
  if (sequence_length == 0 || !output || !input) return invalid();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(pair_count, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    rope_k<float><<<g, 256>>>(tp<float>(output), ctp<float>(input), pair_count, sequence_length, feature_count, start_position, theta, inverse);
  else
    rope_k<double><<<g, 256>>>(tp<double>(output), ctp<double>(input), pair_count, sequence_length, feature_count, start_position, theta, inverse);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_causal_mask(void* output, uint64_t sequence_length,
                                                       int dtype, int device) {
  if (!valid_dtype(dtype) || sequence_length == 0 || sequence_length > UINT64_MAX / sequence_length ||
      !output)
    return invalid();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(sequence_length * sequence_length, device);
  if (dtype == SPAR_CUDA_FLOAT32) causal_mask_k<float><<<g, 256>>>(tp<float>(output), sequence_length);
  else causal_mask_k<double><<<g, 256>>>(tp<double>(output), sequence_length);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_fill_from_scalar(void* output, const void* scalar,
                                                            uint64_t count, int dtype, double scale,
                                                            int device) {
  if (!valid_dtype(dtype) || !scalar || (count != 0 && !output)) return invalid();
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    fill_k<float><<<g, 256>>>(tp<float>(output), ctp<float>(scalar), count, static_cast<float>(scale));
  else
    fill_k<double><<<g, 256>>>(tp<double>(output), ctp<double>(scalar), count, scale);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_add_in_place(void* destination, const void* source,
                                                        uint64_t count, int dtype, int device) {
  if (!valid_dtype(dtype) || (count != 0 && (!destination || !source))) return invalid();
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    add_in_place_k<float><<<g, 256>>>(tp<float>(destination), ctp<float>(source), count);
  else
    add_in_place_k<double><<<g, 256>>>(tp<double>(destination), ctp<double>(source), count);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_strided_copy(void* destination, const void* source,
                                                        uint64_t rank, const uint64_t* extents,
                                                        const uint64_t* strides,
                                                        uint64_t storage_offset, uint64_t count,
                                                        uint64_t element_size, int device) {
  if ((element_size != 4 && element_size != 8) || (count != 0 && (!destination || !source)) ||
      (rank != 0 && (!extents || !strides)) || rank > kMaxRank)
    return invalid();
  if (count == 0) return ok();
  Shape16 sh{};
  for (uint64_t a = 0; a < rank; ++a) {
    if (extents[a] == 0) return invalid();
    sh.extent[a] = extents[a];
    sh.stride[a] = strides[a];
  }
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (element_size == 4)
    strided_copy_k<uint32_t><<<g, 256>>>(tp<uint32_t>(destination), ctp<uint32_t>(source), sh, rank, storage_offset, count);
  else
    strided_copy_k<uint64_t><<<g, 256>>>(tp<uint64_t>(destination), ctp<uint64_t>(source), sh, rank, storage_offset, count);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_broadcast_reduce(
    void* destination, const void* gradient, uint64_t gradient_rank,
    const uint64_t* gradient_extents, uint64_t original_rank, const uint64_t* original_extents,
    const uint64_t* original_strides, uint64_t count, int dtype, int device) {
  if (!valid_dtype(dtype) || original_rank > gradient_rank ||
      (count != 0 && (!destination || !gradient)) || (gradient_rank != 0 && !gradient_extents) ||
      (original_rank != 0 && (!original_extents || !original_strides)) ||
      gradient_rank > kMaxRank)
    return invalid();
  if (count == 0) return ok();
  Shape16 sh{};
  const uint64_t leading = gradient_rank - original_rank;
  uint64_t kept = 1, reduced = 1;
  for (uint64_t a = 0; a < gradient_rank; ++a) {
    if (gradient_extents[a] == 0) return invalid();
    sh.extent[a] = gradient_extents[a];
    const bool is_kept = a >= leading && original_extents[a - leading] != 1;
    (is_kept ? kept : reduced) *= gradient_extents[a];
  }
  for (uint64_t a = 0; a < original_rank; ++a) {
    sh.stride[a] = original_strides[a];
    sh.orig_extent[a] = original_extents[a];
  }
  if (kept * reduced != count) return invalid();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(kept, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    broadcast_reduce_k<float><<<g, 256>>>(tp<float>(destination), ctp<float>(gradient), sh, gradient_rank, original_rank, kept, reduced);
  else
    broadcast_reduce_k<double><<<g, 256>>>(tp<double>(destination), ctp<double>(gradient), sh, gradient_rank, original_rank, kept, reduced);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_validate_targets(int32_t* invalid_target, const void* targets,
                                                     uint64_t count, uint64_t classes,
                                                     int target_dtype, int device) {
  if (!invalid_target || classes == 0 || !valid_index(target_dtype) || (count != 0 && !targets))
    return invalid();
  *invalid_target = 0;
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  int32_t* flag = nullptr;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&flag), sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemset(flag, 0, sizeof(int32_t));
  if (e != cudaSuccess) {
    if (flag) cudaFree(flag);
    return runtime(e);
  }
  const unsigned g = blocks_for(count, device);
  if (target_dtype == SPAR_CUDA_INT32)
    validate_indices_k<int32_t><<<g, 256>>>(flag, ctp<int32_t>(targets), count, classes);
  else
    validate_indices_k<int64_t><<<g, 256>>>(flag, ctp<int64_t>(targets), count, classes);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpy(invalid_target, flag, sizeof(int32_t), cudaMemcpyDeviceToHost);
  const cudaError_t f = cudaFree(flag);
  if (e != cudaSuccess) return runtime(e);
  return f == cudaSuccess ? ok() : runtime(f);
}

static SparCudaStatus nll_common(void* output, const void* src, const void* targets,
                                 uint64_t output_count, uint64_t classes, uint64_t seq, int dtype,
                                 int target_dtype, int lm, int device, int backward) {
  if (!valid_dtype(dtype) || !valid_index(target_dtype) || classes == 0 || (lm != 0 && lm != 1) ||
      (lm != 0 && seq < 2) || (output_count != 0 && (!output || !src || !targets)))
    return invalid();
  if (output_count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(output_count, device);
  if (dtype == SPAR_CUDA_FLOAT32 && target_dtype == SPAR_CUDA_INT32)
    nll_k<float, int32_t><<<g, 256>>>(tp<float>(output), ctp<float>(src), ctp<int32_t>(targets), output_count, classes, seq, lm, backward);
  else if (dtype == SPAR_CUDA_FLOAT32)
    nll_k<float, int64_t><<<g, 256>>>(tp<float>(output), ctp<float>(src), ctp<int64_t>(targets), output_count, classes, seq, lm, backward);
  else if (target_dtype == SPAR_CUDA_INT32)
    nll_k<double, int32_t><<<g, 256>>>(tp<double>(output), ctp<double>(src), ctp<int32_t>(targets), output_count, classes, seq, lm, backward);
  else
    nll_k<double, int64_t><<<g, 256>>>(tp<double>(output), ctp<double>(src), ctp<int64_t>(targets), output_count, classes, seq, lm, backward);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_nll_forward(void* output, const void* log_probabilities,
                                                       const void* targets, uint64_t output_count,
                                                       uint64_t classes, uint64_t sequence_length,
                                                       int dtype, int target_dtype,
                                                       int language_model, int device) {
  return nll_common(output, log_probabilities, targets, output_count, classes, sequence_length,
                    dtype, target_dtype, language_model, device, 0);
}

extern "C" SparCudaStatus spar_cuda_launch_nll_backward(void* output, const void* gradient,
                                                        const void* targets, uint64_t output_count,
                                                        uint64_t classes, uint64_t sequence_length,
                                                        int dtype, int target_dtype,
                                                        int language_model, int device) {
  return nll_common(output, gradient, targets, output_count, classes, sequence_length, dtype,
                    target_dtype, language_model, device, 1);
}

extern "C" SparCudaStatus spar_cuda_gradient_norm_summary(SparCudaNormSummary* host_summary,
                                                          const void* gradient, uint64_t count,
                                                          int dtype, int device) {
  if (!host_summary || !valid_dtype(dtype) || (count != 0 && !gradient)) return invalid();
  *host_summary = SparCudaNormSummary{0.0, 1.0, 0, 0};
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const int parts = static_cast<int>(grid_for(count, 256, sm_count(device) * 2));
  char* scratch = nullptr;
  const size_t bytes = parts * (2 * sizeof(double) + sizeof(int)) + sizeof(SparCudaNormSummary) + 64;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&scratch), bytes);
  if (e != cudaSuccess) return runtime(e);
  SparCudaNormSummary* dsum = reinterpret_cast<SparCudaNormSummary*>(scratch);
  double* pmax = reinterpret_cast<double*>(scratch + 64);
  double* pssq = pmax + parts;
  int* pflags = reinterpret_cast<int*>(pssq + parts);
  if (dtype == SPAR_CUDA_FLOAT32) {
    norm_max_k<float><<<parts, 256>>>(pmax, pflags, ctp<float>(gradient), count);
    norm_ssq_k<float><<<parts, 256>>>(pssq, pmax, parts, ctp<float>(gradient), count);
  } else {
    norm_max_k<double><<<parts, 256>>>(pmax, pflags, ctp<double>(gradient), count);
    norm_ssq_k<double><<<parts, 256>>>(pssq, pmax, parts, ctp<double>(gradient), count);
  }
  norm_final_k<<<1, 1>>>(dsum, pmax, pflags, pssq, parts);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpy(host_summary, dsum, sizeof(SparCudaNormSummary), cudaMemcpyDeviceToHost);
  const cudaError_t f = cudaFree(scratch);
  if (e != cudaSuccess) return runtime(e);
  return f == cudaSuccess ? ok() : runtime(f);
}

extern "C" SparCudaStatus spar_cuda_launch_scale_in_place(void* values, uint64_t count, int dtype,
                                                          double factor, int device) {
  if (!valid_dtype(dtype) || !std::isfinite(factor) || (count != 0 && !values)) return invalid();
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (dtype == SPAR_CUDA_FLOAT32) scale_k<float><<<g, 256>>>(tp<float>(values), count, factor);
  else scale_k<double><<<g, 256>>>(tp<double>(values), count, factor);
  return finish();
}

extern "C" SparCudaStatus spar_cuda_launch_adamw(void* parameter, const void* gradient,
                                                 void* first_moment, void* second_moment,
                                                 uint64_t count, int dtype, double learning_rate,
                                                 double beta1, double beta2, double epsilon,
                                                 double weight_decay, double first_correction,
                                                 double second_correction, int device) {
  if (!valid_dtype(dtype) ||
      (count != 0 && (!parameter || !gradient || !first_moment || !second_moment)))
    return invalid();
  if (count == 0) return ok();
  SPAR_SCOPE(device);
  const unsigned g = blocks_for(count, device);
  if (dtype == SPAR_CUDA_FLOAT32)
    adamw_k<float><<<g, 256>>>(tp<float>(parameter), ctp<float>(gradient), tp<float>(first_moment), tp<float>(second_moment), count, learning_rate, beta1, beta2, epsilon, weight_decay, first_correction, second_correction);
  else
    adamw_k<double><<<g, 256>>>(tp<double>(parameter), ctp<double>(gradient), tp<double>(first_moment), tp<double>(second_moment), count, learning_rate, beta1, beta2, epsilon, weight_decay, first_correction, second_correction);
  return finish();
}

extern "C" const char* spar_cuda_error_string(int cuda_error) {
  return cudaGetErrorString(static_cast<cudaError_t>(cuda_error));
}

extern "C" const char* spar_b200_version(void) { return "spar_b200 0.1 (sm_100a)"; }
