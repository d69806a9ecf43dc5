// GELU and SwiGLU forward/backward, rotary embedding, column sums and a deterministic total sum.
//
// GELU: Spar has no GELU op; the harness writes the tanh form exactly through Spar's stable
// sigmoid (src/ops/unary.cpp:137-148, branch form of cuda_kernels.cu:105-111):
//   gelu(x) = x * sigmoid(u),  u = 2*sqrt(2/pi)*(x + 0.044715 x^3)   (tanh(z) = 2 sigmoid(2z) - 1)
//   gelu'(x) = s + x * s * (1 - s) * du/dx,  du/dx = 2*sqrt(2/pi)*(1 + 3*0.044715 x^2)
// SwiGLU: nn::swiglu (src/nn/functional.cpp:9-11) h = silu(gate) * value, silu(x) = x * s(x) with
// the stable sigmoid; backward through multiply and silu's local derivative s + x s (1 - s)
// (src/ops/unary.cpp:150-160): d gate = (dh * value) * (s + gate * (s * (1 - s))),
// d value = dh * silu(gate), in that operation order.
// RoPE: interleaved pairs (2i, 2i+1) as Spar's apply_rope (src/nn/rope.cpp:35-66); the angle table
// is computed once in double and rounded to fp32 exactly as the reference does per element.
#include <initializer_list>

#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

__global__ void gelu_forward_kernel(float4* __restrict__ y, const float4* __restrict__ x,
                                    uint64_t n4) {
  pdl_begin();
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    const float4 v = ld_stream(x + i);
    st_stream(y + i, make_float4(gelu_value(v.x), gelu_value(v.y), gelu_value(v.z),
                                 gelu_value(v.w)));
  }
}

__global__ void gelu_backward_kernel(float4* __restrict__ dx, const float4* __restrict__ dy,
                                     const float4* __restrict__ x, uint64_t n4) {
  pdl_begin();
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    const float4 v = ld_stream(x + i);
    const float4 g = ld_stream(dy + i);
    st_stream(dx + i, make_float4(g.x * gelu_derivative(v.x), g.y * gelu_derivative(v.y),
                                  g.z * gelu_derivative(v.z), g.w * gelu_derivative(v.w)));
  }
}

__global__ void gelu_tail_kernel(float* y, const float* dy, const float* x, uint64_t begin,
                                 uint64_t n, int backward) {
  pdl_begin();
  const uint64_t i = begin + threadIdx.x;
  if (i >= n) return;
  y[i] = backward ? dy[i] * gelu_derivative(x[i]) : gelu_value(x[i]);
}

// The sigmoid through the hardware exponential and an approximate divide (fast_sigmoid, a few ulp
// from the accurate form): with expf and an IEEE divide the forward was SM-bound (ncu: SM 69 %,
// DRAM 59 % of peak).
__device__ __forceinline__ float silu_value(float g) { return g * fast_sigmoid(g); }

__device__ __forceinline__ void swiglu_grads(float d, float g, float v, float& dg, float& dv) {
  const float sg = fast_sigmoid(g);
  dg = (d * v) * (sg + g * (sg * (1.f - sg)));
  dv = d * (g * sg);
}

// Row-strided SwiGLU over rows x cols. Vector path: every leading dimension and pointer allows
// float4 access (cols % 4 == 0). No per-element index division: the forward gives block (x, y)
// 256 consecutive float4 (or float) columns of rows y, y + gridDim.y, ... with four rows' loads in
// flight per thread; the backward (five streams) cuts the rows into 256-column segments that
// blocks take in grid-stride order, so consecutive blocks stream consecutive memory (each layout
// measured the faster for its kernel).
template <bool kVec>
__global__ void swiglu_forward_kernel(float* __restrict__ h, uint64_t ldh,
                                      const float* __restrict__ gate, uint64_t ldg,
                                      const float* __restrict__ value, uint64_t ldv, uint64_t rows,
                                      uint64_t cols) {
  pdl_begin();
  const uint64_t per_row = kVec ? cols / 4 : cols;
  const uint64_t c = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= per_row) return;
#pragma unroll 4
  for (uint64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    if constexpr (kVec) {
      const float4 g = ld_stream(reinterpret_cast<const float4*>(gate + r * ldg) + c);
      const float4 v = ld_stream(reinterpret_cast<const float4*>(value + r * ldv) + c);
      reinterpret_cast<float4*>(h + r * ldh)[c] =
          make_float4(silu_value(g.x) * v.x, silu_value(g.y) * v.y, silu_value(g.z) * v.z,
                      silu_value(g.w) * v.w);
    } else {
      h[r * ldh + c] = silu_value(gate[r * ldg + c]) * value[r * ldv + c];
    }
  }
}

template <bool kVec>
__global__ void swiglu_backward_kernel(float* __restrict__ dgate, uint64_t lddg,
                                       float* __restrict__ dvalue, uint64_t lddv,
                                       const float* __restrict__ dh, uint64_t lddh,
                                       const float* __restrict__ gate, uint64_t ldg,
                                       const float* __restrict__ value, uint64_t ldv,
                                       uint64_t rows, uint64_t cols) {
  pdl_begin();
  const uint64_t per_row = kVec ? cols / 4 : cols;
  const uint64_t segs_per_row = (per_row + 255) / 256, segs = rows * segs_per_row;
  for (uint64_t seg = blockIdx.x; seg < segs; seg += gridDim.x) {
    const uint64_t r = seg / segs_per_row;
    const uint64_t c = (seg - r * segs_per_row) * 256 + threadIdx.x;
    if (c >= per_row) continue;
    if constexpr (kVec) {
      const float4 d = ld_stream(reinterpret_cast<const float4*>(dh + r * lddh) + c);
      const float4 g = ld_stream(reinterpret_cast<const float4*>(gate + r * ldg) + c);
      const float4 v = ld_stream(reinterpret_cast<const float4*>(value + r * ldv) + c);
      float4 a, b;
      swiglu_grads(d.x, g.x, v.x, a.x, b.x);
      swiglu_grads(d.y, g.y, v.y, a.y, b.y);
      swiglu_grads(d.z, g.z, v.z, a.z, b.z);
      swiglu_grads(d.w, g.w, v.w, a.w, b.w);
      reinterpret_cast<float4*>(dgate + r * lddg)[c] = a;
      reinterpret_cast<float4*>(dvalue + r * lddv)[c] = b;
    } else {
      float a, b;
      swiglu_grads(dh[r * lddh + c], gate[r * ldg + c], value[r * ldv + c], a, b);
      dgate[r * lddg + c] = a;
      dvalue[r * lddv + c] = b;
    }
  }
}

// One thread per (position, pair): cos/sin of pos * theta^(-2i/D), computed in double.
__global__ void rope_table_kernel(float2* table, uint64_t t, uint64_t half, uint64_t d,
                                  double theta, uint64_t start) {
  pdl_begin();
  const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= t * half) return;
  const uint64_t pos = idx / half, pair = idx % half;
  const double position = static_cast<double>(start + pos);
  const double exponent = -2.0 * static_cast<double>(pair) / static_cast<double>(d);
  const double angle = position * pow(theta, exponent);
  table[idx] = make_float2(static_cast<float>(cos(angle)), static_cast<float>(sin(angle)));
}

// x: rows of `heads * d` features per token (row stride ld); rotates each head's pairs.
__global__ void rope_apply_kernel(float* __restrict__ x, const float2* __restrict__ table,
                                  uint64_t tokens, uint64_t t, uint64_t heads, uint64_t half,
                                  uint64_t ld, int inverse, int round) {
  pdl_begin();
  const uint64_t pairs_per_token = heads * half;
  const uint64_t total = tokens * pairs_per_token;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += stride) {
    const uint64_t token = idx / pairs_per_token;
    const uint64_t within = idx % pairs_per_token;  // head * half + pair
    const uint64_t pair = within % half;
    const float2 cs = table[(token % t) * half + pair];
    const float sine = inverse ? -cs.y : cs.y;
    float2* p = reinterpret_cast<float2*>(x + token * ld) + within;
    const float2 v = *p;
    float2 o = make_float2(v.x * cs.x - v.y * sine, v.x * sine + v.y * cs.x);
    if (round) o = make_float2(round_tf32(o.x), round_tf32(o.y));
    *p = o;
  }
}

// Column sums, stage 1: block (cx, ry) sums columns [cx*128, cx*128+128) over its row range.
constexpr int kColWarps = 8;
__global__ void __launch_bounds__(kColWarps * 32)
column_sum_partial_kernel(float* __restrict__ partial, const float* __restrict__ x, uint64_t rows,
                          uint64_t cols, uint64_t ld, uint64_t rows_per_part) {
  pdl_begin();
  __shared__ float4 red[kColWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t col4 = static_cast<uint64_t>(blockIdx.x) * 32 + lane;  // float4 column index
  const uint64_t r0 = static_cast<uint64_t>(blockIdx.y) * rows_per_part;
  uint64_t r1 = r0 + rows_per_part;
  if (r1 > rows) r1 = rows;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col4 * 4 < cols) {
    for (uint64_t r = r0 + warp; r < r1; r += kColWarps) {
      const float4 v = reinterpret_cast<const float4*>(x + r * ld)[col4];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && col4 * 4 < cols) {
    float4 s = red[0][lane];
    for (int w = 1; w < kColWarps; ++w) {
      s.x += red[w][lane].x;
      s.y += red[w][lane].y;
      s.z += red[w][lane].z;
      s.w += red[w][lane].w;
    }
    reinterpret_cast<float4*>(partial + static_cast<uint64_t>(blockIdx.y) * cols)[col4] = s;
  }
}

__global__ void column_sum_final_kernel(float* __restrict__ out, const float* __restrict__ partial,
                                        int parts, uint64_t cols, int accumulate) {
  pdl_begin();
  const uint64_t c = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[static_cast<uint64_t>(p) * cols + c];
  out[c] = accumulate ? out[c] + s : s;
}

__global__ void sum_kernel(float* out, const float* __restrict__ v, uint64_t n) {
  pdl_begin();
  __shared__ double red[32];
  double s = 0.0;
  for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) s += static_cast<double>(v[i]);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    t = warp_sum(t);
    if (threadIdx.x == 0) *out = static_cast<float>(t);
  }
}

}  // namespace

cudaError_t gelu_launch(float* y, const float* dy, const float* x, uint64_t n, int backward,
                        int device, cudaStream_t stream) {
  const uint64_t n4 = n / 4;
  if (n4 > 0) {
    const unsigned grid = grid_for(n4, 256, sm_count(device) * 16);
    if (backward)
      launch(gelu_backward_kernel, dim3(grid), dim3(256), 0, stream, reinterpret_cast<float4*>(y),
                                                     reinterpret_cast<const float4*>(dy),
                                                     reinterpret_cast<const float4*>(x), n4);
    else
      launch(gelu_forward_kernel, dim3(grid), dim3(256), 0, stream, reinterpret_cast<float4*>(y),
                                                    reinterpret_cast<const float4*>(x), n4);
  }
  if (n % 4) launch(gelu_tail_kernel, dim3(1), dim3(32), 0, stream, y, dy, x, n4 * 4, n, backward);
  return cudaGetLastError();
}

cudaError_t rope_table_launch(float* table, uint64_t t, uint64_t d, double theta, uint64_t start,
                              cudaStream_t stream) {
  const uint64_t half = d / 2, n = t * half;
  launch(rope_table_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream, 
      reinterpret_cast<float2*>(table), t, half, d, theta, start);
  return cudaGetLastError();
}

cudaError_t rope_apply_launch(float* x, const float* table, uint64_t tokens, uint64_t t,
                              uint64_t heads, uint64_t d, uint64_t ld, int inverse, int device,
                              cudaStream_t stream, int round) {
  const uint64_t half = d / 2;
  const unsigned grid = grid_for(tokens * heads * half, 256, sm_count(device) * 16);
  launch(rope_apply_kernel, dim3(grid), dim3(256), 0, stream, x, reinterpret_cast<const float2*>(table), tokens,
                                              t, heads, half, ld, inverse, round);
  return cudaGetLastError();
}

int column_sum_parts(uint64_t rows, uint64_t cols, int device) {
  const uint64_t col_blocks = (cols + 127) / 128;
  uint64_t parts = (static_cast<uint64_t>(sm_count(device)) * 4 + col_blocks - 1) / col_blocks;
  const uint64_t max_parts = (rows + kColWarps * 4 - 1) / (kColWarps * 4);
  if (parts > max_parts) parts = max_parts;
  if (parts < 1) parts = 1;
  return static_cast<int>(parts);
}

cudaError_t column_sum_launch(float* out, const float* x, uint64_t rows, uint64_t cols,
                              uint64_t ld, int accumulate, float* workspace, int device,
                              cudaStream_t stream) {
  const int parts = column_sum_parts(rows, cols, device);
  const uint64_t rows_per_part = (rows + parts - 1) / parts;
  dim3 grid(static_cast<unsigned>((cols + 127) / 128), static_cast<unsigned>(parts));
  launch(column_sum_partial_kernel, dim3(grid), dim3(kColWarps * 32), 0, stream, workspace, x, rows, cols, ld,
                                                                 rows_per_part);
  launch(column_sum_final_kernel, dim3(static_cast<unsigned>((cols + 255) / 256)), dim3(256), 0, stream, 
      out, workspace, parts, cols, accumulate);
  return cudaGetLastError();
}

cudaError_t sum_launch(float* out, const float* v, uint64_t n, cudaStream_t stream) {
  launch(sum_kernel, dim3(1), dim3(1024), 0, stream, out, v, n);
  return cudaGetLastError();
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_gelu_forward(float* y, const float* x, uint64_t count,
                                                 int device, void* stream) {
  if (count == 0) return ok();
  if (!y || !x) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = gelu_launch(y, nullptr, x, count, 0, device, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_gelu_backward(float* dx, const float* dy, const float* x,
                                                  uint64_t count, int device, void* stream) {
  if (count == 0) return ok();
  if (!dx || !dy || !x) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = gelu_launch(dx, dy, x, count, 1, device, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}

namespace spar_b200 {
namespace {
// float4 access is possible when cols and every leading dimension are multiples of 4 and every
// pointer is 16-byte aligned.
bool swiglu_vec(uint64_t cols, std::initializer_list<uint64_t> lds,
                std::initializer_list<const void*> ptrs) {
  if (cols % 4) return false;
  for (uint64_t ld : lds)
    if (ld % 4) return false;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return false;
  return true;
}

// Forward: 256-wide column blocks x enough row slots for about eight blocks per SM.
dim3 swiglu_forward_grid(uint64_t rows, uint64_t per_row, int device) {
  const uint64_t gx = (per_row + 255) / 256;
  uint64_t gy = (static_cast<uint64_t>(sm_count(device)) * 8 + gx - 1) / gx;
  if (gy > rows) gy = rows;
  if (gy > 65535) gy = 65535;
  if (gy < 1) gy = 1;
  return dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
}

// Backward: one 256-thread block per 256-column segment, at most eight blocks per SM.
dim3 swiglu_backward_grid(uint64_t rows, uint64_t per_row, int device) {
  return dim3(grid_for(rows * ((per_row + 255) / 256), 1, sm_count(device) * 8));
}
}  // namespace

cudaError_t swiglu_forward_launch(float* h, uint64_t ldh, const float* gate, uint64_t ldg,
                                  const float* value, uint64_t ldv, uint64_t rows, uint64_t cols,
                                  int device, cudaStream_t s) {
  const bool vec = swiglu_vec(cols, {ldh, ldg, ldv}, {h, gate, value});
  const dim3 grid = swiglu_forward_grid(rows, vec ? cols / 4 : cols, device);
  if (vec) return launch(swiglu_forward_kernel<true>, grid, dim3(256), 0, s, h, ldh, gate, ldg, value, ldv, rows, cols);
  return launch(swiglu_forward_kernel<false>, grid, dim3(256), 0, s, h, ldh, gate, ldg, value, ldv, rows, cols);
}

cudaError_t swiglu_backward_launch(float* dgate, uint64_t lddg, float* dvalue, uint64_t lddv,
                                   const float* dh, uint64_t lddh, const float* gate, uint64_t ldg,
                                   const float* value, uint64_t ldv, uint64_t rows, uint64_t cols,
                                   int device, cudaStream_t s) {
  const bool vec = swiglu_vec(cols, {lddg, lddv, lddh, ldg, ldv}, {dgate, dvalue, dh, gate, value});
  const dim3 grid = swiglu_backward_grid(rows, vec ? cols / 4 : cols, device);
  if (vec)
    return launch(swiglu_backward_kernel<true>, grid, dim3(256), 0, s, dgate, lddg, dvalue, lddv,
                  dh, lddh, gate, ldg, value, ldv, rows, cols);
  return launch(swiglu_backward_kernel<false>, grid, dim3(256), 0, s, dgate, lddg, dvalue, lddv,
                dh, lddh, gate, ldg, value, ldv, rows, cols);
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_swiglu_forward(float* h, uint64_t ldh, const float* gate,
                                                   uint64_t ldg, const float* value, uint64_t ldv,
                                                   uint64_t rows, uint64_t cols, int device,
                                                   void* stream) {
  if (rows == 0 || cols == 0) return ok();
  if (!h || !gate || !value || ldh < cols || ldg < cols || ldv < cols) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = swiglu_forward_launch(h, ldh, gate, ldg, value, ldv, rows, cols, device,
                                              static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_swiglu_backward(float* dgate, uint64_t lddg, float* dvalue,
                                                    uint64_t lddv, const float* dh, uint64_t lddh,
                                                    const float* gate, uint64_t ldg,
                                                    const float* value, uint64_t ldv,
                                                    uint64_t rows, uint64_t cols, int device,
                                                    void* stream) {
  if (rows == 0 || cols == 0) return ok();
  if (!dgate || !dvalue || !dh || !gate || !value || lddg < cols || lddv < cols || lddh < cols ||
      ldg < cols || ldv < cols)
    return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = swiglu_backward_launch(dgate, lddg, dvalue, lddv, dh, lddh, gate, ldg,
                                               value, ldv, rows, cols, device,
                                               static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_rope_table(float* table, uint64_t t, uint64_t d,
                                               double theta, uint64_t start_position, int device,
                                               void* stream) {
  if (t == 0) return ok();
  if (!table || d == 0 || d % 2 != 0 || !(theta > 0.0)) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = rope_table_launch(table, t, d, theta, start_position, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_rope_apply(float* x, const float* table, uint64_t batch,
                                               uint64_t t, uint64_t heads, uint64_t d, uint64_t ld,
                                               int inverse, int device, void* stream) {
  if (batch == 0 || t == 0 || heads == 0) return ok();
  if (!x || !table || d == 0 || d % 2 != 0 || ld < heads * d || ld % 2 != 0) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = rope_apply_launch(x, table, batch * t, t, heads, d, ld, inverse, device,
                                          (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_column_sum(float* out, const float* x, uint64_t rows,
                                               uint64_t cols, uint64_t ld, int accumulate,
                                               int device, void* stream) {
  if (cols == 0) return ok();
  if (!out || cols % 4 != 0 || ld % 4 != 0 || ld < cols || (rows != 0 && !x)) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = (cudaStream_t)stream;
  if (rows == 0) {
    if (accumulate) return ok();
    const cudaError_t e = cudaMemsetAsync(out, 0, cols * sizeof(float), s);
    return e == cudaSuccess ? ok() : runtime(e);
  }
  const int parts = column_sum_parts(rows, cols, device);
  float* ws = nullptr;
  cudaError_t e = stream_alloc(reinterpret_cast<void**>(&ws), parts * cols * sizeof(float), s);
  if (e != cudaSuccess) return runtime(e);
  e = column_sum_launch(out, x, rows, cols, ld, accumulate, ws, device, s);
  const cudaError_t f = cudaFreeAsync(ws, s);
  if (e != cudaSuccess) return runtime(e);
  return f == cudaSuccess ? ok() : runtime(f);
}

extern "C" SparCudaStatus spar_b200_sum(float* out, const float* values, uint64_t count,
                                        int device, void* stream) {
  if (!out || (count != 0 && !values)) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = sum_launch(out, values, count, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : runtime(e);
}
