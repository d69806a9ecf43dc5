// qk-norm + RoPE of the Spar-family projection in one pass per token, and its backward.
//
// nn::SelfAttention with qk_norm (src/nn/attention.cpp:183-186, 208-215) normalises every query
// and key head with RMSNorm(head_dim) (src/nn/rmsnorm.cpp:50-52: x / sqrt(mean(x^2) + eps) * w)
// and then applies RoPE (src/nn/rope.cpp:35-66: interleaved pairs (2i, 2i + 1) rotated by
// pos * theta^(-2i / head_dim)). Forward here: one warp per token reads the raw projection row
// [q heads | k heads | v heads] once, normalises each q / k head (a head is DH / 4 consecutive
// lanes' float4, reduced with shuffles inside that lane group), rotates its pairs, rounds q, k, v
// to nearest TF32 (they only feed the attention's tensor-core products) and writes the row once;
// 1 / rms per (token, head) is kept for the backward. Backward (the attention has already rotated
// dq, dk back): dx = rstd * (g - xhat * mean(g * xhat)), g = dy * w, xhat = x * rstd, in place
// over dq | dk; the weight gradients sum dy * xhat over all tokens and heads: each lane keeps the
// running sums of its float4 of the head (the same head offset for every head it visits), the
// block reduces them into one partial row, and a second kernel adds the rows in a fixed order.
#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {
namespace {

constexpr int kWarps = 8;

template <int DH>
__global__ void __launch_bounds__(kWarps * 32)
qk_norm_rope_kernel(float* __restrict__ out, const float* __restrict__ raw, uint64_t tokens,
                    uint32_t seq, uint32_t heads, uint32_t kv_heads, uint64_t ld,
                    const float* __restrict__ wq, const float* __restrict__ wk,
                    float* __restrict__ rstd, const float2* __restrict__ rope, float eps,
                    int round_out) {
  pdl_begin();
  constexpr uint32_t kLanes = DH / 4;  // lanes per head
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t c = lane % kLanes;  // this lane's float4 of every head it visits
  const uint32_t qk_heads = heads + kv_heads, all_heads = heads + 2 * kv_heads;
  const uint32_t chunks = all_heads * kLanes;
  const float4 gq = __ldg(reinterpret_cast<const float4*>(wq) + c);
  const float4 gk = __ldg(reinterpret_cast<const float4*>(wk) + c);
  const uint64_t warp_stride = static_cast<uint64_t>(gridDim.x) * kWarps;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < tokens;
       t += warp_stride) {
    const float4* src = reinterpret_cast<const float4*>(raw + t * ld);
    float4* dst = reinterpret_cast<float4*>(out + t * ld);
    const uint32_t pos = static_cast<uint32_t>(t % seq);
    for (uint32_t j = lane; j < (chunks + 31) / 32 * 32; j += 32) {
      const bool active = j < chunks;
      const uint32_t h = j / kLanes;
      const float4 v = active ? ld_stream(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      float ss = (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
#pragma unroll
      for (uint32_t o = kLanes / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (!active) continue;
      if (h >= qk_heads) {  // value head: copy (rounded to nearest TF32 in TF32 mode)
        dst[j] = round_out ? make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z),
                                         round_tf32(v.w))
                           : v;
        continue;
      }
      const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(DH)) + eps);
      const bool is_q = h < heads;
      const float4 g = is_q ? gq : gk;
      float4 y = make_float4(v.x * r * g.x, v.y * r * g.y, v.z * r * g.z, v.w * r * g.w);
      if (rope) {
        const float2 c0 = __ldg(rope + static_cast<uint64_t>(pos) * (DH / 2) + 2 * c);
        const float2 c1 = __ldg(rope + static_cast<uint64_t>(pos) * (DH / 2) + 2 * c + 1);
        y = make_float4(y.x * c0.x - y.y * c0.y, y.x * c0.y + y.y * c0.x, y.z * c1.x - y.w * c1.y,
                        y.z * c1.y + y.w * c1.x);
      }
      dst[j] = round_out ? make_float4(round_tf32(y.x), round_tf32(y.y), round_tf32(y.z),
                                       round_tf32(y.w))
                         : y;
      if (c == 0)
        rstd[is_q ? t * heads + h : tokens * heads + t * kv_heads + (h - heads)] = r;
    }
  }
}

template <int DH>
__global__ void __launch_bounds__(kWarps * 32)
qk_norm_backward_kernel(float* __restrict__ dqk, const float* __restrict__ raw, uint64_t tokens,
                        uint32_t heads, uint32_t kv_heads, uint64_t ld,
                        const float* __restrict__ wq, const float* __restrict__ wk,
                        const float* __restrict__ rstd, float* __restrict__ partial) {
  pdl_begin();
  constexpr uint32_t kLanes = DH / 4;
  __shared__ float4 red[kWarps][32][2];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t c = lane % kLanes;
  const uint32_t chunks = (heads + kv_heads) * kLanes;
  const float4 gq = __ldg(reinterpret_cast<const float4*>(wq) + c);
  const float4 gk = __ldg(reinterpret_cast<const float4*>(wk) + c);
  float4 aq = make_float4(0.f, 0.f, 0.f, 0.f), ak = aq;
  const uint64_t warp_stride = static_cast<uint64_t>(gridDim.x) * kWarps;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * kWarps + warp; t < tokens; t += warp_stride) {
    float4* dyr = reinterpret_cast<float4*>(dqk + t * ld);
    const float4* xr = reinterpret_cast<const float4*>(raw + t * ld);
    for (uint32_t j = lane; j < (chunks + 31) / 32 * 32; j += 32) {
      const bool active = j < chunks;
      const uint32_t h = j / kLanes;
      const bool is_q = h < heads;
      float4 d = make_float4(0.f, 0.f, 0.f, 0.f), x = d;
      float r = 0.f;
      if (active) {
        d = dyr[j];
        x = ld_stream(xr + j);
        r = __ldg(rstd + (is_q ? t * heads + h : tokens * heads + t * kv_heads + (h - heads)));
      }
      const float4 g = is_q ? gq : gk;
      const float4 xh = make_float4(x.x * r, x.y * r, x.z * r, x.w * r);
      const float4 gy = make_float4(d.x * g.x, d.y * g.y, d.z * g.z, d.w * g.w);
      float s = (gy.x * xh.x + gy.y * xh.y) + (gy.z * xh.z + gy.w * xh.w);
#pragma unroll
      for (uint32_t o = kLanes / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (!active) continue;
      const float m = s * (1.0f / static_cast<float>(DH));
      dyr[j] = make_float4(r * (gy.x - xh.x * m), r * (gy.y - xh.y * m), r * (gy.z - xh.z * m),
                           r * (gy.w - xh.w * m));
      float4& a = is_q ? aq : ak;
      a.x += d.x * xh.x;
      a.y += d.y * xh.y;
      a.z += d.z * xh.z;
      a.w += d.w * xh.w;
    }
  }
  // Block partial of the two weight gradients: lanes with the same head offset c, warp by warp,
  // in a fixed order.
  red[warp][lane][0] = aq;
  red[warp][lane][1] = ak;
  __syncthreads();
  if (threadIdx.x < 2 * kLanes) {
    const uint32_t which = threadIdx.x / kLanes, cc = threadIdx.x % kLanes;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < kWarps; ++w)
      for (uint32_t l = cc; l < 32; l += kLanes) {
        const float4 v = red[w][l][which];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
    reinterpret_cast<float4*>(partial + static_cast<uint64_t>(blockIdx.x) * 2 * DH)[which * kLanes + cc] = s;
  }
}

// out[i] (+)= sum over parts of partial[p][i], parts in order (deterministic); i < 2 * DH:
// the first DH values go to dwq, the rest to dwk.
__global__ void qk_weight_sum_kernel(float* __restrict__ dwq, float* __restrict__ dwk,
                                     const float* __restrict__ partial, int parts, int dh,
                                     int accumulate) {
  pdl_begin();
  const int i = threadIdx.x;
  if (i >= 2 * dh) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[static_cast<uint64_t>(p) * 2 * dh + i];
  float* out = i < dh ? dwq + i : dwk + (i - dh);
  *out = accumulate ? *out + s : s;
}

}  // namespace

int qk_norm_backward_parts(uint64_t tokens, int device) {
  uint64_t g = (tokens + kWarps - 1) / kWarps;
  const uint64_t cap = static_cast<uint64_t>(sm_count(device)) * 2;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

cudaError_t qk_norm_rope_launch(float* out, const float* raw, uint64_t tokens, uint64_t seq,
                                uint64_t heads, uint64_t kv_heads, uint64_t head_dim, uint64_t ld,
                                const float* wq, const float* wk, float* rstd,
                                const float* rope_table, float eps, int device,
                                cudaStream_t stream, bool round_out) {
  const unsigned grid = grid_for(tokens, kWarps, sm_count(device) * 8);
  const float2* rope = reinterpret_cast<const float2*>(rope_table);
  const uint32_t s = static_cast<uint32_t>(seq), h = static_cast<uint32_t>(heads),
                 kv = static_cast<uint32_t>(kv_heads);
  if (head_dim == 64)
    return launch(qk_norm_rope_kernel<64>, dim3(grid), dim3(kWarps * 32), 0, stream, out, raw,
                  tokens, s, h, kv, ld, wq, wk, rstd, rope, eps, round_out ? 1 : 0);
  if (head_dim == 32)
    return launch(qk_norm_rope_kernel<32>, dim3(grid), dim3(kWarps * 32), 0, stream, out, raw,
                  tokens, s, h, kv, ld, wq, wk, rstd, rope, eps, round_out ? 1 : 0);
  return cudaErrorInvalidValue;
}

cudaError_t qk_norm_backward_launch(float* dqk, const float* raw, uint64_t tokens, uint64_t heads,
                                    uint64_t kv_heads, uint64_t head_dim, uint64_t ld,
                                    const float* wq, const float* wk, const float* rstd,
                                    float* dwq, float* dwk, int accumulate, float* workspace,
                                    int device, cudaStream_t stream) {
  const int parts = qk_norm_backward_parts(tokens, device);
  const uint32_t h = static_cast<uint32_t>(heads), kv = static_cast<uint32_t>(kv_heads);
  cudaError_t e;
  if (head_dim == 64)
    e = launch(qk_norm_backward_kernel<64>, dim3(parts), dim3(kWarps * 32), 0, stream, dqk, raw,
               tokens, h, kv, ld, wq, wk, rstd, workspace);
  else if (head_dim == 32)
    e = launch(qk_norm_backward_kernel<32>, dim3(parts), dim3(kWarps * 32), 0, stream, dqk, raw,
               tokens, h, kv, ld, wq, wk, rstd, workspace);
  else
    return cudaErrorInvalidValue;
  if (e != cudaSuccess) return e;
  return launch(qk_weight_sum_kernel, dim3(1), dim3(128), 0, stream, dwq, dwk,
                static_cast<const float*>(workspace), parts, static_cast<int>(head_dim),
                accumulate);
}

// Grouped-query attention on the unfused (3xTF32) path, as Spar's repeat_kv_heads
// (src/nn/attention.cpp:77-94) and its backward: k | v of kv_heads heads, read from the packed
// projection [tokens, ld] at column kcol, expanded to `heads` heads ([tokens, 2 * heads * dh],
// query head h reading key / value head h / group); and the reverse, each key / value head's
// gradient the sum of its group's heads in head order (deterministic).
__global__ void repeat_kv_kernel(float* __restrict__ out, const float* __restrict__ qkv,
                                 uint64_t tokens, uint32_t heads, uint32_t kv_heads, uint32_t dh,
                                 uint64_t ld, uint64_t kcol) {
  pdl_begin();
  const uint32_t group = heads / kv_heads;
  const uint64_t d = static_cast<uint64_t>(heads) * dh, per_token = 2 * d;
  const uint64_t n = tokens * per_token;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t t = i / per_token, c = i % per_token;
    const uint64_t part = c / d, h = (c % d) / dh, e = c % dh;  // part 0 = k, 1 = v
    out[i] = qkv[t * ld + kcol + part * kv_heads * dh + (h / group) * dh + e];
  }
}

__global__ void group_sum_kernel(float* __restrict__ dqkv, const float* __restrict__ drep,
                                 uint64_t tokens, uint32_t heads, uint32_t kv_heads, uint32_t dh,
                                 uint64_t ld, uint64_t kcol) {
  pdl_begin();
  const uint32_t group = heads / kv_heads;
  const uint64_t d = static_cast<uint64_t>(heads) * dh, kvd = static_cast<uint64_t>(kv_heads) * dh;
  const uint64_t n = tokens * 2 * kvd;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t t = i / (2 * kvd), c = i % (2 * kvd);
    const uint64_t part = c / kvd, kh = (c % kvd) / dh, e = c % dh;
    const float* src = drep + t * 2 * d + part * d + kh * group * dh + e;
    float acc = 0.f;
    for (uint32_t g = 0; g < group; ++g) acc += src[static_cast<uint64_t>(g) * dh];
    dqkv[t * ld + kcol + c] = acc;
  }
}

cudaError_t repeat_kv_launch(float* out, const float* qkv, uint64_t tokens, uint64_t heads,
                             uint64_t kv_heads, uint64_t dh, uint64_t ld, uint64_t kcol,
                             int device, cudaStream_t stream) {
  const uint64_t n = tokens * 2 * heads * dh;
  return launch(repeat_kv_kernel, dim3(grid_for(n, 256, sm_count(device) * 16)), dim3(256), 0,
                stream, out, qkv, tokens, static_cast<uint32_t>(heads),
                static_cast<uint32_t>(kv_heads), static_cast<uint32_t>(dh), ld, kcol);
}

cudaError_t group_sum_launch(float* dqkv, const float* drep, uint64_t tokens, uint64_t heads,
                             uint64_t kv_heads, uint64_t dh, uint64_t ld, uint64_t kcol,
                             int device, cudaStream_t stream) {
  const uint64_t n = tokens * 2 * kv_heads * dh;
  return launch(group_sum_kernel, dim3(grid_for(n, 256, sm_count(device) * 16)), dim3(256), 0,
                stream, dqkv, drep, tokens, static_cast<uint32_t>(heads),
                static_cast<uint32_t>(kv_heads), static_cast<uint32_t>(dh), ld, kcol);
}

}  // namespace spar_b200
