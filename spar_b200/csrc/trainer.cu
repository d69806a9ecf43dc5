// Training-step runtime for the pre-LN decoder: parameter/gradient/moment arena, saved
// activations, forward, hand-scheduled backward, gradient accumulation, data-parallel
// all-reduce hooks and the fused clip + AdamW update, all enqueued on one CUDA stream.
//
// Model (Spar modules composed as in src/nn/decoder.cpp:73-90 and
// src/nn/transformer.cpp:53-69, with Spar's RMSNorm/SwiGLU swapped for LayerNorm/GELU):
//   h0 = E[ids]                                        Embedding (src/nn/embedding.cpp:40-42)
//   per block:  a = LN1(x); q,k,v = a W{q,k,v} + b     Linear, weight [in, out] (linear.cpp:48-63)
//               q,k = rope(q,k)                        apply_rope (src/nn/rope.cpp:70-92)
//               P = causal_softmax(q k^T / sqrt(dh))   scaled_dot_product_attention
//               h1 = x + (P v) Wo + bo                   (src/nn/attention.cpp:122-135, 188-225)
//               x' = h1 + gelu(LN2(h1) W1 + b1) W2 + b2
//   logits = LN_f(h_L) E^T (tied, decoder.cpp:88-89); loss = LM cross-entropy
//   (src/loss/cross_entropy.cpp:176-214)
// Backward is the reverse-mode sweep Spar's tape performs (src/autograd/autograd.cpp:201-265),
// written out per layer so every GEMM reads its operands in place (no transposed copies), the
// GELU derivative and residual adds ride in GEMM epilogues, and leaf gradients accumulate on the
// device across micro-steps. Q/K/V weights live fused as one [d, 3d] matrix (columns q | k | v);
// the named-parameter view below splits them back into Spar's q_proj/k_proj/v_proj tensors.
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <string>
#include <vector>

#include "checkpoint.h"
#include "common.cuh"
#include "kernels.cuh"

namespace spar_b200 {

cudaError_t gemm_launch(const SparB200Gemm& g, float* split_workspace, int device,
                        cudaStream_t stream, float* splitk_workspace, uint64_t splitk_floats,
                        uint32_t min_parts = 1);
uint64_t gemm_split_workspace_floats(const SparB200Gemm& g);
uint64_t gemm_splitk_workspace_floats(const SparB200Gemm& g, int device);
cudaError_t comm_allreduce_sum(void* comm, float* data, uint64_t count, cudaStream_t stream);
cudaError_t comm_allreduce_sum_f64(void* comm, double* data, uint64_t count, cudaStream_t stream);
cudaError_t comm_reduce_scatter_sum(void* comm, float* data, uint64_t shard, cudaStream_t stream);
cudaError_t comm_all_gather(void* comm, float* data, uint64_t shard, cudaStream_t stream);
int comm_rank(void* comm);
int comm_size(void* comm);
SparCudaStatus comm_wait(void* comm, cudaStream_t stream);

namespace {

constexpr uint64_t kAlign = 64;  // floats (256 bytes)
uint64_t align_up(uint64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// SplitMix64 draw `counter` (0-based) of a Spar Random seeded with `seed`
// (src/core/random.cpp:22-28: state += golden; mix).
__device__ __forceinline__ uint64_t splitmix_draw(uint64_t seed, uint64_t counter) {
  uint64_t z = seed + (counter + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// N(0, std) by Box-Muller on two uniform_double draws (random.cpp:35-38), element i of a
// [rows, cols] tensor taking draws first + 2i and first + 2i + 1; written at dst[r*ld + c].
__global__ void init_normal_kernel(float* dst, uint64_t rows, uint64_t cols, uint64_t ld,
                                   uint64_t seed, uint64_t first, double std) {
  const uint64_t n = rows * cols;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const double u1 = static_cast<double>(splitmix_draw(seed, first + 2 * i) >> 11) / 9007199254740992.0;
    const double u2 = static_cast<double>(splitmix_draw(seed, first + 2 * i + 1) >> 11) / 9007199254740992.0;
    const double z = sqrt(-2.0 * log1p(-u1)) * cos(2.0 * 3.141592653589793 * u2);
    dst[(i / cols) * ld + i % cols] = static_cast<float>(z * std);
  }
}

// a += b (+ c (+ d)), n float4, summed in that order: the other lanes' gradients into lane 0's.
__global__ void add_lanes_kernel(float4* __restrict__ a, const float4* __restrict__ b,
                                 const float4* __restrict__ c, const float4* __restrict__ d,
                                 uint64_t n) {
  pdl_begin();
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float4 x = a[i];
    const float4* src[3] = {b, c, d};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      if (!src[k]) break;
      const float4 y = src[k][i];
      x.x += y.x;
      x.y += y.y;
      x.z += y.z;
      x.w += y.w;
    }
    a[i] = x;
  }
}

__global__ void fill_kernel(float* dst, uint64_t n, float v) {
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = v;
}

struct NamedTensor {
  std::string name;
  uint64_t offset;  // into the flat arena (floats)
  uint64_t rows, cols;  // cols == 0: 1-D of length rows
  uint64_t ld;          // row stride in the arena (fused qkv: 3d)
  bool draws;           // consumes normal draws at init (weight matrices)
};

struct LayerOffsets {
  uint64_t ln1_g, ln1_b, wqkv, bqkv, wo, bo, ln2_g, ln2_b, w1, b1, w2, b2, begin, end;
  uint64_t qn, kn;  // Spar family with qk_norm: q_norm / k_norm weights [head_dim]
};

struct LayerActs {
  float *x, *mean1, *rstd1, *a1, *qkv, *ctx, *h1, *mean2, *rstd2, *a2, *u, *g;
  float* p;      // attention probabilities [B, H, T, T] (unfused path only)
  float* stats;  // fused attention softmax statistics: row max [B*H*T], 1 / row sum [B*H*T]
  // Spar family: u = [gate | up] projection [N, 2F], g = swiglu output [N, F]; with qk_norm the
  // projection before the q / k norms (qkv_raw) and their 1 / rms (qk_rstd [N * (H + KVH)]).
  float *qkv_raw, *qk_rstd;
};

}  // namespace

// Host-only layout of the parameter arena (no device work): Spar's named_parameters order, every
// tensor 256-byte aligned, fused [d, 3d] QKV. Shared by the runtime and the layout queries.
struct ParamLayout {
  uint64_t flat = 0, off_E = 0, off_lnf_g = 0, off_lnf_b = 0;
  std::vector<NamedTensor> named;
  std::vector<LayerOffsets> lay;
  // Gradient all-reduce buckets in the order the data-parallel step issues them: blocks from last
  // to first (each block's range as soon as its backward finishes), then the tied embedding and
  // the final norm. Together they tile [0, flat).
  std::vector<std::pair<uint64_t, uint64_t>> buckets() const {
    std::vector<std::pair<uint64_t, uint64_t>> b;
    for (size_t l = lay.size(); l-- > 0;) b.push_back({lay[l].begin, lay[l].end - lay[l].begin});
    b.push_back({off_E, lay[0].begin - off_E});
    b.push_back({off_lnf_g, flat - off_lnf_g});
    return b;
  }
};

// One rank's part of a gradient bucket [off, off + count) under the sharded optimiser: `world`
// pieces of `shard` floats (a multiple of 64, so every piece stays 256-byte aligned) are
// reduce-scattered, piece `rank` (at own_off) is this rank's to update, and the tail that does not
// split evenly, [rem_off, rem_off + rem_count), is all-reduced and updated on every rank.
struct BucketShard {
  uint64_t off, shard, own_off, rem_off, rem_count;
};

BucketShard shard_bucket(uint64_t off, uint64_t count, int world, int rank) {
  BucketShard b;
  b.off = off;
  b.shard = count / static_cast<uint64_t>(world) / kAlign * kAlign;
  b.own_off = off + static_cast<uint64_t>(rank) * b.shard;
  b.rem_off = off + static_cast<uint64_t>(world) * b.shard;
  b.rem_count = off + count - b.rem_off;
  return b;
}

// Spar's own decoder (family 1): nn::named_parameters order of DecoderLM (src/nn/parameters.cpp:
// 61-108): embedding; per block attention_norm, q / k / v / out projections (q_norm, k_norm),
// mlp_norm, gate / up / down projections; final_norm. q | k | v are stored as one [d, (H + 2 KVH)
// dh] matrix and gate | up as one [d, 2F] matrix (column views under Spar's names), so each
// projection is one product.
void plan_spar_family(const SparB200LMConfig& c, ParamLayout& pl, uint64_t& o,
                      const std::function<uint64_t(uint64_t)>& take) {
  const uint64_t V = c.vocab_size, d = c.model_dim, F = c.hidden_dim, L = c.num_layers,
                 H = c.num_heads, dh = d / H, KVH = c.num_kv_heads ? c.num_kv_heads : H;
  const uint64_t wq = (H + 2 * KVH) * dh;
  pl.off_E = take(V * d);
  pl.named.push_back({"token_embedding.weight", pl.off_E, V, d, d, true});
  for (uint64_t l = 0; l < L; ++l) {
    LayerOffsets lo{};
    lo.begin = o;
    lo.ln1_g = take(d);
    lo.wqkv = take(d * wq);
    lo.wo = take(d * d);
    if (c.qk_norm) {
      lo.qn = take(dh);
      lo.kn = take(dh);
    }
    lo.ln2_g = take(d);
    lo.w1 = take(d * 2 * F);
    lo.w2 = take(F * d);
    lo.end = o;
    pl.lay.push_back(lo);
    const std::string p = "blocks." + std::to_string(l) + ".";
    pl.named.push_back({p + "attention_norm.weight", lo.ln1_g, d, 0, 0, false});
    pl.named.push_back({p + "attention.q_proj.weight", lo.wqkv, d, H * dh, wq, true});
    pl.named.push_back({p + "attention.k_proj.weight", lo.wqkv + H * dh, d, KVH * dh, wq, true});
    pl.named.push_back({p + "attention.v_proj.weight", lo.wqkv + (H + KVH) * dh, d, KVH * dh, wq,
                        true});
    pl.named.push_back({p + "attention.out_proj.weight", lo.wo, d, d, d, true});
    if (c.qk_norm) {
      pl.named.push_back({p + "attention.q_norm.weight", lo.qn, dh, 0, 0, false});
      pl.named.push_back({p + "attention.k_norm.weight", lo.kn, dh, 0, 0, false});
    }
    pl.named.push_back({p + "mlp_norm.weight", lo.ln2_g, d, 0, 0, false});
    pl.named.push_back({p + "mlp.gate_proj.weight", lo.w1, d, F, 2 * F, true});
    pl.named.push_back({p + "mlp.up_proj.weight", lo.w1 + F, d, F, 2 * F, true});
    pl.named.push_back({p + "mlp.down_proj.weight", lo.w2, F, d, d, true});
  }
  pl.off_lnf_g = take(d);
  pl.off_lnf_b = pl.off_lnf_g;  // no bias: the final-norm bucket is [off_lnf_g, flat)
  pl.named.push_back({"final_norm.weight", pl.off_lnf_g, d, 0, 0, false});
}

SparCudaStatus plan_params(const SparB200LMConfig& c, ParamLayout& pl) {
  const uint64_t V = c.vocab_size, d = c.model_dim, F = c.hidden_dim, L = c.num_layers,
                 H = c.num_heads, T = c.sequence_length, B = c.micro_batch;
  if (V == 0 || d == 0 || F == 0 || L == 0 || H == 0 || T < 2 || B == 0 || d % H != 0)
    return invalid();
  const uint64_t dh = d / H;
  if (d % 32 != 0 || F % 4 != 0 || dh % 32 != 0 || T % 4 != 0) return invalid();
  if (c.precision != SPAR_B200_TF32 && c.precision != SPAR_B200_TF32X3) return invalid();
  if (c.family != SPAR_B200_FAMILY_LN_GELU && c.family != SPAR_B200_FAMILY_SPAR) return invalid();
  // ---- parameter arena in Spar's named_parameters order (src/nn/parameters.cpp:51-132)
  uint64_t o = 0;
  auto take = [&](uint64_t n) {
    const uint64_t at = o;
    o = align_up(o + n);
    return at;
  };
  if (c.family == SPAR_B200_FAMILY_SPAR) {
    // DecoderLM's checks (src/nn/decoder.cpp:17-49) and this runtime's: TF32 with the fused
    // attention (head_dim 32 or 64).
    const uint64_t kvh = c.num_kv_heads ? c.num_kv_heads : H;
    if (kvh > H || H % kvh != 0 || (dh != 32 && dh != 64) ||
        (c.qk_norm && !(c.qk_norm_epsilon > 0.0)) || F % 32 != 0)
      return invalid();
    plan_spar_family(c, pl, o, take);
    pl.flat = o;
    return ok();
  }
  pl.off_E = take(V * d);
  pl.named.push_back({"token_embedding.weight", pl.off_E, V, d, d, true});
  for (uint64_t l = 0; l < L; ++l) {
    LayerOffsets lo{};
    lo.begin = o;
    lo.ln1_g = take(d);
    lo.ln1_b = take(d);
    lo.wqkv = take(d * 3 * d);
    lo.bqkv = take(3 * d);
    lo.wo = take(d * d);
    lo.bo = take(d);
    lo.ln2_g = take(d);
    lo.ln2_b = take(d);
    lo.w1 = take(d * F);
    lo.b1 = take(F);
    lo.w2 = take(F * d);
    lo.b2 = take(d);
    lo.end = o;
    pl.lay.push_back(lo);
    const std::string p = "blocks." + std::to_string(l) + ".";
    pl.named.push_back({p + "attention_norm.weight", lo.ln1_g, d, 0, 0, false});
    pl.named.push_back({p + "attention_norm.bias", lo.ln1_b, d, 0, 0, false});
    const char* proj[3] = {"q_proj", "k_proj", "v_proj"};
    for (int j = 0; j < 3; ++j) {
      pl.named.push_back({p + "attention." + proj[j] + ".weight", lo.wqkv + j * d, d, d, 3 * d, true});
      pl.named.push_back({p + "attention." + proj[j] + ".bias", lo.bqkv + j * d, d, 0, 0, false});
    }
    pl.named.push_back({p + "attention.out_proj.weight", lo.wo, d, d, d, true});
    pl.named.push_back({p + "attention.out_proj.bias", lo.bo, d, 0, 0, false});
    pl.named.push_back({p + "mlp_norm.weight", lo.ln2_g, d, 0, 0, false});
    pl.named.push_back({p + "mlp_norm.bias", lo.ln2_b, d, 0, 0, false});
    pl.named.push_back({p + "mlp.up_proj.weight", lo.w1, d, F, F, true});
    pl.named.push_back({p + "mlp.up_proj.bias", lo.b1, F, 0, 0, false});
    pl.named.push_back({p + "mlp.down_proj.weight", lo.w2, F, d, d, true});
    pl.named.push_back({p + "mlp.down_proj.bias", lo.b2, d, 0, 0, false});
  }
  pl.off_lnf_g = take(d);
  pl.off_lnf_b = take(d);
  pl.named.push_back({"final_norm.weight", pl.off_lnf_g, d, 0, 0, false});
  pl.named.push_back({"final_norm.bias", pl.off_lnf_b, d, 0, 0, false});
  pl.flat = o;
  return ok();
}

#define SPAR_TRY_RAW(expr)              \
  do {                                  \
    const cudaError_t e_ = (expr);      \
    if (e_ != cudaSuccess) return e_;   \
  } while (0)

class LMTrainer {
 public:
  SparB200LMConfig cfg;
  int device = 0;
  uint64_t V, d, F, L, H, T, B, N, dh, Vp;
  // Model family (SPAR_B200_FAMILY_*); Spar family: KVH key/value heads, qkv rows of Wq =
  // (H + 2 KVH) dh floats, [gate | up] rows of Fu = 2F floats (LN family: KVH = H, Wq = 3d, Fu = F).
  int family = SPAR_B200_FAMILY_LN_GELU;
  uint64_t KVH = 0, Wq = 0, Fu = 0;
  bool qk_norm = false;
  uint64_t flat = 0;  // parameter floats (with alignment padding)
  std::vector<NamedTensor> named;
  std::vector<LayerOffsets> lay;
  uint64_t off_E = 0, off_lnf_g = 0, off_lnf_b = 0;
  std::vector<std::pair<uint64_t, uint64_t>> buckets;  // all-reduce buckets in issue order
  float *params = nullptr, *grads = nullptr, *m1 = nullptr, *m2 = nullptr;
  // TF32 mode: the parameters rounded to nearest TF32, which every GEMM reads as its weight
  // operand (the tensor cores would otherwise truncate the fp32 master weights: a systematic
  // shrink of every product). Kept current by AdamW (it writes both), by the sharded optimiser's
  // parameter gather, and, after host writes (wround_dirty), by a rounding pass before the step.
  float* wround = nullptr;
  bool wround_dirty = true;
  cudaError_t refresh_rounded(cudaStream_t s);
  // activations
  char* act_base = nullptr;
  std::vector<LayerActs> acts;
  float *xL = nullptr, *meanf = nullptr, *rstdf = nullptr, *hf = nullptr, *logits = nullptr;
  float *dres = nullptr, *dtmp = nullptr, *dqkv = nullptr, *dS = nullptr, *du = nullptr;
  float* dh_buf = nullptr;  // Spar family: d(swiglu output) [N, F]
  // Bias-gradient partials written by the producers of du and dqkv (per 32-row block column
  // sums, [N / 32, F] then [N / 32, 3d]), so the bias gradients never re-read du or dqkv.
  float* colpart = nullptr;
  // Spar family on the unfused (3xTF32) attention path with grouped key / value heads: k | v
  // expanded to the query heads [N, 2d] (rebuilt in the backward), and its gradient.
  float *kvrep = nullptr, *dkvrep = nullptr;
  // Fused attention (TF32 mode, head_dim 32 / 64): no [T, T] buffers; dS holds the backward's
  // D = rowsum(dO o O) [B*H*T] instead of dS.
  bool fused_attention = false;
  float *ln_ws = nullptr, *col_ws = nullptr, *split_ws = nullptr, *rope_tab = nullptr;
  float* splitk_ws = nullptr;  // split-K partial tiles of the small weight-gradient GEMMs
  float* splitk_ws2 = nullptr;  // the same for products on the weight-gradient stream
  uint64_t splitk_floats = 0;
  // Weight gradients on a second stream: in the backward, dW = X^T dY and dX = dY W^T only share
  // their input, so the dW products (and the bias column sums) run beside the dX chain and fill
  // the SMs the other product leaves idle (a 2048-row product fills under half a wave of SM pairs).
  // Forks and joins are events (captured as graph edges). TF32 mode, not while profiling.
  cudaStream_t wgrad_stream = nullptr;
  cudaEvent_t wg_fork[5] = {}, wg_join[4] = {};
  bool wgrad_enabled = !(getenv("SPAR_B200_WGRAD_STREAM") && getenv("SPAR_B200_WGRAD_STREAM")[0] == '0');
  // Several micro-steps in flight at small micro-batches ("lanes"): each lane owns a full set of
  // activation and workspace buffers, its streams and a gradient arena. Micro-step m runs on lane
  // m % lanes beside the others, so narrow micro-steps fill the SMs like one wider one; the other
  // lanes' gradients are added into lane 0's in lane order (per all-reduce bucket ahead of the
  // data-parallel reduction, or once after the last micro-step), so steps stay deterministic.
  // The working members above (acts, dres, ..., grads, wgrad_stream) are the selected lane's.
  struct Lane {
    std::vector<LayerActs> acts;
    float *xL = nullptr, *meanf = nullptr, *rstdf = nullptr, *hf = nullptr, *logits = nullptr;
    float *dres = nullptr, *dtmp = nullptr, *dqkv = nullptr, *dS = nullptr, *du = nullptr;
    float* dh_buf = nullptr;
    float* colpart = nullptr;
    float *kvrep = nullptr, *dkvrep = nullptr;
    float *ln_ws = nullptr, *col_ws = nullptr, *splitk_ws = nullptr, *splitk_ws2 = nullptr;
    float *row_loss = nullptr, *grads = nullptr;
    void* emb_scratch = nullptr;
    cudaStream_t stream = nullptr, wgrad_stream = nullptr;
    cudaEvent_t wg_fork[5] = {}, wg_join[4] = {};
    cudaStream_t key_stream = nullptr;  // the attention backward's key kernel
    cudaEvent_t key_fork = nullptr, key_join = nullptr;
    std::vector<cudaEvent_t> layer_ev;  // data parallel: block l done in the lane's last micro-step
    cudaEvent_t tail_ev = nullptr;
  };
  static constexpr int kMaxLanes = 4;
  Lane lanes[kMaxLanes];
  int lanes_alloc = 1;  // lanes with buffers (2 or 4 when the micro-batch is small)
  int cur_lane = 0, step_lanes = 1, comm_lane = 0;
  cudaEvent_t lane_fork = nullptr, lane_join[kMaxLanes] = {};
  // SPAR_B200_LANES: 0 = never, 2 / 4 = that many at any micro-batch, unset / 1 = by micro-batch.
  int lanes_mode = getenv("SPAR_B200_LANES") ? getenv("SPAR_B200_LANES")[0] - '0' : 1;
  void select_lane(int i) {
    Lane& ln = lanes[i];
    acts = ln.acts;
    xL = ln.xL; meanf = ln.meanf; rstdf = ln.rstdf; hf = ln.hf; logits = ln.logits;
    dres = ln.dres; dtmp = ln.dtmp; dqkv = ln.dqkv; dS = ln.dS; du = ln.du; dh_buf = ln.dh_buf;
    colpart = ln.colpart;
    kvrep = ln.kvrep;
    dkvrep = ln.dkvrep;
    ln_ws = ln.ln_ws; col_ws = ln.col_ws; splitk_ws = ln.splitk_ws; splitk_ws2 = ln.splitk_ws2;
    row_loss = ln.row_loss; grads = ln.grads; emb_scratch = ln.emb_scratch;
    wgrad_stream = ln.wgrad_stream;
    for (int k = 0; k < 5; ++k) wg_fork[k] = ln.wg_fork[k];
    for (int k = 0; k < 4; ++k) wg_join[k] = ln.wg_join[k];
    cur_lane = i;
  }
  void* emb_scratch = nullptr;
  float* row_loss = nullptr;     // [N]
  float* loss_sums = nullptr;    // [kMaxMicro]
  double* norm_state = nullptr;  // [kNormStateDoubles]
  int32_t* flags = nullptr;      // [0] invalid target/id, [1] non-finite grad norm
  int32_t* ids_dev = nullptr;    // [kMaxMicro * N]
  static constexpr uint64_t kMaxMicro = 64;
  void* comm = nullptr;
  int world = 1;
  bool last_micro = false;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> layer_ev;
  cudaEvent_t tail_ev = nullptr, comm_done = nullptr;
  // Sharded optimiser state (data parallel): each bucket's gradients are reduce-scattered instead
  // of all-reduced, and every rank runs the norm pass (its partial sum of squares all-reduced)
  // and AdamW on its own piece of each bucket only: 1 / world of the optimiser's HBM traffic. The
  // updated parameter pieces are all-gathered at the start of the next step, bucket by bucket in
  // the order the forward pass first reads them (embedding, blocks 0.., final norm), and each
  // micro-step's forward waits for a bucket only where it first reads it, so the gathers overlap
  // the forward pass as the reductions overlap the backward. Moments stay sharded; gradients,
  // moments and parameters read back through the C ABI need spar_b200_lm_gather on every rank.
  // SPAR_B200_SHARD_OPT=0 keeps the replicated all-reduce + whole-arena AdamW; =1 shards with a
  // one-rank communicator too (the path's test on one GPU); default: world > 1.
  int shard_mode = getenv("SPAR_B200_SHARD_OPT") ? getenv("SPAR_B200_SHARD_OPT")[0] - '0' : -1;
  bool sharded = false;       // a communicator is attached and the optimiser is sharded
  bool sharded_step = false;  // the step being issued reduce-scatters (train_step only)
  int rank = 0;
  std::vector<BucketShard> shard_plan;    // per bucket, issue order
  std::vector<Slice> own_slices, norm_slices;
  std::vector<cudaEvent_t> gather_ev;     // per bucket: its parameters gathered
  cudaEvent_t gather_fork = nullptr;
  bool stale[4] = {};  // arena (parameters, gradients, moments) holds other ranks' pieces stale
  cudaError_t gather_params(cudaStream_t s);
  cudaError_t gather_arena(int which, cudaStream_t s);
  cudaError_t reduce_bucket(size_t i, float* g);
  cudaError_t wait_gather(size_t bucket, cudaStream_t s) {
    return sharded_step ? cudaStreamWaitEvent(s, gather_ev[bucket], 0) : cudaSuccess;
  }
  uint64_t split_floats = 0;
  // Live profiling of the tensor-core GEMMs (CUDA events around every launch on its stream).
  bool profiling = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev_pool;
  size_t ev_used = 0;
  std::vector<double> ev_flops;
  uint64_t launches = 0;  // kernels this runtime launched since the counter was reset
  // CUDA-graph replay of whole training steps (zero gradients, micro-steps, clip + AdamW): one
  // graph per micro-step count, captured on the second train_step call (the first runs eagerly
  // and configures every kernel), replayed on an internal stream ordered after the caller's by
  // events. AdamW's step-dependent scalars come from opt_args, refreshed before each replay.
  struct StepGraph {
    cudaGraphExec_t exec;
    uint64_t launches;
  };
  std::map<uint64_t, StepGraph> graphs;
  // A step's bounded wait aborted the communicator: the captured steps hold that communicator's
  // collectives, whose resources the abort released, so they are dropped without being
  // destroyed (destroying them would run the library's clean-up on the released communicator).
  bool comm_aborted = false;
  void drop_graphs() {
    if (!comm_aborted)
      for (auto& g : graphs) cudaGraphExecDestroy(g.second.exec);
    graphs.clear();
  }
  // SPAR_B200_GRAPHS=0 keeps every step eager (for per-kernel profiling of the step).
  bool graphs_enabled = !(getenv("SPAR_B200_GRAPHS") && getenv("SPAR_B200_GRAPHS")[0] == '0');
  uint64_t eager_steps = 0;
  cudaStream_t exec_stream = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  AdamWArgs* opt_args = nullptr;       // device
  AdamWArgs* opt_args_host = nullptr;  // pinned host
  // Pinned host landing area of a step's results. A device-to-host copy into pageable memory
  // returns only once the stream's earlier work has finished, which would hold the host inside
  // the copy (before the communicator's bounded wait) when a peer never joins the step.
  struct StepResults {
    float sums[kMaxMicro];  // loss sum of each micro-step
    double norm_state[2];
    int32_t flags[2];
  };
  StepResults* results_host = nullptr;
  SparCudaStatus step_body(uint64_t micro_steps, float grad_scale, double lr, uint64_t step,
                           cudaStream_t s, bool device_args);

  SparCudaStatus init(const SparB200LMConfig& c, int dev);
  ~LMTrainer();
  SparCudaStatus forward_backward(const int32_t* ids, float grad_scale, uint64_t micro,
                                  cudaStream_t s);
  cudaError_t gemm(uint64_t m, uint64_t n, uint64_t k, const float* a, uint64_t lda, bool at,
                   const float* b, uint64_t ldb, bool bt, float* c, uint64_t ldc,
                   bool accumulate, int epi, const float* bias, float* aux, uint64_t ldaux,
                   cudaStream_t s, int causal = SPAR_B200_CAUSAL_NONE, uint64_t b0 = 1,
                   uint64_t b1 = 1, const uint64_t* a_bs = nullptr, const uint64_t* b_bs = nullptr,
                   const uint64_t* c_bs = nullptr, bool round_out = false, bool rope = false,
                   float* column_partials = nullptr);
  cudaError_t attention_forward(LayerActs& A, cudaStream_t s);
  cudaError_t attention_backward(LayerActs& A, cudaStream_t s);
  cudaError_t layer_backward(uint64_t l, cudaStream_t s);
  // Spar family (nn::DecoderLM): one block forward / backward.
  cudaError_t layer_forward_spar(uint64_t l, float* out, cudaStream_t s);
  cudaError_t layer_backward_spar(uint64_t l, cudaStream_t s);
  // Data-parallel reduction of buckets [b0, b1) on the communication stream once the gradients in
  // them are final on stream s. With two lanes, each lane records lane_ev after its last
  // micro-step has produced them; the lane that issues last (comm_lane) then adds lane 1's
  // buckets into lane 0's and reduces lane 0's.
  cudaError_t reduce_buckets(size_t b0, size_t b1, int layer, cudaEvent_t single_ev,
                             cudaStream_t s);
  // lanes[0].grads[off, off + count) += the other step lanes' gradients, in lane order.
  cudaError_t merge_lanes(uint64_t off, uint64_t count, cudaStream_t s);
};

LMTrainer::~LMTrainer() {
  DeviceScope scope(device);
  cudaDeviceSynchronize();
  for (auto ev : layer_ev) cudaEventDestroy(ev);
  for (auto ev : gather_ev) cudaEventDestroy(ev);
  if (gather_fork) cudaEventDestroy(gather_fork);
  if (tail_ev) cudaEventDestroy(tail_ev);
  if (comm_done) cudaEventDestroy(comm_done);
  if (comm_stream) cudaStreamDestroy(comm_stream);
  for (Lane& ln : lanes) {
    for (auto ev : ln.wg_fork)
      if (ev) cudaEventDestroy(ev);
    for (auto ev : ln.wg_join)
      if (ev) cudaEventDestroy(ev);
    for (auto ev : ln.layer_ev) cudaEventDestroy(ev);
    if (ln.key_fork) cudaEventDestroy(ln.key_fork);
    if (ln.key_join) cudaEventDestroy(ln.key_join);
    if (ln.key_stream) cudaStreamDestroy(ln.key_stream);
    if (ln.tail_ev) cudaEventDestroy(ln.tail_ev);
    if (ln.wgrad_stream) cudaStreamDestroy(ln.wgrad_stream);
    if (&ln != &lanes[0] && ln.stream) cudaStreamDestroy(ln.stream);  // lane 0 borrows the step's
  }
  if (lane_fork) cudaEventDestroy(lane_fork);
  for (auto ev : lane_join)
    if (ev) cudaEventDestroy(ev);
  drop_graphs();
  if (exec_stream) cudaStreamDestroy(exec_stream);
  if (ev_in) cudaEventDestroy(ev_in);
  if (ev_out) cudaEventDestroy(ev_out);
  if (opt_args_host) cudaFreeHost(opt_args_host);
  if (results_host) cudaFreeHost(results_host);
  cudaFree(params);
  if (wround) cudaFree(wround);
  cudaFree(act_base);
}

// The rounded weight copy after host-side parameter writes (not captured into a step graph).
cudaError_t LMTrainer::refresh_rounded(cudaStream_t s) {
  if (!wround || !wround_dirty) return cudaSuccess;
  const cudaError_t e = round_copy_launch(wround, params, flat, device, s);
  if (e == cudaSuccess) wround_dirty = false;
  return e;
}

SparCudaStatus LMTrainer::init(const SparB200LMConfig& c, int dev) {
  cfg = c;
  device = dev;
  V = c.vocab_size;
  d = c.model_dim;
  F = c.hidden_dim;
  L = c.num_layers;
  H = c.num_heads;
  T = c.sequence_length;
  B = c.micro_batch;
  if (V == 0 || d == 0 || F == 0 || L == 0 || H == 0 || T < 2 || B == 0 || d % H != 0)
    return invalid();
  dh = d / H;
  N = B * T;
  Vp = (V + 3) / 4 * 4;
  family = c.family;
  KVH = (family == SPAR_B200_FAMILY_SPAR && c.num_kv_heads) ? c.num_kv_heads : H;
  Wq = (H + 2 * KVH) * (d / H);
  Fu = family == SPAR_B200_FAMILY_SPAR ? 2 * F : F;
  qk_norm = family == SPAR_B200_FAMILY_SPAR && c.qk_norm != 0;
  if (d % 32 != 0 || F % 4 != 0 || dh % 32 != 0 || T % 4 != 0) return invalid();
  if (c.precision != SPAR_B200_TF32 && c.precision != SPAR_B200_TF32X3) return invalid();

  ParamLayout pl;
  const SparCudaStatus ls = plan_params(c, pl);
  if (ls.code) return ls;
  flat = pl.flat;
  off_E = pl.off_E;
  off_lnf_g = pl.off_lnf_g;
  off_lnf_b = pl.off_lnf_b;
  buckets = pl.buckets();
  named = std::move(pl.named);
  lay = std::move(pl.lay);

  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&params), 4 * flat * sizeof(float));
  if (e != cudaSuccess) return runtime(e);
  grads = params + flat;
  m1 = grads + flat;
  m2 = m1 + flat;
  e = cudaMemset(params, 0, 4 * flat * sizeof(float));
  if (e != cudaSuccess) return runtime(e);
  if (c.precision == SPAR_B200_TF32) {
    e = cudaMalloc(reinterpret_cast<void**>(&wround), flat * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(wround, 0, flat * sizeof(float));
    if (e != cudaSuccess) return runtime(e);
  }

  // ---- activation arena
  fused_attention = c.precision == SPAR_B200_TF32 && attention_supported(dh);
  // One layer's attention probabilities (unfused) or softmax statistics (fused).
  const uint64_t PS = fused_attention ? 2 * B * H * T : B * H * T * T;
  const int ln_parts = layernorm_backward_parts(N, device);
  // Column-sum partials: the partition count depends on the width, so take the largest
  // parts x cols over the widths reduced in the backward pass (d, 3d, F).
  uint64_t col_floats = 0;
  for (uint64_t w : {d, 3 * d, F})
    col_floats = std::max<uint64_t>(col_floats, static_cast<uint64_t>(column_sum_parts(N, w, device)) * w);
  std::vector<std::pair<void**, uint64_t>> plan;  // (pointer slot, bytes)
  auto f = [&](float** p, uint64_t n) { plan.push_back({reinterpret_cast<void**>(p), n * 4}); };
  // Two lanes (two micro-steps in flight) when a micro-step is too narrow to fill the GPU.
  // Two lanes at micro-batches of <= 4 sequences (SPAR_B200_LANES=2 / 4 force two / four at any
  // micro-batch; four measured no faster than two at micro-batch 2: the merge grows, the SMs
  // are already shared).
  lanes_alloc = 1;
  if (c.precision == SPAR_B200_TF32) {
    if (lanes_mode == 2 || lanes_mode == 4) lanes_alloc = lanes_mode;
    else if (lanes_mode == 1) lanes_alloc = B <= 4 ? 2 : 1;
  }
  for (int li = 0; li < lanes_alloc; ++li) {
    Lane& ln = lanes[li];
    ln.acts.resize(L);
    for (uint64_t l = 0; l < L; ++l) {
      LayerActs& A = ln.acts[l];
      f(&A.x, N * d);
      f(&A.mean1, N);
      f(&A.rstd1, N);
      f(&A.a1, N * d);
      f(&A.qkv, N * Wq);
      if (qk_norm) {
        f(&A.qkv_raw, N * Wq);
        f(&A.qk_rstd, N * (H + KVH));
      }
      f(fused_attention ? &A.stats : &A.p, PS);
      f(&A.ctx, N * d);
      f(&A.h1, N * d);
      f(&A.mean2, N);
      f(&A.rstd2, N);
      f(&A.a2, N * d);
      f(&A.u, N * Fu);
      f(&A.g, N * F);
    }
    f(&ln.xL, N * d);
    f(&ln.meanf, N);
    f(&ln.rstdf, N);
    f(&ln.hf, N * d);
    f(&ln.logits, N * Vp);
    f(&ln.dres, N * d);
    f(&ln.dtmp, N * d);
    f(&ln.dqkv, N * Wq);
    f(&ln.dS, fused_attention ? B * H * T : PS);
    f(&ln.du, N * Fu);
    if (family == SPAR_B200_FAMILY_SPAR) f(&ln.dh_buf, N * F);
    else f(&ln.colpart, (N + 31) / 32 * (F + Wq));
    if (!fused_attention && KVH != H) {
      f(&ln.kvrep, N * 2 * d);
      f(&ln.dkvrep, N * 2 * d);
    }
    f(&ln.ln_ws, 3ull * ln_parts * d);  // dgamma, dbeta and dx column-sum partials
    f(&ln.col_ws, col_floats);
    f(&ln.row_loss, N);
    plan.push_back({reinterpret_cast<void**>(&ln.emb_scratch), embedding_backward_scratch(N, V)});
    if (li > 0) f(&ln.grads, flat);  // lane 0 accumulates into the trainer's gradient arena
  }
  lanes[0].grads = grads;
  f(&rope_tab, T * dh);
  f(&loss_sums, kMaxMicro);
  plan.push_back({reinterpret_cast<void**>(&norm_state), kNormStateDoubles * sizeof(double)});
  plan.push_back({reinterpret_cast<void**>(&flags), 64});
  plan.push_back({reinterpret_cast<void**>(&opt_args), sizeof(AdamWArgs)});
  plan.push_back({reinterpret_cast<void**>(&ids_dev), kMaxMicro * N * sizeof(int32_t)});
  if (c.precision == SPAR_B200_TF32X3) {
    // 3xTF32 splits both operands of every GEMM into hi/lo copies; size the workspace for the
    // largest of the step's GEMMs (m, n, k, A transposed, B transposed, batch), all listed here.
    struct Shape { uint64_t m, n, k; int at, bt; uint64_t b0, b1; };
    const Shape shapes[] = {
        {N, 3 * d, d, 0, 0, 1, 1},  {T, T, dh, 0, 1, B, H},  {T, dh, T, 0, 0, B, H},
        {N, d, d, 0, 0, 1, 1},      {N, F, d, 0, 0, 1, 1},   {N, d, F, 0, 0, 1, 1},
        {N, V, d, 0, 1, 1, 1},      {V, d, N, 1, 0, 1, 1},   {N, d, V, 0, 0, 1, 1},
        {F, d, N, 1, 0, 1, 1},      {N, F, d, 0, 1, 1, 1},   {d, F, N, 1, 0, 1, 1},
        {N, d, F, 0, 1, 1, 1},      {d, d, N, 1, 0, 1, 1},   {N, d, d, 0, 1, 1, 1},
        {T, dh, T, 1, 0, B, H},     {T, T, dh, 0, 1, B, H},  {T, dh, T, 0, 0, B, H},
        {T, dh, T, 1, 0, B, H},     {d, 3 * d, N, 1, 0, 1, 1}, {N, d, 3 * d, 0, 1, 1, 1},
        // Spar family: packed q | k | v rows of Wq, gate | up rows of Fu
        {N, Wq, d, 0, 0, 1, 1},     {d, Wq, N, 1, 0, 1, 1},  {N, d, Wq, 0, 1, 1, 1},
        {N, Fu, d, 0, 0, 1, 1},     {d, Fu, N, 1, 0, 1, 1},  {N, d, Fu, 0, 1, 1, 1},
    };
    for (const Shape& sh : shapes) {
      SparB200Gemm g{};
      g.m = sh.m; g.n = sh.n; g.k = sh.k; g.a_transposed = sh.at; g.b_transposed = sh.bt;
      g.batch[0] = sh.b0; g.batch[1] = sh.b1;
      g.precision = SPAR_B200_TF32X3;  // the workspace depends on how the product is split
      // The batched attention products are the causal ones (three-section kernel).
      g.causal = sh.b0 * sh.b1 > 1 ? SPAR_B200_CAUSAL_LOWER : SPAR_B200_CAUSAL_NONE;
      split_floats = std::max(split_floats, gemm_split_workspace_floats(g));
    }
    f(&split_ws, split_floats);
  }
  {
    // Partial tiles of every product of the step that may be split along K (few output tiles
    // for the SMs: the weight gradients, and the token-dimension products at small batches).
    struct Shape { uint64_t m, n, k; };
    const Shape shapes[] = {{N, Wq, d}, {N, d, d},  {N, Fu, d}, {N, d, F}, {N, V, d},
                            {V, d, N},  {N, d, V},  {F, d, N},  {d, Fu, N}, {d, d, N},
                            {d, Wq, N}, {N, d, Wq}, {N, F, d},  {N, d, Fu}};
    for (const Shape& sh : shapes) {
      SparB200Gemm g{};
      g.m = sh.m; g.n = sh.n; g.k = sh.k; g.batch[0] = g.batch[1] = 1;
      g.precision = c.precision;
      splitk_floats = std::max(splitk_floats, gemm_splitk_workspace_floats(g, device));
    }
    if (splitk_floats)
      for (int li = 0; li < lanes_alloc; ++li) {
        f(&lanes[li].splitk_ws, splitk_floats);
        f(&lanes[li].splitk_ws2, splitk_floats);
      }
  }
  uint64_t total = 0;
  for (auto& pb : plan) total += (pb.second + 255) / 256 * 256;
  e = cudaMalloc(reinterpret_cast<void**>(&act_base), total);
  if (e != cudaSuccess) return runtime(e);
  uint64_t pos = 0;
  for (auto& pb : plan) {
    *pb.first = act_base + pos;
    pos += (pb.second + 255) / 256 * 256;
  }
  e = cudaMemset(flags, 0, 64);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&exec_stream, cudaStreamNonBlocking);
  for (int li = 0; li < lanes_alloc; ++li) {
    Lane& ln = lanes[li];
    if (li > 0 && e == cudaSuccess) e = cudaStreamCreateWithFlags(&ln.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ln.wgrad_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ln.key_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ln.key_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ln.key_join, cudaEventDisableTiming);
    for (auto& ev : ln.wg_fork)
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    for (auto& ev : ln.wg_join)
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&lane_fork, cudaEventDisableTiming);
  for (int li = 0; li < lanes_alloc; ++li)
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&lane_join[li], cudaEventDisableTiming);
  select_lane(0);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming);
  if (e == cudaSuccess)
    e = cudaMallocHost(reinterpret_cast<void**>(&opt_args_host), sizeof(AdamWArgs));
  if (e == cudaSuccess)
    e = cudaMallocHost(reinterpret_cast<void**>(&results_host), sizeof(StepResults));
  if (e == cudaSuccess) e = rope_table_launch(rope_tab, T, dh, c.rope_theta, 0, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return runtime(e);
  // LayerNorm gamma = 1, beta = 0; biases 0 (BASELINE init, Linear bias init linear.cpp:40-42).
  for (const auto& t : named)
    if (t.name.find("norm.weight") != std::string::npos)
      fill_kernel<<<grid_for(t.rows, 256, 1024), 256>>>(params + t.offset, t.rows, 1.f);
  e = cudaDeviceSynchronize();
  return e == cudaSuccess ? ok() : runtime(e);
}

cudaError_t LMTrainer::gemm(uint64_t m, uint64_t n, uint64_t k, const float* a, uint64_t lda,
                            bool at, const float* b, uint64_t ldb, bool bt, float* c, uint64_t ldc,
                            bool accumulate, int epi, const float* bias, float* aux,
                            uint64_t ldaux, cudaStream_t s, int causal, uint64_t b0, uint64_t b1,
                            const uint64_t* a_bs, const uint64_t* b_bs, const uint64_t* c_bs,
                            bool round_out, bool rope, float* column_partials) {
  SparB200Gemm g{};
  g.m = m;
  g.n = n;
  g.k = k;
  g.batch[0] = b0;
  g.batch[1] = b1;
  g.a = a;
  g.lda = lda;
  g.a_transposed = at;
  g.b = b;
  g.ldb = ldb;
  g.b_transposed = bt;
  g.c = c;
  g.ldc = ldc;
  if (a_bs) g.a_batch_stride[0] = a_bs[0], g.a_batch_stride[1] = a_bs[1];
  if (b_bs) g.b_batch_stride[0] = b_bs[0], g.b_batch_stride[1] = b_bs[1];
  if (c_bs) g.c_batch_stride[0] = c_bs[0], g.c_batch_stride[1] = c_bs[1];
  g.alpha = 1.f;
  g.accumulate = accumulate;
  g.epilogue = epi;
  g.bias = bias;
  g.aux = aux;
  g.ldaux = ldaux;
  g.precision = cfg.precision;
  g.causal = causal;
  g.round_output = round_out;
  g.column_partials = column_partials;
  if (rope) {  // RoPE on the q and k thirds of the fused projection output
    g.rope_table = rope_tab;
    g.rope_seq = T;
    g.rope_dim = dh;
    g.rope_cols = Wq - KVH * dh;  // the q and k parts
  }
  launches += cfg.precision == SPAR_B200_TF32X3 ? 3 : 1;
  // Never let a split copy run past the workspace sized in init().
  if (cfg.precision == SPAR_B200_TF32X3 && gemm_split_workspace_floats(g) > split_floats)
    return cudaErrorInvalidValue;
  float* kws = s == wgrad_stream ? splitk_ws2 : splitk_ws;
  if (!profiling) return gemm_launch(g, split_ws, device, s, kws, splitk_floats);
  if (ev_used == ev_pool.size()) {
    std::pair<cudaEvent_t, cudaEvent_t> pr;
    SPAR_TRY_RAW(cudaEventCreate(&pr.first));
    SPAR_TRY_RAW(cudaEventCreate(&pr.second));
    ev_pool.push_back(pr);
  }
  // Algorithmic FLOPs: 2mnk per batch entry; the causal products do half of that useful work.
  double fl = 2.0 * m * n * k * b0 * b1;
  if (causal != SPAR_B200_CAUSAL_NONE) fl *= 0.5;
  auto& pr = ev_pool[ev_used++];
  ev_flops.push_back(fl);
  SPAR_TRY_RAW(cudaEventRecord(pr.first, s));
  SPAR_TRY_RAW(gemm_launch(g, split_ws, device, s, kws, splitk_floats));
  return cudaEventRecord(pr.second, s);
}

#define SPAR_TRY(expr)                  \
  do {                                  \
    const cudaError_t e_ = (expr);      \
    if (e_ != cudaSuccess) return e_;   \
  } while (0)

// S = QK^T (lower tiles), P = causal softmax in place, ctx = P V (k <= row).
cudaError_t LMTrainer::attention_forward(LayerActs& A, cudaStream_t s) {
  if (fused_attention)  // TF32 mode: ctx only feeds TF32 products, stored rounded to nearest
    return attention_forward_launch(A.qkv, A.ctx, A.stats, A.stats + B * H * T, B, T, H, dh,
                                    device, s, KVH, cfg.precision == SPAR_B200_TF32);
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dh)));
  // q from the packed projection (rows of Wq floats); k, v from it too, or (grouped key / value
  // heads) from their expansion to the query heads, rows of 2d floats.
  const uint64_t ldq = Wq;
  uint64_t ldkv = Wq;
  const float* k = A.qkv + d;
  const float* v = A.qkv + 2 * d;
  if (KVH != H) {
    SPAR_TRY(repeat_kv_launch(kvrep, A.qkv, N, H, KVH, dh, Wq, d, device, s));
    ldkv = 2 * d;
    k = kvrep;
    v = kvrep + d;
  }
  const uint64_t q_bs[2] = {T * ldq, dh};
  const uint64_t kv_bs[2] = {T * ldkv, dh};
  const uint64_t p_bs[2] = {H * T * T, T * T};
  const uint64_t ctx_bs[2] = {T * d, dh};
  const float* q = A.qkv;
  SPAR_TRY(gemm(T, T, dh, q, ldq, false, k, ldkv, true, A.p, T, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_LOWER, B, H, q_bs, kv_bs, p_bs));
  SPAR_TRY(causal_softmax_launch(A.p, A.p, nullptr, B * H, T, T, scale, 128, 0, s));
  SPAR_TRY(gemm(T, dh, T, A.p, T, false, v, ldkv, false, A.ctx, d, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_K_UPTO, B, H, p_bs, kv_bs, ctx_bs));
  return cudaSuccess;
}

cudaError_t LMTrainer::merge_lanes(uint64_t off, uint64_t count, cudaStream_t s) {
  const float4* src[3] = {nullptr, nullptr, nullptr};
  for (int li = 1; li < step_lanes; ++li) src[li - 1] = reinterpret_cast<const float4*>(lanes[li].grads + off);
  launches += 1;
  return launch(add_lanes_kernel, dim3(grid_for(count / 4, 256, sm_count(device) * 8)), dim3(256), 0,
                s, reinterpret_cast<float4*>(lanes[0].grads + off), src[0], src[1], src[2], count / 4);
}

cudaError_t LMTrainer::reduce_buckets(size_t b0, size_t b1, int layer, cudaEvent_t single_ev,
                                      cudaStream_t s) {
  if (step_lanes == 1) {
    SPAR_TRY_RAW(cudaEventRecord(single_ev, s));
    SPAR_TRY_RAW(cudaStreamWaitEvent(comm_stream, single_ev, 0));
    for (size_t i = b0; i < b1; ++i) SPAR_TRY_RAW(reduce_bucket(i, grads));
    return cudaSuccess;
  }
  auto ev = [&](int li) { return layer >= 0 ? lanes[li].layer_ev[layer] : lanes[li].tail_ev; };
  SPAR_TRY_RAW(cudaEventRecord(ev(cur_lane), s));
  if (cur_lane != comm_lane) return cudaSuccess;  // the lane issued last runs the reduction
  // Every other lane's last micro-step was issued earlier, so all events are recorded.
  for (int li = 0; li < step_lanes; ++li) SPAR_TRY_RAW(cudaStreamWaitEvent(comm_stream, ev(li), 0));
  for (size_t i = b0; i < b1; ++i) {
    const uint64_t off = buckets[i].first, cnt = buckets[i].second;
    SPAR_TRY_RAW(merge_lanes(off, cnt, comm_stream));
    SPAR_TRY_RAW(reduce_bucket(i, lanes[0].grads));
  }
  return cudaSuccess;
}

// Bucket i of gradient arena g summed across ranks on the communication stream: all-reduced, or
// (sharded optimiser) reduce-scattered with its uneven tail all-reduced.
cudaError_t LMTrainer::reduce_bucket(size_t i, float* g) {
  if (!sharded_step) return comm_allreduce_sum(comm, g + buckets[i].first, buckets[i].second, comm_stream);
  const BucketShard& b = shard_plan[i];
  if (b.shard) SPAR_TRY_RAW(comm_reduce_scatter_sum(comm, g + b.off, b.shard, comm_stream));
  if (b.rem_count) SPAR_TRY_RAW(comm_allreduce_sum(comm, g + b.rem_off, b.rem_count, comm_stream));
  return cudaSuccess;
}

// Start of a sharded step: the parameter pieces the other ranks updated in the previous step are
// all-gathered on the communication stream (after everything already on s), in the order the
// forward pass first reads the buckets; gather_ev[i] marks bucket i complete.
cudaError_t LMTrainer::gather_params(cudaStream_t s) {
  SPAR_TRY_RAW(cudaEventRecord(gather_fork, s));
  SPAR_TRY_RAW(cudaStreamWaitEvent(comm_stream, gather_fork, 0));
  auto issue = [&](size_t i) -> cudaError_t {
    const BucketShard& b = shard_plan[i];
    if (b.shard) SPAR_TRY_RAW(comm_all_gather(comm, params + b.off, b.shard, comm_stream));
    if (wround && b.shard) {  // the other ranks' pieces arrive unrounded
      launches += 1;
      SPAR_TRY_RAW(round_copy_launch(wround + b.off, params + b.off,
                                     static_cast<uint64_t>(comm_size(comm)) * b.shard, device,
                                     comm_stream));
    }
    return cudaEventRecord(gather_ev[i], comm_stream);
  };
  SPAR_TRY_RAW(issue(L));  // embedding
  for (uint64_t l = 0; l < L; ++l) SPAR_TRY_RAW(issue(L - 1 - l));
  return issue(L + 1);  // final norm
}

// Every bucket's pieces of arena `which` (0 parameters, 1 gradients, 2 / 3 moments) gathered onto
// every rank, ordered after the work on s, which waits for the gather. Collective.
cudaError_t LMTrainer::gather_arena(int which, cudaStream_t s) {
  if (!sharded || !stale[which]) return cudaSuccess;
  float* base = params + static_cast<uint64_t>(which) * flat;
  SPAR_TRY_RAW(cudaEventRecord(gather_fork, s));
  SPAR_TRY_RAW(cudaStreamWaitEvent(comm_stream, gather_fork, 0));
  for (const BucketShard& b : shard_plan)
    if (b.shard) SPAR_TRY_RAW(comm_all_gather(comm, base + b.off, b.shard, comm_stream));
  SPAR_TRY_RAW(cudaEventRecord(comm_done, comm_stream));
  SPAR_TRY_RAW(cudaStreamWaitEvent(s, comm_done, 0));
  stale[which] = false;
  if (which == 0) wround_dirty = true;  // the gathered pieces reach the rounded copy next step
  return cudaSuccess;
}

// One whole optimiser step on stream s with the token ids already in ids_dev: (sharded: gather the
// parameters,) zero the gradient arenas, the micro-step sweeps, the global-norm pass and
// clip + AdamW (scalars by value, or from opt_args when the launches are being captured).
SparCudaStatus LMTrainer::step_body(uint64_t micro_steps, float grad_scale, double lr,
                                    uint64_t step, cudaStream_t s, bool device_args) {
  step_lanes = (lanes_alloc > 1 && micro_steps >= 2 && !profiling)
                   ? static_cast<int>(std::min<uint64_t>(lanes_alloc, micro_steps))
                   : 1;
  comm_lane = static_cast<int>((micro_steps - 1) % step_lanes);  // issues last, runs the reduction
  lanes[0].stream = s;
  sharded_step = sharded && comm;
  struct Reset {  // the caller-driven micro-steps never shard
    bool& f;
    ~Reset() { f = false; }
  } reset{sharded_step};
  // The error flags describe this step only (a skipped update does not taint the next step).
  cudaError_t e = cudaMemsetAsync(flags, 0, 2 * sizeof(int32_t), s);
  if (e == cudaSuccess && sharded_step) e = gather_params(s);
  for (int li = 0; li < step_lanes && e == cudaSuccess; ++li)
    e = cudaMemsetAsync(lanes[li].grads, 0, flat * sizeof(float), s);
  if (e == cudaSuccess && step_lanes > 1) {  // the other lanes start after the zeroing
    e = cudaEventRecord(lane_fork, s);
    for (int li = 1; li < step_lanes && e == cudaSuccess; ++li)
      e = cudaStreamWaitEvent(lanes[li].stream, lane_fork, 0);
  }
  if (e != cudaSuccess) return runtime(e);
  for (uint64_t m = 0; m < micro_steps; ++m) {
    const int li = static_cast<int>(m % step_lanes);
    select_lane(li);
    last_micro = m + step_lanes >= micro_steps;  // the lane's last micro-step
    const SparCudaStatus st = forward_backward(ids_dev + m * N, grad_scale, m, lanes[li].stream);
    if (st.code != 0) {
      select_lane(0);
      lanes[0].stream = nullptr;
      return st;
    }
  }
  select_lane(0);
  lanes[0].stream = nullptr;  // borrowed for this step only
  if (step_lanes > 1) {
    for (int li = 1; li < step_lanes && e == cudaSuccess; ++li) {
      e = cudaEventRecord(lane_join[li], lanes[li].stream);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(s, lane_join[li], 0);
    }
    // Without a communicator the lanes' gradients are added here (with one, per bucket).
    if (e == cudaSuccess && !comm) e = merge_lanes(0, flat, s);
    if (e != cudaSuccess) return runtime(e);
  }
  Slice slice{params, grads, m1, m2, flat};
  if (sharded_step) {
    // This rank's pieces: sum of squares, summed over ranks (the non-finite flags too), then
    // clip + AdamW on the pieces.
    launches += norm_slices.size() + 1 + own_slices.size();
    e = grad_norm_launch(norm_state, norm_slices.data(), norm_slices.size(), device, s,
                         gemm_wait_flag(device), attention_wait_flag(device));
    if (e == cudaSuccess) e = cudaEventRecord(gather_fork, s);  // collectives stay on comm_stream
    if (e == cudaSuccess) e = cudaStreamWaitEvent(comm_stream, gather_fork, 0);
    if (e == cudaSuccess) e = comm_allreduce_sum_f64(comm, norm_state, 2, comm_stream);
    if (e == cudaSuccess) e = cudaEventRecord(comm_done, comm_stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, comm_done, 0);
    if (e == cudaSuccess)
      e = adamw_launch(own_slices.data(), own_slices.size(), norm_state, cfg.max_grad_norm, lr,
                       cfg.beta1, cfg.beta2, cfg.adam_epsilon, cfg.weight_decay, step, flags + 1,
                       device, s, device_args ? opt_args : nullptr, params, wround);
    return e == cudaSuccess ? ok() : runtime(e);
  }
  launches += 3;
  e = grad_norm_launch(norm_state, &slice, 1, device, s, gemm_wait_flag(device),
                       attention_wait_flag(device));
  if (e == cudaSuccess)
    e = adamw_launch(&slice, 1, norm_state, cfg.max_grad_norm, lr, cfg.beta1, cfg.beta2,
                     cfg.adam_epsilon, cfg.weight_decay, step, flags + 1, device, s,
                     device_args ? opt_args : nullptr, params, wround);
  return e == cudaSuccess ? ok() : runtime(e);
}

SparCudaStatus LMTrainer::forward_backward(const int32_t* ids, float grad_scale, uint64_t micro,
                                           cudaStream_t s) {
#define SPAR_CHECK(expr)                              \
  do {                                                \
    const cudaError_t e_ = (expr);                    \
    if (e_ != cudaSuccess) return runtime(e_);        \
  } while (0)
  const float eps = static_cast<float>(cfg.norm_epsilon);
  const bool rn = cfg.precision == SPAR_B200_TF32;
  float* P = params;
  // Weights as the GEMMs read them: the copy rounded to nearest TF32 in TF32 mode.
  const float* Wt = wround ? wround : params;
  float* G = grads;
  // ---------------------------------------------------------------- forward
  launches += 1;
  SPAR_CHECK(wait_gather(L, s));  // sharded optimiser: the embedding's bucket is gathered
  SPAR_CHECK(embedding_forward_launch(acts[0].x, P + off_E, ids, N, V, d, flags, device, s));
  for (uint64_t l = 0; l < L; ++l) {
    LayerActs& A = acts[l];
    const LayerOffsets& lo = lay[l];
    float* out = l + 1 < L ? acts[l + 1].x : xL;
    SPAR_CHECK(wait_gather(L - 1 - l, s));
    if (family == SPAR_B200_FAMILY_SPAR) {
      SPAR_CHECK(layer_forward_spar(l, out, s));
      continue;
    }
    launches += 2 + 1;  // 2 LayerNorms, softmax (or fused attention)
    // TF32 mode: the norm outputs, g, ctx, dlogits, du and dqkv only feed TF32 products and are
    // stored rounded to nearest TF32 (the tensor cores would truncate them: a bias toward zero).
    SPAR_CHECK(layernorm_forward_launch(A.a1, A.mean1, A.rstd1, A.x, P + lo.ln1_g, P + lo.ln1_b,
                                        N, d, eps, device, s, rn));
    // qkv = a1 Wqkv + b, RoPE on the q and k thirds in the epilogue. q, k, v only feed
    // attention products: with fused attention they are stored rounded to nearest TF32.
    SPAR_CHECK(gemm(N, 3 * d, d, A.a1, d, false, Wt + lo.wqkv, 3 * d, false, A.qkv, 3 * d, false,
                    SPAR_B200_EPI_BIAS, P + lo.bqkv, nullptr, 0, s, SPAR_B200_CAUSAL_NONE, 1, 1,
                    nullptr, nullptr, nullptr, fused_attention, cfg.use_rope != 0));
    SPAR_CHECK(attention_forward(A, s));
    SPAR_CHECK(gemm(N, d, d, A.ctx, d, false, Wt + lo.wo, d, false, A.h1, d, false,
                    SPAR_B200_EPI_BIAS_ADD, P + lo.bo, A.x, d, s));
    SPAR_CHECK(layernorm_forward_launch(A.a2, A.mean2, A.rstd2, A.h1, P + lo.ln2_g, P + lo.ln2_b,
                                        N, d, eps, device, s, rn));
    SPAR_CHECK(gemm(N, F, d, A.a2, d, false, Wt + lo.w1, F, false, A.g, F, false,
                    SPAR_B200_EPI_BIAS_GELU, P + lo.b1, A.u, F, s, SPAR_B200_CAUSAL_NONE, 1, 1,
                    nullptr, nullptr, nullptr, rn));
    SPAR_CHECK(gemm(N, d, F, A.g, F, false, Wt + lo.w2, d, false, out, d, false,
                    SPAR_B200_EPI_BIAS_ADD, P + lo.b2, A.h1, d, s));
  }
  launches += 1 + 2 + 2;  // final LayerNorm, cross-entropy + loss sum, final LayerNorm backward
  SPAR_CHECK(wait_gather(L + 1, s));
  if (family == SPAR_B200_FAMILY_SPAR)
    SPAR_CHECK(rmsnorm_forward_launch(hf, rstdf, xL, P + off_lnf_g, N, d, eps, device, s, 0, 1,
                                      rn));
  else
    SPAR_CHECK(layernorm_forward_launch(hf, meanf, rstdf, xL, P + off_lnf_g, P + off_lnf_b, N, d,
                                        eps, device, s, rn));
  SPAR_CHECK(gemm(N, V, d, hf, d, false, Wt + off_E, d, true, logits, Vp, false,
                  SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s));
  // Fused log-softmax + NLL + mean backward; dlogits overwrite the logits in place.
  SPAR_CHECK(cross_entropy_launch(row_loss, logits, logits, ids, N, V, Vp, T, grad_scale,
                                  flags, device, s, rn));
  SPAR_CHECK(sum_launch(loss_sums + micro, row_loss, N, s));
  // ---------------------------------------------------------------- backward
  // dE += dlogits^T hf (weight-gradient stream) ; dhf = dlogits E
  const bool conc = wgrad_enabled && !profiling && cfg.precision == SPAR_B200_TF32;
  cudaStream_t w = conc ? wgrad_stream : s;
  if (conc) {
    SPAR_CHECK(cudaEventRecord(wg_fork[4], s));
    SPAR_CHECK(cudaStreamWaitEvent(w, wg_fork[4], 0));
  }
  SPAR_CHECK(gemm(V, d, N, logits, Vp, true, hf, d, false, G + off_E, d, true, SPAR_B200_EPI_NONE,
                  nullptr, nullptr, 0, w));
  if (conc) SPAR_CHECK(cudaEventRecord(wg_join[3], w));
  SPAR_CHECK(gemm(N, d, V, logits, Vp, false, Wt + off_E, d, false, dtmp, d, false,
                  SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s));
  // The final norm's dx is dL/d(last block output): its column sums are that block's b2 gradient.
  if (family == SPAR_B200_FAMILY_SPAR)
    SPAR_CHECK(rmsnorm_backward_launch(dres, G + off_lnf_g, dtmp, xL, P + off_lnf_g, rstdf, N, d,
                                       1, 0, ln_ws, device, s));
  else
    SPAR_CHECK(layernorm_backward_launch(dres, G + off_lnf_g, G + off_lnf_b, dtmp, xL,
                                         P + off_lnf_g, meanf, rstdf, N, d, 1, 0, ln_ws, device, s,
                                         G + lay[L - 1].b2));
  for (uint64_t l = L; l-- > 0;) {
    SPAR_CHECK(family == SPAR_B200_FAMILY_SPAR ? layer_backward_spar(l, s) : layer_backward(l, s));
  }
  launches += 5;
  // dE's tied-embedding scatter below adds into G + off_E, and the next micro-step rewrites the
  // logits and hf that the dE product reads.
  if (conc) SPAR_CHECK(cudaStreamWaitEvent(s, wg_join[3], 0));
  SPAR_CHECK(embedding_backward_launch(G + off_E, dres, ids, N, V, d, emb_scratch, device, s));
  if (comm && last_micro) {
    // Tied embedding and final norm (first and last gradients of the sweep), then join.
    SPAR_CHECK(reduce_buckets(L, buckets.size(), -1, tail_ev, s));
    if (step_lanes == 1 || cur_lane == comm_lane) {
      SPAR_CHECK(cudaEventRecord(comm_done, comm_stream));
      SPAR_CHECK(cudaStreamWaitEvent(s, comm_done, 0));
    }
  }
  return ok();
#undef SPAR_CHECK
}

// One block of Spar's decoder (TransformerBlock::forward, src/nn/transformer.cpp:53-69):
//   a1 = RMSNorm(x); qkv = a1 [Wq | Wk | Wv]; (qk_norm: RMSNorm of each q / k head); RoPE on q, k;
//   ctx = attention (key/value heads shared by query groups); h1 = x + ctx Wo;
//   a2 = RMSNorm(h1); [gate | up] = a2 [Wgate | Wup]; g = silu(gate) * up; out = h1 + g Wdown.
cudaError_t LMTrainer::layer_forward_spar(uint64_t l, float* out, cudaStream_t s) {
  LayerActs& A = acts[l];
  const LayerOffsets& lo = lay[l];
  float* P = params;
  // Weights as the GEMMs read them: the copy rounded to nearest TF32 in TF32 mode.
  const float* Wt = wround ? wround : params;
  const float eps = static_cast<float>(cfg.norm_epsilon);
  launches += 2 + 1 + 1;  // 2 RMSNorms, attention, SwiGLU
  const bool rn = cfg.precision == SPAR_B200_TF32;  // norm outputs only feed TF32 products
  SPAR_TRY(rmsnorm_forward_launch(A.a1, A.rstd1, A.x, P + lo.ln1_g, N, d, eps, device, s, 0, 1,
                                  rn));
  if (!qk_norm) {
    // RoPE on the q and k parts in the epilogue; q, k, v stored rounded to nearest TF32.
    SPAR_TRY(gemm(N, Wq, d, A.a1, d, false, Wt + lo.wqkv, Wq, false, A.qkv, Wq, false,
                  SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_NONE, 1, 1,
                  nullptr, nullptr, nullptr, rn, cfg.use_rope != 0));
  } else {
    // The q / k norms come before RoPE (attention.cpp:212-215): project, then one pass per
    // token normalises each q / k head, rotates it and writes q | k | v rounded to TF32.
    launches += 1;
    SPAR_TRY(gemm(N, Wq, d, A.a1, d, false, Wt + lo.wqkv, Wq, false, A.qkv_raw, Wq, false,
                  SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s));
    SPAR_TRY(qk_norm_rope_launch(A.qkv, A.qkv_raw, N, T, H, KVH, dh, Wq, P + lo.qn, P + lo.kn,
                                 A.qk_rstd, cfg.use_rope ? rope_tab : nullptr,
                                 static_cast<float>(cfg.qk_norm_epsilon), device, s, rn));
  }
  SPAR_TRY(attention_forward(A, s));
  SPAR_TRY(gemm(N, d, d, A.ctx, d, false, Wt + lo.wo, d, false, A.h1, d, false,
                SPAR_B200_EPI_BIAS_ADD, nullptr, A.x, d, s));
  SPAR_TRY(rmsnorm_forward_launch(A.a2, A.rstd2, A.h1, P + lo.ln2_g, N, d, eps, device, s, 0, 1,
                                  rn));
  SPAR_TRY(gemm(N, Fu, d, A.a2, d, false, Wt + lo.w1, Fu, false, A.u, Fu, false,
                SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s));
  SPAR_TRY(swiglu_forward_launch(A.g, F, A.u, Fu, A.u + F, Fu, N, F, device, s));
  return gemm(N, d, F, A.g, F, false, Wt + lo.w2, d, false, out, d, false, SPAR_B200_EPI_BIAS_ADD,
              nullptr, A.h1, d, s);
}

// Backward of that block, dres = dL/d(block output) in, dres = dL/d(block input) out; weight
// gradients accumulate, on the weight-gradient stream beside the dX chain as in layer_backward.
cudaError_t LMTrainer::layer_backward_spar(uint64_t l, cudaStream_t s) {
  LayerActs& A = acts[l];
  const LayerOffsets& lo = lay[l];
  float* P = params;
  // Weights as the GEMMs read them: the copy rounded to nearest TF32 in TF32 mode.
  const float* Wt = wround ? wround : params;
  float* G = grads;
  launches += 2 * 2 + 1 + 1 + (qk_norm ? 2 : 0);  // RMSNorm bwd, attention, SwiGLU bwd, qk norms
  // (3xTF32 keeps one stream: its hi / lo operand workspace is shared by the products.)
  const bool conc = wgrad_enabled && !profiling && cfg.precision == SPAR_B200_TF32;
  cudaStream_t w = conc ? wgrad_stream : s;
  auto fork = [&](int i) -> cudaError_t {
    if (!conc) return cudaSuccess;
    cudaError_t e = cudaEventRecord(wg_fork[i], s);
    return e == cudaSuccess ? cudaStreamWaitEvent(w, wg_fork[i], 0) : e;
  };
  auto mark = [&](int i) -> cudaError_t { return conc ? cudaEventRecord(wg_join[i], w) : cudaSuccess; };
  auto join = [&](int i) -> cudaError_t { return conc ? cudaStreamWaitEvent(s, wg_join[i], 0) : cudaSuccess; };
  // MLP: out = h1 + g Wdown, g = silu(gate) * up, [gate | up] = a2 [Wgate | Wup]
  SPAR_TRY(fork(0));
  SPAR_TRY(gemm(F, d, N, A.g, F, true, dres, d, false, G + lo.w2, d, true, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, w));
  SPAR_TRY(mark(0));  // dWdown has read dres
  SPAR_TRY(gemm(N, F, d, dres, d, false, Wt + lo.w2, d, true, dh_buf, F, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s));
  SPAR_TRY(swiglu_backward_launch(du, Fu, du + F, Fu, dh_buf, F, A.u, Fu, A.u + F, Fu, N, F,
                                  device, s));
  SPAR_TRY(fork(1));
  SPAR_TRY(gemm(d, Fu, N, A.a2, d, true, du, Fu, false, G + lo.w1, Fu, true, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, w));
  SPAR_TRY(gemm(N, d, Fu, du, Fu, false, Wt + lo.w1, Fu, true, dtmp, d, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s));
  // dres += RMSNorm backward -> dL/dh1 (dWdown read dres first)
  SPAR_TRY(join(0));
  SPAR_TRY(rmsnorm_backward_launch(dres, G + lo.ln2_g, dtmp, A.h1, P + lo.ln2_g, A.rstd2, N, d, 1,
                                   1, ln_ws, device, s));
  // out projection: h1 = x + ctx Wo
  SPAR_TRY(fork(2));
  SPAR_TRY(gemm(d, d, N, A.ctx, d, true, dres, d, false, G + lo.wo, d, true, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, w));
  SPAR_TRY(mark(1));  // dWo has read dres
  SPAR_TRY(gemm(N, d, d, dres, d, false, Wt + lo.wo, d, true, dtmp, d, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_NONE, 1, 1, nullptr, nullptr, nullptr,
                cfg.precision == SPAR_B200_TF32));
  // attention: dctx (dtmp) -> dqkv; the fused kernels rotate dq / dk back through RoPE, the
  // unfused path does it after the products (q and k heads are consecutive in each row).
  SPAR_TRY(attention_backward(A, s));
  if (cfg.use_rope && !fused_attention)
    SPAR_TRY(rope_apply_launch(dqkv, rope_tab, N, T, H + KVH, dh, Wq, 1, device, s));
  if (qk_norm)  // through the q / k norms, in place (weight gradients accumulate)
    SPAR_TRY(qk_norm_backward_launch(dqkv, A.qkv_raw, N, H, KVH, dh, Wq, P + lo.qn, P + lo.kn,
                                     A.qk_rstd, G + lo.qn, G + lo.kn, 1, ln_ws, device, s));
  SPAR_TRY(fork(3));
  SPAR_TRY(gemm(d, Wq, N, A.a1, d, true, dqkv, Wq, false, G + lo.wqkv, Wq, true,
                SPAR_B200_EPI_NONE, nullptr, nullptr, 0, w));
  SPAR_TRY(mark(2));
  SPAR_TRY(gemm(N, d, Wq, dqkv, Wq, false, Wt + lo.wqkv, Wq, true, dtmp, d, false,
                SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s));
  SPAR_TRY(join(1));
  SPAR_TRY(rmsnorm_backward_launch(dres, G + lo.ln1_g, dtmp, A.x, P + lo.ln1_g, A.rstd1, N, d, 1,
                                   1, ln_ws, device, s));
  SPAR_TRY(join(2));
  if (comm && last_micro) SPAR_TRY(reduce_buckets(L - 1 - l, L - l, static_cast<int>(l), layer_ev[l], s));
  return cudaSuccess;
}

// dqkv from dctx (in dtmp): fused kernels, or the six batched GEMMs around the materialised
// probabilities and the softmax backward.
cudaError_t LMTrainer::attention_backward(LayerActs& A, cudaStream_t s) {
  if (fused_attention) {
    launches += 1;  // query and key kernels (one counted with the softmax in layer_backward)
    const Lane& ln = lanes[cur_lane];
    const bool two = !profiling;
    return attention_backward_launch(A.qkv, A.ctx, dtmp, A.stats, A.stats + B * H * T, dS, dqkv,
                                     B, T, H, dh, device, s, cfg.use_rope ? rope_tab : nullptr,
                                     two ? ln.key_stream : nullptr, two ? ln.key_fork : nullptr,
                                     two ? ln.key_join : nullptr, KVH,
                                     cfg.precision == SPAR_B200_TF32,
                                     family == SPAR_B200_FAMILY_SPAR || T % 32
                                         ? nullptr
                                         : colpart + (N + 31) / 32 * F);
  }
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dh)));
  // Grouped key / value heads: the products run on the expansion to the query heads (rebuilt
  // here), their k / v gradients land in dkvrep and are summed per group into dqkv.
  const bool grouped = KVH != H;
  const uint64_t ldq = Wq, ldkv = grouped ? 2 * d : Wq;
  if (grouped) SPAR_TRY(repeat_kv_launch(kvrep, A.qkv, N, H, KVH, dh, Wq, d, device, s));
  const uint64_t q_bs[2] = {T * ldq, dh};
  const uint64_t kv_bs[2] = {T * ldkv, dh};
  const uint64_t p_bs[2] = {H * T * T, T * T};
  const uint64_t ctx_bs[2] = {T * d, dh};
  const float* q = A.qkv;
  const float* k = grouped ? kvrep : A.qkv + d;
  const float* v = grouped ? kvrep + d : A.qkv + 2 * d;
  float* dk = grouped ? dkvrep : dqkv + d;
  float* dv = grouped ? dkvrep + d : dqkv + 2 * d;
  // dV = P^T dctx (k >= row)
  SPAR_TRY(gemm(T, dh, T, A.p, T, true, dtmp, d, false, dv, ldkv, false,
                SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_K_FROM, B, H, p_bs,
                ctx_bs, kv_bs));
  // dP = dctx V^T (lower tiles), dS = softmax backward (scaled) in place
  SPAR_TRY(gemm(T, T, dh, dtmp, d, false, v, ldkv, true, dS, T, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_LOWER, B, H, ctx_bs, kv_bs, p_bs));
  SPAR_TRY(causal_softmax_launch(dS, dS, A.p, B * H, T, T, scale, 128, 1, s));
  // dQ = dS K (k <= row), dK = dS^T Q (k >= row)
  SPAR_TRY(gemm(T, dh, T, dS, T, false, k, ldkv, false, dqkv, ldq, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_K_UPTO, B, H, p_bs, kv_bs, q_bs));
  SPAR_TRY(gemm(T, dh, T, dS, T, true, q, ldq, false, dk, ldkv, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_K_FROM, B, H, p_bs, q_bs, kv_bs));
  if (grouped) SPAR_TRY(group_sum_launch(dqkv, dkvrep, N, H, KVH, dh, Wq, d, device, s));
  return cudaSuccess;
}

cudaError_t LMTrainer::layer_backward(uint64_t l, cudaStream_t s) {
  LayerActs& A = acts[l];
  const LayerOffsets& lo = lay[l];
  float* P = params;
  // Weights as the GEMMs read them: the copy rounded to nearest TF32 in TF32 mode.
  const float* Wt = wround ? wround : params;
  float* G = grads;
  launches += 2 * 2 + 2 * 2 + 1 + (cfg.use_rope && !fused_attention ? 1 : 0);  // col sums, LN bwd, softmax bwd, rope
  // Weight gradients on the second stream (forks: event on s, wait on w; joins: the reverse).
  const bool conc = wgrad_enabled && !profiling && cfg.precision == SPAR_B200_TF32;
  cudaStream_t w = conc ? wgrad_stream : s;
  auto fork = [&](int i) -> cudaError_t {
    if (!conc) return cudaSuccess;
    cudaError_t e = cudaEventRecord(wg_fork[i], s);
    return e == cudaSuccess ? cudaStreamWaitEvent(w, wg_fork[i], 0) : e;
  };
  auto mark = [&](int i) -> cudaError_t { return conc ? cudaEventRecord(wg_join[i], w) : cudaSuccess; };
  auto join = [&](int i) -> cudaError_t { return conc ? cudaStreamWaitEvent(s, wg_join[i], 0) : cudaSuccess; };
  // dres = dL/d(layer output) = dL/d(h1 + mlp)
  // MLP: mlp = g W2 + b2, g = gelu(u), u = a2 W1 + b1. The b2 gradient (column sums of dres)
  // came out of the LayerNorm backward that produced dres (the next block's LN1, or the final
  // norm).
  SPAR_TRY(fork(0));
  SPAR_TRY(gemm(F, d, N, A.g, F, true, dres, d, false, G + lo.w2, d, true, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, w));
  SPAR_TRY(mark(0));  // dW2 has read dres
  // du = (dres W2^T) o gelu'(u); its epilogue also leaves the b1 gradient's column partials.
  SPAR_TRY(gemm(N, F, d, dres, d, false, Wt + lo.w2, d, true, du, F, false, SPAR_B200_EPI_GELU_BWD,
                nullptr, A.u, F, s, SPAR_B200_CAUSAL_NONE, 1, 1, nullptr, nullptr, nullptr,
                cfg.precision == SPAR_B200_TF32, false, colpart));
  SPAR_TRY(fork(1));
  SPAR_TRY(gemm(d, F, N, A.a2, d, true, du, F, false, G + lo.w1, F, true, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, w));
  const uint64_t blocks = (N + 31) / 32;
  SPAR_TRY(column_sum_launch(G + lo.b1, colpart, blocks, F, F, 1, col_ws, device, w));
  SPAR_TRY(gemm(N, d, F, du, F, false, Wt + lo.w1, F, true, dtmp, d, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s));
  // dres += LN2 backward  ->  dL/dh1, whose column sums are the bo gradient (dW2 read dres first)
  SPAR_TRY(join(0));
  SPAR_TRY(layernorm_backward_launch(dres, G + lo.ln2_g, G + lo.ln2_b, dtmp, A.h1, P + lo.ln2_g,
                                     A.mean2, A.rstd2, N, d, 1, 1, ln_ws, device, s, G + lo.bo));
  // out projection: h1 = x + ctx Wo + bo
  SPAR_TRY(fork(2));
  SPAR_TRY(gemm(d, d, N, A.ctx, d, true, dres, d, false, G + lo.wo, d, true, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, w));
  SPAR_TRY(mark(1));  // dWo has read dres
  SPAR_TRY(gemm(N, d, d, dres, d, false, Wt + lo.wo, d, true, dtmp, d, false, SPAR_B200_EPI_NONE,
                nullptr, nullptr, 0, s, SPAR_B200_CAUSAL_NONE, 1, 1, nullptr, nullptr, nullptr,
                fused_attention));
  // attention core: dtmp = dctx [N, d] -> dqkv
  SPAR_TRY(attention_backward(A, s));
  const uint64_t ld = 3 * d;
  // Inverse RoPE on dq, dk (the fused attention kernels apply it in their epilogues).
  if (cfg.use_rope && !fused_attention)
    SPAR_TRY(rope_apply_launch(dqkv, rope_tab, N, T, 2 * H, dh, ld, 1, device, s));
  // QKV projection
  SPAR_TRY(fork(3));
  SPAR_TRY(gemm(d, 3 * d, N, A.a1, d, true, dqkv, ld, false, G + lo.wqkv, ld, true,
                SPAR_B200_EPI_NONE, nullptr, nullptr, 0, w));
  if (fused_attention && T % 32 == 0)  // partials left by the attention backward
    SPAR_TRY(column_sum_launch(G + lo.bqkv, colpart + blocks * F, blocks, 3 * d, 3 * d, 1, col_ws,
                               device, w));
  else
    SPAR_TRY(column_sum_launch(G + lo.bqkv, dqkv, N, 3 * d, ld, 1, col_ws, device, w));
  SPAR_TRY(mark(2));  // every product of this layer on the weight-gradient stream is done
  SPAR_TRY(gemm(N, d, 3 * d, dqkv, ld, false, Wt + lo.wqkv, ld, true, dtmp, d, false,
                SPAR_B200_EPI_NONE, nullptr, nullptr, 0, s));
  // dres += LN1 backward -> dL/dx = dL/d(previous block output): its column sums are the
  // previous block's b2 gradient (dWo read dres first)
  SPAR_TRY(join(1));
  SPAR_TRY(layernorm_backward_launch(dres, G + lo.ln1_g, G + lo.ln1_b, dtmp, A.x, P + lo.ln1_g,
                                     A.mean1, A.rstd1, N, d, 1, 1, ln_ws, device, s,
                                     l > 0 ? G + lay[l - 1].b2 : nullptr));
  // The next layer rewrites du and dqkv, and this layer's gradients are complete.
  SPAR_TRY(join(2));
  if (comm && last_micro) {
    // This layer's gradients are final: reduce them on the communication stream while the
    // remaining layers run backward (bucket = one block's contiguous parameter range).
    SPAR_TRY(reduce_buckets(L - 1 - l, L - l, static_cast<int>(l), layer_ev[l], s));
  }
  return cudaSuccess;
}

}  // namespace spar_b200

// ===================================================================================== C ABI
using namespace spar_b200;

namespace {
LMTrainer* as_trainer(void* h) { return static_cast<LMTrainer*>(h); }
}  // namespace

extern "C" SparCudaStatus spar_b200_lm_create(const SparB200LMConfig* config, int device,
                                              void** handle) {
  if (!config || !handle) return invalid();
  *handle = nullptr;
  LMTrainer* t = new LMTrainer();
  const SparCudaStatus st = t->init(*config, device);
  if (st.code != 0) {
    delete t;
    return st;
  }
  *handle = t;
  return ok();
}

extern "C" void spar_b200_lm_destroy(void* handle) { delete as_trainer(handle); }

extern "C" uint64_t spar_b200_lm_parameter_count(void* handle) {
  return handle ? as_trainer(handle)->named.size() : 0;
}

extern "C" uint64_t spar_b200_lm_flat_size(void* handle) {
  return handle ? as_trainer(handle)->flat : 0;
}

extern "C" float* spar_b200_lm_flat_buffer(void* handle, int which) {
  if (!handle || which < 0 || which > 3) return nullptr;
  LMTrainer* t = as_trainer(handle);
  return t->params + static_cast<uint64_t>(which) * t->flat;
}

extern "C" SparCudaStatus spar_b200_lm_parameter_info(void* handle, uint64_t index, char* name,
                                                      uint64_t name_capacity, uint64_t* rows,
                                                      uint64_t* cols) {
  if (!handle) return invalid();
  LMTrainer* t = as_trainer(handle);
  if (index >= t->named.size()) return invalid();
  const NamedTensor& n = t->named[index];
  if (name && name_capacity) {
    std::strncpy(name, n.name.c_str(), name_capacity - 1);
    name[name_capacity - 1] = 0;
  }
  if (rows) *rows = n.rows;
  if (cols) *cols = n.cols;
  return ok();
}

// which: 0 parameter, 1 gradient, 2 first moment, 3 second moment. Synchronous copy of one
// named tensor between host memory and its (possibly column-strided) place in the arena.
extern "C" SparCudaStatus spar_b200_lm_parameter_copy(void* handle, uint64_t index, int which,
                                                      int to_device, float* host) {
  if (!handle || !host || which < 0 || which > 3) return invalid();
  LMTrainer* t = as_trainer(handle);
  if (index >= t->named.size()) return invalid();
  const NamedTensor& n = t->named[index];
  // Sharded optimiser: other ranks' pieces are out of date until spar_b200_lm_gather.
  if (!to_device && t->stale[which]) return {1, static_cast<int>(cudaErrorNotReady)};
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  float* dev = t->params + static_cast<uint64_t>(which) * t->flat + n.offset;
  const uint64_t cols = n.cols ? n.cols : n.rows, rows = n.cols ? n.rows : 1;
  const uint64_t ld = n.cols ? n.ld : n.rows;
  cudaError_t e = cudaDeviceSynchronize();
  if (to_device && which == 0) t->wround_dirty = true;
  if (e == cudaSuccess) {
    if (to_device)
      e = cudaMemcpy2D(dev, ld * 4, host, cols * 4, cols * 4, rows, cudaMemcpyHostToDevice);
    else
      e = cudaMemcpy2D(host, cols * 4, dev, ld * 4, cols * 4, rows, cudaMemcpyDeviceToHost);
  }
  return e == cudaSuccess ? ok() : runtime(e);
}

// Device-side N(0, std) initialisation of every weight matrix and the embedding, drawing from one
// SplitMix64 stream in named-parameter order (the same stream the CPU oracle uses).
extern "C" SparCudaStatus spar_b200_lm_init_normal(void* handle, uint64_t seed, double std,
                                                   void* stream) {
  if (!handle) return invalid();
  LMTrainer* t = as_trainer(handle);
  t->wround_dirty = true;
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint64_t draws = 0;
  for (const auto& n : t->named) {
    if (!n.draws) continue;
    init_normal_kernel<<<grid_for(n.rows * n.cols, 256, sm_count(t->device) * 16), 256, 0, s>>>(
        t->params + n.offset, n.rows, n.cols, n.ld, seed, draws, std);
    draws += 2 * n.rows * n.cols;
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_lm_zero_grad(void* handle, void* stream) {
  if (!handle) return invalid();
  LMTrainer* t = as_trainer(handle);
  DeviceScope scope(t->device);
  cudaError_t e = cudaMemsetAsync(t->grads, 0, t->flat * sizeof(float),
                                  static_cast<cudaStream_t>(stream));
  // A new accumulation window: the error flags start clear.
  if (e == cudaSuccess)
    e = cudaMemsetAsync(t->flags, 0, 2 * sizeof(int32_t), static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) t->stale[1] = false;
  return e == cudaSuccess ? ok() : runtime(e);
}

// One micro-step: forward, loss, backward; gradients accumulate into the gradient arena.
// ids: device int32 [micro_batch, sequence_length]. grad_scale = upstream gradient of each row
// loss (1 / rows of the whole optimiser batch for Spar's mean reduction).
extern "C" SparCudaStatus spar_b200_lm_forward_backward(void* handle, const int32_t* ids,
                                                        uint64_t micro_index, float grad_scale,
                                                        int last_micro, void* stream) {
  if (!handle || !ids) return invalid();
  LMTrainer* t = as_trainer(handle);
  if (micro_index >= LMTrainer::kMaxMicro) return invalid();
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  t->last_micro = last_micro != 0;
  t->step_lanes = 1;  // a caller-driven micro-step always runs on lane 0
  t->comm_lane = 0;
  t->select_lane(0);
  // After a sharded train step: whole parameters and gradients (collective, like the step).
  cudaError_t e = t->gather_arena(0, static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = t->gather_arena(1, static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = t->refresh_rounded(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return runtime(e);
  return t->forward_backward(ids, grad_scale, micro_index, static_cast<cudaStream_t>(stream));
}

// Global-norm clip + AdamW over every parameter (decoupled decay on all, src/optim/adamw.cpp:
// 83-170); `step` is the 1-based AdamW step used for bias correction.
extern "C" SparCudaStatus spar_b200_lm_optimizer_step(void* handle, double learning_rate,
                                                      uint64_t step, void* stream) {
  if (!handle || step == 0) return invalid();
  LMTrainer* t = as_trainer(handle);
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Slice slice{t->params, t->grads, t->m1, t->m2, t->flat};
  cudaError_t e = cudaSuccess;
  for (int w = 0; w < 4 && e == cudaSuccess; ++w) e = t->gather_arena(w, s);  // whole arenas
  if (e != cudaSuccess) return runtime(e);
  t->launches += 3;
  e = grad_norm_launch(t->norm_state, &slice, 1, t->device, s, gemm_wait_flag(t->device),
                       attention_wait_flag(t->device));
  if (e == cudaSuccess)
    e = adamw_launch(&slice, 1, t->norm_state, t->cfg.max_grad_norm, learning_rate, t->cfg.beta1,
                     t->cfg.beta2, t->cfg.adam_epsilon, t->cfg.weight_decay, step, t->flags + 1,
                     t->device, s, nullptr, t->params, t->wround);
  return e == cudaSuccess ? ok() : runtime(e);
}

// A whole optimiser step: zero gradients, `micro_steps` forward/backward passes over
// ids[micro_steps, micro_batch, T] (host memory when ids_on_host, copied in this call), the
// data-parallel gradient reduction when a communicator is attached, clip + AdamW, then a
// device->host read of the mean loss, the pre-clip gradient norm and the error flags
// ([0] invalid token/target id, [1] non-finite gradient norm). Synchronises `stream`.
extern "C" SparCudaStatus spar_b200_lm_train_step(void* handle, const int32_t* ids,
                                                  int ids_on_host, uint64_t micro_steps,
                                                  double learning_rate, uint64_t step,
                                                  float* loss_out, double* grad_norm_out,
                                                  int32_t* flags_out, void* stream) {
  if (!handle || !ids || micro_steps == 0 || micro_steps > LMTrainer::kMaxMicro || step == 0)
    return invalid();
  LMTrainer* t = as_trainer(handle);
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t n_ids = micro_steps * t->N;
  cudaError_t e = cudaSuccess;
  // The step always reads its ids from ids_dev (fixed address, so a captured step replays).
  if (ids_on_host)
    e = cudaMemcpyAsync(t->ids_dev, ids, n_ids * sizeof(int32_t), cudaMemcpyHostToDevice, s);
  else if (ids != t->ids_dev)
    e = cudaMemcpyAsync(t->ids_dev, ids, n_ids * sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return runtime(e);
  const double rows = static_cast<double>(t->B) * static_cast<double>(t->T - 1) *
                      static_cast<double>(micro_steps) * static_cast<double>(t->world);
  const float grad_scale = static_cast<float>(1.0 / rows);
  e = t->refresh_rounded(s);  // host writes since the last step (eager, never in a graph)
  if (e != cudaSuccess) return runtime(e);
  if (!t->graphs_enabled || t->profiling || t->eager_steps == 0) {
    const SparCudaStatus st = t->step_body(micro_steps, grad_scale, learning_rate, step, s, false);
    if (st.code != 0) return st;
    ++t->eager_steps;
  } else {
    *t->opt_args_host = adamw_args(t->cfg.max_grad_norm, learning_rate, t->cfg.beta1,
                                   t->cfg.beta2, t->cfg.adam_epsilon, t->cfg.weight_decay, step);
    e = cudaMemcpyAsync(t->opt_args, t->opt_args_host, sizeof(AdamWArgs), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(t->ev_in, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(t->exec_stream, t->ev_in, 0);
    if (e != cudaSuccess) return runtime(e);
    auto it = t->graphs.find(micro_steps);
    if (it == t->graphs.end()) {
      const uint64_t before = t->launches;
      cudaGraph_t graph = nullptr;
      cudaGraphExec_t exec = nullptr;
      e = cudaStreamBeginCapture(t->exec_stream, cudaStreamCaptureModeThreadLocal);
      SparCudaStatus st = ok();
      if (e == cudaSuccess) st = t->step_body(micro_steps, grad_scale, learning_rate, step, t->exec_stream, true);
      const cudaError_t ce = cudaStreamEndCapture(t->exec_stream, &graph);
      if (e == cudaSuccess && st.code == 0 && ce == cudaSuccess && graph)
        e = cudaGraphInstantiate(&exec, graph, 0);
      else if (e == cudaSuccess)
        e = ce != cudaSuccess ? ce : cudaErrorStreamCaptureInvalidated;
      if (graph) cudaGraphDestroy(graph);
      const uint64_t captured = t->launches - before;
      t->launches = before;
      if (e != cudaSuccess || !exec) {
        // Capture did not work here (e.g. a library refused it): run this and later steps eagerly.
        cudaGetLastError();
        t->graphs_enabled = false;
        const SparCudaStatus es = t->step_body(micro_steps, grad_scale, learning_rate, step, s, false);
        if (es.code != 0) return es;
        goto done;
      }
      it = t->graphs.emplace(micro_steps, LMTrainer::StepGraph{exec, captured}).first;
    }
    e = cudaGraphLaunch(it->second.exec, t->exec_stream);
    if (e == cudaSuccess) e = cudaEventRecord(t->ev_out, t->exec_stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, t->ev_out, 0);
    if (e != cudaSuccess) return runtime(e);
    t->launches += it->second.launches;
  }
done:
  if (t->sharded && t->comm)  // only this rank's pieces were reduced and updated
    for (auto& st : t->stale) st = true;
  LMTrainer::StepResults* r = t->results_host;
  e = cudaMemcpyAsync(r->sums, t->loss_sums, micro_steps * sizeof(float), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(r->norm_state, t->norm_state, 2 * sizeof(double), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(r->flags, t->flags, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return runtime(e);
  if (t->comm) {
    // Bounded: a peer that left makes the step's collectives wait forever; the communicator is
    // then aborted and the step reports code 3 (the caller destroys the communicator).
    const SparCudaStatus w = comm_wait(t->comm, s);
    if (w.code == 3) {
      t->comm_aborted = true;
      t->drop_graphs();
    }
    if (w.code != 0) return w;
  } else if ((e = cudaStreamSynchronize(s)) != cudaSuccess) {
    return runtime(e);
  }
  const double* norm_state = r->norm_state;
  double total = 0.0;
  for (uint64_t m = 0; m < micro_steps; ++m) total += r->sums[m];
  if (loss_out) *loss_out = static_cast<float>(total / (rows / t->world));
  if (grad_norm_out) *grad_norm_out = std::sqrt(norm_state[0]);
  if (flags_out) {
    flags_out[0] = r->flags[0];
    flags_out[1] = r->flags[1];
  }
  // A GEMM or attention kernel of this step (on any rank) gave up one of its bounded waits: the
  // gradients are not trustworthy and AdamW updated nothing. The flags stay set until cleared
  // (spar_b200_gemm_error / spar_b200_attention_error with clear = 1), so later steps also refuse.
  if (norm_state[1] >= kWaitErrorMark) return runtime(cudaErrorTimeout);
  return ok();
}

// Attaches a communicator from spar_b200_comm_init: gradients of each block are then summed
// across ranks during the last micro-step's backward pass. A one-rank communicator is accepted
// (the bucket reductions then run as identities); comm == nullptr with world_size 1 detaches.
extern "C" SparCudaStatus spar_b200_lm_set_comm(void* handle, void* comm, int world_size) {
  if (!handle || world_size < 1 || (world_size > 1 && !comm)) return invalid();
  LMTrainer* t = as_trainer(handle);
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  // Arenas left sharded by the current communicator must be gathered through it first.
  if (t->comm != comm && (t->stale[0] || t->stale[1] || t->stale[2] || t->stale[3])) return invalid();
  if (t->comm != comm && !t->graphs.empty()) {  // captured steps hold the old reductions
    cudaError_t e = cudaDeviceSynchronize();
    t->drop_graphs();
    if (e != cudaSuccess) return runtime(e);
  }
  t->comm = comm;
  t->world = world_size;
  if (t->comm && !t->comm_stream) {
    cudaError_t e = cudaStreamCreateWithFlags(&t->comm_stream, cudaStreamNonBlocking);
    t->layer_ev.resize(t->L);
    for (auto& ev : t->layer_ev)
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&t->tail_ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&t->comm_done, cudaEventDisableTiming);
    for (int li = 0; li < t->lanes_alloc; ++li) {
      LMTrainer::Lane& ln = t->lanes[li];
      ln.layer_ev.resize(t->L);
      for (auto& ev : ln.layer_ev)
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ln.tail_ev, cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return runtime(e);
  }
  // Sharded optimiser: this rank's piece of every bucket (and the uneven tails, which every rank
  // updates; rank 0 alone counts them in the norm).
  t->sharded = t->comm && (t->shard_mode == 1 || (t->shard_mode < 0 && world_size > 1));
  if (t->sharded && comm_size(t->comm) != world_size) return invalid();
  t->rank = t->sharded ? comm_rank(t->comm) : 0;
  t->shard_plan.clear();
  t->own_slices.clear();
  t->norm_slices.clear();
  if (t->sharded) {
    cudaError_t e = cudaSuccess;
    if (!t->gather_fork) e = cudaEventCreateWithFlags(&t->gather_fork, cudaEventDisableTiming);
    while (e == cudaSuccess && t->gather_ev.size() < t->buckets.size()) {
      cudaEvent_t ev = nullptr;
      e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
      if (e == cudaSuccess) t->gather_ev.push_back(ev);
    }
    if (e != cudaSuccess) return runtime(e);
    auto slice = [t](uint64_t off, uint64_t count) {
      return Slice{t->params + off, t->grads + off, t->m1 + off, t->m2 + off, count};
    };
    for (const auto& bk : t->buckets) {
      const BucketShard b = shard_bucket(bk.first, bk.second, world_size, t->rank);
      t->shard_plan.push_back(b);
      if (b.shard) {
        t->own_slices.push_back(slice(b.own_off, b.shard));
        t->norm_slices.push_back(slice(b.own_off, b.shard));
      }
      if (b.rem_count) {
        t->own_slices.push_back(slice(b.rem_off, b.rem_count));
        if (t->rank == 0) t->norm_slices.push_back(slice(b.rem_off, b.rem_count));
      }
    }
  }
  return ok();
}

// ---------------------------------------------------------------- checkpoints (SPARCKPT v1)
namespace spar_b200 {
// Named tensors (name, shape) of a Spar-family config, in named-parameter order.
bool checkpoint_tensors(const SparB200LMConfig& c, std::vector<CkptTensor>& out) {
  if (c.family != SPAR_B200_FAMILY_SPAR) return false;
  ParamLayout pl;
  if (plan_params(c, pl).code != 0) return false;
  out.clear();
  for (const NamedTensor& n : pl.named)
    out.push_back({n.name, n.cols ? std::vector<uint64_t>{n.rows, n.cols}
                                  : std::vector<uint64_t>{n.rows}});
  return true;
}
}  // namespace spar_b200

namespace {
// Device arena `which` of every named tensor <-> contiguous host arrays.
cudaError_t stage_tensors(LMTrainer* t, int which, std::vector<std::vector<float>>& host,
                          bool to_device) {
  if (!to_device) host.assign(t->named.size(), {});
  for (size_t i = 0; i < t->named.size(); ++i) {
    const NamedTensor& n = t->named[i];
    const uint64_t cols = n.cols ? n.cols : n.rows, rows = n.cols ? n.rows : 1;
    const uint64_t ld = n.cols ? n.ld : n.rows;
    float* dev = t->params + static_cast<uint64_t>(which) * t->flat + n.offset;
    if (!to_device) host[i].resize(rows * cols);
    const cudaError_t e =
        to_device ? cudaMemcpy2D(dev, ld * 4, host[i].data(), cols * 4, cols * 4, rows,
                                 cudaMemcpyHostToDevice)
                  : cudaMemcpy2D(host[i].data(), cols * 4, dev, ld * 4, cols * 4, rows,
                                 cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

std::vector<const float*> cptrs(const std::vector<std::vector<float>>& h) {
  std::vector<const float*> p;
  for (const auto& x : h) p.push_back(x.data());
  return p;
}
std::vector<float*> ptrs(std::vector<std::vector<float>>& h) {
  std::vector<float*> p;
  for (auto& x : h) p.push_back(x.data());
  return p;
}
}  // namespace

extern "C" SparCudaStatus spar_b200_lm_save_checkpoint(void* handle, const char* path,
                                                       const SparB200Checkpoint* meta) {
  if (!handle || !meta) return invalid();
  LMTrainer* t = as_trainer(handle);
  if (t->family != SPAR_B200_FAMILY_SPAR) return invalid();
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaError_t e = cudaDeviceSynchronize();
  for (int w : {0, 2, 3})  // sharded optimiser: whole parameters and moments (collective)
    if (e == cudaSuccess) e = t->gather_arena(w, nullptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return runtime(e);
  if (!path) return ok();
  std::vector<std::vector<float>> p, m, v;
  e = stage_tensors(t, 0, p, false);
  if (e == cudaSuccess && meta->adam_step) e = stage_tensors(t, 2, m, false);
  if (e == cudaSuccess && meta->adam_step) e = stage_tensors(t, 3, v, false);
  if (e != cudaSuccess) return runtime(e);
  const auto pp = cptrs(p), mp = cptrs(m), vp = cptrs(v);
  return checkpoint_write(path, t->cfg, *meta, pp.data(), meta->adam_step ? mp.data() : nullptr,
                          meta->adam_step ? vp.data() : nullptr);
}

extern "C" SparCudaStatus spar_b200_lm_load_checkpoint(void* handle, const char* path,
                                                       SparB200Checkpoint* meta) {
  if (!handle || !path || !meta) return invalid();
  LMTrainer* t = as_trainer(handle);
  if (t->family != SPAR_B200_FAMILY_SPAR) return invalid();
  std::vector<std::vector<float>> p(t->named.size()), m(t->named.size()), v(t->named.size());
  for (size_t i = 0; i < t->named.size(); ++i) {
    const NamedTensor& n = t->named[i];
    const uint64_t numel = n.cols ? n.rows * n.cols : n.rows;
    p[i].resize(numel);
    m[i].resize(numel);
    v[i].resize(numel);
  }
  auto pp = ptrs(p), mp = ptrs(m), vp = ptrs(v);
  const SparCudaStatus st = checkpoint_read(path, t->cfg, *meta, pp.data(), mp.data(), vp.data());
  if (st.code != 0) return st;
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaError_t e = cudaDeviceSynchronize();
  t->wround_dirty = true;
  if (e == cudaSuccess) e = stage_tensors(t, 0, p, true);
  if (e == cudaSuccess) e = stage_tensors(t, 2, m, true);
  if (e == cudaSuccess) e = stage_tensors(t, 3, v, true);
  if (e != cudaSuccess) return runtime(e);
  for (int w : {0, 2, 3}) t->stale[w] = false;  // every rank loads the whole state
  return ok();
}

// Sharded optimiser: gathers every rank's pieces of arena `which` (0 parameters, 1 gradients,
// 2 first moments, 3 second moments) onto every rank, ordered on `stream` (which waits for it).
// After a sharded train step the arenas hold only this rank's pieces up to date; this call (made
// by every rank, in the same order) brings one whole arena up to date for reading. No-op when the
// arena is current or the optimiser is not sharded.
extern "C" SparCudaStatus spar_b200_lm_gather(void* handle, int which, void* stream) {
  if (!handle || which < 0 || which > 3) return invalid();
  LMTrainer* t = as_trainer(handle);
  DeviceScope scope(t->device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = t->gather_arena(which, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : runtime(e);
}

// Mean loss of the micro-steps run since the last train step (host read, synchronous).
extern "C" SparCudaStatus spar_b200_lm_read_losses(void* handle, float* host, uint64_t count) {
  if (!handle || !host || count > LMTrainer::kMaxMicro) return invalid();
  LMTrainer* t = as_trainer(handle);
  DeviceScope scope(t->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(host, t->loss_sums, count * 4, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? ok() : runtime(e);
}

// Warmup-cosine learning rate (training::warmup_cosine_learning_rate,
// src/training/schedule.cpp:9-38). Returns NaN for an invalid configuration.
extern "C" double spar_b200_warmup_cosine(double peak, double minimum, uint64_t warmup_steps,
                                          uint64_t decay_steps, uint64_t completed_steps) {
  if (!std::isfinite(peak) || peak < 0.0 || !std::isfinite(minimum) || minimum < 0.0 ||
      minimum > peak || decay_steps == 0)
    return NAN;
  if (completed_steps < warmup_steps)  // progress first, then scale (schedule.cpp:25-27)
    return peak * (static_cast<double>(completed_steps + 1) / static_cast<double>(warmup_steps));
  const uint64_t idx = completed_steps - warmup_steps;
  if (idx >= decay_steps || decay_steps == 1) return minimum;
  const double progress = static_cast<double>(idx) / static_cast<double>(decay_steps - 1);
  return minimum + 0.5 * (peak - minimum) * (1.0 + std::cos(M_PI * progress));
}

// Enables (1) or disables (0) event timing of every tensor-core GEMM launch; enabling resets the
// accumulators and the launch counter.
extern "C" SparCudaStatus spar_b200_lm_profile(void* handle, int enable) {
  if (!handle) return invalid();
  LMTrainer* t = as_trainer(handle);
  t->profiling = enable != 0;
  if (enable) {
    t->ev_used = 0;
    t->ev_flops.clear();
    t->launches = 0;
  }
  return ok();
}

// Synchronises, then reports the summed device time (ms) and algorithmic FLOPs of the GEMM
// launches timed since profiling was enabled, and the number of kernels launched.
extern "C" SparCudaStatus spar_b200_lm_profile_read(void* handle, double* gemm_ms,
                                                    double* gemm_flops, uint64_t* gemm_launches,
                                                    uint64_t* kernel_launches) {
  if (!handle) return invalid();
  LMTrainer* t = as_trainer(handle);
  DeviceScope scope(t->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return runtime(e);
  double ms = 0.0, fl = 0.0;
  for (size_t i = 0; i < t->ev_used; ++i) {
    float x = 0.f;
    e = cudaEventElapsedTime(&x, t->ev_pool[i].first, t->ev_pool[i].second);
    if (e != cudaSuccess) return runtime(e);
    ms += x;
    fl += t->ev_flops[i];
  }
  if (gemm_ms) *gemm_ms = ms;
  if (gemm_flops) *gemm_flops = fl;
  if (gemm_launches) *gemm_launches = t->ev_used;
  if (kernel_launches) *kernel_launches = t->launches;
  return ok();
}

// ------------------------------------------------------------ host-only layout queries (no GPU)
extern "C" SparCudaStatus spar_b200_lm_layout(const SparB200LMConfig* config, uint64_t* flat_size,
                                              uint64_t* num_tensors, uint64_t* num_buckets) {
  if (!config) return invalid();
  ParamLayout pl;
  const SparCudaStatus st = plan_params(*config, pl);
  if (st.code) return st;
  if (flat_size) *flat_size = pl.flat;
  if (num_tensors) *num_tensors = pl.named.size();
  if (num_buckets) *num_buckets = pl.buckets().size();
  return ok();
}

extern "C" SparCudaStatus spar_b200_lm_layout_tensor(const SparB200LMConfig* config, uint64_t index,
                                                     char* name, uint64_t name_capacity,
                                                     uint64_t* offset, uint64_t* rows,
                                                     uint64_t* cols, uint64_t* ld) {
  if (!config || !name || name_capacity == 0) return invalid();
  ParamLayout pl;
  const SparCudaStatus st = plan_params(*config, pl);
  if (st.code) return st;
  if (index >= pl.named.size()) return invalid();
  const NamedTensor& t = pl.named[index];
  if (t.name.size() + 1 > name_capacity) return invalid();
  memcpy(name, t.name.c_str(), t.name.size() + 1);
  if (offset) *offset = t.offset;
  if (rows) *rows = t.rows;
  if (cols) *cols = t.cols;
  if (ld) *ld = t.ld;
  return ok();
}

extern "C" SparCudaStatus spar_b200_lm_layout_bucket(const SparB200LMConfig* config, uint64_t index,
                                                     uint64_t* offset, uint64_t* count) {
  if (!config || !offset || !count) return invalid();
  ParamLayout pl;
  const SparCudaStatus st = plan_params(*config, pl);
  if (st.code) return st;
  const auto b = pl.buckets();
  if (index >= b.size()) return invalid();
  *offset = b[index].first;
  *count = b[index].second;
  return ok();
}

extern "C" SparCudaStatus spar_b200_lm_layout_shard(const SparB200LMConfig* config, uint64_t index,
                                                    int world, int rank, uint64_t* own_offset,
                                                    uint64_t* shard, uint64_t* tail_offset,
                                                    uint64_t* tail_count) {
  if (!config || !own_offset || !shard || !tail_offset || !tail_count || world < 1 || rank < 0 ||
      rank >= world)
    return invalid();
  ParamLayout pl;
  const SparCudaStatus st = plan_params(*config, pl);
  if (st.code) return st;
  const auto b = pl.buckets();
  if (index >= b.size()) return invalid();
  const BucketShard s = shard_bucket(b[index].first, b[index].second, world, rank);
  *own_offset = s.own_off;
  *shard = s.shard;
  *tail_offset = s.rem_off;
  *tail_count = s.rem_count;
  return ok();
}
