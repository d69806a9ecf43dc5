// Fused causal self-attention on the sm_100a tensor cores: tcgen05.mma kind::tf32 with TMEM
// accumulators, operands staged in shared memory by TMA, the softmax done by the warps that read
// the score tile out of TMEM. The [T, T] score and probability matrices never reach HBM.
//
// This computes what Spar's scaled_dot_product_attention does (src/nn/attention.cpp:121-135:
// scores = (Q K^T) * 1/sqrt(head_dim), causal -inf mask, softmax over the last axis, P V) and its
// autograd backward (matmul / softmax backward), for the packed projection buffer
// qkv [batch, seq, (heads + 2 kv_heads) * head_dim] (Q | K | V, head h at columns h*head_dim of
// each part). With kv_heads < heads (grouped-query attention, repeat_kv_heads of
// src/nn/attention.cpp:77-94) query head h reads key / value head h / (heads / kv_heads); the key
// kernel's items are (batch, key/value head, key tile) and sweep every query head of the group,
// so dK / dV come out summed over the group without the repeated heads ever existing.
//
// Forward (one CTA per SM, persistent; work item = (batch, head, query tiles t and T-1-t), so
// every item costs the same T+1 key-tile products): the two query tiles alternate on the tensor
// cores, S_X = Q_X K_j^T and O_X += P_X V_j, while four softmax warps per tile turn S into
// P = exp2(S * scale * log2(e) - m) in TMEM (the A operand of the P V product). m is a running
// row maximum that only moves, with O and the row sum rescaled, when a tile exceeds it by more
// than 8 (log2 units). m and 1 / row sum are saved for the backward.
// Backward (deterministic: every gradient element is written by exactly one CTA, no atomics):
//   D = rowsum(dO o O) per (row, head) first, by a small streaming kernel.
//   query kernel  per (batch, head, 128-query tile): for each 64-key tile S, dP = dO V^T,
//                 P recomputed from the saved statistics, dS = P o (dP - D) * scale, dQ += dS K.
//   key kernel    per (batch, head, 128-key tile): for each 64-query tile S^T = K Q^T,
//                 dP^T = V dO^T, P^T and dS^T as above, dV += P^T dO, dK += dS^T Q.
// Warp roles in every kernel: warp 0 TMA producer, warp 1 MMA issuer (one elected thread),
// warps 2-9 softmax / epilogue: TMEM lane = tile row (warp w reads lanes 32*(w%4)..+31), and the
// two warps of each lane quarter split the tile's columns. They exchange row partials through
// shared memory, synchronised by an mbarrier with a bounded wait (never bar.sync, which cannot
// time out if a partner warp gave up).
// Every wait is bounded (2 s) and records an error flag instead of hanging.
//
// Precision: products are TF32 with fp32 accumulation. The operands the kernels write themselves
// (P, dS) are rounded to nearest TF32; Q, K, V and dO are read as stored, so the tensor cores drop
// their low 13 mantissa bits (truncation) unless the producer stored them rounded to nearest
// (the training runtime does: QKV projection + RoPE outputs and d ctx are stored TF32-rounded).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <queue>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace spar_b200 {

__device__ int g_attn_error = 0;

namespace {

constexpr int kSoftWarps = 8;  // two column groups x four TMEM lane quarters
constexpr int kThreads = 64 + 32 * kSoftWarps;
constexpr uint32_t kMaxSmem = 232448;  // per-CTA dynamic shared memory limit
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnParams {
  CUtensorMap qk128;   // qkv, K-major boxes {32 cols, 128 rows}
  CUtensorMap qk64;    // qkv, K-major boxes {32, 64}
  CUtensorMap qkv_mn;  // qkv, MN-major boxes {32, 32}
  CUtensorMap do128;   // dO (= d ctx), K-major {32, 128}
  CUtensorMap do64;    // dO, K-major {32, 64}
  CUtensorMap do_mn;   // dO, MN-major {32, 32}
  CUtensorMap out;     // output store boxes {32, 32}: ctx (forward) or dqkv (backward)
  const float* o;      // forward output (backward: D = rowsum(dO o O))
  float* o_out;        // forward: where the output is stored
  const float* d_o;    // dO
  float* row_max;      // [batch*heads, seq]: max of scores * scale * log2(e)
  float* row_inv;      // [batch*heads, seq]: 1 / sum of exponentials
  float* delta;        // [batch*heads, seq]: D
  const float2* rope;  // optional RoPE table [seq, head_dim / 2]: dQ, dK leave inverse-rotated
  uint32_t heads, seq, model_dim, bh;
  // Grouped-query attention (repeat_kv_heads, src/nn/attention.cpp:77-94): query head h reads
  // key / value head h / group; K and V start at columns kcol and vcol of each qkv / dqkv row
  // (group 1: kcol = model_dim, vcol = 2 * model_dim).
  uint32_t group, kv_heads, kv_bh, kcol, vcol;
  // Backward work lists: CTA c processes items sched[sched[c] .. sched[c + 1]) of the item array
  // at sched + grid + 1 (an item idx decodes as tile idx / bh, (batch, head) idx % bh); built on
  // the host by longest-processing-time-first over the items' costs (see backward_schedule).
  const uint32_t* sched;
  uint32_t sched_grid;
  uint64_t ld_o;  // row stride of O and dO
  float scale, scale_log2;
  uint32_t tiles;  // stationary tiles per (batch, head)
  uint32_t adjacent_pairs;  // forward: items pair query tiles (2p, 2p+1), heaviest first
  // Forward, balanced pairs only: the pairs of one (batch, head) are consecutive items, so the
  // CTAs running at the same time share that head's K / V tiles through L2 (otherwise the items of
  // one pair index run together over every head and each K / V tile is fetched once per pair).
  uint32_t head_major;
  uint32_t total;  // work items
  uint32_t round_out;  // store ctx / dqkv rounded to nearest TF32 (they only feed TF32 products)
  // Backward, optional (seq a multiple of 32): per 32-row block column sums of dqkv (the qkv
  // bias gradient's partials), [batch * seq / 32, width of a packed row].
  float* colpart;
  uint32_t colpart_ld;
};

__device__ __forceinline__ void record_error() { atomicExch(&g_attn_error, 1); }

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Byte offset of 16-byte chunk c of row r in a K-major operand block stored with the 128-byte
// swizzle (rows of 128 B = 32 fp32; chunk index XOR the row's low three bits).
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * 128 + ((c ^ (r & 7)) << 4);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// K-major operand (rows of 32 fp32 per 128-byte swizzle row, 32-column blocks `block_bytes`
// apart), K step ks of 8 elements.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, uint32_t block_bytes, int ks) {
  return tc::smem_desc(base + (ks >> 2) * block_bytes + (ks & 3) * 32, 16, 1024, tc::kLayoutSw128);
}

// MN-major operand stored as 32-row K blocks of DH/32 boxes {32 MN, 32 K} (4 KB each).
template <int DH>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int ks) {
  return tc::smem_desc(base + (ks >> 2) * (DH / 32) * 4096 + (ks & 3) * 1024, 4096, 512,
                       tc::kLayoutSw128Base32);
}

// Writes 32 fp32 values (columns c*32..c*32+31 of row r) into a K-major swizzled block.
__device__ __forceinline__ void store_row32(uint8_t* block, uint32_t r, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
    *reinterpret_cast<float4*>(block + swz(r, i)) =
        make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// Rotates 16 (x0, x1) column pairs back by their RoPE angles: (x0 c + x1 s, x1 c - x0 s), the
// transpose of the forward rotation (src/nn/rope.cpp:35-66), so a gradient with respect to
// rotated q / k becomes the gradient with respect to the unrotated projection.
__device__ __forceinline__ void inverse_rope(float (&o)[32], const float2* tab) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 cs = __ldg(tab + i);
    const float x0 = o[2 * i], x1 = o[2 * i + 1];
    o[2 * i] = x0 * cs.x + x1 * cs.y;
    o[2 * i + 1] = x1 * cs.x - x0 * cs.y;
  }
}

struct Item {
  uint32_t b, h, t;
};

// Backward item list of this CTA: [begin, end) into the schedule, and the k-th item there.
__device__ __forceinline__ uint32_t sched_begin(const AttnParams& p) { return p.sched[blockIdx.x]; }
__device__ __forceinline__ uint32_t sched_end(const AttnParams& p) { return p.sched[blockIdx.x + 1]; }
__device__ __forceinline__ uint32_t sched_item(const AttnParams& p, uint32_t k) {
  return p.sched[p.sched_grid + 1 + k];
}

// Key-side items of the backward: (batch, key/value head, 128-key tile).
__device__ __forceinline__ Item decode_kv(const AttnParams& p, uint32_t idx) {
  const uint32_t tile = idx / p.kv_bh;
  const uint32_t bh = idx - tile * p.kv_bh;
  Item it;
  it.b = bh / p.kv_heads;
  it.h = bh - it.b * p.kv_heads;
  it.t = tile;
  return it;
}

__device__ __forceinline__ Item decode(const AttnParams& p, uint32_t idx, bool descending) {
  const uint32_t tile = idx / p.bh;
  const uint32_t bh = idx - tile * p.bh;
  Item it;
  it.b = bh / p.heads;
  it.h = bh - it.b * p.heads;
  it.t = descending ? p.tiles - 1 - tile : tile;
  return it;
}

// Column sums of one stored 32 x 32 box of dqkv (before rounding) into the partials array.
__device__ __forceinline__ void box_partials(const AttnParams& p, const float (&v)[32], int col,
                                             int row, int b) {
  if (!p.colpart || static_cast<uint32_t>(row) >= p.seq) return;
  const float cs = box_column_sum(v, true);
  const uint64_t block = (static_cast<uint64_t>(b) * p.seq + static_cast<uint32_t>(row)) / 32;
  p.colpart[block * p.colpart_ld + static_cast<uint32_t>(col) + (threadIdx.x & 31)] = cs;
}

__device__ __forceinline__ void round_box(float (&v)[32]) {
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = round_tf32(v[e]);
}

// Stages one 32-row x 32-column fp32 box (this warp's rows) and stores it through `map`.
__device__ __forceinline__ void store_box(const CUtensorMap* map, uint8_t* buf, const float (&v)[32],
                                          int col, int row, int b) {
  const uint32_t lane = threadIdx.x & 31;
  store_row32(buf, lane, v);
  tc::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) tc::tma_store_4d(map, buf, col, row, b, 0);
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (tc::mbar_wait(bar, parity)) return true;
  record_error();
  *abort = 1;
  return false;
}

// Rendezvous of the softmax warps (mbarrier with kSoftWarps arrivals, bounded wait). Shared
// memory written before it is visible to every softmax thread after it.
__device__ __forceinline__ bool soft_sync(uint64_t* bar, uint32_t& phase, volatile int* abort) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) tc::mbar_arrive(bar);
  const bool ok = wait_or_abort(bar, phase, abort);
  phase ^= 1;
  return ok;
}

// Identity of a softmax thread: tile row r (= TMEM lane), column group, lane quarter.
struct SoftThread {
  uint32_t quarter, grp, r, lanes;
  __device__ SoftThread(int warp, int lane, uint32_t tmem) {
    quarter = warp & 3;
    grp = (warp - 2) >> 2;
    r = quarter * 32 + lane;
    lanes = tmem + ((quarter * 32) << 16);
  }
};

// Round to nearest TF32 (ties away from zero) a value that only feeds the tensor cores: one
// conversion instruction (the MMA reads the upper 19 bits).
__device__ __forceinline__ uint32_t tf32_operand(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}

// Running maxima of 64 score columns (c0 .. c0+63 of the row) into eight accumulators; on the
// diagonal key tile only columns <= r (the query row) count.
template <bool kDiag>
__device__ __forceinline__ void row_max64(const uint32_t (&v0)[32], const uint32_t (&v1)[32],
                                          uint32_t c0, uint32_t r, float (&mxs)[8]) {
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    if (!kDiag || c0 + e <= r) mxs[e & 7] = fmaxf(mxs[e & 7], __uint_as_float(v0[e]));
    if (!kDiag || c0 + 32 + e <= r) mxs[e & 7] = fmaxf(mxs[e & 7], __uint_as_float(v1[e]));
  }
}

// P = exp2(S * scale_log2 - m) over 64 columns in place (as TF32 operands), adding the unrounded
// values into four partial sums; masked columns of the diagonal tile become 0.
template <bool kDiag>
__device__ __forceinline__ void probs64(uint32_t (&v0)[32], uint32_t (&v1)[32], float scale_log2,
                                        float m, uint32_t c0, uint32_t r, float (&sums)[4]) {
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    float p0 = ex2(fmaf(__uint_as_float(v0[e]), scale_log2, -m));
    float p1 = ex2(fmaf(__uint_as_float(v1[e]), scale_log2, -m));
    if (kDiag && c0 + e > r) p0 = 0.f;
    if (kDiag && c0 + 32 + e > r) p1 = 0.f;
    sums[e & 3] += p0 + p1;
    v0[e] = tf32_operand(p0);
    v1[e] = tf32_operand(p1);
  }
}

// ============================================================================ forward
// Work item = (batch, head, pair of query tiles): t and T-1-t (T+1 key-tile products per item,
// the same for every item, so the causal triangle balances across SMs at any batch), or, with
// at least four items per SM, the adjacent tiles 2q and 2q+1 heaviest first (the two tiles' key
// counts differ by one, so both softmax groups work side by side for the whole item).
// Four softmax warps per query tile (thread = query row, all 128 scores of its row).
// The item is a list of jobs: for each key tile j, (A, j) while j <= t, then (B, j). Job g
// (counted over the CTA's items) computes S = Q_X K_j^T into TMEM score buffer g % 3, its
// softmax warps overwrite S with P there, and O_X += P V_j reads it. With three buffers the
// MMA warp runs up to three S products ahead of the P V products, so a tile's next scores are
// ready when its softmax warps finish, including the stretch where only tile B has keys left.
// One pass over the keys with a running maximum per row: P = exp2(S * scale * log2(e) - m), m the
// maximum in use. m moves (O and the row sum are rescaled by exp2(m_old - m_new)) only when a
// tile's maximum exceeds it by more than 8, so P <= 2^8 and rescaling is rare. The saved
// statistics are that m and 1 / sum, which give the normalised probabilities exactly as the
// backward recomputes them.
template <int DH>
struct Fwd {
  static constexpr uint32_t kTile = DH * 512;  // 128 rows x DH fp32
  // head_dim 64: two K and three V stages (V_j is read last, by the P V products, so its stage
  // frees latest); measured against three K and two V stages: 122.9 vs 124.7 us at 16 sequences,
  // 21.2 vs 22.5 us at 2 (C5 widths).
  static constexpr uint32_t kKStages = DH == 64 ? 2 : 4;
  static constexpr uint32_t kVStages = DH == 64 ? 3 : 2;
  static constexpr uint32_t kQ = 0;  // [2] query tiles A, B
  static constexpr uint32_t kK = kQ + 2 * kTile;
  static constexpr uint32_t kV = kK + kKStages * kTile;
  static constexpr uint32_t kBar = kV + kVStages * kTile;
  static constexpr uint32_t kSmem = kBar + 320 + 1024;
  static_assert(kSmem <= kMaxSmem, "forward shared memory");
};

constexpr float kRescaleLog2 = 8.f;  // move the running maximum only past this margin
constexpr uint32_t kSBufs = 3;       // TMEM score / probability buffers (128 columns each)

// The item's two query tiles: A = t (absent when it equals B, the middle tile of an odd count)
// and B = T-1-t; nA, nB key tiles each.
struct PairItem {
  uint32_t b, h, ta, tb, na, nb;
};

__device__ __forceinline__ PairItem decode_pair(const AttnParams& p, uint32_t idx) {
  uint32_t pair, bh;
  if (p.head_major) {
    const uint32_t pairs = (p.tiles + 1) / 2;
    bh = idx / pairs;
    pair = idx - bh * pairs;
  } else {
    pair = idx / p.bh;
    bh = idx - pair * p.bh;
  }
  PairItem it;
  it.b = bh / p.heads;
  it.h = bh - it.b * p.heads;
  if (p.adjacent_pairs) {
    // Tiles 2q and 2q+1 (q = the pair counted from the end, so the heaviest items come first):
    // the two tiles' key counts differ by one, so both softmax groups stay busy until the last
    // key tile. Used when there are enough items per SM to balance their unequal sizes.
    const uint32_t q = (p.tiles + 1) / 2 - 1 - pair;
    it.ta = 2 * q;
    it.tb = min(2 * q + 1, p.tiles - 1);
  } else {  // tiles t and T-1-t: every item the same T+1 key tiles (balanced at any batch)
    it.ta = pair;
    it.tb = p.tiles - 1 - pair;
  }
  it.na = it.ta != it.tb ? it.ta + 1 : 0;
  it.nb = it.tb + 1;
  return it;
}

// Job i of an item: (A, i / 2) and (B, i / 2) alternate while A has keys, then (B, i - nA).
__device__ __forceinline__ void job_of(const PairItem& it, uint32_t i, uint32_t& x, uint32_t& j) {
  if (i < 2 * it.na) {
    x = i & 1;
    j = i >> 1;
  } else {
    x = 1;
    j = i - it.na;
  }
}

__device__ __forceinline__ uint32_t job_index(const PairItem& it, uint32_t x, uint32_t j) {
  return x == 0 ? 2 * j : (j < it.na ? 2 * j + 1 : it.na + j);
}

// TMEM columns: score / probability buffers at 0, 128, 256; O of tile X at 384 + X * 64.
template <int DH>
__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ AttnParams p) {
  using L = Fwd<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;     // [2]
  uint64_t* q_empty = bars + 2;    // [2]
  uint64_t* o_pv = bars + 4;       // [2] an O_X += P V product finished
  uint64_t* o_full = bars + 6;     // [2]
  uint64_t* o_empty = bars + 8;    // [2]
  // [2 tiles][3 buffers] scores of tile X in the buffer. Per tile: a tile's softmax warps can be
  // many jobs (several uses of a buffer by the other tile) past their previous job, so a
  // barrier shared by both tiles could complete two phases between their waits.
  uint64_t* s_full = bars + 10;
  // bars + 16 .. 18: unused (buffer reuse needs no barrier, see the MMA issuer)
  uint64_t* p_full = bars + 19;    // [3] probabilities in buffer
  uint64_t* drain = bars + 22;
  uint64_t* k_full = bars + 23;                      // [kKStages]
  uint64_t* k_empty = k_full + L::kKStages;          // [kKStages]
  uint64_t* v_full = k_empty + L::kKStages;          // [kVStages]
  uint64_t* v_empty = v_full + L::kVStages;          // [kVStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_empty + L::kVStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int x = 0; x < 2; ++x) {
      tc::mbar_init(q_full + x, 1);
      tc::mbar_init(q_empty + x, 1);
      tc::mbar_init(o_pv + x, 1);
      tc::mbar_init(o_full + x, 1);
      tc::mbar_init(o_empty + x, 4);
    }
    for (uint32_t b = 0; b < kSBufs; ++b) {
      tc::mbar_init(s_full + b, 1);
      tc::mbar_init(s_full + kSBufs + b, 1);
      tc::mbar_init(p_full + b, 4);
    }
    tc::mbar_init(drain, 1);
    for (uint32_t i = 0; i < L::kKStages; ++i) {
      tc::mbar_init(k_full + i, 1);
      tc::mbar_init(k_empty + i, 1);
    }
    for (uint32_t i = 0; i < L::kVStages; ++i) {
      tc::mbar_init(v_full + i, 1);
      tc::mbar_init(v_empty + i, 1);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_begin();  // set-up done; global memory from here on

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    if (tc::elect_one()) {
      tc::tma_prefetch(&p.qk128);
      tc::tma_prefetch(&p.qkv_mn);
      uint32_t kn = 0, vn = 0, qn[2] = {0, 0};
      int last_q[2] = {-1, -1}, last_k[L::kKStages], last_v[L::kVStages];
      for (uint32_t i = 0; i < L::kKStages; ++i) last_k[i] = -1;
      for (uint32_t i = 0; i < L::kVStages; ++i) last_v[i] = -1;
      for (uint32_t idx = blockIdx.x; idx < p.total && !*abort_flag; idx += gridDim.x) {
        const PairItem it = decode_pair(p, idx);
        const int hc = static_cast<int>(it.h * DH), b = static_cast<int>(it.b);
        const int kvc = static_cast<int>(it.h / p.group * DH);
        const int kc = static_cast<int>(p.kcol) + kvc, vc = static_cast<int>(p.vcol) + kvc;
        bool ok = true;
        for (int x = it.na ? 0 : 1; x < 2 && ok; ++x) {
          const uint32_t t = x ? it.tb : it.ta;
          if (!(ok = wait_or_abort(q_empty + x, (qn[x] & 1) ^ 1, abort_flag))) break;
          tc::mbar_arrive_expect_tx(q_full + x, L::kTile);
          last_q[x] = qn[x] & 1;
          ++qn[x];
#pragma unroll
          for (int c = 0; c < DH / 32; ++c)
            tc::tma_load_4d(smem + L::kQ + x * L::kTile + c * 16384, &p.qk128, q_full + x,
                            hc + 32 * c, static_cast<int>(t * 128), b, 0);
        }
        if (!ok) break;
        for (uint32_t j = 0; j < it.nb && !*abort_flag; ++j) {
          const int row = static_cast<int>(j * 128);
          {
            const uint32_t st = kn % L::kKStages, ph = (kn / L::kKStages) & 1;
            if (!wait_or_abort(k_empty + st, ph ^ 1, abort_flag)) break;
            tc::mbar_arrive_expect_tx(k_full + st, L::kTile);
            last_k[st] = static_cast<int>(ph);
#pragma unroll
            for (int c = 0; c < DH / 32; ++c)
              tc::tma_load_4d(smem + L::kK + st * L::kTile + c * 16384, &p.qk128, k_full + st,
                              kc + 32 * c, row, b, 0);
            ++kn;
          }
          {
            const uint32_t st = vn % L::kVStages, ph = (vn / L::kVStages) & 1;
            if (!wait_or_abort(v_empty + st, ph ^ 1, abort_flag)) break;
            tc::mbar_arrive_expect_tx(v_full + st, L::kTile);
            last_v[st] = static_cast<int>(ph);
#pragma unroll
            for (int kb = 0; kb < 4; ++kb)
#pragma unroll
              for (int c = 0; c < DH / 32; ++c)
                tc::tma_load_4d(smem + L::kV + st * L::kTile + (kb * (DH / 32) + c) * 4096,
                                &p.qkv_mn, v_full + st, vc + 32 * c, row + 32 * kb, b, 0);
            ++vn;
          }
        }
      }
      // Every load issued must have landed before the CTA exits.
      for (int x = 0; x < 2; ++x)
        if (last_q[x] >= 0 && !tc::mbar_wait(q_full + x, last_q[x])) record_error();
      for (uint32_t s = 0; s < L::kKStages; ++s)
        if (last_k[s] >= 0 && !tc::mbar_wait(k_full + s, last_k[s])) record_error();
      for (uint32_t s = 0; s < L::kVStages; ++s)
        if (last_v[s] >= 0 && !tc::mbar_wait(v_full + s, last_v[s])) record_error();
    }
    __syncwarp();
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (tc::elect_one()) {
      const uint32_t idesc_s = tc::idesc_tf32(128, 128, 0, 0);
      const uint32_t idesc_o = tc::idesc_tf32(128, DH, 0, 1);
      const uint32_t q_addr = tc::smem_u32(smem + L::kQ);
      const uint32_t k_addr = tc::smem_u32(smem + L::kK);
      const uint32_t v_addr = tc::smem_u32(smem + L::kV);
      uint32_t kn = 0, vn = 0, qn[2] = {0, 0}, on[2] = {0, 0}, gbase = 0;
      bool ok = true;
      for (uint32_t idx = blockIdx.x; idx < p.total && ok && !*abort_flag; idx += gridDim.x) {
        const PairItem it = decode_pair(p, idx);
        const uint32_t n[2] = {it.na, it.nb};
        const uint32_t njobs = it.na + it.nb;
        for (int x = it.na ? 0 : 1; x < 2 && ok; ++x) {
          ok = wait_or_abort(q_full + x, qn[x] & 1, abort_flag);
          ++qn[x];
        }
        int k_ready = -1, v_ready = -1;  // key tiles whose K / V stage has been waited for
        uint32_t is = 0;                 // S jobs issued (P V jobs: ip)
        for (uint32_t ip = 0; ip < njobs && ok; ++ip) {
          // S jobs up to three ahead: job g reuses the buffer of job g - 3, whose P V product
          // this thread issued before (S(g) is issued once ip > g - 3). The tensor core runs
          // one thread's tcgen05.mma operations in issue order, so that product reads P before
          // S(g) overwrites it: no wait for its completion (the softmax warps finished with the
          // buffer before p_full, which the P V product waited for).
          while (is < njobs && is < ip + kSBufs && ok) {
            uint32_t x, j;
            job_of(it, is, x, j);
            const uint32_t g = gbase + is, buf = g % kSBufs;
            const uint32_t kst = (kn + j) % L::kKStages;
            if (static_cast<int>(j) > k_ready) {
              if (!(ok = wait_or_abort(k_full + kst, ((kn + j) / L::kKStages) & 1, abort_flag))) break;
              k_ready = static_cast<int>(j);
            }
            tc::tc_fence_after();
            const uint32_t qa = q_addr + x * L::kTile;
#pragma unroll
            for (int ks = 0; ks < DH / 8; ++ks)
              tc::mma_tf32(tmem + buf * 128, kmajor_desc(qa, 16384, ks),
                           kmajor_desc(k_addr + kst * L::kTile, 16384, ks), idesc_s, ks > 0);
            tc::mma_commit(s_full + x * kSBufs + buf);
            if (j + 1 == n[x]) tc::mma_commit(q_empty + x);  // Q_X no longer read this item
            if (x == 1) tc::mma_commit(k_empty + kst);       // (B, j) is K_j's last product
            ++is;
          }
          if (!ok) break;
          uint32_t x, j;
          job_of(it, ip, x, j);
          const uint32_t g = gbase + ip, buf = g % kSBufs;
          if (!(ok = wait_or_abort(p_full + buf, (g / kSBufs) & 1, abort_flag))) break;
          if (j == 0 && !(ok = wait_or_abort(o_empty + x, (on[x] & 1) ^ 1, abort_flag))) break;
          const uint32_t vst = (vn + j) % L::kVStages;
          if (static_cast<int>(j) > v_ready) {
            if (!(ok = wait_or_abort(v_full + vst, ((vn + j) / L::kVStages) & 1, abort_flag))) break;
            v_ready = static_cast<int>(j);
          }
          tc::tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 16; ++ks)
            tc::mma_tf32_ts(tmem + 384 + x * 64, tmem + buf * 128 + ks * 8,
                            mnmajor_desc<DH>(v_addr + vst * L::kTile, ks), idesc_o, (j | ks) != 0);
          tc::mma_commit(o_pv + x);
          if (j + 1 == n[x]) {
            tc::mma_commit(o_full + x);
            ++on[x];
          }
          if (x == 1) tc::mma_commit(v_empty + vst);  // (B, j) is V_j's last product
        }
        kn += it.nb;
        vn += it.nb;
        gbase += njobs;
      }
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0)) record_error();
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax + epilogue
    // Warps 2-5 serve tile A, warps 6-9 tile B; thread = row r of its tile (TMEM lane).
    const uint32_t x = static_cast<uint32_t>(warp - 2) >> 2;
    const uint32_t quarter = warp & 3;
    const uint32_t r = quarter * 32 + lane;
    const uint32_t lanes = tmem + ((quarter * 32) << 16);
    const uint32_t o_col = lanes + 384 + x * 64;
    uint32_t gbase = 0, pv_done = 0, on = 0, scnt[kSBufs] = {0, 0, 0};  // this tile's uses per buffer
    bool ok = true;
    for (uint32_t idx = blockIdx.x; idx < p.total && ok; idx += gridDim.x) {
      const PairItem it = decode_pair(p, idx);
      const uint32_t njobs = it.na + it.nb;
      const uint32_t n = x ? it.nb : it.na;
      const uint32_t t = x ? it.tb : it.ta;
      float m = -INFINITY, sum = 0.f;
      for (uint32_t j = 0; j < n && ok; ++j) {
        const uint32_t g = gbase + job_index(it, x, j), buf = g % kSBufs;
        const uint32_t s_col = lanes + buf * 128;
        if (!(ok = wait_or_abort(s_full + x * kSBufs + buf, scnt[buf] & 1, abort_flag))) break;
        ++scnt[buf];
        tc::tc_fence_after();
        // Scores in two 64-column halves (64 registers each): half 0 is read for its maximum
        // only, half 1 is kept, turned into P first, and half 0 is read again. Eight running
        // maxima and four sums keep the dependent chains short.
        uint32_t v0[32], v1[32];
        const bool diag = j == t;
        float mxs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mxs[i] = -INFINITY;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          tc::tmem_load_2x32(s_col + 64 * half, s_col + 64 * half + 32, v0, v1);
          if (diag) row_max64<true>(v0, v1, 64 * half, r, mxs);
          else row_max64<false>(v0, v1, 64 * half, r, mxs);
        }
        const float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                               fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
        const float mx2 = mx * p.scale_log2;
        if (j == 0) {
          m = mx2;
        } else {
          const bool move = mx2 > m + kRescaleLog2;
          if (__any_sync(0xffffffffu, move)) {
            // O_X and the row sum follow the new maximum: the last O_X += P V must be done.
            if (!(ok = wait_or_abort(o_pv + x, (pv_done + j - 1) & 1, abort_flag))) break;
            tc::tc_fence_after();
            const float f = move ? ex2(m - mx2) : 1.f;
#pragma unroll 1
            for (int c = 0; c < DH / 32; ++c) {
              uint32_t o[32];
              tc::tmem_load_32x32(o_col + c * 32, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
              tc::tmem_store_32x32(o_col + c * 32, o);
            }
            sum *= f;
            if (move) m = mx2;
          }
        }
        float sums[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int half = 1; half >= 0; --half) {
          if (half == 0) tc::tmem_load_2x32(s_col, s_col + 32, v0, v1);
          const uint32_t c0 = static_cast<uint32_t>(half) * 64;
          // The P V operand, rounded to nearest instead of truncated.
          if (diag) probs64<true>(v0, v1, p.scale_log2, m, c0, r, sums);
          else probs64<false>(v0, v1, p.scale_log2, m, c0, r, sums);
          tc::tmem_store_2x32(s_col + c0, s_col + c0 + 32, v0, v1);
        }
        sum += (sums[0] + sums[1]) + (sums[2] + sums[3]);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(p_full + buf);
      }
      if (!ok) break;
      gbase += njobs;
      if (n == 0) continue;  // no tile A in this item
      pv_done += n;
      if (!(ok = wait_or_abort(o_full + x, on & 1, abort_flag))) break;
      ++on;
      tc::tc_fence_after();
      const float inv = 1.f / sum;
      const uint32_t qrow = t * 128 + r;
      float* dst = p.o_out + (static_cast<uint64_t>(it.b) * p.seq + qrow) * p.ld_o + it.h * DH;
#pragma unroll
      for (int c = 0; c < DH / 32; ++c) {
        uint32_t o[32];
        tc::tmem_load_32x32(o_col + c * 32, o);
        if (qrow < p.seq) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4 w = make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                                   __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            if (p.round_out)
              w = make_float4(round_tf32(w.x), round_tf32(w.y), round_tf32(w.z), round_tf32(w.w));
            *reinterpret_cast<float4*>(dst + c * 32 + e) = w;
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(o_empty + x);
      if (qrow < p.seq) {
        const uint64_t s = static_cast<uint64_t>(it.b * p.heads + it.h) * p.seq + qrow;
        p.row_max[s] = m;
        p.row_inv[s] = inv;
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ============================================================================ backward: queries
template <int DH>
struct BwdQ {
  static constexpr uint32_t kTile128 = DH * 512;  // 128 rows x DH
  static constexpr uint32_t kTile64 = DH * 256;   // 64 rows x DH
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kDO = kQ + kTile128;
  static constexpr uint32_t kStage = 3 * kTile64;  // K (K-major), V (K-major), K (MN-major)
  static constexpr uint32_t kStages = 3;
  static constexpr uint32_t kKV = kDO + kTile128;
  static constexpr uint32_t kDS = kKV + kStages * kStage;  // dQ staging: 4 warps x 4 KB
  static constexpr uint32_t kBar = kDS + 16384;
  static constexpr uint32_t kSmem = kBar + 256 + 1024;
  static_assert(kSmem <= kMaxSmem, "query-kernel shared memory");
};

template <int DH>
__global__ void __launch_bounds__(kThreads, 1) attn_bwd_q_kernel(const __grid_constant__ AttnParams p) {
  using L = BwdQ<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;   // [kStages]
  uint64_t* kv_empty = bars + 5;  // [kStages]
  uint64_t* s_full = bars + 8;    // [2]
  // bars + 10, 11: unused (S / dP buffer reuse needs no barrier, see issue_s)
  uint64_t* ds_full = bars + 12;  // [2] dS ready, alternating by step (see p_full above)
  uint64_t* acc_full = bars + 14;
  uint64_t* acc_empty = bars + 15;
  uint64_t* drain = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    tc::mbar_init(q_empty, 1);
    for (uint32_t i = 0; i < L::kStages; ++i) {
      tc::mbar_init(kv_full + i, 1);
      tc::mbar_init(kv_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(s_full + i, 1);
    }
    tc::mbar_init(ds_full, kSoftWarps);
    tc::mbar_init(ds_full + 1, kSoftWarps);
    tc::mbar_init(acc_full, 1);
    tc::mbar_init(acc_empty, kSoftWarps);
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_begin();  // set-up done; global memory from here on
  const uint32_t seq = p.seq;

  if (warp == 0) {
    if (tc::elect_one()) {
      uint32_t n = 0, item = 0, st = 0, ph = 0;
      int last_q = -1, last_kv[L::kStages];
      for (uint32_t i = 0; i < L::kStages; ++i) last_kv[i] = -1;
      for (uint32_t k = sched_begin(p); k < sched_end(p) && !*abort_flag; ++k, ++item) {
        const uint32_t idx = sched_item(p, k);
        const Item it = decode(p, idx, false);
        const int hc = static_cast<int>(it.h * DH), b = static_cast<int>(it.b);
        const int kvc = static_cast<int>(it.h / p.group * DH);
        const int kc = static_cast<int>(p.kcol) + kvc, vc = static_cast<int>(p.vcol) + kvc;
        if (!wait_or_abort(q_empty, (item & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(q_full, 2 * L::kTile128);
        last_q = item & 1;
        const int q0 = static_cast<int>(it.t * 128);
#pragma unroll
        for (int c = 0; c < DH / 32; ++c) {
          tc::tma_load_4d(smem + L::kQ + c * 16384, &p.qk128, q_full, hc + 32 * c, q0, b, 0);
          tc::tma_load_4d(smem + L::kDO + c * 16384, &p.do128, q_full, hc + 32 * c, q0, b, 0);
        }
        const uint32_t nkv = (min(seq, it.t * 128 + 128) + 63) / 64;
        for (uint32_t j = 0; j < nkv; ++j, ++n) {
          if (!wait_or_abort(kv_empty + st, ph ^ 1, abort_flag)) break;
          tc::mbar_arrive_expect_tx(kv_full + st, L::kStage);
          last_kv[st] = static_cast<int>(ph);
          uint8_t* s = smem + L::kKV + st * L::kStage;
          const int row = static_cast<int>(j * 64);
#pragma unroll
          for (int c = 0; c < DH / 32; ++c) {
            tc::tma_load_4d(s + c * 8192, &p.qk64, kv_full + st, kc + 32 * c, row, b, 0);
            tc::tma_load_4d(s + L::kTile64 + c * 8192, &p.qk64, kv_full + st, vc + 32 * c, row, b,
                            0);
          }
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int c = 0; c < DH / 32; ++c)
              tc::tma_load_4d(s + 2 * L::kTile64 + (kb * (DH / 32) + c) * 4096, &p.qkv_mn,
                              kv_full + st, kc + 32 * c, row + 32 * kb, b, 0);
          if (++st == L::kStages) {
            st = 0;
            ph ^= 1;
          }
        }
      }
      if (last_q >= 0 && !tc::mbar_wait(q_full, last_q)) record_error();
      for (uint32_t s = 0; s < L::kStages; ++s)
        if (last_kv[s] >= 0 && !tc::mbar_wait(kv_full + s, last_kv[s])) record_error();
    }
    __syncwarp();
  } else if (warp == 1) {
    if (tc::elect_one()) {
      const uint32_t idesc_s = tc::idesc_tf32(128, 64, 0, 0);
      const uint32_t idesc_q = tc::idesc_tf32(128, DH, 0, 1);
      const uint32_t q_addr = tc::smem_u32(smem + L::kQ);
      const uint32_t do_addr = tc::smem_u32(smem + L::kDO);
      const uint32_t kv_addr = tc::smem_u32(smem + L::kKV);
      uint32_t n = 0, sn = 0, dn = 0, item = 0;
      bool ok = true;
      // kv load number kn sits in stage kn % kStages, phase (kn / kStages) & 1.
      // Buffer sb was last read by the dQ product of two steps back (dS over S), which this
      // thread issued before; one thread's tcgen05.mma operations run in issue order, so S and
      // dP can be issued into it without waiting for that product (the softmax warps were done
      // with it before ds_full, which the dQ product waited for).
      auto issue_s = [&](uint32_t kn) -> bool {  // S and dP for kv load number kn
        const uint32_t st = kn % L::kStages, sb = sn & 1;
        if (!wait_or_abort(kv_full + st, (kn / L::kStages) & 1, abort_flag)) return false;
        tc::tc_fence_after();
        const uint32_t s = kv_addr + st * L::kStage;
#pragma unroll
        for (int ks = 0; ks < DH / 8; ++ks) {
          tc::mma_tf32(tmem + sb * 64, kmajor_desc(q_addr, 16384, ks), kmajor_desc(s, 8192, ks),
                       idesc_s, ks > 0);
          tc::mma_tf32(tmem + 128 + sb * 64, kmajor_desc(do_addr, 16384, ks),
                       kmajor_desc(s + L::kTile64, 8192, ks), idesc_s, ks > 0);
        }
        tc::mma_commit(s_full + sb);
        ++sn;
        return true;
      };
      for (uint32_t k = sched_begin(p); k < sched_end(p) && ok && !*abort_flag; ++k, ++item) {
        const uint32_t idx = sched_item(p, k);
        const Item it = decode(p, idx, false);
        const uint32_t nkv = (min(seq, it.t * 128 + 128) + 63) / 64;
        if (!(ok = wait_or_abort(q_full, item & 1, abort_flag))) break;
        tc::tc_fence_after();
        const uint32_t n0 = n, sn0 = sn;
        if (!(ok = issue_s(n0))) break;
        for (uint32_t j = 0; j < nkv && ok; ++j) {
          if (j + 1 < nkv) {
            if (!(ok = issue_s(n0 + j + 1))) break;
          }
          if (j + 1 == nkv) tc::mma_commit(q_empty);  // Q, dO no longer read in this item
          if (!(ok = wait_or_abort(ds_full + (dn & 1), (dn >> 1) & 1, abort_flag))) break;
          ++dn;
          if (j == 0 && !(ok = wait_or_abort(acc_empty, (item & 1) ^ 1, abort_flag))) break;
          tc::tc_fence_after();
          const uint32_t st = (n0 + j) % L::kStages, sb = (sn0 + j) & 1;
          const uint32_t kmn = kv_addr + st * L::kStage + 2 * L::kTile64;
          // dQ += dS K with dS read from TMEM, where the softmax warps wrote it over S.
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc::mma_tf32_ts(tmem + 256, tmem + sb * 64 + ks * 8, mnmajor_desc<DH>(kmn, ks),
                            idesc_q, (j | ks) != 0);
          tc::mma_commit(kv_empty + st);
        }
        n = n0 + nkv;
        if (ok) tc::mma_commit(acc_full);
      }
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0)) record_error();
    }
    __syncwarp();
  } else {
    // Thread (r, grp) owns key columns [32*grp, 32*grp + 32) of every 128 x 64 tile.
    const SoftThread th(warp, lane, tmem);
    const uint32_t r = th.r, grp = th.grp;
    uint8_t* dsbuf = smem + L::kDS;
    uint32_t sn = 0, item = 0;
    bool ok = true;
    for (uint32_t k = sched_begin(p); k < sched_end(p) && ok; ++k, ++item) {
        const uint32_t idx = sched_item(p, k);
      const Item it = decode(p, idx, false);
      const uint32_t nkv = (min(seq, it.t * 128 + 128) + 63) / 64;
      const uint32_t q = it.t * 128 + r;
      const bool valid = q < seq;
      const uint64_t srow = static_cast<uint64_t>(it.b * p.heads + it.h) * seq + q;
      // Rows past the sequence: mx = 0, inv = 0 make every probability 0 (their scores are 0).
      // D = rowsum(dO o O) comes precomputed (attn_delta_kernel).
      float mx = 0.f, inv = 0.f, dd = 0.f;
      if (valid) {
        mx = p.row_max[srow];
        inv = p.row_inv[srow];
        dd = p.delta[srow];
      }
      const float ninv_scale = inv * p.scale;
      if (lane == 0) tc::bulk_wait_read<0>();
      __syncwarp();
      for (uint32_t j = 0; j < nkv && ok; ++j, ++sn) {
        if (!(ok = wait_or_abort(s_full + (sn & 1), (sn >> 1) & 1, abort_flag))) break;
        tc::tc_fence_after();
        uint32_t sv[32], pv[32];
        tc::tmem_load_2x32(th.lanes + (sn & 1) * 64 + grp * 32,
                           th.lanes + 128 + (sn & 1) * 64 + grp * 32, sv, pv);
        const uint32_t kv0 = j * 64 + grp * 32;
        float ds[32];
        if (kv0 + 31 <= it.t * 128) {  // every key of this chunk precedes every row of the tile
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float pr = ex2(fmaf(__uint_as_float(sv[e]), p.scale_log2, -mx));
            ds[e] = round_tf32(pr * ninv_scale * (__uint_as_float(pv[e]) - dd));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float pr = ex2(fmaf(__uint_as_float(sv[e]), p.scale_log2, -mx));
            if (kv0 + e > q) pr = 0.f;
            ds[e] = round_tf32(pr * ninv_scale * (__uint_as_float(pv[e]) - dd));
          }
        }
        // dS overwrites this thread's S columns in TMEM: the A operand of dQ += dS K.
        uint32_t dsu[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) dsu[e] = __float_as_uint(ds[e]);
        tc::tmem_store_32x32(th.lanes + (sn & 1) * 64 + grp * 32, dsu);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(ds_full + (sn & 1));
      }
      if (!ok) break;
      if (!(ok = wait_or_abort(acc_full, item & 1, abort_flag))) break;
      tc::tc_fence_after();
      if (grp == 0) {  // the four warps of column group 0 store dQ, one 32-column box at a time
        uint8_t* stg = dsbuf + th.quarter * 4096;
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t v[32];
          tc::tmem_load_32x32(th.lanes + 256 + c * 32, v);
          float o[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __uint_as_float(v[e]);
          if (p.rope && valid) inverse_rope(o, p.rope + static_cast<uint64_t>(q) * (DH / 2) + c * 16);
          box_partials(p, o, static_cast<int>(it.h * DH + 32 * c),
                       static_cast<int>(it.t * 128 + th.quarter * 32), static_cast<int>(it.b));
          if (p.round_out) round_box(o);
          if (c > 0) {
            if (lane == 0) tc::bulk_wait_read<0>();
            __syncwarp();
          }
          store_box(&p.out, stg, o, static_cast<int>(it.h * DH + 32 * c),
                    static_cast<int>(it.t * 128 + th.quarter * 32), static_cast<int>(it.b));
          if (lane == 0) tc::bulk_commit();
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acc_empty);
    }
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ============================================================================ backward: keys
template <int DH>
struct BwdKV {
  static constexpr uint32_t kTile128 = DH * 512;
  static constexpr uint32_t kTile64 = DH * 256;
  static constexpr uint32_t kK = 0;
  static constexpr uint32_t kV = kK + kTile128;
  static constexpr uint32_t kKQ = kV + kTile128;      // 2 stages: Q and dO K-major (64 rows)
  static constexpr uint32_t kMN = kKQ + 4 * kTile64;  // 2 stages: Q and dO MN-major
  static constexpr uint32_t kStg = kMN + 4 * kTile64;  // output staging, 4 KB per softmax warp
  static constexpr uint32_t kStats = kStg + kSoftWarps * 4096;  // [2 steps][max, 1/sum, D][64]
  static constexpr uint32_t kBar = kStats + 2 * 3 * 64 * 4;
  static constexpr uint32_t kSmem = kBar + 192 + 1024;
  static_assert(kSmem <= kMaxSmem, "key-kernel shared memory");
};

// TMEM columns: S^T / P^T [2][64] at 0, dP^T / dS^T [2][64] at 128, dV at 256, dK at 256 + DH.
// P^T and dS^T overwrite S^T and dP^T in place and are the A operands of dV += P^T dO and
// dK += dS^T Q, read straight from TMEM.
template <int DH>
__global__ void __launch_bounds__(kThreads, 1) attn_bwd_kv_kernel(const __grid_constant__ AttnParams p) {
  using L = BwdKV<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* kv_empty = bars + 1;
  uint64_t* kq_full = bars + 2;   // [2]
  uint64_t* kq_empty = bars + 4;  // [2]
  uint64_t* s_full = bars + 6;    // [2]
  // bars + 8, 9: unused (S^T / dP^T buffer reuse needs no barrier, see issue_s)
  uint64_t* mn_full = bars + 10;  // [2]
  uint64_t* mn_empty = bars + 12;  // [2]
  uint64_t* pd_full = bars + 14;  // [2] P^T / dS^T ready, alternating by step (see p_full above)
  uint64_t* acc_full = bars + 16;
  uint64_t* acc_empty = bars + 17;
  uint64_t* drain = bars + 18;
  uint64_t* xbar = bars + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tc::mbar_init(kv_full, 1);
    tc::mbar_init(kv_empty, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(kq_full + i, 1);
      tc::mbar_init(kq_empty + i, 1);
      tc::mbar_init(s_full + i, 1);
      tc::mbar_init(mn_full + i, 1);
      tc::mbar_init(mn_empty + i, 1);
    }
    tc::mbar_init(pd_full, kSoftWarps);
    tc::mbar_init(pd_full + 1, kSoftWarps);
    tc::mbar_init(acc_full, 1);
    tc::mbar_init(acc_empty, kSoftWarps);
    tc::mbar_init(drain, 1);
    tc::mbar_init(xbar, kSoftWarps);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_begin();  // set-up done; global memory from here on
  const uint32_t seq = p.seq;
  const uint32_t nq_all = (seq + 63) / 64;

  if (warp == 0) {
    if (tc::elect_one()) {
      uint32_t n = 0, item = 0;
      int last_kv = -1, last_kq[2] = {-1, -1}, last_mn[2] = {-1, -1};
      for (uint32_t k = sched_begin(p); k < sched_end(p) && !*abort_flag; ++k, ++item) {
        const uint32_t idx = sched_item(p, k);
        const Item it = decode_kv(p, idx);  // it.h: the key / value head
        const int b = static_cast<int>(it.b);
        const int kc = static_cast<int>(p.kcol + it.h * DH), vc = static_cast<int>(p.vcol + it.h * DH);
        if (!wait_or_abort(kv_empty, (item & 1) ^ 1, abort_flag)) break;
        tc::mbar_arrive_expect_tx(kv_full, 2 * L::kTile128);
        last_kv = item & 1;
        const int k0 = static_cast<int>(it.t * 128);
#pragma unroll
        for (int c = 0; c < DH / 32; ++c) {
          tc::tma_load_4d(smem + L::kK + c * 16384, &p.qk128, kv_full, kc + 32 * c, k0, b, 0);
          tc::tma_load_4d(smem + L::kV + c * 16384, &p.qk128, kv_full, vc + 32 * c, k0, b, 0);
        }
        // Every query head of the group, each over the query tiles at or after the key tile.
        const uint32_t steps = nq_all - 2 * it.t;
        for (uint32_t j = 0; j < steps * p.group; ++j, ++n) {
          const uint32_t i = 2 * it.t + j % steps;
          const int hc = static_cast<int>((it.h * p.group + j / steps) * DH);
          const uint32_t st = n & 1, ph = (n >> 1) & 1;
          const int row = static_cast<int>(i * 64);
          if (!wait_or_abort(kq_empty + st, ph ^ 1, abort_flag)) break;
          tc::mbar_arrive_expect_tx(kq_full + st, 2 * L::kTile64);
          last_kq[st] = ph;
          uint8_t* s = smem + L::kKQ + st * 2 * L::kTile64;
#pragma unroll
          for (int c = 0; c < DH / 32; ++c) {
            tc::tma_load_4d(s + c * 8192, &p.qk64, kq_full + st, hc + 32 * c, row, b, 0);
            tc::tma_load_4d(s + L::kTile64 + c * 8192, &p.do64, kq_full + st, hc + 32 * c, row, b, 0);
          }
          if (!wait_or_abort(mn_empty + st, ph ^ 1, abort_flag)) break;
          tc::mbar_arrive_expect_tx(mn_full + st, 2 * L::kTile64);
          last_mn[st] = ph;
          uint8_t* m = smem + L::kMN + st * 2 * L::kTile64;
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int c = 0; c < DH / 32; ++c) {
              const uint32_t o = (kb * (DH / 32) + c) * 4096;
              tc::tma_load_4d(m + o, &p.qkv_mn, mn_full + st, hc + 32 * c, row + 32 * kb, b, 0);
              tc::tma_load_4d(m + L::kTile64 + o, &p.do_mn, mn_full + st, hc + 32 * c,
                              row + 32 * kb, b, 0);
            }
        }
      }
      if (last_kv >= 0 && !tc::mbar_wait(kv_full, last_kv)) record_error();
      for (int s = 0; s < 2; ++s) {
        if (last_kq[s] >= 0 && !tc::mbar_wait(kq_full + s, last_kq[s])) record_error();
        if (last_mn[s] >= 0 && !tc::mbar_wait(mn_full + s, last_mn[s])) record_error();
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (tc::elect_one()) {
      const uint32_t idesc_s = tc::idesc_tf32(128, 64, 0, 0);
      const uint32_t idesc_g = tc::idesc_tf32(128, DH, 0, 1);
      const uint32_t k_addr = tc::smem_u32(smem + L::kK);
      const uint32_t v_addr = tc::smem_u32(smem + L::kV);
      const uint32_t kq_addr = tc::smem_u32(smem + L::kKQ);
      const uint32_t mn_addr = tc::smem_u32(smem + L::kMN);
      uint32_t n = 0, sn = 0, item = 0;
      bool ok = true;
      // Buffer sb was last read by the dV / dK products of two steps back (P^T, dS^T over S^T,
      // dP^T), issued before by this thread; in-order tcgen05.mma execution makes the wait for
      // their completion unnecessary (the softmax warps were done before pd_full).
      auto issue_s = [&](uint32_t qn) -> bool {  // S^T and dP^T for query load number qn
        const uint32_t st = qn & 1, sb = sn & 1;
        if (!wait_or_abort(kq_full + st, (qn >> 1) & 1, abort_flag)) return false;
        tc::tc_fence_after();
        const uint32_t s = kq_addr + st * 2 * L::kTile64;
#pragma unroll
        for (int ks = 0; ks < DH / 8; ++ks) {
          tc::mma_tf32(tmem + sb * 64, kmajor_desc(k_addr, 16384, ks), kmajor_desc(s, 8192, ks),
                       idesc_s, ks > 0);
          tc::mma_tf32(tmem + 128 + sb * 64, kmajor_desc(v_addr, 16384, ks),
                       kmajor_desc(s + L::kTile64, 8192, ks), idesc_s, ks > 0);
        }
        tc::mma_commit(kq_empty + st);
        tc::mma_commit(s_full + sb);
        ++sn;
        return true;
      };
      for (uint32_t k = sched_begin(p); k < sched_end(p) && ok && !*abort_flag; ++k, ++item) {
        const uint32_t idx = sched_item(p, k);
        const Item it = decode_kv(p, idx);
        // >= 1 query tile per head (every 128-key tile starts below seq), for each head of the group
        const uint32_t steps = (nq_all - 2 * it.t) * p.group;
        if (!(ok = wait_or_abort(kv_full, item & 1, abort_flag))) break;
        tc::tc_fence_after();
        const uint32_t n0 = n, sn0 = sn;
        if (!(ok = issue_s(n0))) break;
        for (uint32_t i = 0; i < steps && ok; ++i) {
          if (i + 1 < steps) {
            if (!(ok = issue_s(n0 + i + 1))) break;
          }
          if (i + 1 == steps) tc::mma_commit(kv_empty);
          const uint32_t qn = n0 + i, st = qn & 1, sb = (sn0 + i) & 1;
          if (!(ok = wait_or_abort(pd_full + (qn & 1), (qn >> 1) & 1, abort_flag))) break;
          if (!(ok = wait_or_abort(mn_full + st, (qn >> 1) & 1, abort_flag))) break;
          if (i == 0 && !(ok = wait_or_abort(acc_empty, (item & 1) ^ 1, abort_flag))) break;
          tc::tc_fence_after();
          const uint32_t m = mn_addr + st * 2 * L::kTile64;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            tc::mma_tf32_ts(tmem + 256, tmem + sb * 64 + ks * 8,
                            mnmajor_desc<DH>(m + L::kTile64, ks), idesc_g, (i | ks) != 0);
            tc::mma_tf32_ts(tmem + 256 + DH, tmem + 128 + sb * 64 + ks * 8,
                            mnmajor_desc<DH>(m, ks), idesc_g, (i | ks) != 0);
          }
          tc::mma_commit(mn_empty + st);
        }
        n = n0 + steps;
        if (ok) tc::mma_commit(acc_full);
      }
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0)) record_error();
    }
    __syncwarp();
  } else {
    // Thread (r, grp) owns query columns [32*grp, 32*grp + 32) of every 128 x 64 tile (rows are
    // keys). The 64 queries' statistics are staged in shared memory once per step: softmax thread
    // u < 192 fetches value u % 64 of array u / 64 (row max, 1 / sum, D) one step ahead.
    const SoftThread th(warp, lane, tmem);
    const uint32_t r = th.r, grp = th.grp;
    const uint32_t u = (warp - 2) * 32 + lane;
    const float* src = u < 64 ? p.row_max : (u < 128 ? p.row_inv : p.delta);
    float* stats = reinterpret_cast<float*>(smem + L::kStats);  // [2][3][64]
    uint8_t* stg = smem + L::kStg + (warp - 2) * 4096;
    uint32_t n = 0, item = 0, xphase = 0;
    bool ok = true;
    // Queries past the sequence get zero statistics: their probabilities come out 0.
    auto fetch = [&](uint64_t sbase, uint32_t q0) -> float {
      const uint32_t q = q0 + (u & 63);
      return (u < 192 && q < seq) ? __ldg(src + sbase + q) : 0.f;
    };
    for (uint32_t k = sched_begin(p); k < sched_end(p) && ok; ++k, ++item) {
        const uint32_t idx = sched_item(p, k);
      const Item it = decode_kv(p, idx);
      const uint32_t i0 = 2 * it.t;
      const uint32_t per_head = nq_all - i0;
      const uint32_t steps = per_head * p.group;
      const uint32_t kv = it.t * 128 + r;
      // Statistics of query head it.h * group + j / per_head, query tile i0 + j % per_head.
      auto stat_base = [&](uint32_t j) {
        return static_cast<uint64_t>(it.b * p.heads + it.h * p.group + j / per_head) * seq;
      };
      float next = fetch(stat_base(0), i0 * 64);
      for (uint32_t j = 0; j < steps && ok; ++j, ++n) {
        const uint32_t i = j % per_head;  // query tile i0 + i
        float* st = stats + (n & 1) * 192;
        if (u < 192) st[u] = next;
        if (!(ok = soft_sync(xbar, xphase, abort_flag))) break;
        if (j + 1 < steps) next = fetch(stat_base(j + 1), (i0 + (j + 1) % per_head) * 64);
        if (!(ok = wait_or_abort(s_full + (n & 1), (n >> 1) & 1, abort_flag))) break;
        tc::tc_fence_after();
        uint32_t sv[32], pv[32];
        const uint32_t s_col = th.lanes + (n & 1) * 64 + grp * 32;
        tc::tmem_load_2x32(s_col, s_col + 128, sv, pv);
        const uint32_t q0 = (i0 + i) * 64 + grp * 32;
        const float4* mx4 = reinterpret_cast<const float4*>(st + grp * 32);
        const float4* inv4 = reinterpret_cast<const float4*>(st + 64 + grp * 32);
        const float4* dd4 = reinterpret_cast<const float4*>(st + 128 + grp * 32);
        const bool full = q0 >= it.t * 128 + 127;  // every query of the chunk follows every key
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const float4 m4 = mx4[g], i4 = inv4[g], d4 = dd4[g];
          const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
          const float iv[4] = {i4.x, i4.y, i4.z, i4.w};
          const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const int e = 4 * g + e4;
            float pr = ex2(fmaf(__uint_as_float(sv[e]), p.scale_log2, -mv[e4])) * iv[e4];
            if (!full && q0 + e < kv) pr = 0.f;
            const float ds = pr * (__uint_as_float(pv[e]) - dv[e4]) * p.scale;
            sv[e] = __float_as_uint(round_tf32(pr));
            pv[e] = __float_as_uint(round_tf32(ds));
          }
        }
        // P^T and dS^T overwrite S^T and dP^T: the TMEM A operands of dV and dK.
        tc::tmem_store_2x32(s_col, s_col + 128, sv, pv);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(pd_full + (n & 1));
      }
      if (!ok) break;
      if (!(ok = wait_or_abort(acc_full, item & 1, abort_flag))) break;
      tc::tc_fence_after();
      if (grp < DH / 32) {
        const int row = static_cast<int>(it.t * 128 + th.quarter * 32);
        uint32_t v[32], w[32];
        tc::tmem_load_2x32(th.lanes + 256 + grp * 32, th.lanes + 256 + DH + grp * 32, v, w);
        float o[32];
        if (lane == 0) tc::bulk_wait_read<0>();  // this warp's staging box is free again
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __uint_as_float(v[e]);  // dV
        box_partials(p, o, static_cast<int>(p.vcol + it.h * DH + 32 * grp), row,
                     static_cast<int>(it.b));
        if (p.round_out) round_box(o);
        store_box(&p.out, stg, o, static_cast<int>(p.vcol + it.h * DH + 32 * grp), row,
                  static_cast<int>(it.b));
        if (lane == 0) {
          tc::bulk_commit();
          tc::bulk_wait_read<0>();
        }
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __uint_as_float(w[e]);  // dK
        if (p.rope && kv < seq) inverse_rope(o, p.rope + static_cast<uint64_t>(kv) * (DH / 2) + grp * 16);
        box_partials(p, o, static_cast<int>(p.kcol + it.h * DH + 32 * grp), row,
                     static_cast<int>(it.b));
        if (p.round_out) round_box(o);
        store_box(&p.out, stg, o, static_cast<int>(p.kcol + it.h * DH + 32 * grp), row,
                  static_cast<int>(it.b));
        if (lane == 0) tc::bulk_commit();
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acc_empty);
    }
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ============================================================================ D = rowsum(dO o O)
// One warp per (token row, head): the dot product of the head's dO and O slices (coalesced 128-
// and 256-byte reads), written as D[(b * heads + h) * seq + t] for the backward kernels.
// D[b, h, t] = sum over the head's columns of dO * O: one warp per token row covering every head
// with coalesced float4 loads (lane l takes float4 chunks l, l + 32, ...); the dh / 4 lanes that
// hold one head's chunks combine their products with butterfly shuffles.
__global__ void __launch_bounds__(256) attn_delta_kernel(float* __restrict__ delta,
                                                         const float* __restrict__ d_o,
                                                         const float* __restrict__ o, uint64_t rows,
                                                         uint32_t seq, uint32_t heads, uint32_t dh,
                                                         uint64_t ld) {
  pdl_begin();
  const uint64_t row = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint32_t group = dh / 4;  // lanes per head: 8, 16 or 32
  const uint32_t n4 = heads * group;
  const float4* a = reinterpret_cast<const float4*>(d_o + row * ld);
  const float4* b = reinterpret_cast<const float4*>(o + row * ld);
  const uint64_t bb = row / seq, t = row - bb * seq;
#pragma unroll 4
  for (uint32_t f0 = 0; f0 < n4; f0 += 32) {
    const uint32_t f = f0 + lane;
    float acc = 0.f;
    if (f < n4) {
      const float4 x = __ldg(a + f), y = __ldg(b + f);
      acc = (x.x * y.x + x.y * y.y) + (x.z * y.z + x.w * y.w);
    }
    for (uint32_t off = group / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (f < n4 && lane % group == 0) delta[(bb * heads + f / group) * seq + t] = acc;
  }
}

// ============================================================================ host side
template <typename K>
cudaError_t launch_attn(K kernel, uint32_t smem, const AttnParams& p, int device,
                        cudaStream_t stream, bool* configured) {
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  if (!configured[device]) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[device] = true;
  }
  const unsigned grid =
      p.sched ? p.sched_grid : std::min<uint32_t>(p.total, static_cast<uint32_t>(sm_count(device)));
  if (grid == 0) return cudaSuccess;
  return launch(kernel, dim3(grid), dim3(kThreads), smem, stream, p);
}

// Work lists for the persistent backward kernels, longest processing time first: the items
// (tile, batch-head) are sorted by cost (the 64-row steps the item loops over: key tiles up to the
// query tile's end for the query kernel, query tiles from the key tile on times the query group for
// the key kernel), then each goes to the CTA with the least cost assigned so far. Round-robin over
// tiles in cost order left CTAs with one heavy and one medium item beside others with one light
// item (at 2 sequences x 16 heads x 8 tiles, 24 steps on the busiest CTA against 15.6 on average).
// That is for the two kernels run one after the other (18 % faster at 2 x 16 x 1024 x 64). When
// they run side by side on two streams (lpt = false, the training runtime), the CTAs that finish
// early in cost-ordered round robin hand their SMs to the other kernel, which measured as good or
// slightly better than balanced lists, so that order is kept there.
// Stored as CSR in device memory [grid + 1 offsets | items], built once per (device, side, shape,
// kind): the first backward call of a shape allocates, so make it before any stream capture.
// With head_pairs (the kOrderHead order) the lists are instead made of tile pairs (T-1-t, t) of
// one (batch, head), heavier tile first; pair k (counted head by head) goes to CTA k % grid. A
// pair's cost is the same for every t (the triangle's rows and columns sum to T+1 tiles), so the
// lists balance without sorting, and the CTAs that start together work on the same heads.
cudaError_t backward_schedule(int device, bool key_side, uint32_t bh, uint32_t tiles, uint32_t seq,
                              uint32_t group, bool lpt, const uint32_t** out, uint32_t* grid_out,
                              bool head_pairs = false) {
  using Key = std::tuple<int, bool, uint32_t, uint32_t, uint32_t, uint32_t, bool, bool>;
  static std::mutex mu;
  static std::map<Key, std::pair<uint32_t*, uint32_t>> cache;
  std::lock_guard<std::mutex> lock(mu);
  const Key key{device, key_side, bh, tiles, seq, group, lpt, head_pairs};
  auto it = cache.find(key);
  if (it == cache.end()) {
    const uint32_t total = bh * tiles;
    const uint32_t pairs = (tiles + 1) / 2;
    const uint32_t grid = std::min<uint32_t>(head_pairs ? bh * pairs : total,
                                             static_cast<uint32_t>(sm_count(device)));
    const uint32_t nq_all = (seq + 63) / 64;
    auto cost = [&](uint32_t t) -> uint64_t {
      if (key_side) return static_cast<uint64_t>(nq_all - 2 * t) * group;
      return (std::min<uint64_t>(seq, 128ull * t + 128) + 63) / 64;
    };
    std::vector<std::vector<uint32_t>> lists(grid);
    if (head_pairs) {
      for (uint32_t h = 0; h < bh; ++h)
        for (uint32_t q = 0; q < pairs; ++q) {
          const uint32_t lo = q, hi = tiles - 1 - q;
          const uint32_t heavy = cost(lo) >= cost(hi) ? lo : hi, light = heavy == lo ? hi : lo;
          std::vector<uint32_t>& l = lists[(h * pairs + q) % grid];
          l.push_back(heavy * bh + h);
          if (light != heavy) l.push_back(light * bh + h);
        }
    } else {
      std::vector<uint32_t> items(total);
      for (uint32_t i = 0; i < total; ++i) items[i] = i;
      std::stable_sort(items.begin(), items.end(), [&](uint32_t a, uint32_t b) {
        return cost(a / bh) > cost(b / bh);
      });
      using Slot = std::pair<uint64_t, uint32_t>;  // (assigned cost, cta)
      std::priority_queue<Slot, std::vector<Slot>, std::greater<Slot>> heap;
      for (uint32_t c = 0; c < grid; ++c) heap.push({0, c});
      for (uint32_t k = 0; k < total; ++k) {  // !lpt: CTA c takes items c, c + grid, ...
        const uint32_t i = items[k];
        if (!lpt) {
          lists[k % grid].push_back(i);
          continue;
        }
        Slot sl = heap.top();
        heap.pop();
        lists[sl.second].push_back(i);
        sl.first += cost(i / bh);
        heap.push(sl);
      }
    }
    std::vector<uint32_t> host(grid + 1 + total);
    uint32_t pos = 0;
    for (uint32_t c = 0; c < grid; ++c) {
      host[c] = pos;
      for (uint32_t i : lists[c]) host[grid + 1 + pos++] = i;
    }
    host[grid] = pos;
    uint32_t* dev = nullptr;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&dev), host.size() * sizeof(uint32_t));
    if (e == cudaSuccess)
      e = cudaMemcpy(dev, host.data(), host.size() * sizeof(uint32_t), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(dev);
      return e;
    }
    it = cache.emplace(key, std::make_pair(dev, grid)).first;
  }
  *out = it->second.first;
  *grid_out = it->second.second;
  return cudaSuccess;
}

void base_params(AttnParams& p, uint64_t batch, uint64_t seq, uint64_t heads, uint64_t head_dim,
                 uint64_t kv_heads) {
  memset(&p, 0, sizeof(p));
  p.heads = static_cast<uint32_t>(heads);
  p.seq = static_cast<uint32_t>(seq);
  p.model_dim = static_cast<uint32_t>(heads * head_dim);
  p.bh = static_cast<uint32_t>(batch * heads);
  p.kv_heads = static_cast<uint32_t>(kv_heads);
  p.kv_bh = static_cast<uint32_t>(batch * kv_heads);
  p.group = static_cast<uint32_t>(heads / kv_heads);
  p.kcol = p.model_dim;
  p.vcol = static_cast<uint32_t>((heads + kv_heads) * head_dim);
  p.ld_o = heads * head_dim;
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)));
  p.scale_log2 = p.scale * kLog2e;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Work orders of the persistent kernels. kOrderAuto: the forward pairs adjacent query tiles
// heaviest first when there are at least four items per SM, else tiles t and T-1-t; the backward
// lists are cost-ordered (longest first). kOrderHead: forward tiles t and T-1-t with the pairs of
// one (batch, head) consecutive; backward lists of tile pairs (t, T-1-t) of one (batch, head)
// handed to consecutive CTAs, so the CTAs that run together read the same head's tiles and L2
// serves the repeats. SPAR_B200_ATTN_ORDER=head | auto overrides the default.
enum AttnOrder { kOrderAuto = 0, kOrderHead = 1 };

AttnOrder attn_order() {
  static const AttnOrder order = [] {
    const char* e = getenv("SPAR_B200_ATTN_ORDER");
    if (e && std::strcmp(e, "head") == 0) return kOrderHead;
    return kOrderAuto;
  }();
  return order;
}

}  // namespace

bool attention_supported(uint64_t head_dim) { return head_dim == 32 || head_dim == 64; }

cudaError_t attention_forward_launch(const float* qkv, float* ctx, float* row_max, float* row_inv,
                                     uint64_t batch, uint64_t seq, uint64_t heads,
                                     uint64_t head_dim, int device, cudaStream_t stream,
                                     uint64_t kv_heads, bool round_out) {
  if (kv_heads == 0) kv_heads = heads;
  AttnParams p;
  base_params(p, batch, seq, heads, head_dim, kv_heads);
  p.round_out = round_out ? 1u : 0u;
  const uint64_t w = (heads + 2 * kv_heads) * head_dim;  // packed q | k | v row
  if (!make_map(&p.qk128, qkv, w, seq, batch, 1, w, seq * w, 0, 128, false) ||
      !make_map(&p.qkv_mn, qkv, w, seq, batch, 1, w, seq * w, 0, 32, true))
    return cudaErrorInvalidValue;
  p.o_out = ctx;
  p.row_max = row_max;
  p.row_inv = row_inv;
  p.tiles = static_cast<uint32_t>((seq + 127) / 128);
  p.total = (p.tiles + 1) / 2 * p.bh;  // pairs of query tiles
  if (attn_order() == kOrderHead)
    p.head_major = 1u;
  else
    p.adjacent_pairs = p.total >= 4u * static_cast<uint32_t>(sm_count(device)) ? 1u : 0u;
  static bool cfg32[64] = {}, cfg64[64] = {};
  return head_dim == 64 ? launch_attn(attn_fwd_kernel<64>, Fwd<64>::kSmem, p, device, stream, cfg64)
                        : launch_attn(attn_fwd_kernel<32>, Fwd<32>::kSmem, p, device, stream, cfg32);
}

cudaError_t attention_backward_launch(const float* qkv, const float* ctx, const float* dctx,
                                      const float* row_max, const float* row_inv, float* delta,
                                      float* dqkv, uint64_t batch, uint64_t seq, uint64_t heads,
                                      uint64_t head_dim, int device, cudaStream_t stream,
                                      const float* rope_table, cudaStream_t key_stream,
                                      cudaEvent_t fork, cudaEvent_t join, uint64_t kv_heads,
                                      bool round_out, float* column_partials) {
  if (kv_heads == 0) kv_heads = heads;
  if (column_partials && seq % 32) return cudaErrorInvalidValue;
  AttnParams p;
  base_params(p, batch, seq, heads, head_dim, kv_heads);
  p.round_out = round_out ? 1u : 0u;
  p.colpart = column_partials;
  p.colpart_ld = static_cast<uint32_t>((heads + 2 * kv_heads) * head_dim);
  const uint64_t d = heads * head_dim;
  const uint64_t w = (heads + 2 * kv_heads) * head_dim;  // packed q | k | v row
  if (!make_map(&p.qk128, qkv, w, seq, batch, 1, w, seq * w, 0, 128, false) ||
      !make_map(&p.qk64, qkv, w, seq, batch, 1, w, seq * w, 0, 64, false) ||
      !make_map(&p.qkv_mn, qkv, w, seq, batch, 1, w, seq * w, 0, 32, true) ||
      !make_map(&p.do128, dctx, d, seq, batch, 1, d, seq * d, 0, 128, false) ||
      !make_map(&p.do64, dctx, d, seq, batch, 1, d, seq * d, 0, 64, false) ||
      !make_map(&p.do_mn, dctx, d, seq, batch, 1, d, seq * d, 0, 32, true) ||
      !make_map(&p.out, dqkv, w, seq, batch, 1, w, seq * w, 0, 32, false))
    return cudaErrorInvalidValue;
  p.o = ctx;
  p.d_o = dctx;
  p.row_max = const_cast<float*>(row_max);
  p.row_inv = const_cast<float*>(row_inv);
  p.delta = delta;
  p.rope = reinterpret_cast<const float2*>(rope_table);
  static bool q32[64] = {}, q64[64] = {}, k32[64] = {}, k64[64] = {};
  const uint64_t warps = batch * seq;  // one per token row
  cudaError_t e = launch(attn_delta_kernel, dim3(static_cast<unsigned>((warps + 7) / 8)),
                         dim3(256), 0, stream, delta, static_cast<const float*>(dctx),
                         static_cast<const float*>(ctx), batch * seq,
                         static_cast<uint32_t>(seq), static_cast<uint32_t>(heads),
                         static_cast<uint32_t>(head_dim), static_cast<uint64_t>(d));
  if (e != cudaSuccess) return e;
  p.tiles = static_cast<uint32_t>((seq + 127) / 128);
  p.total = p.tiles * p.bh;
  AttnParams pk = p;  // the key kernel's items: one per key / value head
  pk.total = p.tiles * p.kv_bh;
  const bool side_by_side = key_stream && fork && join;
  const bool head_pairs = attn_order() == kOrderHead;
  e = backward_schedule(device, false, p.bh, p.tiles, p.seq, p.group, !side_by_side, &p.sched,
                        &p.sched_grid, head_pairs);
  if (e == cudaSuccess)
    e = backward_schedule(device, true, pk.kv_bh, pk.tiles, pk.seq, pk.group, !side_by_side,
                          &pk.sched, &pk.sched_grid, head_pairs);
  if (e != cudaSuccess) return e;
  // The query and key kernels only share inputs (they write dq and dk / dv): on a second stream
  // the key kernel's CTAs take the SMs that the query kernel's last items leave idle.
  cudaStream_t ks = stream;
  if (key_stream && fork && join) {
    e = cudaEventRecord(fork, stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(key_stream, fork, 0);
    if (e != cudaSuccess) return e;
    ks = key_stream;
  }
  e = head_dim == 64
          ? launch_attn(attn_bwd_q_kernel<64>, BwdQ<64>::kSmem, p, device, stream, q64)
          : launch_attn(attn_bwd_q_kernel<32>, BwdQ<32>::kSmem, p, device, stream, q32);
  if (e != cudaSuccess) return e;
  e = head_dim == 64 ? launch_attn(attn_bwd_kv_kernel<64>, BwdKV<64>::kSmem, pk, device, ks, k64)
                     : launch_attn(attn_bwd_kv_kernel<32>, BwdKV<32>::kSmem, pk, device, ks, k32);
  if (e != cudaSuccess || ks == stream) return e;
  e = cudaEventRecord(join, ks);
  return e == cudaSuccess ? cudaStreamWaitEvent(stream, join, 0) : e;
}

namespace {
SparCudaStatus attention_validate(const float* const* ptrs, int count, uint64_t batch,
                                  uint64_t seq, uint64_t heads, uint64_t head_dim,
                                  uint64_t kv_heads) {
  for (int i = 0; i < count; ++i)
    if (!ptrs[i] || !aligned16(ptrs[i])) return invalid();
  if (batch == 0 || seq == 0 || heads == 0 || !attention_supported(head_dim)) return invalid();
  // repeat_kv_heads' requirement (src/nn/attention.cpp:26-75): kv heads divide the query heads.
  if (kv_heads == 0 || kv_heads > heads || heads % kv_heads != 0) return invalid();
  if (batch * heads > (1ull << 31) || seq > (1ull << 31) ||
      batch * seq * (heads + 2 * kv_heads) * head_dim >= (1ull << 40))
    return invalid();
  return ok();
}
}  // namespace

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_attention_forward_gqa(const float* qkv, float* ctx,
                                                          float* row_max, float* row_inv,
                                                          uint64_t batch, uint64_t seq,
                                                          uint64_t heads, uint64_t kv_heads,
                                                          uint64_t head_dim, int device,
                                                          void* stream) {
  const float* ptrs[4] = {qkv, ctx, row_max, row_inv};
  const SparCudaStatus v = attention_validate(ptrs, 4, batch, seq, heads, head_dim, kv_heads);
  if (v.code) return v;
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = attention_forward_launch(qkv, ctx, row_max, row_inv, batch, seq, heads,
                                                 head_dim, device, static_cast<cudaStream_t>(stream),
                                                 kv_heads);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_attention_forward(const float* qkv, float* ctx, float* row_max,
                                                      float* row_inv, uint64_t batch, uint64_t seq,
                                                      uint64_t heads, uint64_t head_dim, int device,
                                                      void* stream) {
  return spar_b200_attention_forward_gqa(qkv, ctx, row_max, row_inv, batch, seq, heads, heads,
                                         head_dim, device, stream);
}

extern "C" SparCudaStatus spar_b200_attention_backward_gqa(
    const float* qkv, const float* ctx, const float* dctx, const float* row_max,
    const float* row_inv, float* delta, float* dqkv, uint64_t batch, uint64_t seq, uint64_t heads,
    uint64_t kv_heads, uint64_t head_dim, const float* rope_table, int device, void* stream) {
  const float* ptrs[7] = {qkv, ctx, dctx, row_max, row_inv, delta, dqkv};
  const SparCudaStatus v = attention_validate(ptrs, 7, batch, seq, heads, head_dim, kv_heads);
  if (v.code) return v;
  if (rope_table && (reinterpret_cast<uintptr_t>(rope_table) & 7)) return invalid();
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  const cudaError_t e = attention_backward_launch(qkv, ctx, dctx, row_max, row_inv, delta, dqkv,
                                                  batch, seq, heads, head_dim, device,
                                                  static_cast<cudaStream_t>(stream), rope_table,
                                                  nullptr, nullptr, nullptr, kv_heads);
  return e == cudaSuccess ? ok() : runtime(e);
}

extern "C" SparCudaStatus spar_b200_attention_backward(const float* qkv, const float* ctx,
                                                       const float* dctx, const float* row_max,
                                                       const float* row_inv, float* delta,
                                                       float* dqkv, uint64_t batch, uint64_t seq,
                                                       uint64_t heads, uint64_t head_dim,
                                                       const float* rope_table, int device,
                                                       void* stream) {
  return spar_b200_attention_backward_gqa(qkv, ctx, dctx, row_max, row_inv, delta, dqkv, batch,
                                          seq, heads, heads, head_dim, rope_table, device, stream);
}

namespace spar_b200 {
int* attention_wait_flag(int device) {
  static std::mutex mu;
  static int* addr[64] = {};
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    DeviceScope scope(device);
    void* p = nullptr;
    if (scope.error() == cudaSuccess && cudaGetSymbolAddress(&p, g_attn_error) == cudaSuccess)
      addr[device] = static_cast<int*>(p);
    else
      cudaGetLastError();
  }
  return addr[device];
}
}  // namespace spar_b200

extern "C" int spar_b200_attention_error(int device, int clear) {
  DeviceScope scope(device);
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_attn_error, &zero, sizeof(int));
  }
  return v;
}
