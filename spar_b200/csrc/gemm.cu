// Dense fp32 contractions on the sm_100a tensor cores: tcgen05.mma kind::tf32, operands staged
// in shared memory by TMA (128-byte swizzle), fp32 accumulators in TMEM.
//
// This replaces Spar's cuBLAS seam (src/backend/cuda_blas.cppm:122-194: a fresh handle and one
// cublasSgemm per batch matrix, plus permute().contiguous() copies for every transposed operand,
// src/ops/matmul.cpp:140-153). Both operand majors are read in place: a row-major [m, k] A is
// "K-major" for the MMA, a row-major [k, m] (transposed) A is "MN-major"; the same for B. So
// Y = X*W, dX = dY*W^T and dW = X^T*dY run without transposed copies, and the attention products
// run on head-strided views of the fused QKV buffer through 4-D tensor maps.
//
// Kernel shape (persistent, one CTA per SM, 192 threads):
//   warp 0     TMA producer: one elected thread fills a STAGES-deep ring of A/B k-slices
//   warp 1     MMA issuer: one elected thread issues tcgen05.mma (M=128, N=BN, K=8) into one of
//              two TMEM accumulators; tcgen05.commit releases ring slots and publishes tiles
//   warps 2-5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)..+31),
//              alpha/bias/GELU/GELU'/accumulate applied in registers, 128-bit global stores
// The double-buffered accumulator lets the epilogue of tile i overlap the mainloop of tile i+1.
//
// 3xTF32 ("fp32-faithful") mode: A = Ah + Al, B = Bh + Bl with Ah = A rounded to TF32 and
// Al = A - Ah rounded to TF32; the kernel runs over three K sections reading (Ah,Bh), (Ah,Bl),
// (Al,Bh) from split copies made by a streaming kernel, so A*B ~ Ah*Bh + Ah*Bl + Al*Bh
// (error-compensated TF32, Ootomo & Yokota 2022). The tensor cores' fp32 accumulation rounds
// toward zero, so this mode accumulates in chunks of 128 K elements per TMEM accumulator and
// sums the chunks in registers with round-to-nearest adds.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace spar_b200 {

__device__ int g_gemm_error = 0;  // set when a bounded wait expires (read by the host)

namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // 32 fp32 = 128 bytes = one swizzle row
// Threads: producer warp, MMA warp, EW epilogue warps (4: one per TMEM lane quarter; 8: two per
// quarter, splitting each tile's columns, for epilogues with real per-element work).
__host__ __device__ constexpr int threads_for(int ew) { return 64 + 32 * ew; }
__host__ __device__ constexpr uint32_t epi_bytes(int ew) { return ew * 2 * 4096; }  // 2 staging boxes of 4 KB per warp

struct GemmParams {
  CUtensorMap a_map[3];
  CUtensorMap b_map[3];
  CUtensorMap c_map;    // output, {32 cols, 32 rows} boxes, 128-byte swizzle
  CUtensorMap aux_map;  // epilogue side input/output (residual, pre-activation), same boxes
  CUtensorMap part_map;  // split-K partial tiles [kparts][m][n] (raw sums, no epilogue)
  int sections;
  int a_mn_major, b_mn_major;
  uint32_t m, n, k;
  uint32_t batch1;  // inner batch extent (b1); b0 derived
  uint32_t tiles_m, tiles_n;
  uint32_t total_tiles;
  float* c;
  uint64_t ldc, c_bs0, c_bs1;
  float* aux;
  uint64_t ldaux;
  const float* bias;
  float alpha;
  int accumulate, epilogue, causal;
  uint32_t kchunk;  // k-blocks per accumulation chunk (chunked kernels only)
  uint32_t kparts;  // split-K factor (1: no split); partial sums go to part_map
  int round_out;    // round the stored C to nearest TF32
  const float2* rope;  // optional RoPE table [rope_seq, rope_half]
  uint32_t rope_seq, rope_half, rope_dim, rope_cols;
  float* colpart;  // optional [ceil(m / 32), n] per-32-row-block column sums of the output
  int l2_hints;    // paired kernel: operand loads evict_last, C / aux stores evict_first in L2
};

struct TileCoord {
  uint32_t b0, b1, mt, nt, ks;
};

template <int BN>
__device__ __forceinline__ bool decode_tile(const GemmParams& p, uint32_t idx, TileCoord& t) {
  const uint32_t per_split = p.total_tiles / p.kparts;
  t.ks = idx / per_split;
  idx -= t.ks * per_split;
  const uint32_t per_batch = p.tiles_m * p.tiles_n;
  const uint32_t bidx = idx / per_batch;
  const uint32_t r = idx - bidx * per_batch;
  t.b1 = bidx % p.batch1;
  t.b0 = bidx / p.batch1;
  // Grouped raster: 8 M-tiles share each sweep over N for L2 reuse of B.
  constexpr uint32_t G = 8;
  const uint32_t per_group = G * p.tiles_n;
  const uint32_t group = r / per_group;
  const uint32_t first_m = group * G;
  const uint32_t gsize = min(p.tiles_m - first_m, G);
  const uint32_t in_group = r - group * per_group;
  t.mt = first_m + in_group % gsize;
  t.nt = in_group / gsize;
  if (p.causal == SPAR_B200_CAUSAL_LOWER && t.nt * BN >= (t.mt + 1) * BM) return false;
  return true;
}

__device__ __forceinline__ void k_range(const GemmParams& p, const TileCoord& t, uint32_t& kb0,
                                        uint32_t& kb1) {
  const uint32_t mt = t.mt;
  const uint32_t kb_total = (p.k + BK - 1) / BK;
  kb0 = 0;
  kb1 = kb_total;
  if (p.causal == SPAR_B200_CAUSAL_K_UPTO) {
    const uint32_t kend = min(p.k, (mt + 1) * BM);
    kb1 = (kend + BK - 1) / BK;
  } else if (p.causal == SPAR_B200_CAUSAL_K_FROM) {
    kb0 = min((mt * BM) / BK, kb_total);
  }
  if (p.kparts > 1) {  // split t.ks of kparts (the host guarantees every split is non-empty)
    const uint32_t per = (kb1 - kb0 + p.kparts - 1) / p.kparts;
    kb0 = kb0 + t.ks * per;
    kb1 = min(kb1, kb0 + per);
  }
}

__device__ __forceinline__ void record_error() { atomicExch(&g_gemm_error, 1); }

// Byte offset of 16-byte chunk `c` of row `r` in a 32x32 fp32 box stored with the 128-byte
// swizzle (the layout TMA reads and writes for a {32, 32} box): rows of 128 B, chunk index
// XOR-ed with the row's low three bits, so the 8 threads of a shared-memory phase hit 8
// different bank groups.
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) { return r * 128 + ((c ^ (r & 7)) << 4); }

struct EpiState {
  uint8_t* bufs;      // this warp's two 4 KB staging boxes
  uint64_t* aux_bar;  // this warp's two mbarriers for aux-tile loads
  uint32_t aux_phase[2];
  uint32_t sel;
  bool prefetched;    // the aux box of the next epilogue_box call is already on its way
};

__device__ __forceinline__ bool epilogue_needs_aux(const GemmParams& p) {
  return p.kparts == 1 &&
         (p.epilogue == SPAR_B200_EPI_BIAS_ADD || p.epilogue == SPAR_B200_EPI_GELU_BWD);
}

// Starts the TMA load of the aux box that the next epilogue_box call (box at col0, row0) reads,
// into the staging box it will use, so the load overlaps the current box's work. That staging
// box was last written by the store two boxes back: wait until at most one store still reads.
__device__ __forceinline__ void aux_prefetch(const GemmParams& p, EpiState& st, uint32_t col0,
                                             uint32_t row0, uint32_t b1, uint32_t b0) {
  if (!epilogue_needs_aux(p) || st.prefetched) return;
  if ((threadIdx.x & 31) == 0) {
    tc::bulk_wait_read<1>();
    tc::mbar_arrive_expect_tx(st.aux_bar + st.sel, 4096);
    tc::tma_load_4d(st.bufs + st.sel * 4096, &p.aux_map, st.aux_bar + st.sel, col0, row0, b1, b0);
  }
  st.prefetched = true;
}

// Epilogue of one 32 x 32 box (this warp's 32 accumulator rows x 32 columns): optional aux tile
// brought in by TMA, alpha/bias/GELU/GELU'/residual applied in registers (thread = row), the
// result staged in shared memory and written by a TMA store (TMA reduce-add when accumulating).
// Rows/columns outside the matrix are clipped by the tensor maps.
__device__ __forceinline__ void epilogue_box(const GemmParams& p, EpiState& st, float (&v)[32],
                                             uint32_t col0, uint32_t row0, uint32_t b1,
                                             uint32_t b0, uint32_t ks, bool& ok) {
  const int lane = threadIdx.x & 31;
  if (p.kparts > 1) {  // raw partial sum of this K split; the reduction applies the epilogue
    uint8_t* buf = st.bufs + st.sel * 4096;
    if (lane == 0) tc::bulk_wait_read<1>();
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(buf + swz(lane, c)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tc::tma_store_4d(&p.part_map, buf, col0, row0, ks, 0);
      tc::bulk_commit();
    }
    st.sel ^= 1;
    return;
  }
  const bool needs_aux = p.epilogue == SPAR_B200_EPI_BIAS_ADD || p.epilogue == SPAR_B200_EPI_GELU_BWD;
  const bool two_outputs = p.epilogue == SPAR_B200_EPI_BIAS_GELU;
  uint8_t* buf = st.bufs + st.sel * 4096;
  uint8_t* buf2 = st.bufs + (st.sel ^ 1) * 4096;
  // The staging box (both boxes for two outputs) must be free of earlier stores.
  if (lane == 0) {
    if (two_outputs) tc::bulk_wait_read<0>();
    else tc::bulk_wait_read<1>();
  }
  __syncwarp();
  if (needs_aux && !st.prefetched) {
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(st.aux_bar + st.sel, 4096);
      tc::tma_load_4d(buf, &p.aux_map, st.aux_bar + st.sel, col0, row0, b1, b0);
    }
  }
  st.prefetched = false;
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] *= p.alpha;
  if (p.bias && (p.epilogue == SPAR_B200_EPI_BIAS || p.epilogue == SPAR_B200_EPI_BIAS_GELU ||
                 p.epilogue == SPAR_B200_EPI_BIAS_ADD)) {
    if (col0 + 32 <= p.n && (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0) {
      // Same 32 values for every lane: eight broadcast 16-byte loads.
      const float4* b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 b = __ldg(b4 + i);
        v[4 * i] += b.x;
        v[4 * i + 1] += b.y;
        v[4 * i + 2] += b.z;
        v[4 * i + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (col0 + e < p.n) v[e] += __ldg(p.bias + col0 + e);
    }
  }
  if (needs_aux) {
    if (!tc::mbar_wait(st.aux_bar + st.sel, st.aux_phase[st.sel])) {
      record_error();
      ok = false;
    }
    st.aux_phase[st.sel] ^= 1;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 q = *reinterpret_cast<const float4*>(buf + swz(lane, c));
      const float a4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (p.epilogue == SPAR_B200_EPI_BIAS_ADD) v[4 * c + e] += a4[e];
        else v[4 * c + e] *= gelu_derivative_fast(a4[e]);
      }
    }
  }
  if (two_outputs) {  // pre-activation to aux, gelu(pre) to C
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(buf2 + swz(lane, c)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = gelu_value_fast(v[e]);
  }
  if (p.rope && col0 < p.rope_cols) {  // RoPE on this row's 16 column pairs
    const uint32_t pos = (row0 + lane) % p.rope_seq;
    const float2* tab = p.rope + static_cast<uint64_t>(pos) * p.rope_half;
    const uint32_t pair0 = (col0 % p.rope_dim) / 2;
    const bool one_head = pair0 + 16 <= p.rope_half;  // the box does not cross a head boundary
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t pair = one_head ? pair0 + i : ((col0 + 2 * i) % p.rope_dim) / 2;
      const float2 cs = __ldg(tab + pair);
      const float x0 = v[2 * i], x1 = v[2 * i + 1];
      v[2 * i] = x0 * cs.x - x1 * cs.y;
      v[2 * i + 1] = x0 * cs.y + x1 * cs.x;
    }
  }
  // This box's column sums (a bias gradient's partials), before rounding. Boxes wholly below
  // row m (the rest of a tile that overhangs the matrix) have no row of the partials array.
  if (p.colpart && row0 < p.m) {
    const float cs = box_column_sum(v, row0 + lane < p.m);
    if (col0 + lane < p.n) p.colpart[static_cast<uint64_t>(row0 / 32) * p.n + col0 + lane] = cs;
  }
  if (p.round_out) {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = round_tf32(v[e]);
  }
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<float4*>(buf + swz(lane, c)) =
        make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  tc::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (p.l2_hints) {
      const uint64_t pol = tc::policy_evict_first();
      if (two_outputs) tc::tma_store_4d_hint(&p.aux_map, buf2, col0, row0, b1, b0, pol);
      if (p.accumulate) tc::tma_reduce_add_4d(&p.c_map, buf, col0, row0, b1, b0);
      else tc::tma_store_4d_hint(&p.c_map, buf, col0, row0, b1, b0, pol);
    } else {
      if (two_outputs) tc::tma_store_4d(&p.aux_map, buf2, col0, row0, b1, b0);
      if (p.accumulate) tc::tma_reduce_add_4d(&p.c_map, buf, col0, row0, b1, b0);
      else tc::tma_store_4d(&p.c_map, buf, col0, row0, b1, b0);
    }
    tc::bulk_commit();
  }
  st.sel ^= 1;
}

// CHUNKED (3xTF32): the tile's K range is accumulated in chunks of p.kchunk k-blocks, each chunk
// into a fresh TMEM accumulator that the epilogue adds into fp32 registers with round-to-nearest
// adds. The tensor cores' own accumulation rounds toward zero, so long hardware-accumulated
// sums drift; chunking bounds that drift to one chunk, which keeps the split mode fp32-faithful
// at any K.
template <int BN, int STAGES, bool CHUNKED, int EW>
__global__ void __launch_bounds__(threads_for(EW), 1) gemm_tf32_kernel(const __grid_constant__ GemmParams p) {
  static_assert(EW == 4 || (EW == 8 && !CHUNKED), "epilogue warps");
  constexpr uint32_t kEpiBytes = epi_bytes(EW);
  constexpr uint32_t A_BYTES = BM * BK * 4;
  constexpr uint32_t B_BYTES = BN * BK * 4;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + STAGES * STAGE_BYTES;  // EW warps x 2 staging boxes x 4 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + kEpiBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* aux_bars = drain + 1;  // EW warps x 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bars + 2 * EW);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full + s, 1);
      tc::mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(tfull + b, 1);
      tc::mbar_init(tempty + b, EW);
    }
    tc::mbar_init(drain, 1);
    for (int b = 0; b < 2 * EW; ++b) tc::mbar_init(aux_bars + b, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < p.sections; ++s) {
      tc::tma_prefetch(&p.a_map[s]);
      tc::tma_prefetch(&p.b_map[s]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_begin();  // set-up done; global memory from here on

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (tc::elect_one()) {
      uint32_t stage = 0, phase = 0;
      int last_phase[STAGES];  // parity of the last fill issued into each slot (-1: never)
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
      for (uint32_t idx = blockIdx.x; idx < p.total_tiles && !*abort_flag; idx += gridDim.x) {
        TileCoord t;
        if (!decode_tile<BN>(p, idx, t)) continue;
        uint32_t kb0, kb1;
        k_range(p, t, kb0, kb1);
        const int m0 = static_cast<int>(t.mt * BM), n0 = static_cast<int>(t.nt * BN);
        for (uint32_t kb = kb0; kb < kb1 && !*abort_flag; ++kb) {
          const int k0 = static_cast<int>(kb * BK);
          for (int sec = 0; sec < p.sections; ++sec) {
            if (!tc::mbar_wait(empty + stage, phase ^ 1)) {
              record_error();
              *abort_flag = 1;
              break;
            }
            uint8_t* a_s = smem + stage * STAGE_BYTES;
            uint8_t* b_s = a_s + A_BYTES;
            tc::mbar_arrive_expect_tx(full + stage, STAGE_BYTES);
            last_phase[stage] = static_cast<int>(phase);
            if (p.a_mn_major) {
#pragma unroll
              for (int j = 0; j < BM / 32; ++j)
                tc::tma_load_4d(a_s + j * 4096, &p.a_map[sec], full + stage, m0 + 32 * j, k0,
                                t.b1, t.b0);
            } else {
              tc::tma_load_4d(a_s, &p.a_map[sec], full + stage, k0, m0, t.b1, t.b0);
            }
            if (p.b_mn_major) {
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                tc::tma_load_4d(b_s + j * 4096, &p.b_map[sec], full + stage, n0 + 32 * j, k0,
                                t.b1, t.b0);
            } else {
              tc::tma_load_4d(b_s, &p.b_map[sec], full + stage, k0, n0, t.b1, t.b0);
            }
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      // Every copy issued into a slot must have landed before the CTA exits (this matters only
      // when a consumer gave up early; in the normal path these phases completed long ago).
#pragma unroll
      for (int s = 0; s < STAGES; ++s)
        if (last_phase[s] >= 0 && !tc::mbar_wait(full + s, static_cast<uint32_t>(last_phase[s])))
          record_error();
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t idesc = tc::idesc_tf32(BM, BN, p.a_mn_major, p.b_mn_major);
    if (tc::elect_one()) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      for (uint32_t idx = blockIdx.x; idx < p.total_tiles && !*abort_flag; idx += gridDim.x) {
        TileCoord t;
        if (!decode_tile<BN>(p, idx, t)) continue;
        uint32_t kb0, kb1;
        k_range(p, t, kb0, kb1);
        const uint32_t chunk = CHUNKED ? p.kchunk : (kb1 - kb0);
        for (uint32_t c0 = kb0; c0 < kb1 && !*abort_flag; c0 += chunk) {
          const uint32_t c1 = min(c0 + chunk, kb1);
          if (!tc::mbar_wait(tempty + acc, acc_phase ^ 1)) {
            record_error();
            *abort_flag = 1;
            break;
          }
          tc::tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          uint32_t issued = 0;
          for (uint32_t kb = c0; kb < c1 && !*abort_flag; ++kb) {
            for (int sec = 0; sec < p.sections; ++sec) {
              if (!tc::mbar_wait(full + stage, phase)) {
                record_error();
                *abort_flag = 1;
                break;
              }
              tc::tc_fence_after();
              const uint32_t a_addr = tc::smem_u32(smem + stage * STAGE_BYTES);
              const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
              for (int ks = 0; ks < BK / 8; ++ks) {
                // K-major: 8 rows of 128 B per 1024 B atom, K step = 32 B inside the row.
                // MN-major: 32-element MN chunks (one TMA box of 32 K-rows = 4 KB) at LBO, 4-row
                // K groups at SBO = 512 B, K step = 8 rows = 1024 B.
                const uint64_t a_desc =
                    p.a_mn_major
                        ? tc::smem_desc(a_addr + ks * 1024, 4096, 512, tc::kLayoutSw128Base32)
                        : tc::smem_desc(a_addr + ks * 32, 16, 1024, tc::kLayoutSw128);
                const uint64_t b_desc =
                    p.b_mn_major
                        ? tc::smem_desc(b_addr + ks * 1024, 4096, 512, tc::kLayoutSw128Base32)
                        : tc::smem_desc(b_addr + ks * 32, 16, 1024, tc::kLayoutSw128);
                tc::mma_tf32(d_tmem, a_desc, b_desc, idesc, (issued | ks) != 0 ? 1u : 0u);
              }
              issued = 1;
              tc::mma_commit(empty + stage);
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1;
              }
            }
          }
          tc::mma_commit(tfull + acc);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
      // Make sure every MMA has retired before TMEM is released.
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0)) record_error();
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..)
    const uint32_t quarter = static_cast<uint32_t>(warp & 3);
    const uint32_t ew = static_cast<uint32_t>(warp - 2);
    constexpr int kChunks = BN / 32 / (EW / 4);  // 32-column boxes per warp and tile
    const int chunk0 = static_cast<int>(ew / 4) * kChunks;
    EpiState st;
    st.bufs = epi_smem + ew * 8192;
    st.aux_bar = aux_bars + ew * 2;
    st.aux_phase[0] = st.aux_phase[1] = 0;
    st.sel = 0;
    st.prefetched = false;
    bool ok = true;
    uint32_t acc = 0, acc_phase = 0;
    for (uint32_t idx = blockIdx.x; idx < p.total_tiles && ok; idx += gridDim.x) {
      TileCoord t;
      if (!decode_tile<BN>(p, idx, t)) continue;
      if (*abort_flag) break;
      const uint32_t row0 = t.mt * BM + quarter * 32;
      const uint32_t lane_base = tmem_base + ((quarter * 32) << 16);
      if constexpr (!CHUNKED) {
        if (t.nt * BN + chunk0 * 32 < p.n) aux_prefetch(p, st, t.nt * BN + chunk0 * 32, row0, t.b1, t.b0);
        if (!tc::mbar_wait(tfull + acc, acc_phase)) {
          record_error();
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
#pragma unroll 1
        for (int chunk = chunk0; chunk < chunk0 + kChunks; ++chunk) {
          const uint32_t col0 = t.nt * BN + chunk * 32;
          uint32_t r[32];
          tc::tmem_load_32x32(lane_base + acc * BN + chunk * 32, r);
          if (col0 >= p.n) continue;
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
          epilogue_box(p, st, v, col0, row0, t.b1, t.b0, t.ks, ok);
          if (chunk + 1 < chunk0 + kChunks && col0 + 32 < p.n)
            aux_prefetch(p, st, col0 + 32, row0, t.b1, t.b0);
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(tempty + acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      } else {
        uint32_t kb0, kb1;
        k_range(p, t, kb0, kb1);
        float sum[BN];
        for (uint32_t c0 = kb0; c0 < kb1; c0 += p.kchunk) {
          if (!tc::mbar_wait(tfull + acc, acc_phase)) {
            record_error();
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc::tc_fence_after();
#pragma unroll
          for (int chunk = 0; chunk < BN / 32; ++chunk) {
            uint32_t r[32];
            tc::tmem_load_32x32(lane_base + acc * BN + chunk * 32, r);
#pragma unroll
            for (int e = 0; e < 32; ++e)
              sum[chunk * 32 + e] = c0 == kb0 ? __uint_as_float(r[e])
                                              : sum[chunk * 32 + e] + __uint_as_float(r[e]);
          }
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(tempty + acc);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
        if (!ok) break;
#pragma unroll
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          const uint32_t col0 = t.nt * BN + chunk * 32;
          if (col0 >= p.n) continue;
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = sum[chunk * 32 + e];
          epilogue_box(p, st, v, col0, row0, t.b1, t.b0, t.ks, ok);
        }
      }
    }
    if (!ok) *abort_flag = 1;
    // A prefetched aux load left unused (the loop was abandoned) must land before the CTA exits.
    if (st.prefetched && !tc::mbar_wait(st.aux_bar + st.sel, st.aux_phase[st.sel])) record_error();
    // All staged stores must have finished before the CTA (and its shared memory) goes away.
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem_base, TMEM_COLS);
}

// ----------------------------------------------------------------- paired-SM GEMM
// A cluster of two CTAs on two SMs computes one 256 x 256 tile with tcgen05.mma.cta_group::2:
// CTA r loads rows [128r, 128r + 128) of the A tile and rows [128r, 128r + 128) of the B tile's
// N extent into its own shared memory, and its TMEM receives its 128 rows of the 256 x 256
// accumulator. Per FLOP this moves a third fewer operand bytes from L2 than two independent
// 128 x 256 tiles, and each stage is 32 KB instead of 48 KB, so more stages fit.
// Roles (both CTAs): warp 0 TMA producer into its own shared memory, completing on the even CTA's
// "full" barrier (armed by the even CTA for both CTAs' bytes); warp 1 of the even CTA issues every
// MMA; warps 2.. epilogue of the CTA's own rows.
// Completions: the MMA commits each stage's "empty" and each accumulator's "full" to the barrier
// of the same name in both CTAs (two plain commits); both CTAs' epilogue warps arrive on the even
// CTA's accumulator-empty barrier. Every wait is bounded; the closing cluster barrier keeps each
// CTA (and its shared memory) alive until the even CTA has drained or given up.
// DRAIN (concatenated 3xTF32 products): the tile's K range is accumulated in chunks of p.kchunk
// k-blocks, alternating between the two TMEM accumulators; the epilogue warps add each chunk into
// fp32 registers (round-to-nearest adds) and apply the epilogue to those sums after the last
// chunk. The tensor cores' accumulation rounds toward zero, so the drift of a long hardware sum
// is bounded by one chunk, without partial tiles in HBM.
template <int BN, int STAGES, int EW, bool DRAIN = false>
__global__ void __launch_bounds__(threads_for(EW), 1) gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  static_assert(BN == 256 || BN == 128, "paired tile N");
  static_assert(!DRAIN || BN / 32 / (EW / 4) <= 2, "drained sums: at most 64 registers a thread");
  constexpr int BNH = BN / 2;  // B rows (N) staged by each CTA
  constexpr uint32_t A_BYTES = BM * BK * 4;
  constexpr uint32_t B_BYTES = BNH * BK * 4;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t kEpiBytes = epi_bytes(EW);
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulator buffers of BN columns

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + kEpiBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* aux_bars = drain + 1;  // EW warps x 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bars + 2 * EW);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full + s, 1);  // even CTA: armed by its producer with both CTAs' bytes
      tc::mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(tfull + b, 1);
      tc::mbar_init(tempty + b, 2 * EW);  // epilogue warps of both CTAs (even CTA's barrier)
    }
    tc::mbar_init(drain, 1);
    for (int b = 0; b < 2 * EW; ++b) tc::mbar_init(aux_bars + b, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tc::tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tc::tma_prefetch(&p.a_map[0]);
    tc::tma_prefetch(&p.b_map[0]);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrival
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_begin();  // set-up done; global memory from here on

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (tc::elect_one()) {
      uint32_t stage = 0, phase = 0;
      int last_phase[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = -1;
      const uint64_t keep = p.l2_hints ? tc::policy_evict_last() : 0;
      for (uint32_t idx = cluster; idx < p.total_tiles && !*abort_flag; idx += nclusters) {
        TileCoord t;
        if (!decode_tile<BN>(p, idx, t)) continue;
        uint32_t kb0, kb1;
        k_range(p, t, kb0, kb1);
        const int m0 = static_cast<int>(t.mt * 256 + rank * BM);
        const int n0 = static_cast<int>(t.nt * BN + rank * BNH);
        for (uint32_t kb = kb0; kb < kb1 && !*abort_flag; ++kb) {
          const int k0 = static_cast<int>(kb * BK);
          if (!tc::mbar_wait_cluster(empty + stage, phase ^ 1)) {
            record_error();
            *abort_flag = 1;
            break;
          }
          uint8_t* a_s = smem + stage * STAGE_BYTES;
          uint8_t* b_s = a_s + A_BYTES;
          const uint32_t fb = tc::map_to_rank(tc::smem_u32(full + stage), 0);
          if (leader) {
            tc::mbar_arrive_expect_tx(full + stage, 2 * STAGE_BYTES);
            last_phase[stage] = static_cast<int>(phase);
          }
          if (p.l2_hints) {
            if (p.a_mn_major) {
#pragma unroll
              for (int j = 0; j < BM / 32; ++j)
                tc::tma_load_4d_pair_hint(a_s + j * 4096, &p.a_map[0], fb, m0 + 32 * j, k0, 0, 0,
                                          keep);
            } else {
              tc::tma_load_4d_pair_hint(a_s, &p.a_map[0], fb, k0, m0, 0, 0, keep);
            }
            if (p.b_mn_major) {
#pragma unroll
              for (int j = 0; j < BNH / 32; ++j)
                tc::tma_load_4d_pair_hint(b_s + j * 4096, &p.b_map[0], fb, n0 + 32 * j, k0, 0, 0,
                                          keep);
            } else {
              tc::tma_load_4d_pair_hint(b_s, &p.b_map[0], fb, k0, n0, 0, 0, keep);
            }
          } else {
            if (p.a_mn_major) {
#pragma unroll
              for (int j = 0; j < BM / 32; ++j)
                tc::tma_load_4d_pair(a_s + j * 4096, &p.a_map[0], fb, m0 + 32 * j, k0, 0, 0);
            } else {
              tc::tma_load_4d_pair(a_s, &p.a_map[0], fb, k0, m0, 0, 0);
            }
            if (p.b_mn_major) {
#pragma unroll
              for (int j = 0; j < BNH / 32; ++j)
                tc::tma_load_4d_pair(b_s + j * 4096, &p.b_map[0], fb, n0 + 32 * j, k0, 0, 0);
            } else {
              tc::tma_load_4d_pair(b_s, &p.b_map[0], fb, k0, n0, 0, 0);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every armed stage (both CTAs' bytes) must have landed before the pair exits.
#pragma unroll
      for (int s = 0; s < STAGES; ++s)
        if (last_phase[s] >= 0 && !tc::mbar_wait_cluster(full + s, static_cast<uint32_t>(last_phase[s])))
          record_error();
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA;
    // warp 1 of the odd CTA has no role after the TMEM allocation)
    const uint32_t idesc = tc::idesc_tf32(256, BN, p.a_mn_major, p.b_mn_major);
    if (leader && tc::elect_one()) {
      const uint32_t peer = 1;
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      for (uint32_t idx = cluster; idx < p.total_tiles && !*abort_flag; idx += nclusters) {
        TileCoord t;
        if (!decode_tile<BN>(p, idx, t)) continue;
        uint32_t kb0, kb1;
        k_range(p, t, kb0, kb1);
        const uint32_t chunk = DRAIN ? p.kchunk : kb1 - kb0;
        for (uint32_t c0 = kb0; c0 < kb1 && !*abort_flag; c0 += chunk) {
          const uint32_t c1 = min(kb1, c0 + chunk);
          if (!tc::mbar_wait_cluster(tempty + acc, acc_phase ^ 1)) {
            record_error();
            *abort_flag = 1;
            break;
          }
          tc::tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          for (uint32_t kb = c0; kb < c1 && !*abort_flag; ++kb) {
            if (!tc::mbar_wait_cluster(full + stage, phase)) {
              record_error();
              *abort_flag = 1;
              break;
            }
            tc::tc_fence_after();
            const uint32_t a_addr = tc::smem_u32(smem + stage * STAGE_BYTES);
            const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
            for (int ks = 0; ks < BK / 8; ++ks) {
              const uint64_t a_desc =
                  p.a_mn_major ? tc::smem_desc(a_addr + ks * 1024, 4096, 512, tc::kLayoutSw128Base32)
                               : tc::smem_desc(a_addr + ks * 32, 16, 1024, tc::kLayoutSw128);
              const uint64_t b_desc =
                  p.b_mn_major ? tc::smem_desc(b_addr + ks * 1024, 4096, 512, tc::kLayoutSw128Base32)
                               : tc::smem_desc(b_addr + ks * 32, 16, 1024, tc::kLayoutSw128);
              tc::mma_tf32_pair(d_tmem, a_desc, b_desc, idesc, (kb != c0 || ks != 0) ? 1u : 0u);
            }
            const uint32_t e = tc::smem_u32(empty + stage);
            tc::mma_commit_pair(e);
            tc::mma_commit_pair(tc::map_to_rank(e, peer));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          const uint32_t f = tc::smem_u32(tfull + acc);
          tc::mma_commit_pair(f);
          tc::mma_commit_pair(tc::map_to_rank(f, peer));
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
      tc::mma_commit_pair(tc::smem_u32(drain));
      if (!tc::mbar_wait(drain, 0)) record_error();
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..)
    const uint32_t quarter = static_cast<uint32_t>(warp & 3);
    const uint32_t ew = static_cast<uint32_t>(warp - 2);
    constexpr int kChunks = BN / 32 / (EW / 4);
    const int chunk0 = static_cast<int>(ew / 4) * kChunks;
    EpiState st;
    st.bufs = epi_smem + ew * 8192;
    st.aux_bar = aux_bars + ew * 2;
    st.aux_phase[0] = st.aux_phase[1] = 0;
    st.sel = 0;
    st.prefetched = false;
    bool ok = true;
    uint32_t acc = 0, acc_phase = 0;
    const uint32_t tempty_leader = tc::map_to_rank(tc::smem_u32(tempty), 0);
    for (uint32_t idx = cluster; idx < p.total_tiles && ok; idx += nclusters) {
      TileCoord t;
      if (!decode_tile<BN>(p, idx, t)) continue;
      if (*abort_flag) break;
      const uint32_t row0 = t.mt * 256 + rank * BM + quarter * 32;
      const uint32_t lane_base = tmem_base + ((quarter * 32) << 16);
      if (t.nt * BN + chunk0 * 32 < p.n) aux_prefetch(p, st, t.nt * BN + chunk0 * 32, row0, t.b1, t.b0);
      if constexpr (DRAIN) {
        constexpr int kC = kChunks;
        uint32_t kb0, kb1;
        k_range(p, t, kb0, kb1);
        const uint32_t nchunks = (kb1 - kb0 + p.kchunk - 1) / p.kchunk;
        float sum[kC][32];
#pragma unroll
        for (int c = 0; c < kC; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) sum[c][e] = 0.f;
        for (uint32_t ci = 0; ci < nchunks; ++ci) {
          if (!tc::mbar_wait_cluster(tfull + acc, acc_phase)) {
            record_error();
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc::tc_fence_after();
#pragma unroll
          for (int c = 0; c < kC; ++c) {
            uint32_t r[32];
            tc::tmem_load_32x32(lane_base + acc * BN + (chunk0 + c) * 32, r);
#pragma unroll
            for (int e = 0; e < 32; ++e) sum[c][e] += __uint_as_float(r[e]);
          }
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive_cluster(tempty_leader + acc * 8);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < kC; ++c) {
          const uint32_t col0 = t.nt * BN + (chunk0 + c) * 32;
          if (col0 >= p.n) continue;
          epilogue_box(p, st, sum[c], col0, row0, t.b1, t.b0, t.ks, ok);
          if (c + 1 < kC && col0 + 32 < p.n) aux_prefetch(p, st, col0 + 32, row0, t.b1, t.b0);
        }
        continue;
      }
      if (!tc::mbar_wait_cluster(tfull + acc, acc_phase)) {
        record_error();
        *abort_flag = 1;
        break;
      }
      tc::tc_fence_after();
#pragma unroll 1
      for (int chunk = chunk0; chunk < chunk0 + kChunks; ++chunk) {
        const uint32_t col0 = t.nt * BN + chunk * 32;
        uint32_t r[32];
        tc::tmem_load_32x32(lane_base + acc * BN + chunk * 32, r);
        if (col0 >= p.n) continue;
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
        epilogue_box(p, st, v, col0, row0, t.b1, t.b0, t.ks, ok);
        if (chunk + 1 < chunk0 + kChunks && col0 + 32 < p.n)
          aux_prefetch(p, st, col0 + 32, row0, t.b1, t.b0);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(tempty_leader + acc * 8);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (!ok) *abort_flag = 1;
    if (st.prefetched && !tc::mbar_wait(st.aux_bar + st.sel, st.aux_phase[st.sel])) record_error();
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // the pair's MMAs and both epilogues are done with TMEM
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

// ----------------------------------------------------------------- 3xTF32 operand split
// Both halves are rounded to nearest TF32 (round_tf32), so the tensor cores see exact TF32
// values and the split error is unbiased: hi = rn(x), lo = rn(x - hi).

__global__ void split_tf32_kernel(float* __restrict__ hi, float* __restrict__ lo,
                                  const float* __restrict__ src, uint64_t inner, uint64_t rows,
                                  uint64_t b1, uint64_t b0, uint64_t ld, uint64_t bs1,
                                  uint64_t bs0, uint64_t out_ld) {
  pdl_begin();
  const uint64_t total = inner * rows * b1 * b0;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const uint64_t x = i % inner;
    uint64_t rest = i / inner;
    const uint64_t r = rest % rows;
    rest /= rows;
    const uint64_t q1 = rest % b1, q0 = rest / b1;
    const float v = src[q0 * bs0 + q1 * bs1 + r * ld + x];
    const float h = round_tf32(v);
    const uint64_t o = ((q0 * b1 + q1) * rows + r) * out_ld + x;
    hi[o] = h;
    lo[o] = round_tf32(v - h);
  }
}

// 3xTF32 as one TF32 product of depth 3 kp (kp = k rounded up to a multiple of 4): the operands
// are written with their three K sections side by side, A' = [hi | hi | lo] and B' = [hi; lo; hi]
// (sections zero-padded from k to kp), so A' B' = hi hi + hi lo + lo hi accumulated in fp32 by the
// fast TF32 kernels (paired-SM 256-column tiles, split-K, every epilogue) instead of a dedicated
// three-section kernel. `k_inner`: K runs along the source rows' contiguous dimension (the
// section offset s * kp is added to the column; otherwise to the row). parts: 0 = (hi, hi, lo),
// 1 = (hi, lo, hi).
__global__ void split_concat_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                    uint64_t inner, uint64_t rows, uint64_t ld, uint64_t out_ld,
                                    uint64_t kp, int k_inner, int parts) {
  pdl_begin();
  // Covers the padded extent along K (kp instead of k) so the pad is written as zeros.
  const uint64_t inner_p = k_inner ? kp : inner, rows_p = k_inner ? rows : kp;
  const uint64_t total = inner_p * rows_p;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const uint64_t x = i % inner_p, r = i / inner_p;
    const bool real = x < inner && r < rows;
    const float v = real ? src[r * ld + x] : 0.f;
    const float h = round_tf32(v);
    const float l = round_tf32(v - h);
    const float sec[3] = {h, parts == 0 ? h : l, parts == 0 ? l : h};
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const uint64_t o = k_inner ? r * out_ld + q * kp + x : (q * kp + r) * out_ld + x;
      dst[o] = sec[q];
    }
  }
}

// Whether a 3xTF32 product runs as one TF32 product over K-concatenated split operands (unbatched,
// non-causal) rather than in the three-section kernel.
bool concat_x3(const SparB200Gemm& g) {
  return g.precision == SPAR_B200_TF32X3 && (g.batch[0] ? g.batch[0] : 1) == 1 &&
         (g.batch[1] ? g.batch[1] : 1) == 1 && g.causal == SPAR_B200_CAUSAL_NONE;
}

// The operand layouts of that product: A' and B' sizes in floats and their leading dimensions.
struct ConcatShape {
  uint64_t kp, a_ld, a_floats, b_ld, b_floats;
};
ConcatShape concat_shape(const SparB200Gemm& g) {
  auto pad = [](uint64_t x) { return (x + 3) & ~3ull; };
  ConcatShape c;
  c.kp = pad(g.k);
  // A logical [m, k]: stored [m, k] (K inner) or [k, m] (K along rows).
  c.a_ld = g.a_transposed ? pad(g.m) : 3 * c.kp;
  c.a_floats = g.a_transposed ? 3 * c.kp * c.a_ld : g.m * c.a_ld;
  // B logical [k, n]: stored [k, n] (K along rows) or [n, k] (K inner).
  c.b_ld = g.b_transposed ? 3 * c.kp : pad(g.n);
  c.b_floats = g.b_transposed ? g.n * c.b_ld : 3 * c.kp * c.b_ld;
  return c;
}

// Split-K reduction and epilogue: the partial tiles [kparts][m][ldp] are summed in split order
// (deterministic), then the GEMM's epilogue is applied exactly as the tile epilogue does it
// (alpha, bias, residual / GELU' aux, bias + GELU with the pre-activation to aux, RoPE,
// rounding to TF32, accumulate into C). A thread owns four adjacent columns of a row; the last
// group of a row may hold fewer (n not a multiple of 4), and C / aux are accessed element by
// element unless their rows are 16-byte aligned (`vec`). ldp is a multiple of 4, so the partials
// are always read four at a time (the columns past n there are never used).
struct SplitEpilogue {
  float* c;
  uint64_t ldc;
  const float* part;
  uint64_t ldp;
  uint32_t kparts, m, n;
  float alpha;
  int accumulate, epilogue, round_out, vec;
  const float* bias;
  float* aux;
  uint64_t ldaux;
  const float2* rope;
  uint32_t rope_seq, rope_dim, rope_cols, rope_half;
  float* colpart;  // optional [ceil(m / 32)][n] column sums of each 32-row block
};

// One row's group of up to four columns: the partial sums added in split order, the epilogue,
// the store. `pre` receives the values before rounding (what the column partials sum).
__device__ __forceinline__ void reduce_group(const SplitEpilogue& q, uint64_t r, uint32_t col,
                                             float (&pre)[4]) {
  const uint32_t cnt = min(4u, q.n - col);  // columns of this group inside the matrix
  const bool vec = q.vec && cnt == 4;
  const uint64_t plane = static_cast<uint64_t>(q.m) * q.ldp;
  const bool bias = q.bias && (q.epilogue == SPAR_B200_EPI_BIAS ||
                               q.epilogue == SPAR_B200_EPI_BIAS_GELU ||
                               q.epilogue == SPAR_B200_EPI_BIAS_ADD);
  const float* src = q.part + r * q.ldp + col;
  float4 acc = *reinterpret_cast<const float4*>(src);
  for (uint32_t s = 1; s < q.kparts; ++s) {
    const float4 x = *reinterpret_cast<const float4*>(src + s * plane);
    acc.x += x.x;
    acc.y += x.y;
    acc.z += x.z;
    acc.w += x.w;
  }
  float v[4] = {q.alpha * acc.x, q.alpha * acc.y, q.alpha * acc.z, q.alpha * acc.w};
  if (bias) {
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (static_cast<uint32_t>(e) < cnt) v[e] += __ldg(q.bias + col + e);
  }
  float* auxp = q.aux ? q.aux + r * q.ldaux + col : nullptr;
  if (q.epilogue == SPAR_B200_EPI_BIAS_ADD || q.epilogue == SPAR_B200_EPI_GELU_BWD) {
    float a4[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec) {
      const float4 x = *reinterpret_cast<const float4*>(auxp);
      a4[0] = x.x; a4[1] = x.y; a4[2] = x.z; a4[3] = x.w;
    } else {
      for (uint32_t e = 0; e < cnt; ++e) a4[e] = auxp[e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (q.epilogue == SPAR_B200_EPI_BIAS_ADD) v[e] += a4[e];
      else v[e] *= gelu_derivative_fast(a4[e]);
    }
  } else if (q.epilogue == SPAR_B200_EPI_BIAS_GELU) {
    if (vec) {
      *reinterpret_cast<float4*>(auxp) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      for (uint32_t e = 0; e < cnt; ++e) auxp[e] = v[e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = gelu_value_fast(v[e]);
  }
  if (q.rope && col < q.rope_cols) {  // rope_cols and the head width are even: whole pairs
    const float2* tab = q.rope + (r % q.rope_seq) * q.rope_half;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float2 cs = __ldg(tab + ((col + 2 * k) % q.rope_dim) / 2);
      const float x0 = v[2 * k], x1 = v[2 * k + 1];
      v[2 * k] = x0 * cs.x - x1 * cs.y;
      v[2 * k + 1] = x0 * cs.y + x1 * cs.x;
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) pre[e] = static_cast<uint32_t>(e) < cnt ? v[e] : 0.f;
  if (q.round_out) {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = round_tf32(v[e]);
  }
  float* out = q.c + r * q.ldc + col;
  if (vec) {
    float4* dst = reinterpret_cast<float4*>(out);
    float4 o = make_float4(v[0], v[1], v[2], v[3]);
    if (q.accumulate) {
      const float4 prev = *dst;
      o.x += prev.x;
      o.y += prev.y;
      o.z += prev.z;
      o.w += prev.w;
    }
    *dst = o;
  } else {
    for (uint32_t e = 0; e < cnt; ++e) out[e] = q.accumulate ? out[e] + v[e] : v[e];
  }
}

// Thread = (row, four-column group); with column partials, thread = (32-row block, four-column
// group), which walks the block's rows and writes the block's column sums of the epilogue output
// (before rounding) to colpart[block][n], as the tile epilogue does for an unsplit product.
__global__ void splitk_reduce_kernel(const __grid_constant__ SplitEpilogue q) {
  pdl_begin();
  const uint32_t n4 = (q.n + 3) / 4;
  const uint64_t rows = q.colpart ? (static_cast<uint64_t>(q.m) + 31) / 32 : q.m;
  const uint64_t total = rows * n4;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const uint64_t r = i / n4;
    const uint32_t col = static_cast<uint32_t>(i % n4) * 4;
    float pre[4];
    if (!q.colpart) {
      reduce_group(q, r, col, pre);
      continue;
    }
    float cs[4] = {0.f, 0.f, 0.f, 0.f};
    const uint64_t r1 = r * 32 + 32 < q.m ? r * 32 + 32 : q.m;
    for (uint64_t row = r * 32; row < r1; ++row) {
      reduce_group(q, row, col, pre);
#pragma unroll
      for (int e = 0; e < 4; ++e) cs[e] += pre[e];
    }
    const uint32_t cnt = min(4u, q.n - col);
    for (uint32_t e = 0; e < cnt; ++e) q.colpart[r * q.n + col + e] = cs[e];
  }
}

}  // namespace

// ----------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Stored operand view: element (x, r) of batch (q1, q0) at base + q0*bs0 + q1*bs1 + r*ld + x,
// x the contiguous index. Box = 32 contiguous elements x box_rows rows.
// MN-major boxes use the 32-byte-atom 128-byte swizzle that the MMA descriptor above expects.
bool make_map(CUtensorMap* map, const float* base, uint64_t inner, uint64_t rows, uint64_t b1,
              uint64_t b0, uint64_t ld, uint64_t bs1, uint64_t bs0, uint32_t box_rows,
              bool mn_major) {
  auto fn = encode_fn();
  if (!fn) return false;
  if (bs1 == 0) bs1 = ld * rows;
  if (bs0 == 0) bs0 = bs1 * b1;
  cuuint64_t dims[4] = {inner, rows, b1, b0};
  cuuint64_t strides[3] = {ld * 4, bs1 * 4, bs0 * 4};
  cuuint32_t box[4] = {32, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

template <int BN, int STAGES, bool CHUNKED, int EW = 4>
cudaError_t launch_kernel(const GemmParams& p, int device, cudaStream_t stream) {
  constexpr size_t smem = STAGES * (BM * BK * 4 + BN * BK * 4) + epi_bytes(EW) + 1024 + 256;
  static_assert(smem <= 232448, "GEMM shared memory");
  static bool configured[64] = {false};
  auto k = gemm_tf32_kernel<BN, STAGES, CHUNKED, EW>;
  if (device < 0 || device >= 64 || !configured[device]) {
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    if (device >= 0 && device < 64) configured[device] = true;
  }
  const unsigned grid = std::min<uint32_t>(p.total_tiles, static_cast<uint32_t>(sm_count(device)));
  return launch(k, dim3(grid), dim3(threads_for(EW)), smem, stream, p);
}

// Paired-SM launch: clusters of two CTAs, at most as many clusters as fit at once.
template <int BN, int STAGES, int EW, bool DRAIN = false>
cudaError_t launch_pair(const GemmParams& p, int device, cudaStream_t stream) {
  constexpr size_t smem = STAGES * (BM * BK * 4 + (BN / 2) * BK * 4) + epi_bytes(EW) + 1024 + 256;
  static_assert(smem <= 232448, "paired GEMM shared memory");
  static int max_clusters[64] = {0};
  auto k = gemm_pair_kernel<BN, STAGES, EW, DRAIN>;
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(threads_for(EW));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!max_clusters[device]) {
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(2 * (sm_count(device) / 2));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, k, &cfg);
    if (e != cudaSuccess) return e;
    max_clusters[device] = n > 0 ? n : 1;
  }
  const uint32_t clusters = std::min<uint32_t>(p.total_tiles, static_cast<uint32_t>(max_clusters[device]));
  cfg.gridDim = dim3(2 * clusters);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, k, p);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

uint64_t gemm_split_workspace_floats(const SparB200Gemm& g) {
  if (concat_x3(g)) {
    const ConcatShape c = concat_shape(g);
    return c.a_floats + c.b_floats;
  }
  const uint64_t b = g.batch[0] * g.batch[1];
  const uint64_t a_inner = g.a_transposed ? g.m : g.k, a_rows = g.a_transposed ? g.k : g.m;
  const uint64_t b_inner = g.b_transposed ? g.k : g.n, b_rows = g.b_transposed ? g.n : g.k;
  auto pad = [](uint64_t x) { return (x + 3) & ~3ull; };
  return 2 * b * (pad(a_inner) * a_rows + pad(b_inner) * b_rows);
}

// How a TF32 product runs, from a small timing model of the persistent kernels: tiles of
// tile_m x tile_n on `units` parallel units (SM pairs or SMs) that each finish a tile of depth k in
// 2 * tile_m * tile_n * k / rate + overhead, optionally split `parts` ways along K into partial
// tiles that a reduction pass then streams (parts + 1 planes of m x n floats, plus the aux plane).
// Rates and overheads are per unit, measured on B200 at C5 shapes.
struct TileModel {
  uint64_t tm, tn;
  double rate;         // FLOP/s per unit
  double overhead_us;  // per tile: accumulator hand-off, epilogue tail
  int units;
};

double model_us(const SparB200Gemm& g, const TileModel& t, uint32_t parts) {
  const uint64_t tiles = ((g.m + t.tm - 1) / t.tm) * ((g.n + t.tn - 1) / t.tn);
  const uint64_t kb = (g.k + BK - 1) / BK;
  const double kper = static_cast<double>((kb + parts - 1) / parts) * BK;
  const double rounds = static_cast<double>((tiles * parts + t.units - 1) / t.units);
  double us = rounds * (2.0 * t.tm * t.tn * kper / t.rate * 1e6 + t.overhead_us);
  if (parts > 1) {
    const bool aux_in = g.epilogue == SPAR_B200_EPI_BIAS_ADD || g.epilogue == SPAR_B200_EPI_GELU_BWD;
    us += 3.0 + (parts + 1 + (aux_in ? 1 : 0)) * static_cast<double>(g.m) * g.n * 4.0 / 5.0e12 * 1e6;
  }
  return us;
}

// Whether K may be split: TF32 products without causal limits or batching (the reduction pass
// applies any epilogue).
bool splittable(const SparB200Gemm& g) {
  return g.precision == SPAR_B200_TF32 && g.causal == SPAR_B200_CAUSAL_NONE && g.batch[0] <= 1 &&
         g.batch[1] <= 1 && g.n % 4 == 0;
}

// The paired kernel marks its operand loads evict_last and its C / aux stores evict_first in L2,
// so streamed outputs do not push reused operand tiles out (measured at 16384 x 4096 x 1024 with
// the bias + GELU epilogue: 0.251 -> 0.246 ms; the C5 step +0.45 %). SPAR_B200_L2_HINTS=0: no hints.
bool l2_hints_enabled() {
  static const bool on = [] {
    const char* e = getenv("SPAR_B200_L2_HINTS");
    return !(e && e[0] == '0');
  }();
  return on;
}

// SPAR_B200_SPLITK_MAX caps the K splits the planner may choose (1: never split); default 8.
uint32_t max_splits() {
  static const uint32_t v = [] {
    const char* e = getenv("SPAR_B200_SPLITK_MAX");
    const int n = e ? atoi(e) : 8;
    return static_cast<uint32_t>(n < 1 ? 1 : (n > 8 ? 8 : n));
  }();
  return v;
}

// Fewest modelled microseconds over K splits 1..8 (at least 8 k-blocks per split) for tile model t.
uint32_t best_parts(const SparB200Gemm& g, const TileModel& t, double* best_us) {
  const uint64_t kblocks = (g.k + BK - 1) / BK;
  uint32_t best = 1;
  double us = model_us(g, t, 1);
  if (splittable(g))
    for (uint32_t parts = 2; parts <= max_splits() && parts * 8 <= kblocks; ++parts) {
      const double u = model_us(g, t, parts);
      if (u < 0.97 * us) {
        us = u;
        best = parts;
      }
    }
  if (best_us) *best_us = us;
  return best;
}

// How a GEMM runs: unbatched non-causal TF32 products with m >= 256 on SM pairs (256 x 256 or
// 256 x 128 tiles over 2-CTA clusters, whichever the model finishes first), everything else
// (batched, causal, 3xTF32, short) on single SMs; either may split K.
struct GemmPlan {
  bool pair;
  int bn;
  uint32_t kparts;
};

GemmPlan gemm_plan(const SparB200Gemm& g, int device, bool narrow_only = false) {
  const bool x3 = g.precision == SPAR_B200_TF32X3;
  const uint64_t b = (g.batch[0] ? g.batch[0] : 1) * (g.batch[1] ? g.batch[1] : 1);
  const int sms = sm_count(device);
  GemmPlan pl;
  pl.pair = false;
  pl.bn = x3 ? 64 : (g.n > 128 ? 256 : (g.n > 64 ? 128 : 64));
  pl.kparts = 1;
  if (x3) return pl;
  if (b == 1 && g.causal == SPAR_B200_CAUSAL_NONE && g.m >= 256 && g.n > 64) {
    const TileModel wide{256, 256, 10.0e12, 1.0, sms / 2};
    const TileModel narrow{256, 128, 7.0e12, 1.0, sms / 2};  // half the reuse of each A stage
    double us_wide = 1e30, us_narrow = 0.0;
    uint32_t parts_wide = 1;
    if (g.n > 128 && !narrow_only) parts_wide = best_parts(g, wide, &us_wide);
    const uint32_t parts_narrow = best_parts(g, narrow, &us_narrow);
    pl.pair = true;
    if (us_wide <= us_narrow) {
      pl.bn = 256;
      pl.kparts = parts_wide;
    } else {
      pl.bn = 128;
      pl.kparts = parts_narrow;
    }
    return pl;
  }
  const TileModel single{BM, static_cast<uint64_t>(pl.bn), pl.bn == 256 ? 5.0e12 : 3.5e12, 1.0, sms};
  pl.kparts = best_parts(g, single, nullptr);
  return pl;
}

// Longest K (in 32-element blocks) a concatenated 3xTF32 product accumulates in one tensor-core
// accumulator. The accumulator's adds round toward zero, so the error grows with the number of
// K = 8 steps added into it. Measured on a C5-width training step against float64: K' = 3 x 16384
// in one accumulator 1.3e-4, at most 3072 per accumulator 1.9e-5, sums moved to fp32 registers
// every 3 x 128 (the three-section kernel) 2.4e-6. On SM pairs the kernel itself moves the sums
// into fp32 registers every kX3DrainBlocks k-blocks (DRAIN); single-SM plans split K into parts of
// at most kX3MaxBlocks k-blocks whose partial tiles the reduction pass sums in fp32.
constexpr uint32_t kX3DrainBlocks = 8;  // 256 K' elements (32 accumulator steps) per drain
constexpr uint32_t kX3MaxBlocks = 16;   // 512 K' elements (64 accumulator steps) per partial

uint32_t x3_min_parts(uint64_t k) {
  const uint64_t kb = (k + BK - 1) / BK;
  return static_cast<uint32_t>((kb + kX3MaxBlocks - 1) / kX3MaxBlocks);
}

// The concatenated product t (TF32 over K' = 3 kp) drains its accumulator on SM pairs when the
// plan puts it there (256 x 128 tiles, eight epilogue warps: 64 fp32 sums a thread).
bool x3_drains(const SparB200Gemm& t, int device) { return gemm_plan(t, device, true).pair; }

// A K split hands the epilogue, column partials included, to the reduction kernel.
GemmPlan gemm_plan_for(const SparB200Gemm& g, int device, uint32_t min_parts = 1,
                       bool drain = false) {
  GemmPlan pl = gemm_plan(g, device, drain);
  if (pl.kparts < min_parts) {
    pl.kparts = min_parts;
    // every split non-empty: (parts - 1) full splits of ceil(kb / parts) blocks stay below kb
    const uint64_t kb = (g.k + BK - 1) / BK;
    while (pl.kparts > 1 && (pl.kparts - 1) * ((kb + pl.kparts - 1) / pl.kparts) >= kb)
      --pl.kparts;
  }
  return pl;
}

uint64_t gemm_splitk_workspace_floats(const SparB200Gemm& g, int device) {
  uint32_t min_parts = 1;
  SparB200Gemm t = g;
  bool drain = false;
  if (concat_x3(g)) {  // planned as the TF32 product it becomes
    t.precision = SPAR_B200_TF32;
    t.k = 3 * concat_shape(g).kp;
    drain = x3_drains(t, device);
    if (!drain) min_parts = x3_min_parts(t.k);
  }
  const GemmPlan pl = gemm_plan_for(t, device, min_parts, drain);
  return pl.kparts > 1 ? static_cast<uint64_t>(pl.kparts) * t.m * ((t.n + 3) / 4 * 4) : 0;
}

cudaError_t gemm_launch_plan(const SparB200Gemm& g, float* split_workspace, int device,
                             cudaStream_t stream, float* splitk_workspace, uint64_t splitk_floats,
                             uint32_t min_parts, bool drain);

cudaError_t gemm_launch(const SparB200Gemm& g, float* split_workspace, int device,
                        cudaStream_t stream, float* splitk_workspace = nullptr,
                        uint64_t splitk_floats = 0, uint32_t min_parts = 1) {
  return gemm_launch_plan(g, split_workspace, device, stream, splitk_workspace, splitk_floats,
                          min_parts, false);
}

cudaError_t gemm_launch_plan(const SparB200Gemm& g, float* split_workspace, int device,
                             cudaStream_t stream, float* splitk_workspace, uint64_t splitk_floats,
                             uint32_t min_parts, bool drain) {
  if (concat_x3(g)) {
    const ConcatShape c = concat_shape(g);
    float* a2 = split_workspace;
    float* b2 = split_workspace + c.a_floats;
    const int sms = sm_count(device);
    const uint64_t a_inner = g.a_transposed ? g.m : g.k, a_rows = g.a_transposed ? g.k : g.m;
    const uint64_t b_inner = g.b_transposed ? g.k : g.n, b_rows = g.b_transposed ? g.n : g.k;
    cudaError_t e = launch(split_concat_kernel, dim3(sms * 8), dim3(256), 0, stream, a2, g.a,
                           a_inner, a_rows, g.lda, c.a_ld, c.kp, g.a_transposed ? 0 : 1, 0);
    if (e == cudaSuccess)
      e = launch(split_concat_kernel, dim3(sms * 8), dim3(256), 0, stream, b2, g.b, b_inner,
                 b_rows, g.ldb, c.b_ld, c.kp, g.b_transposed ? 1 : 0, 1);
    if (e != cudaSuccess) return e;
    SparB200Gemm t = g;
    t.precision = SPAR_B200_TF32;
    t.k = 3 * c.kp;
    t.a = a2;
    t.lda = c.a_ld;
    t.b = b2;
    t.ldb = c.b_ld;
    const bool d = x3_drains(t, device);
    return gemm_launch_plan(t, nullptr, device, stream, splitk_workspace, splitk_floats,
                            d ? 1 : x3_min_parts(t.k), d);
  }
  GemmParams p;
  memset(&p, 0, sizeof(p));
  const uint64_t b1 = g.batch[1] ? g.batch[1] : 1, b0 = g.batch[0] ? g.batch[0] : 1;
  const bool split = g.precision == SPAR_B200_TF32X3;
  // 3xTF32 keeps its running sums in registers (one 64-column row segment per thread).
  const GemmPlan plan = gemm_plan_for(g, device, min_parts, drain);
  const int bn = plan.bn;
  drain = drain && plan.pair && bn == 128;
  p.sections = split ? 3 : 1;
  p.a_mn_major = g.a_transposed ? 1 : 0;
  p.b_mn_major = g.b_transposed ? 0 : 1;

  const uint64_t a_inner = g.a_transposed ? g.m : g.k, a_rows = g.a_transposed ? g.k : g.m;
  const uint64_t b_inner = g.b_transposed ? g.k : g.n, b_rows = g.b_transposed ? g.n : g.k;
  const bool pair = plan.pair;
  const uint32_t a_box_rows = p.a_mn_major ? BK : BM;
  const uint32_t b_box_rows = p.b_mn_major ? BK : static_cast<uint32_t>(pair ? bn / 2 : bn);

  if (!split) {
    if (!make_map(&p.a_map[0], g.a, a_inner, a_rows, b1, b0, g.lda, g.a_batch_stride[1],
                  g.a_batch_stride[0], a_box_rows, p.a_mn_major) ||
        !make_map(&p.b_map[0], g.b, b_inner, b_rows, b1, b0, g.ldb, g.b_batch_stride[1],
                  g.b_batch_stride[0], b_box_rows, p.b_mn_major))
      return cudaErrorInvalidValue;
  } else {
    auto pad = [](uint64_t x) { return (x + 3) & ~3ull; };
    const uint64_t a_ld = pad(a_inner), b_ld = pad(b_inner);
    float* ah = split_workspace;
    float* al = ah + b0 * b1 * a_ld * a_rows;
    float* bh = al + b0 * b1 * a_ld * a_rows;
    float* bl = bh + b0 * b1 * b_ld * b_rows;
    const int sms = sm_count(device);
    cudaError_t e = launch(split_tf32_kernel, dim3(sms * 8), dim3(256), 0, stream, ah, al, g.a,
                           a_inner, a_rows, b1, b0, g.lda, g.a_batch_stride[1],
                           g.a_batch_stride[0], a_ld);
    if (e == cudaSuccess)
      e = launch(split_tf32_kernel, dim3(sms * 8), dim3(256), 0, stream, bh, bl, g.b, b_inner,
                 b_rows, b1, b0, g.ldb, g.b_batch_stride[1], g.b_batch_stride[0], b_ld);
    if (e != cudaSuccess) return e;
    const uint64_t abs1 = a_ld * a_rows, abs0 = abs1 * b1;
    const uint64_t bbs1 = b_ld * b_rows, bbs0 = bbs1 * b1;
    const float* am[3] = {ah, ah, al};
    const float* bm[3] = {bh, bl, bh};
    for (int s = 0; s < 3; ++s) {
      if (!make_map(&p.a_map[s], am[s], a_inner, a_rows, b1, b0, a_ld, abs1, abs0, a_box_rows,
                    p.a_mn_major) ||
          !make_map(&p.b_map[s], bm[s], b_inner, b_rows, b1, b0, b_ld, bbs1, bbs0, b_box_rows,
                    p.b_mn_major))
        return cudaErrorInvalidValue;
    }
  }
  if (!make_map(&p.c_map, g.c, g.n, g.m, b1, b0, g.ldc, g.c_batch_stride[1], g.c_batch_stride[0],
                32, false))
    return cudaErrorInvalidValue;
  if (g.aux && !make_map(&p.aux_map, g.aux, g.n, g.m, b1, b0, g.ldaux, g.c_batch_stride[1],
                         g.c_batch_stride[0], 32, false))
    return cudaErrorInvalidValue;
  p.m = static_cast<uint32_t>(g.m);
  p.n = static_cast<uint32_t>(g.n);
  p.k = static_cast<uint32_t>(g.k);
  p.batch1 = static_cast<uint32_t>(b1);
  p.tiles_m = static_cast<uint32_t>(pair ? (g.m + 255) / 256 : (g.m + BM - 1) / BM);
  p.tiles_n = static_cast<uint32_t>((g.n + bn - 1) / bn);
  p.total_tiles = static_cast<uint32_t>(p.tiles_m * p.tiles_n * b0 * b1);
  p.c = g.c;
  p.ldc = g.ldc;
  p.c_bs0 = g.c_batch_stride[0];
  p.c_bs1 = g.c_batch_stride[1];
  p.aux = g.aux;
  p.ldaux = g.ldaux;
  p.bias = g.bias;
  p.alpha = g.alpha;
  p.accumulate = g.accumulate;
  p.epilogue = g.epilogue;
  p.causal = g.causal;
  p.kchunk = 4;  // 4 k-blocks = 128 K elements x 3 sections per hardware-accumulated chunk
  p.kparts = 1;
  p.round_out = g.round_output != 0;
  p.colpart = g.column_partials;
  p.l2_hints = l2_hints_enabled() && pair ? 1 : 0;
  if (g.rope_table) {
    p.rope = reinterpret_cast<const float2*>(g.rope_table);
    p.rope_seq = static_cast<uint32_t>(g.rope_seq);
    p.rope_half = static_cast<uint32_t>(g.rope_dim / 2);
    p.rope_dim = static_cast<uint32_t>(g.rope_dim);
    p.rope_cols = static_cast<uint32_t>(g.rope_cols);
  }
  const uint32_t kparts = plan.kparts;
  const uint64_t ldp = (g.n + 3) / 4 * 4;
  if (kparts > 1 && splitk_workspace && splitk_floats >= kparts * g.m * ldp) {
    if (!make_map(&p.part_map, splitk_workspace, g.n, g.m, kparts, 1, ldp, g.m * ldp,
                  kparts * g.m * ldp, 32, false))
      return cudaErrorInvalidValue;
    p.kparts = kparts;
    p.total_tiles *= kparts;
    if (drain) p.kchunk = kX3DrainBlocks;
    const cudaError_t e = drain     ? launch_pair<128, 6, 8, true>(p, device, stream)
                        : pair      ? (bn == 256 ? launch_pair<256, 6, 4>(p, device, stream)
                                                 : launch_pair<128, 8, 4>(p, device, stream))
                        : bn == 256 ? launch_kernel<256, 4, false>(p, device, stream)
                        : bn == 128 ? launch_kernel<128, 6, false>(p, device, stream)
                                    : launch_kernel<64, 8, false>(p, device, stream);
    if (e != cudaSuccess) return e;
    SplitEpilogue q;
    q.c = g.c;
    q.ldc = g.ldc;
    q.part = splitk_workspace;
    q.ldp = ldp;
    q.kparts = kparts;
    q.m = static_cast<uint32_t>(g.m);
    q.n = static_cast<uint32_t>(g.n);
    q.alpha = g.alpha;
    q.accumulate = g.accumulate;
    q.epilogue = g.epilogue;
    q.round_out = g.round_output != 0;
    q.bias = g.bias;
    q.aux = g.aux;
    q.ldaux = g.ldaux;
    const auto rows16 = [](const void* ptr, uint64_t ld) {
      return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ld % 4 == 0;
    };
    q.vec = rows16(g.c, g.ldc) && (!g.aux || rows16(g.aux, g.ldaux)) ? 1 : 0;
    q.colpart = g.column_partials;
    q.rope = p.rope;
    q.rope_seq = p.rope_seq;
    q.rope_dim = p.rope_dim;
    q.rope_cols = p.rope_cols;
    q.rope_half = p.rope_half;
    const uint64_t work = (g.column_partials ? (g.m + 31) / 32 : g.m) * ((g.n + 3) / 4);
    return launch(splitk_reduce_kernel, dim3(grid_for(work, 256, sm_count(device) * 8)), dim3(256),
                  0, stream, q);
  }
  if (split) return launch_kernel<64, 8, true>(p, device, stream);
  if (drain) {
    p.kchunk = kX3DrainBlocks;
    return launch_pair<128, 6, 8, true>(p, device, stream);
  }
  // Epilogues with per-element work beyond a bias add (GELU, GELU', residual / aux tiles, RoPE)
  // get eight epilogue warps (one fewer operand stage makes room for their staging boxes).
  const bool heavy = g.epilogue == SPAR_B200_EPI_BIAS_GELU || g.epilogue == SPAR_B200_EPI_GELU_BWD ||
                     g.epilogue == SPAR_B200_EPI_BIAS_ADD || g.rope_table;
  if (pair)
    return bn == 256 ? (heavy ? launch_pair<256, 5, 8>(p, device, stream)
                              : launch_pair<256, 6, 4>(p, device, stream))
                     : (heavy ? launch_pair<128, 6, 8>(p, device, stream)
                              : launch_pair<128, 8, 4>(p, device, stream));
  if (heavy) {
    switch (bn) {
      case 256:
        return launch_kernel<256, 3, false, 8>(p, device, stream);
      case 128:
        return launch_kernel<128, 5, false, 8>(p, device, stream);
      default:
        return launch_kernel<64, 6, false, 8>(p, device, stream);
    }
  }
  switch (bn) {
    case 256:
      return launch_kernel<256, 4, false>(p, device, stream);
    case 128:
      return launch_kernel<128, 6, false>(p, device, stream);
    default:
      return launch_kernel<64, 8, false>(p, device, stream);
  }
}

SparCudaStatus gemm_validate(const SparB200Gemm* g) {
  if (!g) return invalid();
  const SparB200Gemm& x = *g;
  const uint64_t b1 = x.batch[1] ? x.batch[1] : 1, b0 = x.batch[0] ? x.batch[0] : 1;
  if (x.m == 0 || x.n == 0 || x.k == 0) return invalid();
  if (x.m > 0x7fffffffull || x.n > 0x7fffffffull || x.k > 0x7fffffffull) return invalid();
  if ((x.m + BM - 1) / BM * ((x.n + 63) / 64) * b0 * b1 > 0xffffffffull) return invalid();
  if (!x.a || !x.b || !x.c) return invalid();
  if (!aligned16(x.a) || !aligned16(x.b) || !aligned16(x.c)) return invalid();
  if (x.lda % 4 || x.ldb % 4 || x.ldc % 4 || x.a_batch_stride[0] % 4 || x.a_batch_stride[1] % 4 ||
      x.b_batch_stride[0] % 4 || x.b_batch_stride[1] % 4 || x.c_batch_stride[0] % 4 ||
      x.c_batch_stride[1] % 4)
    return invalid();
  const uint64_t a_inner = x.a_transposed ? x.m : x.k;
  const uint64_t b_inner = x.b_transposed ? x.k : x.n;
  if (x.lda < a_inner || x.ldb < b_inner || x.ldc < x.n) return invalid();
  if (x.epilogue < 0 || x.epilogue > SPAR_B200_EPI_BIAS_ADD) return invalid();
  if ((x.epilogue == SPAR_B200_EPI_BIAS || x.epilogue == SPAR_B200_EPI_BIAS_GELU) && !x.bias)
    return invalid();
  if ((x.epilogue == SPAR_B200_EPI_BIAS_GELU || x.epilogue == SPAR_B200_EPI_GELU_BWD ||
       x.epilogue == SPAR_B200_EPI_BIAS_ADD) &&
      (!x.aux || !aligned16(x.aux) || x.ldaux % 4 || x.ldaux < x.n))
    return invalid();
  if (x.precision != SPAR_B200_TF32 && x.precision != SPAR_B200_TF32X3) return invalid();
  if (x.causal < 0 || x.causal > SPAR_B200_CAUSAL_K_FROM) return invalid();
  if (x.causal == SPAR_B200_CAUSAL_LOWER && x.m != x.n) return invalid();
  if (x.rope_table &&
      (x.rope_seq == 0 || x.rope_dim == 0 || x.rope_dim % 2 || x.rope_cols % x.rope_dim ||
       x.rope_cols > x.n || b0 * b1 != 1 || x.accumulate || x.rope_seq > 0x7fffffffull ||
       x.rope_cols > 0x7fffffffull || (x.epilogue != SPAR_B200_EPI_NONE && x.epilogue != SPAR_B200_EPI_BIAS)))
    return invalid();
  if ((x.causal == SPAR_B200_CAUSAL_K_UPTO || x.causal == SPAR_B200_CAUSAL_K_FROM) && x.m != x.k)
    return invalid();
  if (x.column_partials && (b0 * b1 != 1 || x.causal != SPAR_B200_CAUSAL_NONE)) return invalid();
  return ok();
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_gemm(const SparB200Gemm* gemm, int device, void* stream) {
  const SparCudaStatus v = gemm_validate(gemm);
  if (v.code != 0) return v;
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return runtime(scope.error());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* ws = nullptr;
  float* kws = nullptr;
  if (gemm->precision == SPAR_B200_TF32X3) {
    const cudaError_t e = stream_alloc(reinterpret_cast<void**>(&ws),
                                          gemm_split_workspace_floats(*gemm) * sizeof(float), s);
    if (e != cudaSuccess) return runtime(e);
  }
  const uint64_t kfloats = gemm_splitk_workspace_floats(*gemm, device);
  if (kfloats) {
    const cudaError_t e = stream_alloc(reinterpret_cast<void**>(&kws), kfloats * sizeof(float), s);
    if (e != cudaSuccess) return runtime(e);
  }
  const cudaError_t e = gemm_launch(*gemm, ws, device, s, kws, kfloats);
  if (ws) cudaFreeAsync(ws, s);
  if (kws) cudaFreeAsync(kws, s);
  return e == cudaSuccess ? ok() : runtime(e);
}

namespace spar_b200 {
int* gemm_wait_flag(int device) {
  static std::mutex mu;
  static int* addr[64] = {};
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    DeviceScope scope(device);
    void* p = nullptr;
    if (scope.error() == cudaSuccess && cudaGetSymbolAddress(&p, g_gemm_error) == cudaSuccess)
      addr[device] = static_cast<int*>(p);
    else
      cudaGetLastError();
  }
  return addr[device];
}
}  // namespace spar_b200

extern "C" int spar_b200_gemm_error(int device, int clear) {
  DeviceScope scope(device);
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int));
  }
  return v;
}

// Host-side fault injection for tests of the error path: sets (or clears) the flag that a GEMM
// (kernel 0) or attention (kernel 1) kernel raises when one of its bounded waits expires, without
// running a kernel that waits. No GPU work is left in an undefined state.
extern "C" int spar_b200_set_wait_error(int device, int kernel, int value) {
  if (kernel != 0 && kernel != 1) return -1;
  DeviceScope scope(device);
  if (scope.error() != cudaSuccess) return -1;
  const int v = value ? 1 : 0;
  int* flag = kernel == 0 ? gemm_wait_flag(device) : attention_wait_flag(device);
  if (!flag) return -1;
  const cudaError_t e = cudaMemcpy(flag, &v, sizeof(int), cudaMemcpyHostToDevice);
  return e == cudaSuccess ? 0 : -1;
}
