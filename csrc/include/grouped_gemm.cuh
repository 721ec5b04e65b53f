// Persistent, warp-specialised grouped GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   out[row_map(r), n] = epilogue( sum_k A[r, k] * B[expert(seg), n, k] )
//
// A is a row-major [rows_total, K] activation buffer whose rows are grouped in
// "segments" (one segment = consecutive rows that share an expert weight, e.g.
// the rows that source rank s sent to local expert e).  B is the stacked
// expert weight tensor [E * N, K] (K-major, i.e. nn.Linear layout).
//
// Roles inside one CTA (kGemmThreads = 320 threads, one CTA per SM):
//   warp 0      TMA producer: streams 128-row A tiles and BN-row B tiles into
//               an S-stage shared-memory ring (128-byte swizzle, per-CTA loads).
//   warp 1      owns the TMEM allocation; one elected lane issues tcgen05.mma
//               (M=128, N=BN, fp32 accumulators in TMEM, two accumulator
//               buffers so the epilogue of tile i overlaps the MMAs of i+1).
//   warps 2..9  epilogue: tcgen05.ld of the accumulator rows, bias, activation,
//               optional per-row scale, and vector stores to a local or
//               NVLink-peer output pointer chosen per segment (two warps per
//               row quarter, each on half of the tile's columns).
//
// Reference behaviour being replaced: the per-expert index_select / two
// torch matmuls / index_copy_ loop of rlccl/transport/reference_full_moe.py:271-280.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sm100_ptx.cuh"

namespace raiccl {

template <int BN, bool TF32>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int ELEM = TF32 ? 4 : 2;
  static constexpr int BK = 128 / ELEM;           // one 128-byte swizzle atom of K
  static constexpr int UK = 32 / ELEM;            // K per tcgen05.mma (32 bytes)
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM_BUDGET = 200 * 1024;
  static constexpr int STAGES_RAW = SMEM_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int TMEM_COLS = (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64 : (2 * BN) <= 128 ? 128 : (2 * BN) <= 256 ? 256 : 512;
  static constexpr uint32_t IDESC = umma_idesc(TF32 ? 2u : 1u, BM, BN);
  static constexpr int SMEM_TOTAL = 1024 /*align slack*/ + STAGES * STAGE_BYTES + 256 /*barriers*/;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
  static_assert(STAGES >= 2, "pipeline needs two stages");
};

__device__ __forceinline__ float apply_act(float x, Act a) {
  switch (a) {
    case Act::kRelu: return x > 0.f ? x : 0.f;
    case Act::kGelu: return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
    case Act::kSilu: return x / (1.f + __expf(-x));
    default: return x;
  }
}

__device__ __forceinline__ int find_segment(const int* prefix, int nseg, int tile) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;  // plain load: written by the previous launch
  }
  return lo;
}

// Epilogue warps per CTA.  tcgen05.ld lets warp w read TMEM lanes
// [32 (w % 4), 32 (w % 4) + 32), so warps w and w + 4 share a row quarter and
// split its columns: two warps per SM sub-partition hide each other's TMEM-load,
// bias and store latency.
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kSplitMinKBlocks = 4;  // K blocks per split at least (split-K)

// bar.sync on a named barrier among `threads` threads (the epilogue warps).
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The same barrier, returning whether `pred` holds in every participating thread.
__device__ __forceinline__ bool named_barrier_and(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %3, 0;\n\t"
      "bar.red.and.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(threads), "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void store16(float* dst, const float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 16; j += 4) *(float4*)(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}

__device__ __forceinline__ void store16(__nv_bfloat16* dst, const float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 16; j += 8) {
    uint4 w;
    __nv_bfloat162 h0 = __floats2bfloat162_rn(v[j], v[j + 1]);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(v[j + 2], v[j + 3]);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[j + 4], v[j + 5]);
    __nv_bfloat162 h3 = __floats2bfloat162_rn(v[j + 6], v[j + 7]);
    w.x = *(uint32_t*)&h0; w.y = *(uint32_t*)&h1; w.z = *(uint32_t*)&h2; w.w = *(uint32_t*)&h3;
    *(uint4*)(dst + j) = w;
  }
}

// 16 bias values as four 16-byte loads (zeros without a bias).
__device__ __forceinline__ void load_bias16(const float* bias, float (&b)[16]) {
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    const float4 q = bias ? __ldg((const float4*)(bias + j)) : make_float4(0.f, 0.f, 0.f, 0.f);
    b[j] = q.x; b[j + 1] = q.y; b[j + 2] = q.z; b[j + 3] = q.w;
  }
}

// Epilogue of one accumulator row (one thread per row) over the tile columns
// [c0, c1) (multiples of 16; for SwiGLU, columns of the gate half): bias,
// activation, optional per-row scale, vector stores to the segment's output
// pointer at the mapped row.  Two 16-column TMEM loads are in flight per wait.
// t_row: TMEM address of the row's first column.
template <int BN, Act ACT, typename OutT>
__device__ __forceinline__ void gemm_epilogue_row(const GroupedGemmParams& p, const GemmSegment& seg, int nb,
                                                  int r_local, uint32_t t_row, int c0, int c1) {
  const bool valid = r_local < seg.rows;
  const int arow = seg.a_row0 + r_local;
  long long orow = 0;
  float scale = 1.f;
  if (valid) {
    orow = p.row_map ? (long long)__ldg(p.row_map + arow) : (long long)(seg.out_row0 + r_local);
    if (p.row_scale) scale = __ldg(p.row_scale + arow);
  }
  OutT* out = (OutT*)p.out_ptrs[seg.out_slot];
  const float* bias = p.bias ? p.bias + (long long)seg.expert * p.N + nb * BN : nullptr;
  if constexpr (ACT == Act::kSwiGLU) {
    // Tile columns [0, BN/2) hold gate features, [BN/2, BN) the matching up features.
    constexpr int HALF = BN / 2;
    static_assert(HALF % 16 == 0, "SwiGLU tile needs BN multiple of 32");
#pragma unroll 1
    for (int c = c0; c < c1; c += 16) {
      uint32_t g[16], u[16];
      tmem_ld16(t_row + c, g);
      tmem_ld16(t_row + HALF + c, u);
      tmem_ld_wait();
      if (valid) {
        float bg[16], bu[16], v[16];
        load_bias16(bias ? bias + c : nullptr, bg);
        load_bias16(bias ? bias + HALF + c : nullptr, bu);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float gv = __uint_as_float(g[j]) + bg[j];
          const float uv = __uint_as_float(u[j]) + bu[j];
          v[j] = (gv / (1.f + __expf(-gv))) * uv * scale;
        }
        store16(out + orow * p.ldo + nb * HALF + c, v);
      }
    }
  } else {
#pragma unroll 1
    for (int c = c0; c < c1; c += 32) {
      const bool two = c + 16 < c1;
      uint32_t r0[16], r1[16];
      tmem_ld16(t_row + c, r0);
      if (two) tmem_ld16(t_row + c + 16, r1);
      tmem_ld_wait();
      if (valid) {
        float b[16], v[16];
        load_bias16(bias ? bias + c : nullptr, b);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = apply_act(__uint_as_float(r0[j]) + b[j], ACT) * scale;
        store16(out + orow * p.ldo + nb * BN + c, v);
        if (two) {
          load_bias16(bias ? bias + c + 16 : nullptr, b);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = apply_act(__uint_as_float(r1[j]) + b[j], ACT) * scale;
          store16(out + orow * p.ldo + nb * BN + c + 16, v);
        }
      }
    }
  }
}

// Split-K epilogue, partial part: the row's accumulator columns [c0, c1) as
// fp32 into its split's partial tile (rows of 128, BN columns).
template <int BN>
__device__ __forceinline__ void gemm_partial_row(float* part_row, uint32_t t_row, int c0, int c1) {
#pragma unroll 1
  for (int c = c0; c < c1; c += 16) {
    uint32_t r[16];
    tmem_ld16(t_row + c, r);
    tmem_ld_wait();
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
    store16(part_row + c, v);
  }
}

// Split-K epilogue, final part (the tile's last split): the row's columns
// [c0, c1) summed over the S partial tiles in split order (read through L2:
// other SMs wrote them), then bias, activation, row scale and the output
// store as in gemm_epilogue_row.  part0: the row in split 0's partial tile;
// stride: floats from one split's partial tile to the next.
template <int BN, Act ACT, typename OutT>
__device__ __forceinline__ void gemm_sum_row(const GroupedGemmParams& p, const GemmSegment& seg, int nb, int r_local,
                                             const float* part0, long long stride, int S, int c0, int c1) {
  if (r_local >= seg.rows) return;
  const int arow = seg.a_row0 + r_local;
  const long long orow = p.row_map ? (long long)__ldg(p.row_map + arow) : (long long)(seg.out_row0 + r_local);
  const float scale = p.row_scale ? __ldg(p.row_scale + arow) : 1.f;
  OutT* out = (OutT*)p.out_ptrs[seg.out_slot];
  const float* bias = p.bias ? p.bias + (long long)seg.expert * p.N + nb * BN : nullptr;
#pragma unroll 1
  for (int c = c0; c < c1; c += 16) {
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.f;
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
      const float4* src = (const float4*)(part0 + s * stride + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 q = __ldcg(src + j);
        acc[4 * j] += q.x;
        acc[4 * j + 1] += q.y;
        acc[4 * j + 2] += q.z;
        acc[4 * j + 3] += q.w;
      }
    }
    float b[16], v[16];
    load_bias16(bias ? bias + c : nullptr, b);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = apply_act(acc[j] + b[j], ACT) * scale;
    store16(out + orow * p.ldo + nb * BN + c, v);
  }
}

// Staged epilogue (CTA-pair kernel): per 64-byte row piece (16 fp32 or 32
// bf16 columns) the warp writes its 32 rows into a padded shared-memory tile
// (row pitch 80 bytes: the row-wise 16-byte writes of eight lanes hit eight
// distinct bank quads), then reads it back so that each store instruction
// covers eight whole 64-byte row pieces instead of 32 scattered 16-byte
// pieces.  Rows keep their own mapped output row and validity (shuffled from
// the row's lane).  A 2.5 KB tile per warp leaves room for a sixth 32 KB
// operand stage at BN = 256.
template <typename OutT>
struct EpiTile {
  static constexpr int ROW_BYTES = 64;
  static constexpr int COLS = ROW_BYTES / (int)sizeof(OutT);
  static constexpr int PITCH = ROW_BYTES + 16;
  static constexpr int BYTES = 32 * PITCH;  // per epilogue warp
  static constexpr int CH = ROW_BYTES / 16;
  static constexpr int ROWS_PER_PASS = 32 / CH;
};

template <int BN, Act ACT, typename OutT>
__device__ __forceinline__ void gemm_epilogue_staged(const GroupedGemmParams& p, const GemmSegment& seg, int nb,
                                                     int r_local, uint32_t t_row, int c0, int c1, uint8_t* tile) {
  using TL = EpiTile<OutT>;
  static_assert(TL::COLS == 16 || TL::COLS == 32, "a row piece holds one or two 16-column TMEM loads");
  const int lane = threadIdx.x & 31;
  const bool valid = r_local < seg.rows;
  const int arow = seg.a_row0 + r_local;
  long long orow = 0;
  float scale = 1.f;
  if (valid) {
    orow = p.row_map ? (long long)__ldg(p.row_map + arow) : (long long)(seg.out_row0 + r_local);
    if (p.row_scale) scale = __ldg(p.row_scale + arow);
  }
  OutT* out = (OutT*)p.out_ptrs[seg.out_slot];
  const float* bias = p.bias ? p.bias + (long long)seg.expert * p.N + nb * BN : nullptr;
  uint8_t* my_row = tile + lane * TL::PITCH;
  // store the staged row pieces of columns [col, col + COLS)
  auto flush = [&](int col) {
    __syncwarp();
#pragma unroll
    for (int pass = 0; pass < TL::CH; ++pass) {
      const int row = pass * TL::ROWS_PER_PASS + lane / TL::CH;  // tile row this lane stores
      const int k = lane % TL::CH;                                 // its 16-byte chunk
      const long long orow_r = __shfl_sync(0xffffffffu, orow, row);
      const int valid_r = __shfl_sync(0xffffffffu, (int)valid, row);
      const uint4 q = *(const uint4*)(tile + row * TL::PITCH + k * 16);
      if (valid_r) *(uint4*)((uint8_t*)(out + orow_r * p.ldo + nb * BN + col) + k * 16) = q;
    }
    __syncwarp();
  };
#pragma unroll 1
  for (int c = c0; c < c1; c += 32) {
    uint32_t r0[16], r1[16];
    tmem_ld16(t_row + c, r0);
    tmem_ld16(t_row + c + 16, r1);
    tmem_ld_wait();
    float b[16], v[16];
    load_bias16(bias ? bias + c : nullptr, b);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = apply_act(__uint_as_float(r0[j]) + b[j], ACT) * scale;
    store16((OutT*)my_row, v);
    if constexpr (TL::COLS == 16) flush(c);
    load_bias16(bias ? bias + c + 16 : nullptr, b);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = apply_act(__uint_as_float(r1[j]) + b[j], ACT) * scale;
    if constexpr (TL::COLS == 16) {
      store16((OutT*)my_row, v);
      flush(c + 16);
    } else {
      store16((OutT*)my_row + 16, v);
      flush(c);
    }
  }
}

// Column range [c0, c1) of epilogue warp `ew` (0..kEpiWarps-1) in a tile
// whose epilogue covers `cols` columns: warps ew and ew + 4 split the range
// at a 16-column boundary.
__device__ __forceinline__ void epi_columns(int ew, int cols, int& c0, int& c1) {
  const int chunks = cols / 16;
  const int first = (chunks + 1) / 2;
  if (ew < 4) { c0 = 0; c1 = first * 16; }
  else { c0 = first * 16; c1 = cols; }
}

template <int BN, bool TF32, Act ACT, typename OutT>
__global__ void __launch_bounds__(kGemmThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b,
                    GroupedGemmParams p) {
  using C = GemmCfg<BN, TF32>;
  constexpr int kKernelId = 100 + BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint64_t* bars = (uint64_t*)(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + C::STAGES;
  uint64_t* tfull_bar = bars + 2 * C::STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = (uint32_t*)(drain_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull_bar[a], 1); mbar_init(&tempty_bar[a], kEpiWarps); }
    mbar_init(drain_bar, 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, C::TMEM_COLS); tmem_relinquish(); }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // The prologue above touches only this CTA's shared memory and TMEM; the
  // tile table, segments and A rows are the previous launch's outputs.
  griddep_wait();
  griddep_launch_dependents();
  if (p.trace != nullptr && threadIdx.x == 0) atomicMin(&p.trace->t_start, (unsigned long long)globaltimer_ns());

  const int total_tiles = p.tile_prefix[p.num_segs];
  const int nblocks = p.N / BN;
  const int kblocks = (p.K + C::BK - 1) / C::BK;
  const uint64_t lim = p.timeout_ns;
  // split K: every CTA derives the same split count from the tile count;
  // work item t is tile t % total_tiles, split t / total_tiles, K blocks
  // [split * kbs, min(kblocks, (split + 1) * kbs)) (no split is empty)
  int S = 1;
  if (ACT != Act::kSwiGLU && p.ksplit_partial != nullptr && p.ksplit_ticket != nullptr && total_tiles > 0) {
    S = min(p.ksplit_max, (int)gridDim.x / total_tiles);
    S = min(S, kblocks / kSplitMinKBlocks);
    S = min(S, p.ksplit_entries / total_tiles);
    if (S < 1) S = 1;
  }
  const int kbs = (kblocks + S - 1) / S;
  if (S > 1) S = (kblocks + kbs - 1) / kbs;
  const int work = total_tiles * S;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      int stage = 0; uint32_t phase = 0;
      for (int t = blockIdx.x; t < work; t += gridDim.x) {
        const int tile = t % total_tiles, split = t / total_tiles;
        const int s = find_segment(p.tile_prefix, p.num_segs, tile);
        const GemmSegment seg = p.segs[s];
        const int local = tile - p.tile_prefix[s];
        const int mb = local / nblocks, nb = local % nblocks;
        const int arow = seg.a_row0 + mb * C::BM;
        const int brow = seg.expert * p.N + nb * BN;
        const int kb0 = split * kbs, kb1 = min(kblocks, kb0 + kbs);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.status, kKernelId, lim)) { ok = false; break; }
          uint8_t* sa = stage_base + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], C::STAGE_BYTES);
          tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * C::BK, arow);
          tma_load_2d(sa + C::A_BYTES, &tmap_b, &full_bar[stage], kb * C::BK, brow);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      int stage = 0; uint32_t phase = 0; int iter = 0;
      for (int t = blockIdx.x; t < work; t += gridDim.x, ++iter) {
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1u, p.status, kKernelId, lim)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int kb0 = (t / total_tiles) * kbs, kb1 = min(kblocks, kb0 + kbs);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, p.status, kKernelId, lim)) { ok = false; break; }
          tc_fence_after_sync();
          const uint32_t a_addr = smem_u32(stage_base + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < C::BK / C::UK; ++k) {
            const uint64_t ad = umma_desc_k_sw128(a_addr + k * 32);
            const uint64_t bd = umma_desc_k_sw128(b_addr + k * 32);
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            if (TF32) umma_tf32(d_tmem, ad, bd, C::IDESC, accum);
            else umma_f16(d_tmem, ad, bd, C::IDESC, accum);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
      }
      // Drain: every MMA issued above has completed before TMEM is freed.
      umma_commit(drain_bar);
      mbar_wait_bounded(drain_bar, 0, p.status, kKernelId, lim);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int c0, c1;
    epi_columns(warp - 2, ACT == Act::kSwiGLU ? BN / 2 : BN, c0, c1);
    int iter = 0;
    __shared__ int s_last;  // split K: this CTA holds the tile's last split
    for (int t = blockIdx.x; t < work; t += gridDim.x, ++iter) {
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      const int tile = t % total_tiles, split = t / total_tiles;
      const int s = find_segment(p.tile_prefix, p.num_segs, tile);
      const GemmSegment seg = p.segs[s];
      const int local = tile - p.tile_prefix[s];
      const int mb = local / nblocks, nb = local % nblocks;
      bool ok = mbar_wait_bounded(&tfull_bar[acc], acc_phase, p.status, kKernelId, lim);
      // split K: the epilogue warps meet at named barriers, so they stop together
      if (S > 1) ok = named_barrier_and(2, kEpiWarps * 32, ok);
      if (!ok) break;
      tc_fence_after_sync();
      const int r_local = mb * C::BM + row_in_tile;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (S == 1) {
        gemm_epilogue_row<BN, ACT, OutT>(p, seg, nb, r_local, t_row, c0, c1);
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        continue;
      }
      // split K: this split's partial tile, then one ticket per tile; the
      // last split adds every partial in split order and runs the epilogue
      const long long stride = (long long)total_tiles * C::BM * BN;
      float* part_row = p.ksplit_partial + ((long long)tile * C::BM + row_in_tile) * BN;
      gemm_partial_row<BN>(part_row + split * stride, t_row, c0, c1);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      __threadfence();  // this thread's partial stores before the tile's ticket
      named_barrier_sync(1, kEpiWarps * 32);
      if (warp == 2 && lane == 0) s_last = atomicAdd(&p.ksplit_ticket[tile], 1) == S - 1 ? 1 : 0;
      named_barrier_sync(1, kEpiWarps * 32);
      if (s_last) {
        __threadfence();  // every split's partial stores (ordered by their tickets) before the reads
        gemm_sum_row<BN, ACT, OutT>(p, seg, nb, r_local, part_row, stride, S, c0, c1);
      }
      named_barrier_sync(1, kEpiWarps * 32);  // s_last is read before the next tile's ticket
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
  if (p.trace != nullptr && threadIdx.x == 0) {  // after the CTA-wide barrier: every role is done
    atomicMax(&p.trace->t_end, (unsigned long long)globaltimer_ns());
    atomicAdd(&p.trace->ctas, 1);
  }
}

// ---------------------------------------------------------------------------
// Host-side dispatch over the compile-time tile width and activation.
// ---------------------------------------------------------------------------
template <int BN, bool TF32, Act ACT, typename OutT>
inline void launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const GroupedGemmParams& p,
                       int grid, cudaStream_t stream) {
  using C = GemmCfg<BN, TF32>;
  auto kern = grouped_gemm_kernel<BN, TF32, ACT, OutT>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_TOTAL);
    configured = true;
  }
  launch_with_pdl(kern, dim3(grid), dim3(kGemmThreads), C::SMEM_TOTAL, stream, p.pdl != 0, ta, tb, p);
}

template <bool TF32, Act ACT, typename OutT>
inline void dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GroupedGemmParams& p, int grid, cudaStream_t stream) {
  switch (bn) {
    case 16: if constexpr (ACT != Act::kSwiGLU) { launch_one<16, TF32, ACT, OutT>(ta, tb, p, grid, stream); return; } break;
    case 32: launch_one<32, TF32, ACT, OutT>(ta, tb, p, grid, stream); return;
    case 64: launch_one<64, TF32, ACT, OutT>(ta, tb, p, grid, stream); return;
    case 128: launch_one<128, TF32, ACT, OutT>(ta, tb, p, grid, stream); return;
    case 256: launch_one<256, TF32, ACT, OutT>(ta, tb, p, grid, stream); return;
    default: break;
  }
  throw std::runtime_error("grouped_gemm: unsupported BN " + std::to_string(bn));
}

template <bool TF32, typename OutT>
inline void dispatch_act(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                         const GroupedGemmParams& p, int grid, cudaStream_t stream) {
  switch ((Act)act) {
    case Act::kNone: dispatch_bn<TF32, Act::kNone, OutT>(bn, ta, tb, p, grid, stream); return;
    case Act::kRelu: dispatch_bn<TF32, Act::kRelu, OutT>(bn, ta, tb, p, grid, stream); return;
    case Act::kGelu: dispatch_bn<TF32, Act::kGelu, OutT>(bn, ta, tb, p, grid, stream); return;
    case Act::kSilu: dispatch_bn<TF32, Act::kSilu, OutT>(bn, ta, tb, p, grid, stream); return;
    case Act::kSwiGLU: dispatch_bn<TF32, Act::kSwiGLU, OutT>(bn, ta, tb, p, grid, stream); return;
  }
  throw std::runtime_error("grouped_gemm: unknown activation");
}


}  // namespace raiccl
