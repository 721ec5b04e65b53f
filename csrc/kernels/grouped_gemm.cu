// Host launchers for the tcgen05 grouped GEMM (see grouped_gemm.cuh) and the
// single-CTA tile planner that turns per-segment row counts into the
// cumulative tile table the persistent kernel walks.
#include <stdexcept>
#include <string>

#include "grouped_gemm.cuh"
#include "sm100_ptx.cuh"
#include "launchers.h"

namespace raiccl {

// Tiles of one segment: ceil(rows / bm) row tiles times nblocks; with swap > 0
// a last row tile of at most swap rows is counted apart as the tail.
__device__ __forceinline__ void segment_tiles(int rows, int bm, int nblocks, int swap, int& full, int& tail) {
  rows = rows > 0 ? rows : 0;
  const int mt = (rows + bm - 1) / bm;
  const bool sw = swap > 0 && mt > 0 && rows - (mt - 1) * bm <= swap;
  full = (mt - (sw ? 1 : 0)) * nblocks;
  tail = sw ? nblocks : 0;
}

// One CTA: prefix[s] = sum_{j<s} full tiles of j, tail[s] = sum_{j<s} tail tiles of j.
__global__ void gemm_tile_plan_kernel(const GemmSegment* segs, int num_segs, int nblocks,
                                      int* prefix, TraceSlot* trace, int bm, int* tail, int swap) {
  TraceScope trace_scope(trace);
  __shared__ int partial[2][1024];
  const int tid = threadIdx.x;
  if (tail == nullptr) swap = 0;
  int local[2] = {0, 0};
  // each thread owns a contiguous run of segments
  const int per = (num_segs + blockDim.x - 1) / blockDim.x;
  const int s0 = tid * per;
  for (int s = s0; s < s0 + per && s < num_segs; ++s) {
    int f, t;
    segment_tiles(segs[s].rows, bm, nblocks, swap, f, t);
    local[0] += f;
    local[1] += t;
  }
  partial[0][tid] = local[0];
  partial[1][tid] = local[1];
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    const int v0 = tid >= off ? partial[0][tid - off] : 0;
    const int v1 = tid >= off ? partial[1][tid - off] : 0;
    __syncthreads();
    partial[0][tid] += v0;
    partial[1][tid] += v1;
    __syncthreads();
  }
  int run0 = tid > 0 ? partial[0][tid - 1] : 0;
  int run1 = tid > 0 ? partial[1][tid - 1] : 0;
  for (int s = s0; s < s0 + per && s < num_segs; ++s) {
    prefix[s] = run0;
    if (tail != nullptr) tail[s] = run1;
    int f, t;
    segment_tiles(segs[s].rows, bm, nblocks, swap, f, t);
    run0 += f;
    run1 += t;
  }
  if (tid == blockDim.x - 1) {
    prefix[num_segs] = partial[0][tid];
    if (tail != nullptr) tail[num_segs] = partial[1][tid];
  }
}

void launch_tile_plan(const GemmSegment* segs, int num_segs, int nblocks, int* prefix,
                      cudaStream_t stream, TraceSlot* trace, int bm, int* tail, int swap) {
  gemm_tile_plan_kernel<<<1, 1024, 0, stream>>>(segs, num_segs, nblocks, prefix, trace, bm, tail, swap);
}

// Instantiated combinations: tf32 inputs -> fp32 outputs; bf16 inputs -> bf16
// or fp32 outputs.  Every activation is available for every tile width except
// SwiGLU at BN=16 (a SwiGLU tile holds gate and up halves of >=16 columns).
void launch_grouped_gemm(bool in_tf32, bool out_bf16, int act, int bn, const CUtensorMap& ta,
                         const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                         cudaStream_t stream, const CUtensorMap* ta8) {
  if (p.pair) {
    if (p.tail_prefix != nullptr && ta8 == nullptr)
      throw std::runtime_error("grouped_gemm: swapped tail tiles need the 8-row A tensor map");
    const CUtensorMap& a8 = ta8 != nullptr ? *ta8 : ta;  // unused without swapped tiles
    if (in_tf32) {
      if (out_bf16) throw std::runtime_error("grouped_gemm: tf32 inputs produce fp32 outputs");
      launch_gg_pair_tf32_f32(act, bn, ta, a8, tb, p, grid, stream);
    } else if (out_bf16) {
      launch_gg_pair_bf16_bf16(act, bn, ta, a8, tb, p, grid, stream);
    } else {
      launch_gg_pair_bf16_f32(act, bn, ta, a8, tb, p, grid, stream);
    }
    return;
  }
  if (in_tf32) {
    if (out_bf16) throw std::runtime_error("grouped_gemm: tf32 inputs produce fp32 outputs");
    launch_gg_tf32_f32(act, bn, ta, tb, p, grid, stream);
  } else if (out_bf16) {
    launch_gg_bf16_bf16(act, bn, ta, tb, p, grid, stream);
  } else {
    launch_gg_bf16_f32(act, bn, ta, tb, p, grid, stream);
  }
}

}  // namespace raiccl
