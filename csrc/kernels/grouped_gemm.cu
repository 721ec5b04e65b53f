// Host launchers for the tcgen05 grouped GEMM (see grouped_gemm.cuh) and the
// single-CTA tile planner that turns per-segment row counts into the
// cumulative tile table the persistent kernel walks.
#include <stdexcept>
#include <string>

#include "grouped_gemm.cuh"
#include "sm100_ptx.cuh"
#include "launchers.h"

namespace raiccl {

// One CTA: prefix[s] = sum_{j<s} ceil(rows_j / 128) * nblocks.
__global__ void gemm_tile_plan_kernel(const GemmSegment* segs, int num_segs, int nblocks,
                                      int* prefix, TraceSlot* trace, int bm) {
  TraceScope trace_scope(trace);
  __shared__ int partial[1024];
  const int tid = threadIdx.x;
  int local = 0;
  // each thread owns a contiguous run of segments
  const int per = (num_segs + blockDim.x - 1) / blockDim.x;
  const int s0 = tid * per;
  for (int s = s0; s < s0 + per && s < num_segs; ++s) {
    const int rows = segs[s].rows > 0 ? segs[s].rows : 0;
    local += ((rows + bm - 1) / bm) * nblocks;
  }
  partial[tid] = local;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    int v = tid >= off ? partial[tid - off] : 0;
    __syncthreads();
    partial[tid] += v;
    __syncthreads();
  }
  int run = tid > 0 ? partial[tid - 1] : 0;
  for (int s = s0; s < s0 + per && s < num_segs; ++s) {
    prefix[s] = run;
    const int rows = segs[s].rows > 0 ? segs[s].rows : 0;
    run += ((rows + bm - 1) / bm) * nblocks;
  }
  if (tid == blockDim.x - 1) prefix[num_segs] = partial[tid];
}

void launch_tile_plan(const GemmSegment* segs, int num_segs, int nblocks, int* prefix,
                      cudaStream_t stream, TraceSlot* trace, int bm) {
  gemm_tile_plan_kernel<<<1, 1024, 0, stream>>>(segs, num_segs, nblocks, prefix, trace, bm);
}

// Instantiated combinations: tf32 inputs -> fp32 outputs; bf16 inputs -> bf16
// or fp32 outputs.  Every activation is available for every tile width except
// SwiGLU at BN=16 (a SwiGLU tile holds gate and up halves of >=16 columns).
void launch_grouped_gemm(bool in_tf32, bool out_bf16, int act, int bn, const CUtensorMap& ta,
                         const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                         cudaStream_t stream) {
  if (p.pair) {
    if (in_tf32) {
      if (out_bf16) throw std::runtime_error("grouped_gemm: tf32 inputs produce fp32 outputs");
      launch_gg_pair_tf32_f32(act, bn, ta, tb, p, grid, stream);
    } else if (out_bf16) {
      launch_gg_pair_bf16_bf16(act, bn, ta, tb, p, grid, stream);
    } else {
      launch_gg_pair_bf16_f32(act, bn, ta, tb, p, grid, stream);
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
