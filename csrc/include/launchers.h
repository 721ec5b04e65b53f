// C-style launch entry points of the sm_100a kernels.  The .cu files that
// define them include no torch headers (fast, parallel nvcc builds); the torch
// bindings in csrc/kernels/bindings.cpp validate tensors and call these.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "types.h"

namespace raiccl {

void launch_tile_plan(const GemmSegment* segs, int num_segs, int nblocks, int* prefix,
                      cudaStream_t stream, TraceSlot* trace = nullptr);

// in_tf32: A/B hold fp32 (tf32 math) else bf16; out_bf16 selects the output dtype.
void launch_gg_tf32_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GroupedGemmParams& p, int grid, cudaStream_t stream);
void launch_gg_bf16_bf16(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                         const GroupedGemmParams& p, int grid, cudaStream_t stream);
void launch_gg_bf16_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GroupedGemmParams& p, int grid, cudaStream_t stream);
void launch_grouped_gemm(bool in_tf32, bool out_bf16, int act, int bn, const CUtensorMap& ta,
                         const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                         cudaStream_t stream);

}  // namespace raiccl
