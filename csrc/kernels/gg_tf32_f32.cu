// Instantiation unit of the tcgen05 grouped GEMM: tf32 inputs -> f32 outputs.
#include "grouped_gemm.cuh"

namespace raiccl {

void launch_gg_tf32_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GroupedGemmParams& p, int grid, cudaStream_t stream) {
  dispatch_act<true, float>(act, bn, ta, tb, p, grid, stream);
}

}  // namespace raiccl
