// Instantiation unit of the CTA-pair tcgen05 grouped GEMM: tf32 inputs -> f32 outputs.
#include "grouped_gemm_pair.cuh"

namespace raiccl {

void launch_gg_pair_tf32_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& ta8,
                             const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                             cudaStream_t stream) {
  dispatch_act_pair<true, float>(act, bn, ta, ta8, tb, p, grid, stream);
}

}  // namespace raiccl
