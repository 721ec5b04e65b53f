// Instantiation unit of the CTA-pair tcgen05 grouped GEMM: bf16 inputs -> bf16 outputs.
#include "grouped_gemm_pair.cuh"

namespace raiccl {

void launch_gg_pair_bf16_bf16(int act, int bn, const CUtensorMap& ta, const CUtensorMap& ta8,
                              const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                              cudaStream_t stream) {
  dispatch_act_pair<false, __nv_bfloat16>(act, bn, ta, ta8, tb, p, grid, stream);
}

}  // namespace raiccl
