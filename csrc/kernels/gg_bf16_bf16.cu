// Instantiation unit of the tcgen05 grouped GEMM: bf16 inputs -> bf16 outputs.
#include "grouped_gemm.cuh"

namespace raiccl {

void launch_gg_bf16_bf16(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                         const GroupedGemmParams& p, int grid, cudaStream_t stream) {
  dispatch_act<false, __nv_bfloat16>(act, bn, ta, tb, p, grid, stream);
}

}  // namespace raiccl
