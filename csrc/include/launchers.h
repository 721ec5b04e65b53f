// C-style launch entry points of the sm_100a kernels.  The .cu files that
// define them include no torch headers (fast, parallel nvcc builds); the torch
// bindings in csrc/kernels/bindings.cpp validate tensors and call these.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "types.h"

namespace raiccl {

// prefix[s] = sum over segments j < s of ceil(rows_j / bm) * nblocks (bm = 128 for
// the one-CTA kernel, 256 for the CTA-pair kernel).  With tail != nullptr and
// swap > 0, a segment's last row tile of at most swap rows is counted in
// tail[] instead of prefix[] (GroupedGemmParams::tail_prefix).
void launch_tile_plan(const GemmSegment* segs, int num_segs, int nblocks, int* prefix,
                      cudaStream_t stream, TraceSlot* trace = nullptr, int bm = 128,
                      int* tail = nullptr, int swap = 0);

// in_tf32: A/B hold fp32 (tf32 math) else bf16; out_bf16 selects the output dtype.
void launch_gg_tf32_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GroupedGemmParams& p, int grid, cudaStream_t stream);
void launch_gg_bf16_bf16(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                         const GroupedGemmParams& p, int grid, cudaStream_t stream);
void launch_gg_bf16_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GroupedGemmParams& p, int grid, cudaStream_t stream);
void launch_gg_pair_tf32_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& ta8,
                             const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                             cudaStream_t stream);
void launch_gg_pair_bf16_bf16(int act, int bn, const CUtensorMap& ta, const CUtensorMap& ta8,
                              const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                              cudaStream_t stream);
void launch_gg_pair_bf16_f32(int act, int bn, const CUtensorMap& ta, const CUtensorMap& ta8,
                             const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                             cudaStream_t stream);
// p.pair selects the CTA-pair kernel (BN in {64, 128, 256}; A tensor map box of
// 128 rows, B box of bn / 2 rows; tile_prefix counted in 256-row tiles).  With
// swapped tail tiles (p.tail_prefix) the pair kernel also needs ta8: the A
// tensor with a box of 8 rows, so a tail tile stages only the rows it uses.
void launch_grouped_gemm(bool in_tf32, bool out_bf16, int act, int bn, const CUtensorMap& ta,
                         const CUtensorMap& tb, const GroupedGemmParams& p, int grid,
                         cudaStream_t stream, const CUtensorMap* ta8 = nullptr);

// Peer primitives (csrc/kernels/peer_ops.cu).  src / dst: 16-byte aligned,
// bytes a multiple of 16; dst and flag may be another GPU's mapped memory;
// done_counter: a zeroed device int of this GPU, one per concurrent put.
void launch_peer_put_signal(const void* src, void* dst, long long bytes, unsigned long long* flag,
                            unsigned long long seq, int* done_counter, int grid, cudaStream_t s);
// Waits (bounded) until *flag >= seq; waited_ns (optional) receives the wait
// time, or ~0 after a timeout (the status then holds kTimeoutPeerSignal).
void launch_peer_wait(const unsigned long long* flag, unsigned long long seq, unsigned long long timeout_ns,
                      DeviceStatus* status, unsigned long long* waited_ns, cudaStream_t s);

}  // namespace raiccl
