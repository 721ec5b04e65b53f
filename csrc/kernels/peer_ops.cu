// Standalone NVLink peer primitives: one-sided put with a completion signal,
// and a bounded wait for a signal.
//
// These are the put_and_signal / wait operations of the reference's MSCCL++
// shim (extensions/r6_mscclpp/mscclpp_runtime.cu: put + signal on a memory
// channel, wait on its semaphore), written as plain CUDA over the peer
// mappings of the symmetric region (revealaiccl_b200/parallel/peer.py):
//
//   peer_put_signal: CTAs copy `bytes` from a local buffer into a peer's
//     buffer with 16-byte stores (P2P over NVLink/NVSwitch, or local for the
//     own rank), then the last CTA to finish (device-scope acq_rel counter)
//     stores `seq` to the peer's 64-bit flag with st.release.sys.  The CTAs'
//     stores happen before their acq_rel increments; the last CTA's acquiring
//     increment sees them all, and its system-scope release is cumulative, so
//     a reader that acquires the flag sees every byte.
//   peer_wait: one thread polls a local flag (ld.acquire.sys) until it holds
//     at least `seq`, for at most timeout_ns; on timeout it records a status
//     and returns, leaving the context usable.
//
// Every access of another GPU's memory is a plain generic load or store: no
// TMA and no multicast.
#include <cuda_runtime.h>

#include <cstdint>

#include "launchers.h"
#include "sm100_ptx.cuh"

namespace raiccl {
namespace {

constexpr int kPeerOpsKernelId = 90;

__global__ void __launch_bounds__(256) peer_put_signal_kernel(const uint4* __restrict__ src, uint4* dst, long long n16,
                                                              unsigned long long* flag, unsigned long long seq,
                                                              int* done_counter) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  // four 16-byte loads in flight per thread before their stores
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = __ldg(src + i), b = __ldg(src + i + stride), c = __ldg(src + i + 2 * stride),
                d = __ldg(src + i + 3 * stride);
    dst[i] = a;
    dst[i + stride] = b;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; i < n16; i += stride) dst[i] = __ldg(src + i);
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atom_add_acq_rel_gpu(done_counter, 1);
    if (prev == (int)gridDim.x - 1) {
      st_release_sys_u64(reinterpret_cast<uint64_t*>(flag), seq);
      *done_counter = 0;  // ready for the next put (stream order)
    }
  }
}

__global__ void peer_wait_kernel(const unsigned long long* flag, unsigned long long seq, unsigned long long timeout_ns,
                                 DeviceStatus* status, unsigned long long* waited_ns) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  const bool ok = wait_flag_geq_sys(reinterpret_cast<const uint64_t*>(flag), seq, status, kTimeoutPeerSignal,
                                    kPeerOpsKernelId, 0, timeout_ns);
  if (waited_ns != nullptr) *waited_ns = ok ? globaltimer_ns() - t0 : ~0ULL;
}

}  // namespace

void launch_peer_put_signal(const void* src, void* dst, long long bytes, unsigned long long* flag,
                            unsigned long long seq, int* done_counter, int grid, cudaStream_t s) {
  const long long n16 = bytes / 16;
  peer_put_signal_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), static_cast<uint4*>(dst), n16, flag,
                                               seq, done_counter);
}

void launch_peer_wait(const unsigned long long* flag, unsigned long long seq, unsigned long long timeout_ns,
                      DeviceStatus* status, unsigned long long* waited_ns, cudaStream_t s) {
  peer_wait_kernel<<<1, 32, 0, s>>>(flag, seq, timeout_ns, status, waited_ns);
}

}  // namespace raiccl
