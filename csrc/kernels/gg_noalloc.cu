// ===========================================================================
// raiccl_grouped_gemm_noalloc — grouped GEMM entry point that allocates nothing
//
// No counterpart in the reference: it has no C entry point of this kind.
//
// Who it is for.  The ordinary entry point (module `_kernels`, function
// `grouped_gemm`) takes a tile-table tensor and a status tensor that the caller
// allocates, normally through torch.  Some callers cannot do that: a C or C++
// program that links neither torch nor an allocator of its own, or code that
// runs where no new device allocation may happen (a fixed memory budget, an
// out-of-memory path).  This entry point takes raw device pointers and keeps
// its working memory in a file-scope `__device__` array instead, so it calls
// no cudaMalloc, no cudaFree and no allocating library routine.
//
// Scratch.  `g_gg_noalloc_scratch` (kNoAllocScratchBytes = 4608 bytes per
// device) holds the DeviceStatus record, the output-pointer table (one entry)
// and the per-segment tile table, so at most kNoAllocMaxSegs = 1024 segments
// per call; a call with more is rejected (RAICCL_NOALLOC_TOO_MANY_SEGMENTS)
// before anything is launched.
//
// What must start at zero.  Only the status record, and the call zeroes it
// itself: the planning kernel below clears it, stream-ordered, before the GEMM
// kernel (which gives up as soon as the status holds an error) starts.  The
// tile table and the pointer table are overwritten by every call.  Output rows
// named by a segment are written, not accumulated, so `out` needs no clearing.
//
// First call.  The first call on each device resolves the scratch address with
// cudaGetSymbolAddress (with the device current), and the first call of each
// kernel variant sets its shared-memory attribute; both are one-time setup.
// Make the first call on a device before beginning any stream capture.
//
// Overlapping calls race.  There is ONE scratch array per device.  Two calls
// on the same device whose work can overlap (different streams without an
// ordering between them, or several host threads) use the same tile table and
// status record and corrupt each other.  Order the calls on one stream, or
// otherwise make sure one finishes before the next starts.
// ===========================================================================
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <mutex>

#include "gg_noalloc.h"
#include "launchers.h"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace raiccl {
namespace {

constexpr int kNoAllocMaxSegs = 1024;
constexpr int kNoAllocScratchBytes = 4608;
constexpr int kOffStatus = 0;     // DeviceStatus (32 bytes)
constexpr int kOffOutPtrs = 64;   // void* [1]
constexpr int kOffPrefix = 256;   // int [kNoAllocMaxSegs + 1]
static_assert(kOffPrefix + 4 * (kNoAllocMaxSegs + 1) <= kNoAllocScratchBytes, "scratch layout");
static_assert(sizeof(DeviceStatus) <= kOffOutPtrs - kOffStatus, "scratch layout");

constexpr int kMaxDevices = 64;
constexpr int kPlanKernelId = 40;

static __device__ __align__(256) unsigned char g_gg_noalloc_scratch[kNoAllocScratchBytes];

// Clears the status record, stores the output pointer, checks every segment
// against the caller's extents and writes the cumulative tile table
// (prefix[s] = tiles of segments < s).  Any failed check records a status and
// turns the whole call into a no-op (prefix[num_segs] = 0): the GEMM kernel
// then runs no tile, so no out-of-range row, expert or output is touched.
__device__ __forceinline__ bool gg_noalloc_seg_ok(const GemmSegment& g, long long rows_a, int experts,
                                                  long long out_rows, bool mapped) {
  if (g.rows < 0 || g.a_row0 < 0 || (long long)g.a_row0 + g.rows > rows_a) return false;
  if (g.expert < 0 || g.expert >= experts) return false;
  if (!mapped && (g.out_row0 < 0 || (long long)g.out_row0 + g.rows > out_rows)) return false;
  return true;
}

__global__ void gg_noalloc_plan_kernel(const GemmSegment* segs, int num_segs, int nblocks, void* out,
                                       long long rows_a, int experts, long long out_rows, const int* row_map,
                                       unsigned char* scratch) {
  __shared__ int partial[1024];
  DeviceStatus* st = reinterpret_cast<DeviceStatus*>(scratch + kOffStatus);
  int* prefix = reinterpret_cast<int*>(scratch + kOffPrefix);
  if (threadIdx.x == 0) {
    st->code = 0; st->kernel_id = 0; st->block = 0; st->thread = 0; st->index = 0; st->bound = 0;
    reinterpret_cast<void**>(scratch + kOffOutPtrs)[0] = out;
  }
  __syncthreads();
  const int tid = threadIdx.x;
  const int per = (num_segs + blockDim.x - 1) / blockDim.x;
  const int s0 = tid * per;
  const bool mapped = row_map != nullptr;
  int local = 0;
  for (int s = s0; s < s0 + per && s < num_segs; ++s) {
    const GemmSegment g = segs[s];
    if (g.out_slot != 0) record_status(st, kBadConfig, kPlanKernelId, s, 0);
    if (!gg_noalloc_seg_ok(g, rows_a, experts, out_rows, mapped)) record_status(st, kBoundsViolation, kPlanKernelId, s, rows_a);
    const int rows = g.rows > 0 ? g.rows : 0;
    local += ((rows + 127) / 128) * nblocks;
  }
  if (mapped) {
    // every mapped output row of an in-range segment must exist
    for (int s = 0; s < num_segs; ++s) {
      const GemmSegment g = segs[s];
      if (!gg_noalloc_seg_ok(g, rows_a, experts, out_rows, true)) continue;
      for (int r = tid; r < g.rows; r += blockDim.x) {
        const int o = row_map[g.a_row0 + r];
        if (o < 0 || (long long)o >= out_rows) record_status(st, kBoundsViolation, kPlanKernelId, g.a_row0 + r, out_rows);
      }
    }
  }
  partial[tid] = local;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    const int v = tid >= off ? partial[tid - off] : 0;
    __syncthreads();
    partial[tid] += v;
    __syncthreads();
  }
  int run = tid > 0 ? partial[tid - 1] : 0;
  for (int s = s0; s < s0 + per && s < num_segs; ++s) {
    prefix[s] = run;
    const int rows = segs[s].rows > 0 ? segs[s].rows : 0;
    run += ((rows + 127) / 128) * nblocks;
  }
  if (tid == blockDim.x - 1) {
    // a rejected segment turns the whole call into a no-op
    prefix[num_segs] = st->code == 0 ? partial[tid] : 0;
  }
}

std::mutex g_scratch_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {};

// Scratch address on the current device (resolved once per device).
int scratch_for_current_device(unsigned char** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return -4;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gg_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace
}  // namespace raiccl

extern "C" {

// Declared, with the return codes, in csrc/include/gg_noalloc.h.

__attribute__((visibility("default"))) int raiccl_grouped_gemm_noalloc_max_segments(void) {
  return raiccl::kNoAllocMaxSegs;
}

__attribute__((visibility("default"))) const char* raiccl_grouped_gemm_noalloc_error_string(int code) {
  switch (code) {
    case 0: return "ok";
    case RAICCL_NOALLOC_TOO_MANY_SEGMENTS: return "num_segs exceeds the 1024-segment scratch capacity";
    case RAICCL_NOALLOC_BAD_ARGUMENT: return "invalid argument (shape, dtype, tile width, activation or alignment)";
    case RAICCL_NOALLOC_LAUNCH_FAILED: return "tensor-map encoding or kernel launch failed";
    case RAICCL_NOALLOC_BAD_DEVICE: return "current device index outside the supported range";
    default: return code > 0 ? cudaGetErrorString(static_cast<cudaError_t>(code)) : "unknown error";
  }
}

// The contract (shapes, alignment, segment checks) is written out beside the
// declaration in csrc/include/gg_noalloc.h.  The call only enqueues work on
// `stream`; read the device status afterwards with
// raiccl_grouped_gemm_noalloc_status.
__attribute__((visibility("default"))) int raiccl_grouped_gemm_noalloc(
    int in_fp32, const void* A, long long rows_a, long long K, long long lda, const void* B,
    long long rows_b, long long ldb, const void* segs, int num_segs, int N, int bn, int act,
    const float* bias, const int* row_map, const float* row_scale, void* out, long long out_rows, long long ldo,
    int out_bf16, int grid, unsigned long long timeout_ns, cudaStream_t stream) {
  using namespace raiccl;
  if (num_segs > kNoAllocMaxSegs) return RAICCL_NOALLOC_TOO_MANY_SEGMENTS;
  if (num_segs < 1 || A == nullptr || B == nullptr || segs == nullptr || out == nullptr) return RAICCL_NOALLOC_BAD_ARGUMENT;
  if (rows_a < 1 || K < 1 || rows_b < 1 || N < 1 || lda < K || ldb < K || ldo < 1) return RAICCL_NOALLOC_BAD_ARGUMENT;
  if (!(bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256) || N % bn != 0 || rows_b % N != 0)
    return RAICCL_NOALLOC_BAD_ARGUMENT;
  if (act < 0 || act > 4 || (act == 4 && bn < 32)) return RAICCL_NOALLOC_BAD_ARGUMENT;
  if (in_fp32 && out_bf16) return RAICCL_NOALLOC_BAD_ARGUMENT;
  // 16-byte vector accesses: segment records, bias loads, output row stores,
  // TMA operand rows; 4-byte loads of row_map / row_scale
  auto misaligned = [](const void* q, uintptr_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) != 0; };
  if (misaligned(segs, 16) || misaligned(A, 16) || misaligned(B, 16) || misaligned(out, 16)) return RAICCL_NOALLOC_BAD_ARGUMENT;
  if ((bias != nullptr && misaligned(bias, 16)) || (row_map != nullptr && misaligned(row_map, 4)) ||
      (row_scale != nullptr && misaligned(row_scale, 4)))
    return RAICCL_NOALLOC_BAD_ARGUMENT;
  {
    const long long in_elem = in_fp32 ? 4 : 2, out_elem = out_bf16 ? 2 : 4;
    const long long out_width = act == 4 ? N / 2 : N;
    if ((lda * in_elem) % 16 != 0 || (ldb * in_elem) % 16 != 0) return RAICCL_NOALLOC_BAD_ARGUMENT;
    if (out_rows < 1 || ldo < out_width || (ldo * out_elem) % 16 != 0) return RAICCL_NOALLOC_BAD_ARGUMENT;
    if (rows_a > 0x7fffffffLL || rows_b / N > 0x7fffffffLL || out_rows > 0x7fffffffLL) return RAICCL_NOALLOC_BAD_ARGUMENT;
  }
  unsigned char* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != 0) return rc;
  int sms = grid;
  if (sms <= 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  try {
    const int elem = in_fp32 ? 4 : 2;
    const CUtensorMapDataType dt = in_fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUtensorMap ta = make_tmap_2d_sw128(A, dt, elem, rows_a, K, lda, 128, 128 / elem);
    const CUtensorMap tb = make_tmap_2d_sw128(B, dt, elem, rows_b, K, ldb, (uint32_t)bn, 128 / elem);
    const GemmSegment* sg = static_cast<const GemmSegment*>(segs);
    gg_noalloc_plan_kernel<<<1, 1024, 0, stream>>>(sg, num_segs, N / bn, out, rows_a, (int)(rows_b / N), out_rows,
                                                    row_map, scratch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    GroupedGemmParams p{};  // value-initialised: fields this call does not set (trace, ...) are null
    p.segs = sg;
    p.tile_prefix = reinterpret_cast<const int*>(scratch + kOffPrefix);
    p.num_segs = num_segs;
    p.N = N;
    p.K = (int)K;
    p.bias = bias;
    p.row_map = row_map;
    p.row_scale = row_scale;
    p.out_ptrs = reinterpret_cast<void* const*>(scratch + kOffOutPtrs);
    p.ldo = ldo;
    p.status = reinterpret_cast<DeviceStatus*>(scratch + kOffStatus);
    p.timeout_ns = timeout_ns ? timeout_ns : 2000000000ULL;
    launch_grouped_gemm(in_fp32 != 0, out_bf16 != 0, act, bn, ta, tb, p, sms, stream);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
  } catch (const std::exception&) {
    return RAICCL_NOALLOC_LAUNCH_FAILED;
  }
  return 0;
}

// Waits for `stream`, copies the device status record of the current device
// (32 bytes: code, kernel id, block, thread, index, bound) to `host_status`
// when it is not NULL, and returns the status code (0 = no error recorded) or,
// if the wait or the copy failed, minus the cudaError_t value.
__attribute__((visibility("default"))) int raiccl_grouped_gemm_noalloc_status(void* host_status,
                                                                                cudaStream_t stream) {
  using namespace raiccl;
  unsigned char* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != 0) return rc > 0 ? -rc : rc;
  DeviceStatus s{};
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess) e = cudaMemcpy(&s, scratch + kOffStatus, sizeof(s), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return -(int)e;
  if (host_status != nullptr) std::memcpy(host_status, &s, sizeof(s));
  return s.code;
}

}  // extern "C"
