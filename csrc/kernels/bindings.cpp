// Python bindings of the sm_100a kernel library (module revealaiccl_b200._kernels).
//
// Tensor validation and TMA descriptor creation live here (host C++); the
// kernels themselves are launched through the C-style entry points declared
// in launchers.h so that the .cu translation units stay free of torch headers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "launchers.h"
#include "tma_host.h"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

// A:        [rows_total, K] fp32 (tf32 math) or bf16, contiguous rows
// B:        [E * N, K] same dtype as A (K-major expert weights)
// segs:     int32 [S, 8] GemmSegment records (device)
// prefix:   int32 [S + 1] tile table scratch (device, filled by the planner)
// out_ptrs: int64 [P] device pointers of the outputs (local or NVLink peer)
void grouped_gemm(torch::Tensor A, torch::Tensor B, torch::Tensor segs, torch::Tensor prefix,
                  int64_t N, int64_t bn, int64_t act, c10::optional<torch::Tensor> bias,
                  c10::optional<torch::Tensor> row_map, c10::optional<torch::Tensor> row_scale,
                  torch::Tensor out_ptrs, int64_t ldo, bool out_bf16, torch::Tensor status,
                  int64_t grid, int64_t timeout_ns, bool pair, int64_t swap_max) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && segs.is_cuda() && prefix.is_cuda() &&
                  out_ptrs.is_cuda() && status.is_cuda(),
              "grouped_gemm: CUDA tensors required");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "grouped_gemm: shape");
  TORCH_CHECK(A.scalar_type() == B.scalar_type(), "grouped_gemm: A and B dtypes must match");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "grouped_gemm: K must be contiguous");
  TORCH_CHECK(segs.scalar_type() == torch::kInt32 && segs.dim() == 2 && segs.size(1) == 8 &&
                  segs.is_contiguous(),
              "grouped_gemm: segs must be contiguous int32 [S, 8]");
  TORCH_CHECK(prefix.scalar_type() == torch::kInt32 && prefix.numel() >= segs.size(0) + 1,
              "grouped_gemm: prefix int32 [S+1]");
  TORCH_CHECK(segs.size(0) >= 1, "grouped_gemm: at least one segment");
  TORCH_CHECK(bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256, "grouped_gemm: BN");
  TORCH_CHECK(N % bn == 0, "grouped_gemm: N must be a multiple of BN");
  TORCH_CHECK(!pair || bn >= 64, "grouped_gemm: the CTA-pair kernel needs BN >= 64");
  TORCH_CHECK(B.size(0) % N == 0, "grouped_gemm: B rows must be E * N");
  TORCH_CHECK(out_ptrs.scalar_type() == torch::kInt64, "grouped_gemm: out_ptrs int64");
  TORCH_CHECK(status.numel() * status.element_size() >= (int64_t)sizeof(raiccl::DeviceStatus),
              "grouped_gemm: status buffer too small");
  if (bias) TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->is_contiguous() &&
                            bias->numel() == B.size(0) && (reinterpret_cast<uintptr_t>(bias->data_ptr()) & 15) == 0,
                        "grouped_gemm: bias fp32 [E*N], 16-byte aligned");
  if (row_map) TORCH_CHECK(row_map->scalar_type() == torch::kInt32 && row_map->numel() >= A.size(0),
                           "grouped_gemm: row_map int32 [rows_total]");
  if (row_scale) TORCH_CHECK(row_scale->scalar_type() == torch::kFloat32 &&
                                 row_scale->numel() >= A.size(0),
                             "grouped_gemm: row_scale fp32 [rows_total]");
  const bool tf32 = A.scalar_type() == torch::kFloat32;
  TORCH_CHECK(tf32 || A.scalar_type() == torch::kBFloat16, "grouped_gemm: fp32 or bf16 inputs");
  const int elem = tf32 ? 4 : 2;
  const int bk = 128 / elem;
  c10::cuda::CUDAGuard guard(A.device());
  const CUtensorMapDataType dt =
      tf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta = raiccl::make_tmap_2d_sw128(A.data_ptr(), dt, elem, A.size(0), A.size(1),
                                              A.stride(0), 128, bk);
  CUtensorMap tb = raiccl::make_tmap_2d_sw128(B.data_ptr(), dt, elem, B.size(0), B.size(1),
                                              B.stride(0), (uint32_t)(pair ? bn / 2 : bn), bk);
  CUtensorMap ta8 = raiccl::make_tmap_2d_sw128(A.data_ptr(), dt, elem, A.size(0), A.size(1),
                                               A.stride(0), 8, bk);
  const int S = (int)segs.size(0);
  const int nblocks = (int)(N / bn);
  // swapped tail tiles: CTA-pair kernel at BN = 256 without SwiGLU; their
  // table follows the full-tile table in `prefix`
  const bool swapping = swap_max > 0;
  if (swapping) {
    TORCH_CHECK(pair && bn == 256 && act != (int64_t)raiccl::Act::kSwiGLU && swap_max <= 256,
                "grouped_gemm: swap_max needs the CTA-pair kernel at BN 256 without SwiGLU, swap_max <= 256");
    TORCH_CHECK(prefix.numel() >= 2 * (segs.size(0) + 1), "grouped_gemm: prefix int32 [2 (S+1)] with swap_max");
  }
  int* tail = swapping ? prefix.data_ptr<int>() + S + 1 : nullptr;
  raiccl::launch_tile_plan((const raiccl::GemmSegment*)segs.data_ptr<int>(), S, nblocks,
                           prefix.data_ptr<int>(), cur_stream(), nullptr, pair ? 256 : 128,
                           tail, (int)swap_max);
  raiccl::GroupedGemmParams p{};  // value-initialised: fields this call does not set (trace, ...) are null
  p.segs = (const raiccl::GemmSegment*)segs.data_ptr<int>();
  p.tile_prefix = prefix.data_ptr<int>();
  p.num_segs = S;
  p.N = (int)N;
  p.K = (int)A.size(1);
  p.bias = bias ? bias->data_ptr<float>() : nullptr;
  p.row_map = row_map ? row_map->data_ptr<int>() : nullptr;
  p.row_scale = row_scale ? row_scale->data_ptr<float>() : nullptr;
  p.out_ptrs = (void* const*)out_ptrs.data_ptr<int64_t>();
  p.ldo = ldo;
  p.status = (raiccl::DeviceStatus*)status.data_ptr();
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.pair = pair ? 1 : 0;
  p.tail_prefix = tail;
  p.swap_max = (int)swap_max;
  raiccl::launch_grouped_gemm(tf32, out_bf16, (int)act, (int)bn, ta, tb, p, (int)grid,
                              cur_stream(), &ta8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

void register_moe(py::module_& m);

// Peer put + signal: copies src (a CUDA tensor, 16-byte aligned, bytes a
// multiple of 16) to the device address dst_ptr (own or peer mapping), then
// releases seq at flag_ptr.  counter: zeroed int32 CUDA tensor [1].
void peer_put_signal(torch::Tensor src, int64_t dst_ptr, int64_t flag_ptr, int64_t seq, torch::Tensor counter,
                     int64_t grid) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "peer_put_signal: contiguous CUDA source");
  const long long bytes = src.numel() * src.element_size();
  TORCH_CHECK(bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0 && (dst_ptr & 15) == 0,
              "peer_put_signal: 16-byte aligned buffers and a multiple of 16 bytes");
  TORCH_CHECK(flag_ptr != 0 && (flag_ptr & 7) == 0, "peer_put_signal: 8-byte aligned flag");
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == torch::kInt32, "peer_put_signal: int32 counter");
  TORCH_CHECK(grid >= 1 && grid <= 65535, "peer_put_signal: grid");
  c10::cuda::CUDAGuard guard(src.device());
  raiccl::launch_peer_put_signal(src.data_ptr(), reinterpret_cast<void*>(dst_ptr), bytes,
                                 reinterpret_cast<unsigned long long*>(flag_ptr), (unsigned long long)seq,
                                 counter.data_ptr<int>(), (int)grid, cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Bounded wait until the 64-bit word at flag_ptr (this GPU) is >= seq; the
// waited time (ns, or -1 after a timeout) goes to waited[0].
void peer_wait(int64_t flag_ptr, int64_t seq, int64_t timeout_ns, torch::Tensor status, torch::Tensor waited) {
  TORCH_CHECK(flag_ptr != 0 && (flag_ptr & 7) == 0, "peer_wait: 8-byte aligned flag");
  TORCH_CHECK(status.is_cuda() && status.numel() * status.element_size() >= (int64_t)sizeof(raiccl::DeviceStatus),
              "peer_wait: status buffer");
  TORCH_CHECK(waited.is_cuda() && waited.scalar_type() == torch::kInt64, "peer_wait: int64 waited");
  c10::cuda::CUDAGuard guard(status.device());
  raiccl::launch_peer_wait(reinterpret_cast<const unsigned long long*>(flag_ptr), (unsigned long long)seq,
                           (unsigned long long)timeout_ns, reinterpret_cast<raiccl::DeviceStatus*>(status.data_ptr()),
                           reinterpret_cast<unsigned long long*>(waited.data_ptr<int64_t>()), cur_stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "revealaiccl_b200 sm_100a kernels (tcgen05/TMEM/TMA, NVLink peer stores)";
  m.def("grouped_gemm", &grouped_gemm, "tcgen05 grouped GEMM with fused epilogue",
        py::arg("A"), py::arg("B"), py::arg("segs"), py::arg("prefix"), py::arg("N"),
        py::arg("bn"), py::arg("act"), py::arg("bias"), py::arg("row_map"), py::arg("row_scale"),
        py::arg("out_ptrs"), py::arg("ldo"), py::arg("out_bf16"), py::arg("status"),
        py::arg("grid"), py::arg("timeout_ns"), py::arg("pair") = false, py::arg("swap_max") = 0);
  register_moe(m);
  m.def("peer_put_signal", &peer_put_signal, py::arg("src"), py::arg("dst_ptr"), py::arg("flag_ptr"), py::arg("seq"),
        py::arg("counter"), py::arg("grid") = 64);
  m.def("peer_wait", &peer_wait, py::arg("flag_ptr"), py::arg("seq"), py::arg("timeout_ns"), py::arg("status"),
        py::arg("waited"));
}
