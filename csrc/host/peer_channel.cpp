// Host side of the NVLink peer channel: symmetric device allocations whose
// CUDA-IPC handles are exported to every peer rank and opened there, plus
// host-mapped pinned words used as device->host completion mirrors.
//
// The handle exchange itself runs over the torch process group (Python,
// revealaiccl_b200/parallel/peer.py); this file owns every CUDA runtime call.
// It replaces the MSCCL++ TcpBootstrap / registerMemory / MemoryChannel setup
// of extensions/r6_mscclpp/mscclpp_runtime.cu:20-90, which was hard-wired to
// two ranks, with an N-rank mapping of every peer's buffer.
#include <cuda_runtime_api.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <tuple>

namespace py = pybind11;

namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// cudaMalloc'd, zeroed, 256-byte aligned buffer plus its IPC handle bytes.
std::tuple<uintptr_t, py::bytes> alloc_symmetric(size_t nbytes, int device) {
  check(cudaSetDevice(device), "cudaSetDevice");
  void* p = nullptr;
  check(cudaMalloc(&p, nbytes), "cudaMalloc(symmetric)");
  check(cudaMemset(p, 0, nbytes), "cudaMemset(symmetric)");
  check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  return {reinterpret_cast<uintptr_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

void free_symmetric(uintptr_t ptr, int device) {
  check(cudaSetDevice(device), "cudaSetDevice");
  check(cudaFree(reinterpret_cast<void*>(ptr)), "cudaFree(symmetric)");
}

uintptr_t open_peer(py::bytes handle, int device) {
  std::string raw = handle;
  if (raw.size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, raw.data(), sizeof(h));
  check(cudaSetDevice(device), "cudaSetDevice");
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<uintptr_t>(p);
}

void close_peer(uintptr_t ptr, int device) {
  check(cudaSetDevice(device), "cudaSetDevice");
  check(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

bool can_access_peer(int device, int peer) {
  int ok = 0;
  check(cudaDeviceCanAccessPeer(&ok, device, peer), "cudaDeviceCanAccessPeer");
  return ok != 0;
}

// Pinned host memory mapped into the device address space; returns
// (host pointer, device pointer).  Zeroed.
std::tuple<uintptr_t, uintptr_t> alloc_mapped(size_t nbytes) {
  void* h = nullptr;
  check(cudaHostAlloc(&h, nbytes, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc");
  std::memset(h, 0, nbytes);
  void* d = nullptr;
  check(cudaHostGetDevicePointer(&d, h, 0), "cudaHostGetDevicePointer");
  return {reinterpret_cast<uintptr_t>(h), reinterpret_cast<uintptr_t>(d)};
}

void free_mapped(uintptr_t host_ptr) {
  check(cudaFreeHost(reinterpret_cast<void*>(host_ptr)), "cudaFreeHost");
}

uint64_t read_u64(uintptr_t host_ptr) {
  return reinterpret_cast<const volatile uint64_t*>(host_ptr)[0];
}

void write_u64(uintptr_t host_ptr, uint64_t value) {
  __atomic_store_n(reinterpret_cast<uint64_t*>(host_ptr), value, __ATOMIC_RELEASE);
}

}  // namespace

void register_peer_channel(py::module_& m) {
  m.def("alloc_symmetric", &alloc_symmetric, py::arg("nbytes"), py::arg("device"));
  m.def("free_symmetric", &free_symmetric, py::arg("ptr"), py::arg("device"));
  m.def("open_peer", &open_peer, py::arg("handle"), py::arg("device"));
  m.def("close_peer", &close_peer, py::arg("ptr"), py::arg("device"));
  m.def("can_access_peer", &can_access_peer, py::arg("device"), py::arg("peer"));
  m.def("alloc_mapped", &alloc_mapped, py::arg("nbytes"));
  m.def("free_mapped", &free_mapped, py::arg("host_ptr"));
  m.def("read_u64", &read_u64, py::arg("host_ptr"));
  m.def("write_u64", &write_u64, py::arg("host_ptr"), py::arg("value"));
}
