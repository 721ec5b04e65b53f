// revealaiccl_b200._host: host C++ runtime (compiled scheduler core, native
// completion bridge, NVLink peer channel set-up).
#include <pybind11/pybind11.h>

namespace py = pybind11;

void register_scheduler(py::module_& m);
void register_event_bridge(py::module_& m);
void register_peer_channel(py::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "revealaiccl_b200 host runtime: scheduler core, event bridge, peer channel";
  register_scheduler(m);
  register_event_bridge(m);
  register_peer_channel(m);
}
