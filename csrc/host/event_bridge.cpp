// Native completion bridge: a pinned host thread that turns GPU-side
// completion into host-visible per-slot READY states.
//
// Capabilities of extensions/r2_event_bridge/{event_bridge,integrated_event_bridge}.cpp
// (slot array, arm / ready / ready_ns / wait_ready / wait_all / snapshot /
// reset_all / stop, GIL-free waits that throw on timeout or CUDA error, and a
// conservative completion -> host-visible upper bound) with a second source
// added for the B200 path:
//   * event slots poll cudaEventQuery on an armed cudaEvent_t;
//   * flag slots poll a 64-bit word in host memory (pinned + device-mapped,
//     written by a kernel with st.release.sys) until it reaches the armed
//     sequence number — no CUDA API call on the polling path at all.
// Slot states: 0 idle, 1 armed, 2 ready, 3 error.
#include <cuda_runtime_api.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#ifdef __linux__
#include <pthread.h>
#include <sched.h>
#endif

namespace py = pybind11;

namespace {

inline uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

enum SlotState : int { kIdle = 0, kArmed = 1, kReady = 2, kError = 3 };
enum SlotSource : int { kEvent = 0, kFlag = 1 };

struct alignas(64) Slot {
  std::atomic<int> state{kIdle};
  std::atomic<int> source{kEvent};
  std::atomic<uintptr_t> handle{0};      // cudaEvent_t or const uint64_t* flag
  std::atomic<uint64_t> expected{0};     // flag sequence number to wait for
  std::atomic<uint64_t> armed_ns{0};
  std::atomic<uint64_t> last_miss_start_ns{0};
  std::atomic<uint64_t> ready_ns{0};
  std::atomic<uint64_t> upper_bound_ns{0};
  std::atomic<uint64_t> hit_query_ns{0};
  std::atomic<uint64_t> max_query_ns{0};
  std::atomic<uint64_t> polls{0};
  std::atomic<int> cuda_error{0};
  std::atomic<int> upper_bound_valid{0};
};

class EventBridge {
 public:
  EventBridge(size_t capacity, int cpu_core, int cuda_device)
      : capacity_(capacity), cpu_core_(cpu_core), cuda_device_(cuda_device) {
    if (capacity == 0) throw std::invalid_argument("capacity must be positive");
    slots_.reset(new Slot[capacity]);
    running_.store(true, std::memory_order_release);
    worker_ = std::thread(&EventBridge::poll_loop, this);
  }
  ~EventBridge() { stop(); }
  EventBridge(const EventBridge&) = delete;
  EventBridge& operator=(const EventBridge&) = delete;

  void arm(size_t i, uintptr_t event_handle) {
    if (event_handle == 0) throw std::invalid_argument("event handle must be nonzero");
    need_device_.store(true, std::memory_order_release);
    arm_slot(i, kEvent, event_handle, 0);
  }

  void arm_flag(size_t i, uintptr_t host_flag_ptr, uint64_t expected) {
    if (host_flag_ptr == 0 || (host_flag_ptr & 7u) != 0)
      throw std::invalid_argument("flag pointer must be nonzero and 8-byte aligned");
    arm_slot(i, kFlag, host_flag_ptr, expected);
  }

  bool ready(size_t i) const { return at(i).state.load(std::memory_order_acquire) == kReady; }
  uint64_t ready_ns(size_t i) const { return at(i).ready_ns.load(std::memory_order_acquire); }
  int state(size_t i) const { return at(i).state.load(std::memory_order_acquire); }

  uint64_t wait_ready(size_t i, uint64_t timeout_ns) {
    Slot& s = at(i);
    const uint64_t start = now_ns();
    py::gil_scoped_release nogil;
    while (true) {
      const int st = s.state.load(std::memory_order_acquire);
      if (st == kReady) return s.ready_ns.load(std::memory_order_acquire);
      if (st == kError) throw std::runtime_error("event bridge slot failed: CUDA error " +
                                                 std::to_string(s.cuda_error.load()));
      if (st == kIdle) throw std::runtime_error("event bridge slot is not armed");
      if (now_ns() - start > timeout_ns) throw std::runtime_error("event bridge timeout");
    }
  }

  void wait_all(uint64_t timeout_ns) {
    const uint64_t start = now_ns();
    py::gil_scoped_release nogil;
    while (true) {
      bool done = true;
      for (size_t i = 0; i < capacity_; ++i) {
        const int st = slots_[i].state.load(std::memory_order_acquire);
        if (st == kError) throw std::runtime_error("event bridge slot failed");
        if (st == kArmed) done = false;
      }
      if (done) return;
      if (now_ns() - start > timeout_ns) throw std::runtime_error("event bridge timeout");
    }
  }

  std::vector<py::dict> snapshot() const {
    std::vector<py::dict> out;
    for (size_t i = 0; i < capacity_; ++i) {
      const Slot& s = slots_[i];
      py::dict d;
      d["slot"] = i;
      d["state"] = s.state.load();
      d["source"] = s.source.load() == kFlag ? "flag" : "event";
      d["armed_ns"] = s.armed_ns.load();
      d["ready_ns"] = s.ready_ns.load();
      d["last_not_ready_query_start_ns"] = s.last_miss_start_ns.load();
      d["visibility_upper_bound_ns"] = s.upper_bound_ns.load();
      d["upper_bound_valid"] = (bool)s.upper_bound_valid.load();
      d["success_query_duration_ns"] = s.hit_query_ns.load();
      d["max_query_duration_ns"] = s.max_query_ns.load();
      d["poll_count"] = s.polls.load();
      d["cuda_error"] = s.cuda_error.load();
      out.push_back(d);
    }
    return out;
  }

  void reset_all() {
    for (size_t i = 0; i < capacity_; ++i) {
      if (slots_[i].state.load(std::memory_order_acquire) == kArmed)
        throw std::runtime_error("cannot reset while a slot is armed");
    }
    for (size_t i = 0; i < capacity_; ++i) slots_[i].state.store(kIdle, std::memory_order_release);
  }

  void stop() {
    if (running_.exchange(false)) {
      if (worker_.joinable()) worker_.join();
    }
  }

  bool pinned() const { return pinned_.load(); }
  int cpu_core() const { return cpu_core_; }
  int cuda_device() const { return cuda_device_; }
  size_t capacity() const { return capacity_; }

 private:
  Slot& at(size_t i) {
    if (i >= capacity_) throw std::out_of_range("slot index out of range");
    return slots_[i];
  }
  const Slot& at(size_t i) const {
    if (i >= capacity_) throw std::out_of_range("slot index out of range");
    return slots_[i];
  }

  void arm_slot(size_t i, int source, uintptr_t handle, uint64_t expected) {
    Slot& s = at(i);
    if (s.state.load(std::memory_order_acquire) == kArmed) throw std::runtime_error("slot is already armed");
    s.source.store(source, std::memory_order_relaxed);
    s.handle.store(handle, std::memory_order_relaxed);
    s.expected.store(expected, std::memory_order_relaxed);
    s.armed_ns.store(now_ns(), std::memory_order_relaxed);
    s.last_miss_start_ns.store(0, std::memory_order_relaxed);
    s.ready_ns.store(0, std::memory_order_relaxed);
    s.upper_bound_ns.store(0, std::memory_order_relaxed);
    s.hit_query_ns.store(0, std::memory_order_relaxed);
    s.max_query_ns.store(0, std::memory_order_relaxed);
    s.polls.store(0, std::memory_order_relaxed);
    s.cuda_error.store(0, std::memory_order_relaxed);
    s.upper_bound_valid.store(0, std::memory_order_relaxed);
    s.state.store(kArmed, std::memory_order_release);
  }

  void pin_self() {
#ifdef __linux__
    if (cpu_core_ >= 0) {
      cpu_set_t set;
      CPU_ZERO(&set);
      CPU_SET(cpu_core_, &set);
      pinned_.store(pthread_setaffinity_np(pthread_self(), sizeof(set), &set) == 0);
    }
#endif
  }

  void poll_loop() {
    pin_self();
    bool device_set = false;
    while (running_.load(std::memory_order_acquire)) {
      if (!device_set && cuda_device_ >= 0 && need_device_.load(std::memory_order_acquire)) {
        const cudaError_t e = cudaSetDevice(cuda_device_);
        if (e != cudaSuccess) {
          fail_armed_events((int)e);
          need_device_.store(false);
          continue;
        }
        device_set = true;
      }
      for (size_t i = 0; i < capacity_; ++i) {
        Slot& s = slots_[i];
        if (s.state.load(std::memory_order_acquire) != kArmed) continue;
        const uint64_t q0 = now_ns();
        bool hit = false;
        int err = 0;
        if (s.source.load(std::memory_order_relaxed) == kFlag) {
          const auto* flag = reinterpret_cast<const std::atomic<uint64_t>*>(s.handle.load());
          hit = flag->load(std::memory_order_acquire) >= s.expected.load(std::memory_order_relaxed);
        } else {
          if (!device_set) continue;
          const cudaError_t r = cudaEventQuery(reinterpret_cast<cudaEvent_t>(s.handle.load()));
          if (r == cudaSuccess) hit = true;
          else if (r != cudaErrorNotReady) err = (int)r;
        }
        const uint64_t q1 = now_ns();
        const uint64_t dq = q1 - q0;
        s.polls.fetch_add(1, std::memory_order_relaxed);
        if (dq > s.max_query_ns.load(std::memory_order_relaxed)) s.max_query_ns.store(dq, std::memory_order_relaxed);
        if (err) {
          s.cuda_error.store(err, std::memory_order_relaxed);
          s.state.store(kError, std::memory_order_release);
        } else if (hit) {
          const uint64_t miss = s.last_miss_start_ns.load(std::memory_order_relaxed);
          s.hit_query_ns.store(dq, std::memory_order_relaxed);
          if (miss != 0) {
            s.upper_bound_ns.store(q1 - miss, std::memory_order_relaxed);
            s.upper_bound_valid.store(1, std::memory_order_relaxed);
          }
          s.ready_ns.store(q1, std::memory_order_relaxed);
          s.state.store(kReady, std::memory_order_release);
        } else {
          s.last_miss_start_ns.store(q0, std::memory_order_relaxed);
        }
      }
    }
  }

  void fail_armed_events(int err) {
    for (size_t i = 0; i < capacity_; ++i) {
      Slot& s = slots_[i];
      if (s.state.load() == kArmed && s.source.load() == kEvent) {
        s.cuda_error.store(err);
        s.state.store(kError, std::memory_order_release);
      }
    }
  }

  size_t capacity_;
  int cpu_core_;
  int cuda_device_;
  std::unique_ptr<Slot[]> slots_;
  std::atomic<bool> running_{false};
  std::atomic<bool> pinned_{false};
  std::atomic<bool> need_device_{false};
  std::thread worker_;
};

}  // namespace

void register_event_bridge(py::module_& m) {
  py::class_<EventBridge>(m, "EventBridge")
      .def(py::init<size_t, int, int>(), py::arg("capacity"), py::arg("cpu_core") = -1,
           py::arg("cuda_device") = -1)
      .def("arm", &EventBridge::arm, py::arg("index"), py::arg("event_handle"))
      .def("arm_flag", &EventBridge::arm_flag, py::arg("index"), py::arg("host_flag_ptr"),
           py::arg("expected"))
      .def("ready", &EventBridge::ready)
      .def("ready_ns", &EventBridge::ready_ns)
      .def("state", &EventBridge::state)
      .def("wait_ready", &EventBridge::wait_ready, py::arg("index"), py::arg("timeout_ns"))
      .def("wait_all", &EventBridge::wait_all, py::arg("timeout_ns"))
      .def("snapshot", &EventBridge::snapshot)
      .def("reset_all", &EventBridge::reset_all)
      .def("stop", &EventBridge::stop)
      .def_property_readonly("pinned", &EventBridge::pinned)
      .def_property_readonly("cpu_core", &EventBridge::cpu_core)
      .def_property_readonly("cuda_device", &EventBridge::cuda_device)
      .def_property_readonly("capacity", &EventBridge::capacity);
}
