// Python binding of the compiled-scheduler core (csrc/include/sched_core.h)
// operating in place on the NumPy arrays owned by the Python IncrementalState.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "sched_core.h"

namespace py = pybind11;

namespace {

template <typename T>
T* mut_ptr(const py::dict& d, const char* key) {
  py::object o = d[key];
  if (!py::isinstance<py::array>(o)) throw std::invalid_argument(std::string("not an array: ") + key);
  py::array a = o.cast<py::array>();
  if (!a.dtype().is(py::dtype::of<T>())) throw std::invalid_argument(std::string("wrong dtype for ") + key);
  if (!(a.flags() & py::array::c_style)) throw std::invalid_argument(std::string("not contiguous: ") + key);
  if (!a.writeable()) throw std::invalid_argument(std::string("read-only: ") + key);
  return static_cast<T*>(a.mutable_data());
}

template <typename T>
const T* ro_ptr(const py::dict& d, const char* key, py::ssize_t* n = nullptr) {
  py::array a = d[key].cast<py::array>();
  if (!a.dtype().is(py::dtype::of<T>())) throw std::invalid_argument(std::string("wrong dtype for ") + key);
  if (!(a.flags() & py::array::c_style)) throw std::invalid_argument(std::string("not contiguous: ") + key);
  if (n) *n = a.size();
  return static_cast<const T*>(a.data());
}

using raiccl::sched::Cand;
using raiccl::sched::PlanView;
using raiccl::sched::StateView;

PlanView load_plan(const py::dict& f) {
  PlanView p;
  py::ssize_t n = 0;
  p.edge_src = ro_ptr<int32_t>(f, "edge_src", &n);
  p.E = (int)n;
  p.edge_tgt = ro_ptr<int32_t>(f, "edge_tgt");
  p.cap_units = ro_ptr<int64_t>(f, "cap_units");
  p.group_limits = ro_ptr<int64_t>(f, "group_limits", &n);
  p.G = (int)n;
  p.group_ptr = ro_ptr<int32_t>(f, "group_ptr");
  p.group_members = ro_ptr<int32_t>(f, "group_members");
  p.edge_group_ptr = ro_ptr<int32_t>(f, "edge_group_ptr");
  p.edge_group_members = ro_ptr<int32_t>(f, "edge_group_members");
  p.tmpl_ptr = ro_ptr<int32_t>(f, "tmpl_ptr", &n);
  p.V = (int)n - 1;
  p.distances = ro_ptr<int32_t>(f, "distances");
  p.tmpl_edge = ro_ptr<int32_t>(f, "tmpl_edge");
  p.tmpl_src = ro_ptr<int32_t>(f, "tmpl_src");
  p.tmpl_tgt = ro_ptr<int32_t>(f, "tmpl_tgt");
  p.tmpl_tdist = ro_ptr<int32_t>(f, "tmpl_tdist");
  return p;
}

StateView load_state(const py::dict& s) {
  StateView v;
  py::array src = s["sources"].cast<py::array>();
  v.max_tokens = (int)src.size();
  v.sources = mut_ptr<int32_t>(s, "sources");
  v.destinations = mut_ptr<int32_t>(s, "destinations");
  v.holders = mut_ptr<uint8_t>(s, "holders");
  v.ready = mut_ptr<uint8_t>(s, "ready");
  v.committed = mut_ptr<uint8_t>(s, "committed");
  v.residual = mut_ptr<uint8_t>(s, "residual");
  v.remaining_hops = mut_ptr<int32_t>(s, "remaining_hops");
  v.residual_demand = mut_ptr<int64_t>(s, "residual_demand");
  v.link_credits = mut_ptr<int64_t>(s, "link_credits");
  v.group_credits = mut_ptr<int64_t>(s, "group_credits");
  v.scratch_selected = mut_ptr<uint8_t>(s, "scratch_selected");
  v.scratch_seen = mut_ptr<uint8_t>(s, "scratch_seen");
  v.scratch_edge_load = mut_ptr<int64_t>(s, "scratch_edge_load");
  return v;
}

std::vector<std::tuple<int, int, int, int>> sched_enumerate(const py::dict& flat, const py::dict& sd,
                                                            int revealed, int nodes) {
  PlanView p = load_plan(flat);
  StateView st = load_state(sd);
  if (nodes != p.V) throw std::invalid_argument("node count mismatch");
  int n = raiccl::sched::enumerate(p, st, revealed, nullptr, 0);
  std::vector<Cand> buf((size_t)n);
  raiccl::sched::enumerate(p, st, revealed, buf.data(), n);
  std::vector<std::tuple<int, int, int, int>> out;
  out.reserve(buf.size());
  for (const Cand& c : buf) out.emplace_back(c.ordinal, c.edge, c.before, c.after);
  return out;
}

std::vector<int> sched_select(const py::dict& flat, const py::dict& sd,
                              py::array_t<int32_t, py::array::c_style> cands, int revealed) {
  PlanView p = load_plan(flat);
  StateView st = load_state(sd);
  auto c = cands.unchecked<2>();
  std::vector<Cand> buf((size_t)c.shape(0));
  for (py::ssize_t i = 0; i < c.shape(0); ++i) buf[i] = Cand{c(i, 0), c(i, 1), 0, 0};
  std::vector<int> keep(buf.size());
  const int k = raiccl::sched::select(p, st, buf.data(), (int)buf.size(), revealed, keep.data());
  keep.resize((size_t)k);
  return keep;
}

int sched_check(const py::dict& flat, const py::dict& sd,
                py::array_t<int64_t, py::array::c_style> actions, int revealed, bool require_sched) {
  PlanView p = load_plan(flat);
  StateView st = load_state(sd);
  return raiccl::sched::check(p, st, actions.data(), (int)actions.shape(0), revealed, require_sched);
}

void sched_apply(const py::dict& flat, const py::dict& sd,
                 py::array_t<int64_t, py::array::c_style> actions, int nodes) {
  PlanView p = load_plan(flat);
  StateView st = load_state(sd);
  if (nodes != p.V) throw std::invalid_argument("node count mismatch");
  raiccl::sched::apply(p, st, actions.data(), (int)actions.shape(0));
}

}  // namespace

void register_scheduler(py::module_& m) {
  m.def("sched_enumerate", &sched_enumerate, "FastBinder.enumerate_candidates core");
  m.def("sched_select", &sched_select, "FastBinder.select_batch core (indices kept)");
  m.def("sched_check", &sched_check, "DynamicGuard.check core (0 = accept, else reason code)");
  m.def("sched_apply", &sched_apply, "DynamicGuard.apply core (state updated in place)");
}
