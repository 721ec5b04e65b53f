// C++ core of the compiled scheduler: FastBinder enumerate/select and
// DynamicGuard check/apply over the preallocated IncrementalState arrays.
//
// Semantics are those of rlccl/scheduling/compiled_event_driven.py:465-638
// (also restated in revealaiccl_b200/scheduling/compiled.py, the NumPy
// reference this core is differentially tested against):
//   enumerate: for each revealed ordinal that is ready and still residual with
//     0 < remaining_hops < INF, every route template of its destination whose
//     source is a holder, whose target is not, and whose target distance is
//     remaining_hops - 1; order = (ordinal, template order).
//   select: reset slot credits, then greedy in candidate order, one hop per
//     token, needing >= 1 link credit and >= 1 credit in every group of the edge.
//   check: per action unrevealed / duplicate_in_slot / edge_range /
//     source_holder / duplicate_commit / (residual_demand), then aggregate edge
//     capacity and bandwidth groups.
//   apply: reset slot credits; per action set holder + committed bit, consume
//     credits, retire residual demand on arrival, recompute remaining hops.
// The arrays are NumPy buffers owned by the Python IncrementalState and are
// updated in place, so both implementations observe identical state.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace py = pybind11;

namespace {

constexpr int32_t kInf = 2147483647 / 4;

template <typename T>
T* mut_ptr(const py::dict& d, const char* key) {
  py::object o = d[key];
  if (!py::isinstance<py::array>(o)) throw std::invalid_argument(std::string("not an array: ") + key);
  py::array a = o.cast<py::array>();
  if (!a.dtype().is(py::dtype::of<T>()))
    throw std::invalid_argument(std::string("wrong dtype for ") + key);
  if (!(a.flags() & py::array::c_style)) throw std::invalid_argument(std::string("not contiguous: ") + key);
  if (!a.writeable()) throw std::invalid_argument(std::string("read-only: ") + key);
  return static_cast<T*>(a.mutable_data());
}

template <typename T>
const T* ro_ptr(const py::dict& d, const char* key, py::ssize_t* n = nullptr) {
  py::object o = d[key];
  py::array a = o.cast<py::array>();
  if (!a.dtype().is(py::dtype::of<T>()))
    throw std::invalid_argument(std::string("wrong dtype for ") + key);
  if (!(a.flags() & py::array::c_style)) throw std::invalid_argument(std::string("not contiguous: ") + key);
  if (n) *n = a.size();
  return static_cast<const T*>(a.data());
}

struct Plan {
  int E = 0, G = 0, V = 0;
  const int32_t* edge_src;
  const int32_t* edge_tgt;
  const int64_t* cap_units;
  const int64_t* group_limits;
  const int32_t* group_ptr;
  const int32_t* group_members;
  const int32_t* edge_group_ptr;
  const int32_t* edge_group_members;
  const int32_t* distances;  // [V, V]
  const int32_t* tmpl_ptr;   // [V + 1]
  const int32_t* tmpl_edge;
  const int32_t* tmpl_src;
  const int32_t* tmpl_tgt;
  const int32_t* tmpl_tdist;
};

Plan load_plan(const py::dict& f) {
  Plan p;
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

struct State {
  int32_t* sources;
  int32_t* destinations;
  uint8_t* holders;    // [T, V]
  uint8_t* ready;
  uint8_t* committed;  // [T, E]
  uint8_t* residual;
  int32_t* remaining_hops;
  int64_t* residual_demand;  // [V, V]
  int64_t* link_credits;
  int64_t* group_credits;
  uint8_t* scratch_selected;
  uint8_t* scratch_seen;
  int64_t* scratch_edge_load;
};

State load_state(const py::dict& s) {
  return State{mut_ptr<int32_t>(s, "sources"),        mut_ptr<int32_t>(s, "destinations"),
               mut_ptr<uint8_t>(s, "holders"),        mut_ptr<uint8_t>(s, "ready"),
               mut_ptr<uint8_t>(s, "committed"),      mut_ptr<uint8_t>(s, "residual"),
               mut_ptr<int32_t>(s, "remaining_hops"), mut_ptr<int64_t>(s, "residual_demand"),
               mut_ptr<int64_t>(s, "link_credits"),   mut_ptr<int64_t>(s, "group_credits"),
               mut_ptr<uint8_t>(s, "scratch_selected"), mut_ptr<uint8_t>(s, "scratch_seen"),
               mut_ptr<int64_t>(s, "scratch_edge_load")};
}

void reset_slot_credits(const Plan& p, State& st, int max_tokens) {
  for (int e = 0; e < p.E; ++e) st.link_credits[e] = p.cap_units[e];
  for (int g = 0; g < p.G; ++g) st.group_credits[g] = p.group_limits[g];
  for (int t = 0; t < max_tokens; ++t) st.scratch_selected[t] = 0;
}

int max_tokens_of(const py::dict& s) {
  py::array a = s["sources"].cast<py::array>();
  return (int)a.size();
}

std::vector<std::tuple<int, int, int, int>> sched_enumerate(const py::dict& flat, const py::dict& sd,
                                                            int revealed, int nodes) {
  Plan p = load_plan(flat);
  State st = load_state(sd);
  if (nodes != p.V) throw std::invalid_argument("node count mismatch");
  std::vector<std::tuple<int, int, int, int>> out;
  for (int o = 0; o < revealed; ++o) {
    if (!st.ready[o] || !st.residual[o]) continue;
    const int d = st.destinations[o];
    const int before = st.remaining_hops[o];
    if (before <= 0 || before >= kInf) continue;
    const uint8_t* h = st.holders + (size_t)o * p.V;
    for (int k = p.tmpl_ptr[d]; k < p.tmpl_ptr[d + 1]; ++k) {
      if (h[p.tmpl_src[k]] && !h[p.tmpl_tgt[k]] && p.tmpl_tdist[k] == before - 1)
        out.emplace_back(o, p.tmpl_edge[k], before, before - 1);
    }
  }
  return out;
}

std::vector<int> sched_select(const py::dict& flat, const py::dict& sd,
                              py::array_t<int32_t, py::array::c_style> cands, int revealed) {
  Plan p = load_plan(flat);
  State st = load_state(sd);
  reset_slot_credits(p, st, max_tokens_of(sd));
  auto c = cands.unchecked<2>();
  std::vector<int> keep;
  for (py::ssize_t i = 0; i < c.shape(0); ++i) {
    const int o = c(i, 0), e = c(i, 1);
    if (o < 0 || o >= revealed || st.scratch_selected[o]) continue;
    if (e < 0 || e >= p.E) continue;
    if (st.link_credits[e] < 1) continue;
    bool ok = true;
    for (int k = p.edge_group_ptr[e]; k < p.edge_group_ptr[e + 1]; ++k)
      if (st.group_credits[p.edge_group_members[k]] < 1) { ok = false; break; }
    if (!ok) continue;
    st.scratch_selected[o] = 1;
    st.link_credits[e] -= 1;
    for (int k = p.edge_group_ptr[e]; k < p.edge_group_ptr[e + 1]; ++k)
      st.group_credits[p.edge_group_members[k]] -= 1;
    keep.push_back((int)i);
  }
  return keep;
}

// Reason codes match GUARD_REASONS in revealaiccl_b200/scheduling/compiled.py.
enum Reason { kAccept = 0, kUnrevealed = 4, kDupInSlot = 5, kEdgeRange = 6, kSourceHolder = 7,
              kDupCommit = 8, kResidual = 9, kEdgeCap = 10, kGroup = 11 };

int sched_check(const py::dict& flat, const py::dict& sd,
                py::array_t<int64_t, py::array::c_style> actions, int revealed, bool require_sched) {
  Plan p = load_plan(flat);
  State st = load_state(sd);
  const int T = max_tokens_of(sd);
  for (int t = 0; t < T; ++t) st.scratch_seen[t] = 0;
  for (int e = 0; e < p.E; ++e) st.scratch_edge_load[e] = 0;
  auto a = actions.unchecked<2>();
  for (py::ssize_t i = 0; i < a.shape(0); ++i) {
    const int64_t o = a(i, 0), e = a(i, 1);
    if (o < 0 || o >= revealed || !st.ready[o]) return kUnrevealed;
    if (st.scratch_seen[o]) return kDupInSlot;
    st.scratch_seen[o] = 1;
    if (e < 0 || e >= p.E) return kEdgeRange;
    const int s = p.edge_src[e], t = p.edge_tgt[e];
    const uint8_t* h = st.holders + (size_t)o * p.V;
    if (!h[s]) return kSourceHolder;
    if (h[t] || st.committed[(size_t)o * p.E + e]) return kDupCommit;
    if (require_sched) {
      const int d = st.destinations[o];
      const int before = st.remaining_hops[o];
      if (!st.residual[o] || before <= 0 || p.distances[(size_t)t * p.V + d] != before - 1)
        return kResidual;
    }
    st.scratch_edge_load[e] += 1;
  }
  for (int e = 0; e < p.E; ++e)
    if (st.scratch_edge_load[e] > p.cap_units[e]) return kEdgeCap;
  for (int g = 0; g < p.G; ++g) {
    int64_t load = 0;
    for (int k = p.group_ptr[g]; k < p.group_ptr[g + 1]; ++k) load += st.scratch_edge_load[p.group_members[k]];
    if (load > p.group_limits[g]) return kGroup;
  }
  return kAccept;
}

void sched_apply(const py::dict& flat, const py::dict& sd,
                 py::array_t<int64_t, py::array::c_style> actions, int nodes) {
  Plan p = load_plan(flat);
  State st = load_state(sd);
  if (nodes != p.V) throw std::invalid_argument("node count mismatch");
  reset_slot_credits(p, st, max_tokens_of(sd));
  auto a = actions.unchecked<2>();
  for (py::ssize_t i = 0; i < a.shape(0); ++i) {
    const int64_t o = a(i, 0), e = a(i, 1);
    const int t = p.edge_tgt[e];
    uint8_t* h = st.holders + (size_t)o * p.V;
    h[t] = 1;
    st.committed[(size_t)o * p.E + e] = 1;
    st.link_credits[e] -= 1;
    for (int k = p.edge_group_ptr[e]; k < p.edge_group_ptr[e + 1]; ++k)
      st.group_credits[p.edge_group_members[k]] -= 1;
    const int d = st.destinations[o];
    if (t == d && st.residual[o]) {
      st.residual_demand[(size_t)st.sources[o] * p.V + d] -= 1;
      st.residual[o] = 0;
    }
    int best = kInf;
    for (int v = 0; v < p.V; ++v)
      if (h[v] && p.distances[(size_t)v * p.V + d] < best) best = p.distances[(size_t)v * p.V + d];
    st.remaining_hops[o] = best;
  }
}

}  // namespace

void register_scheduler(py::module_& m) {
  m.def("sched_enumerate", &sched_enumerate, "FastBinder.enumerate_candidates core");
  m.def("sched_select", &sched_select, "FastBinder.select_batch core (indices kept)");
  m.def("sched_check", &sched_check, "DynamicGuard.check core (0 = accept, else reason code)");
  m.def("sched_apply", &sched_apply, "DynamicGuard.apply core (state updated in place)");
}
