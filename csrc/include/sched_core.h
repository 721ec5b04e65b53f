// Compiled-scheduler core shared by the host C++ runtime and the device
// control-plane kernel (one source, compiled by g++ and by nvcc).
//
// Semantics are those of rlccl/scheduling/compiled_event_driven.py:465-638,
// restated in revealaiccl_b200/scheduling/compiled.py (the NumPy reference
// every backend is differentially tested against):
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
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define SCHED_HD __host__ __device__ __forceinline__
#else
#define SCHED_HD inline
#endif

namespace raiccl {
namespace sched {

constexpr int32_t kInf = 2147483647 / 4;

// Reason codes (index into GUARD_REASONS of the Python layer).
enum Reason : int {
  kAccept = 0, kStale = 1, kProposalType = 2, kScenarioOnly = 3, kUnrevealed = 4,
  kDupInSlot = 5, kEdgeRange = 6, kSourceHolder = 7, kDupCommit = 8, kResidual = 9,
  kEdgeCap = 10, kGroup = 11
};

struct PlanView {
  int E, G, V;
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

struct StateView {
  int max_tokens;
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

struct Cand {
  int32_t ordinal, edge, before, after;
};

SCHED_HD void reset_slot_credits(const PlanView& p, StateView& st) {
  for (int e = 0; e < p.E; ++e) st.link_credits[e] = p.cap_units[e];
  for (int g = 0; g < p.G; ++g) st.group_credits[g] = p.group_limits[g];
  for (int t = 0; t < st.max_tokens; ++t) st.scratch_selected[t] = 0;
}

// Writes up to `cap` candidates; returns how many exist (may exceed cap).
SCHED_HD int enumerate(const PlanView& p, const StateView& st, int revealed, Cand* out, int cap) {
  int n = 0;
  for (int o = 0; o < revealed; ++o) {
    if (!st.ready[o] || !st.residual[o]) continue;
    const int d = st.destinations[o];
    const int before = st.remaining_hops[o];
    if (before <= 0 || before >= kInf) continue;
    const uint8_t* h = st.holders + (long long)o * p.V;
    for (int k = p.tmpl_ptr[d]; k < p.tmpl_ptr[d + 1]; ++k) {
      if (h[p.tmpl_src[k]] && !h[p.tmpl_tgt[k]] && p.tmpl_tdist[k] == before - 1) {
        if (n < cap) out[n] = Cand{o, p.tmpl_edge[k], before, before - 1};
        ++n;
      }
    }
  }
  return n;
}

// Candidates of one ordinal in template order (the device control plane
// enumerates ordinals in parallel: ordinal o's candidates land at
// out[prefix(o) ...], the same positions the sequential loop gives them).
SCHED_HD int enumerate_one(const PlanView& p, const StateView& st, int o, Cand* out, int cap) {
  if (!st.ready[o] || !st.residual[o]) return 0;
  const int d = st.destinations[o];
  const int before = st.remaining_hops[o];
  if (before <= 0 || before >= kInf) return 0;
  const uint8_t* h = st.holders + (long long)o * p.V;
  int n = 0;
  for (int k = p.tmpl_ptr[d]; k < p.tmpl_ptr[d + 1]; ++k) {
    if (h[p.tmpl_src[k]] && !h[p.tmpl_tgt[k]] && p.tmpl_tdist[k] == before - 1) {
      if (out != nullptr && n < cap) out[n] = Cand{o, p.tmpl_edge[k], before, before - 1};
      ++n;
    }
  }
  return n;
}

// Greedy selection; writes the kept candidate indices to keep[]; returns count.
// `credits_reset`: the caller already reset the slot credits and selection scratch.
SCHED_HD int select(const PlanView& p, StateView& st, const Cand* c, int n, int revealed, int* keep,
                    bool credits_reset = false) {
  if (!credits_reset) reset_slot_credits(p, st);
  int kept = 0;
  for (int i = 0; i < n; ++i) {
    const int o = c[i].ordinal, e = c[i].edge;
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
    keep[kept++] = i;
  }
  return kept;
}

// actions: n pairs (ordinal or -1, edge).  Returns a Reason.
SCHED_HD int check(const PlanView& p, StateView& st, const int64_t* actions, int n, int revealed,
                   bool require_sched, bool scratch_reset = false) {
  if (!scratch_reset) {
    for (int t = 0; t < st.max_tokens; ++t) st.scratch_seen[t] = 0;
    for (int e = 0; e < p.E; ++e) st.scratch_edge_load[e] = 0;
  }
  for (int i = 0; i < n; ++i) {
    const int64_t o = actions[2 * i], e = actions[2 * i + 1];
    if (o < 0 || o >= revealed || !st.ready[o]) return kUnrevealed;
    if (st.scratch_seen[o]) return kDupInSlot;
    st.scratch_seen[o] = 1;
    if (e < 0 || e >= p.E) return kEdgeRange;
    const int s = p.edge_src[e], t = p.edge_tgt[e];
    const uint8_t* h = st.holders + (long long)o * p.V;
    if (!h[s]) return kSourceHolder;
    if (h[t] || st.committed[(long long)o * p.E + e]) return kDupCommit;
    if (require_sched) {
      const int d = st.destinations[o];
      const int before = st.remaining_hops[o];
      if (!st.residual[o] || before <= 0 || p.distances[(long long)t * p.V + d] != before - 1)
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

SCHED_HD void apply(const PlanView& p, StateView& st, const int64_t* actions, int n,
                    bool credits_reset = false) {
  if (!credits_reset) reset_slot_credits(p, st);
  for (int i = 0; i < n; ++i) {
    const int64_t o = actions[2 * i], e = actions[2 * i + 1];
    const int t = p.edge_tgt[e];
    uint8_t* h = st.holders + (long long)o * p.V;
    h[t] = 1;
    st.committed[(long long)o * p.E + e] = 1;
    st.link_credits[e] -= 1;
    for (int k = p.edge_group_ptr[e]; k < p.edge_group_ptr[e + 1]; ++k)
      st.group_credits[p.edge_group_members[k]] -= 1;
    const int d = st.destinations[o];
    if (t == d && st.residual[o]) {
      st.residual_demand[(long long)st.sources[o] * p.V + d] -= 1;
      st.residual[o] = 0;
    }
    int best = kInf;
    for (int v = 0; v < p.V; ++v)
      if (h[v] && p.distances[(long long)v * p.V + d] < best) best = p.distances[(long long)v * p.V + d];
    st.remaining_hops[o] = best;
  }
}

// Stage `count` tokens at ordinals [start, start+count) (holders = {source}).
SCHED_HD void write_token(const PlanView& p, StateView& st, int ordinal, int source, int destination) {
  st.sources[ordinal] = source;
  st.destinations[ordinal] = destination;
  uint8_t* h = st.holders + (long long)ordinal * p.V;
  for (int v = 0; v < p.V; ++v) h[v] = 0;
  h[source] = 1;
}

// Activate ordinals [start, start+count): ready, residual, remaining hops.
SCHED_HD void activate_range(const PlanView& p, StateView& st, int start, int count) {
  for (int o = start; o < start + count; ++o) {
    const int s = st.sources[o], d = st.destinations[o];
    st.ready[o] = 1;
    const uint8_t* h = st.holders + (long long)o * p.V;
    const bool residual = !h[d];
    st.residual[o] = residual ? 1 : 0;
    if (residual) st.residual_demand[(long long)s * p.V + d] += 1;
    int best = kInf;
    for (int v = 0; v < p.V; ++v)
      if (h[v] && p.distances[(long long)v * p.V + d] < best) best = p.distances[(long long)v * p.V + d];
    st.remaining_hops[o] = best;
  }
}

}  // namespace sched
}  // namespace raiccl
