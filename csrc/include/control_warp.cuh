// Single-warp device control plane (the launch path whenever the plan fits: at
// most 64 edges, 32 bandwidth groups, 32 route templates per destination and
// 32 control tokens per chunk, each edge in a group at most once).
//
// control_warp_run executes the triggers [q0, q1) of one layer call on the
// compiled plan and scheduler state held in shared memory (the control blob
// layout), with the same decisions, state updates and log rows as the CTA
// kernel moe_control_kernel (the host's differential replay checks every
// trigger): lanes over tokens, templates and actions; the greedy selection
// walks the eligible ordinals in order, each step taking the first template
// whose edge still has link and group credit (credits in lane registers,
// exhausted resources as warp ballots).  Selections of more than 32 actions
// run the guard check and apply on lane 0 with the shared scheduler core.
//
// Hooks: before(desc) -> bool (false ends the loop: e.g. a bounded wait for
// the trigger's router chunks ran out) and after(desc, permitted), called by
// every lane of the warp.  The one-trigger kernel passes no-op hooks; the
// persistent front-end kernel waits for router chunks and publishes dispatch
// bases there.
#pragma once

#include <cstdint>

#include "control_layout.h"
#include "moe_kernels.h"
#include "sched_core.h"
#include "sm100_ptx.cuh"

namespace raiccl {
namespace ctl {

enum Scalar : int {
  kStaged = 0, kRevealedCount = 1, kVersion = 2, kCompleted = 3, kRevealedBits = 4,
  kDispatched = 5, kFuture = 6, kUnrevealed = 7, kDuplicate = 8, kStale = 9, kPending = 10,
  kChunkStarts = kCtlScalarHeader
};
constexpr int kLogHeader = 16;      // [0..7] decision record, [8..15] phase clocks
constexpr int kCtlStageMax = 1024;  // control-token destinations staged per trigger
constexpr int kCtlMaxChunks = 64;   // chunk bitmaps are 64-bit words
constexpr int kWarpMaxE = 64;
constexpr int kWarpMaxG = 32;
constexpr int kWarpMaxTmpl = 32;
constexpr int kWarpMaxPerChunk = 32;

// 16-byte vector copy, four loads in flight per thread before the stores.
__device__ __forceinline__ void copy16(uint4* dst, const uint4* src, long long n) {
  #pragma unroll 1
  for (long long i0 = threadIdx.x; i0 < n; i0 += 4LL * blockDim.x) {
    uint4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long i = i0 + (long long)u * blockDim.x;
      if (i < n) r[u] = src[i];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long i = i0 + (long long)u * blockDim.x;
      if (i < n) dst[i] = r[u];
    }
  }
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// kFetchesTokens: before(desc) has already placed the control-token
// destinations of every chunk the trigger needs in s_dst[c * cpc + j].
// kPublishesPermit: after(desc, permitted) writes the descriptor's permit
// word itself (the control warp then leaves it alone).
struct NoHooks {
  static constexpr bool kFetchesTokens = false;
  static constexpr bool kPublishesPermit = false;
  __device__ __forceinline__ bool before(int) { return true; }
  __device__ __forceinline__ void after(int, bool) {}
};

// Called by one full warp.  csm holds the staged control blob; s_dst
// (kCtlStageMax >= chunks x ctl_per_chunk), s_coff (kCtlMaxChunks + 1) and
// s_egmask (kWarpMaxE) are shared scratch.  reset: start a layer call (fresh scheduler state).
// s_vmc (kCtlStageMax, optional): per-ordinal template masks kept across the
// triggers of this call.  An ordinal's mask depends only on its own state
// (ready, residual, destination, remaining hops, holders), which changes only
// when it is revealed or one of its actions is applied, so each trigger
// recomputes just those ordinals; without it every trigger recomputes all.
// Rare paths, kept out of line: the warp executes its hot path once per
// trigger, so every instruction line of it is fetched once per trigger, and
// inlined fallbacks would spread that path over more lines.
static __device__ __noinline__ void cold_status(DeviceStatus* st, int code, int id, long long index, long long bound) {
  record_status(st, code, id, index, bound);
}
// The views are taken by value: a reference would make the caller's views
// address-taken, so they would live in local memory for the whole trigger loop
// and every field use on the hot path would be a local load.
static __device__ __noinline__ int cold_select(sched::PlanView plan, sched::StateView st, const sched::Cand* cand,
                                        int n, int revealed, int* keep) {
  return sched::select(plan, st, cand, n, revealed, keep, true);
}
static __device__ __noinline__ int cold_check(sched::PlanView plan, sched::StateView st, const int64_t* actions,
                                       int kept, int revealed) {
  return sched::check(plan, st, actions, kept, revealed, true, true);
}
static __device__ __noinline__ void cold_apply(sched::PlanView plan, sched::StateView st, const int64_t* actions,
                                        int kept) {
  sched::apply(plan, st, actions, kept, true);
}

// Edge -> group bitmasks of the plan (lanes over edges); returns whether an
// edge lists a group twice (the selection then needs the serial core).
// Called by one full warp.
__device__ inline int edge_group_masks(const int32_t* egptr, const int32_t* egmem, int E, uint32_t* s_egmask) {
  int dup_local = 0;
  #pragma unroll 1
  for (int e = threadIdx.x & 31; e < E; e += 32) {
    uint32_t m = 0;
    #pragma unroll 1
    for (int k = egptr[e]; k < egptr[e + 1]; ++k) {
      const uint32_t b = 1u << egmem[k];
      dup_local |= (m & b) ? 1 : 0;
      m |= b;
    }
    s_egmask[e] = m;
  }
  return __any_sync(0xffffffffu, dup_local) ? 1 : 0;
}

template <class Hooks>
__device__ void control_warp_run(const ControlParams& p, const ControlDims& dims, uint8_t* csm, int* s_dst,
                                 int* s_coff, uint32_t* s_egmask, int q0, int q1, bool reset, Hooks& hooks,
                                 uint32_t* s_vmc = nullptr) {
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const ControlLayout Lt = control_layout(dims);
  const int E = dims.E, G = dims.G, V = dims.V, T = dims.T, C = dims.chunks;
  const int P = p.partial_chunks;
  const int cpc = p.ctl_per_chunk;
  const unsigned long long epoch_v = *p.epoch;
  #pragma unroll 1
  for (int c = lane; c <= C; c += 32) s_coff[c] = p.chunk_offsets[c];
  auto at = [&](int a) { return csm + Lt.off[a]; };
  sched::PlanView plan = p.plan;
  const int64_t* s_cap = reinterpret_cast<const int64_t*>(at(kCtlCap));
  const int64_t* s_glim = reinterpret_cast<const int64_t*>(at(kCtlGroupLimits));
  const int32_t* edge_src = reinterpret_cast<const int32_t*>(at(kCtlEdgeSrc));
  const int32_t* edge_tgt = reinterpret_cast<const int32_t*>(at(kCtlEdgeTgt));
  const int32_t* gptr = reinterpret_cast<const int32_t*>(at(kCtlGroupPtr));
  const int32_t* gmem = reinterpret_cast<const int32_t*>(at(kCtlGroupMembers));
  const int32_t* egptr = reinterpret_cast<const int32_t*>(at(kCtlEdgeGroupPtr));
  const int32_t* egmem = reinterpret_cast<const int32_t*>(at(kCtlEdgeGroupMembers));
  const int32_t* dist = reinterpret_cast<const int32_t*>(at(kCtlDistances));
  const int32_t* tptr = reinterpret_cast<const int32_t*>(at(kCtlTmplPtr));
  const int32_t* tedge = reinterpret_cast<const int32_t*>(at(kCtlTmplEdge));
  const int32_t* tsrc = reinterpret_cast<const int32_t*>(at(kCtlTmplSrc));
  const int32_t* ttgt = reinterpret_cast<const int32_t*>(at(kCtlTmplTgt));
  const int32_t* ttd = reinterpret_cast<const int32_t*>(at(kCtlTmplTdist));
  plan.edge_src = edge_src; plan.edge_tgt = edge_tgt; plan.cap_units = s_cap; plan.group_limits = s_glim;
  plan.group_ptr = gptr; plan.group_members = gmem; plan.edge_group_ptr = egptr;
  plan.edge_group_members = egmem; plan.distances = dist; plan.tmpl_ptr = tptr; plan.tmpl_edge = tedge;
  plan.tmpl_src = tsrc; plan.tmpl_tgt = ttgt; plan.tmpl_tdist = ttd;
  sched::StateView st;
  st.max_tokens = T;
  st.sources = reinterpret_cast<int32_t*>(at(kCtlSources));
  st.destinations = reinterpret_cast<int32_t*>(at(kCtlDestinations));
  st.holders = at(kCtlHolders);
  st.ready = at(kCtlReady);
  st.committed = at(kCtlCommitted);
  st.residual = at(kCtlResidual);
  st.remaining_hops = reinterpret_cast<int32_t*>(at(kCtlRemainingHops));
  st.residual_demand = reinterpret_cast<int64_t*>(at(kCtlResidualDemand));
  st.link_credits = reinterpret_cast<int64_t*>(at(kCtlLinkCredits));
  st.group_credits = reinterpret_cast<int64_t*>(at(kCtlGroupCredits));
  st.scratch_selected = at(kCtlScratchSelected);
  st.scratch_seen = at(kCtlScratchSeen);
  st.scratch_edge_load = reinterpret_cast<int64_t*>(at(kCtlScratchEdgeLoad));
  long long* S = reinterpret_cast<long long*>(at(kCtlScalars));
  sched::Cand* cand = reinterpret_cast<sched::Cand*>(at(kCtlCands));
  int* keep = reinterpret_cast<int*>(at(kCtlKeep));
  int64_t* actions = reinterpret_cast<int64_t*>(at(kCtlActions));
  // per-ordinal template bitmask / first candidate index, in the action scratch
  // (free until the selection has been turned into actions)
  uint32_t* vmask = s_vmc ? s_vmc : reinterpret_cast<uint32_t*>(actions);
  int* cbase = reinterpret_cast<int*>(actions) + T;
  // template bitmask of ordinal o: templates j of its destination that take it
  // one hop closer, from a node holding it to one that does not
  auto ordinal_vm = [&](int o) -> uint32_t {
    uint32_t vm = 0;
    if (st.ready[o] && st.residual[o]) {
      const int d = st.destinations[o];
      const int before = st.remaining_hops[o];
      if (before > 0 && before < sched::kInf) {
        const uint8_t* h = st.holders + (long long)o * V;
        const int k0 = tptr[d], nt = tptr[d + 1] - k0;
        #pragma unroll 1
        for (int j = 0; j < nt; ++j) {
          const int k = k0 + j;
          if (h[tsrc[k]] && !h[ttgt[k]] && ttd[k] == before - 1) vm |= 1u << j;
        }
      }
    }
    return vm;
  };
  bool vm_valid = false;  // s_vmc holds the mask of every revealed ordinal
  __syncwarp();
  if (reset) {
    #pragma unroll 1
    for (int i = lane; i < T; i += 32) {
      st.sources[i] = -1; st.destinations[i] = -1; st.ready[i] = 0; st.residual[i] = 0;
      st.remaining_hops[i] = sched::kInf; st.scratch_selected[i] = 0; st.scratch_seen[i] = 0;
    }
    #pragma unroll 1
    for (long long i = lane; i < (long long)T * V; i += 32) st.holders[i] = 0;
    #pragma unroll 1
    for (long long i = lane; i < (long long)T * E; i += 32) st.committed[i] = 0;
    #pragma unroll 1
    for (int i = lane; i < V * V; i += 32) st.residual_demand[i] = 0;
    #pragma unroll 1
    for (int i = lane; i < E; i += 32) { st.link_credits[i] = s_cap[i]; st.scratch_edge_load[i] = 0; }
    #pragma unroll 1
    for (int i = lane; i < G; i += 32) st.group_credits[i] = s_glim[i];
    #pragma unroll 1
    for (int i = lane; i < kChunkStarts + 2 * C; i += 32)
      S[i] = (i >= kChunkStarts && i < kChunkStarts + C) ? -1 : 0;
  }
  // edge -> group bitmask (a repeated group falls back to the serial selection)
  const bool dup_groups = edge_group_masks(egptr, egmem, E, s_egmask) != 0;
  __syncwarp();
  #pragma unroll 1
  for (int desc = q0; desc < q1; ++desc) {
  if (!hooks.before(desc)) break;
  const long long clk0 = clock64();
  int clk[7] = {0, 0, 0, 0, 0, 0, 0};
  const bool final_trigger = desc >= P;
  const int c_lo = final_trigger ? P : desc;
  const int c_hi = final_trigger ? C - 1 : desc;
  // control-token destinations of the trigger's chunks (router output), kept
  // by absolute chunk: s_dst[c * cpc + j]
  if constexpr (!Hooks::kFetchesTokens) {
    const int n_stage = (c_hi - c_lo + 1) * cpc;
    #pragma unroll 1
    for (int i = lane; i < n_stage; i += 32) {
      const int c = c_lo + i / cpc, j = i % cpc;
      const int off = s_coff[c];
      const int size = s_coff[c + 1] - off;
      s_dst[c * cpc + j] = j < size ? p.expert_ids[(long long)(off + j) * p.top_k] % p.ctl_nodes : -1;
    }
  }
  __syncwarp();
  // trigger scalars live in (warp-uniform) registers until the end of the trigger
  long long completed = S[kCompleted], revealed_bits = S[kRevealedBits], pending = S[kPending];
  long long dispatched = S[kDispatched], staged = S[kStaged], revealed_count = S[kRevealedCount];
  long long version = S[kVersion], future = S[kFuture], unrevealed = S[kUnrevealed], stale = S[kStale];
  long long* starts = S + kChunkStarts;
  long long* counts = S + kChunkStarts + C;
  bool gate_ok = true;
  if (lane == 0) clk[0] = (int)(clock64() - clk0);

  // ---- complete: stage the control tokens of the trigger's chunks
  #pragma unroll 1
  for (int c = c_lo; c <= c_hi; ++c) {
    const long long bit = 1LL << c;
    if (completed & bit) { gate_ok = false; continue; }  // completed-chunk replay
    completed |= bit;
    const int off = s_coff[c];
    const int size = s_coff[c + 1] - off;
    const int limit = size < cpc ? size : cpc;
    const long long start = staged;
    const int pos = off + lane;
    const int src = pos % p.ctl_nodes;
    const int dst = lane < limit ? s_dst[c * cpc + lane] : -1;
    const bool keep_tok = lane < limit && src != dst;
    const unsigned bal = __ballot_sync(FULL, keep_tok);
    const int nk = __popc(bal);
    const long long room = T - start > 0 ? T - start : 0;
    const int n = nk <= room ? nk : (int)room;
    if (nk > room) {
      if (lane == 0) cold_status(p.status, kBoundsViolation, 60, start + n, T);
      gate_ok = false;
    }
    const int rank = __popc(bal & lanemask_lt());
    if (keep_tok && rank < n) {
      const int o = (int)(start + rank);
      st.sources[o] = src;
      st.destinations[o] = dst;
      uint8_t* h = st.holders + (long long)o * V;
      #pragma unroll 1
      for (int v = 0; v < V; ++v) h[v] = 0;
      h[src] = 1;
    }
    if (lane == 0) { starts[c] = start; counts[c] = n; }
    staged = start + n;
    pending |= bit;
    __syncwarp();
  }
  // ---- reveal pending chunks strictly in ordinal order
  #pragma unroll 1
  for (int c = c_lo; c <= c_hi; ++c) {
    const long long bit = 1LL << c;
    if (!(completed & bit)) { future += 1; gate_ok = false; continue; }
    if (revealed_bits & bit) { gate_ok = false; continue; }  // revealed-chunk replay
    const long long s0 = starts[c], cn = counts[c];
    if (!(pending & bit) || s0 != revealed_count) { gate_ok = false; continue; }
    revealed_bits |= bit;
    #pragma unroll 1
    for (long long o = s0 + lane; o < s0 + cn; o += 32) {
      const int s = st.sources[o], d = st.destinations[o];
      st.ready[o] = 1;
      const uint8_t* h = st.holders + o * V;
      const bool residual = !h[d];
      st.residual[o] = residual ? 1 : 0;
      if (residual) atomicAdd(reinterpret_cast<unsigned long long*>(&st.residual_demand[(long long)s * V + d]), 1ULL);
      int best = sched::kInf;
      #pragma unroll 1
      for (int v = 0; v < V; ++v)
        if (h[v] && dist[(long long)v * V + d] < best) best = dist[(long long)v * V + d];
      st.remaining_hops[o] = best;
      if (vm_valid) s_vmc[o] = ordinal_vm((int)o);
    }
    revealed_count += cn;
    pending &= ~bit;
    __syncwarp();
  }
  const int revealed = (int)revealed_count;
  if (lane == 0) clk[1] = (int)(clock64() - clk0);

  // ---- enumerate: per-ordinal template bitmask and candidate prefix
  #pragma unroll 1
  for (int t = lane; t < T; t += 32) st.scratch_selected[t] = 0;
  const bool cached = vm_valid;
  int carry = 0;
  #pragma unroll 1
  for (int o0 = 0; o0 < revealed; o0 += 32) {
    const int o = o0 + lane;
    uint32_t vm = 0;
    if (o < revealed) vm = cached ? s_vmc[o] : ordinal_vm(o);
    const int cnt = __popc(vm);
    int incl = cnt;
    for (int s = 1; s < 32; s <<= 1) {
      const int v = __shfl_up_sync(FULL, incl, s);
      if (lane >= s) incl += v;
    }
    const int base = carry + incl - cnt;
    if (o < revealed) {
      if (!cached) vmask[o] = vm;
      cbase[o] = base;
      if (vm) {
        const int d = st.destinations[o];
        const int before = st.remaining_hops[o];
        const int k0 = tptr[d];
        int i = base;
        #pragma unroll 1
        for (uint32_t m = vm; m; m &= m - 1, ++i)
          if (i < p.max_cands) cand[i] = sched::Cand{o, tedge[k0 + __ffs(m) - 1], before, before - 1};
      }
    }
    carry += __shfl_sync(FULL, incl, 31);
  }
  vm_valid = s_vmc != nullptr;
  int n = carry;
  if (n > p.max_cands) {
    if (lane == 0) cold_status(p.status, kBoundsViolation, 61, n, p.max_cands);
    n = p.max_cands;
    gate_ok = false;
  }
  __syncwarp();
  if (lane == 0) clk[2] = (int)(clock64() - clk0);

  // ---- select: greedy over candidates in (ordinal, template) order
  // An edge is usable while it has link credit and none of its groups is
  // exhausted; a candidate is viable iff its edge is usable.  Each lane holds
  // the edge set of its ordinal's candidates, so one ballot finds the next
  // ordinal with a viable candidate and ordinals without one cost nothing;
  // once no edge is usable nothing further can be taken.
  int kept = 0;
  if (!dup_groups) {
    long long cred_lo = lane < E ? s_cap[lane] : 0, cred_hi = lane + 32 < E ? s_cap[lane + 32] : 0;
    long long gcred = lane < G ? s_glim[lane] : 0;
    const uint32_t eg_lo = lane < E ? s_egmask[lane] : 0u, eg_hi = lane + 32 < E ? s_egmask[lane + 32] : 0u;
    uint32_t lack_grp = __ballot_sync(FULL, lane < G && gcred < 1);
    auto usable_edges = [&]() -> unsigned long long {
      const bool ulo = lane < E && cred_lo >= 1 && !(eg_lo & lack_grp);
      const bool uhi = lane + 32 < E && cred_hi >= 1 && !(eg_hi & lack_grp);
      return (unsigned long long)__ballot_sync(FULL, ulo) | ((unsigned long long)__ballot_sync(FULL, uhi) << 32);
    };
    unsigned long long usable = usable_edges();
    #pragma unroll 1
    for (int o0 = 0; o0 < revealed && usable != 0ull; o0 += 32) {
      const int my_o = o0 + lane;
      const uint32_t my_vm = my_o < revealed ? vmask[my_o] : 0u;
      const int my_base = my_o < revealed ? cbase[my_o] : 0;
      const int my_k0 = (my_o < revealed && my_vm) ? tptr[st.destinations[my_o]] : 0;
      unsigned long long my_edges = 0;  // edges of this ordinal's candidates inside the bound n
      {
        int i = my_base;
        #pragma unroll 1
        for (uint32_t m = my_vm; m && i < n; m &= m - 1, ++i) my_edges |= 1ull << tedge[my_k0 + __ffs(m) - 1];
      }
      uint32_t todo = __ballot_sync(FULL, (my_edges & usable) != 0ull);
      #pragma unroll 1
      while (todo) {
        const int src_lane = __ffs(todo) - 1;
        const uint32_t vm = __shfl_sync(FULL, my_vm, src_lane);
        const int b = __shfl_sync(FULL, my_base, src_lane);
        const int k0 = __shfl_sync(FULL, my_k0, src_lane);
        const int ci = b + __popc(vm & lanemask_lt());
        const bool valid = ((vm >> lane) & 1u) && ci < n;
        const int e = valid ? tedge[k0 + lane] : 0;
        const unsigned vb = __ballot_sync(FULL, valid && ((usable >> e) & 1ull));
        const uint32_t later = ~((2u << src_lane) - 1u);  // lanes after src_lane
        if (!vb) { todo &= later; continue; }
        const int jl = __ffs(vb) - 1;
        const int es = __shfl_sync(FULL, e, jl);
        const int cs = __shfl_sync(FULL, ci, jl);
        if (lane == 0) { keep[kept] = cs; st.scratch_selected[o0 + src_lane] = 1; }
        ++kept;
        if (lane == (es & 31)) { if (es < 32) cred_lo -= 1; else cred_hi -= 1; }
        const uint32_t egs = __shfl_sync(FULL, es < 32 ? eg_lo : eg_hi, es & 31);
        if (lane < G && ((egs >> lane) & 1u)) gcred -= 1;
        lack_grp = __ballot_sync(FULL, lane < G && gcred < 1);
        usable = usable_edges();
        todo = __ballot_sync(FULL, (my_edges & usable) != 0ull) & later;
      }
    }
    if (lane < E) st.link_credits[lane] = cred_lo;
    if (lane + 32 < E) st.link_credits[lane + 32] = cred_hi;
    if (lane < G) st.group_credits[lane] = gcred;
    __syncwarp();
  } else {
    #pragma unroll 1
    for (int e = lane; e < E; e += 32) st.link_credits[e] = s_cap[e];
    #pragma unroll 1
    for (int g = lane; g < G; g += 32) st.group_credits[g] = s_glim[g];
    __syncwarp();
    if (lane == 0) kept = cold_select(plan, st, cand, n, revealed, keep);
    kept = __shfl_sync(FULL, kept, 0);
  }
  __syncwarp();
  #pragma unroll 1
  for (int i = lane; i < kept; i += 32) {
    const sched::Cand cc = cand[keep[i]];
    actions[2 * i] = cc.ordinal;
    actions[2 * i + 1] = cc.edge;
  }
  __syncwarp();
  if (lane == 0) clk[3] = (int)(clock64() - clk0);

  // ---- guard check
  #pragma unroll 1
  for (int t = lane; t < T; t += 32) st.scratch_seen[t] = 0;
  #pragma unroll 1
  for (int e = lane; e < E; e += 32) st.scratch_edge_load[e] = 0;
  __syncwarp();
  int code = sched::kAccept;
  const bool fast_actions = kept <= 32 && !dup_groups;
  if (fast_actions) {
    const bool act = lane < kept;
    const int o = act ? (int)actions[2 * lane] : -1;
    const int e = act ? (int)actions[2 * lane + 1] : -1;
    int reason = 0;
    if (act) {
      if (o < 0 || o >= revealed || !st.ready[o]) reason = sched::kUnrevealed;
    }
    const unsigned peers = __match_any_sync(FULL, act ? o : -1 - lane);
    if (act && !reason) {
      const uint8_t* h = st.holders + (long long)o * V;
      if (peers & lanemask_lt()) reason = sched::kDupInSlot;
      else if (e < 0 || e >= E) reason = sched::kEdgeRange;
      else if (!h[edge_src[e]]) reason = sched::kSourceHolder;
      else if (h[edge_tgt[e]] || st.committed[(long long)o * E + e]) reason = sched::kDupCommit;
      else {
        const int d = st.destinations[o], before = st.remaining_hops[o];
        if (!st.residual[o] || before <= 0 || dist[(long long)edge_tgt[e] * V + d] != before - 1)
          reason = sched::kResidual;
      }
    }
    const unsigned fb = __ballot_sync(FULL, reason != 0);
    if (fb) {
      code = __shfl_sync(FULL, reason, __ffs(fb) - 1);
    } else {
      const unsigned epeers = __match_any_sync(FULL, act ? e : -1 - lane);
      if (act) {
        st.scratch_seen[o] = 1;
        if ((epeers & lanemask_lt()) == 0) st.scratch_edge_load[e] = __popc(epeers);
      }
      __syncwarp();
      const bool over_lo = lane < E && st.scratch_edge_load[lane] > s_cap[lane];
      const bool over_hi = lane + 32 < E && st.scratch_edge_load[lane + 32] > s_cap[lane + 32];
      const unsigned olo = __ballot_sync(FULL, over_lo), ohi = __ballot_sync(FULL, over_hi);
      if (olo || ohi) {
        code = sched::kEdgeCap;
      } else {
        long long load = 0;
        if (lane < G)
          #pragma unroll 1
          for (int k = gptr[lane]; k < gptr[lane + 1]; ++k) load += st.scratch_edge_load[gmem[k]];
        if (__ballot_sync(FULL, lane < G && load > s_glim[lane])) code = sched::kGroup;
      }
    }
  } else {
    if (lane == 0) code = cold_check(plan, st, actions, kept, revealed);
    code = __shfl_sync(FULL, code, 0);
  }
  const bool accepted = code == sched::kAccept;
  __syncwarp();
  if (lane == 0) clk[4] = (int)(clock64() - clk0);

  // ---- packing gate and permit, then the release: the descriptor's dispatch
  // does not depend on the state update below, so it starts while it runs
  if (accepted && kept > 0) version += 1;
  #pragma unroll 1
  for (int c = c_lo; c <= c_hi; ++c) {
    const long long bit = 1LL << c;
    if (!(completed & bit)) { future += 1; gate_ok = false; }
    else if (!(revealed_bits & bit)) { unrevealed += 1; gate_ok = false; }
    else if (dispatched & bit) { stale += 1; gate_ok = false; }
  }
  if (gate_ok)
    #pragma unroll 1
    for (int c = c_lo; c <= c_hi; ++c) dispatched |= 1LL << c;
  if (lane == 0) {
    if (!Hooks::kPublishesPermit) p.permit[desc] = (accepted && gate_ok) ? epoch_v : 0ULL;
    if (!(accepted && gate_ok)) cold_status(p.status, kTimeoutPermit, 62, desc, code);
  }
  __syncwarp();
  hooks.after(desc, accepted && gate_ok);

  // ---- apply (accepted actions)
  if (accepted && kept > 0 && fast_actions) {
    // credits after the slot = reset credits minus the committed usage
    if (lane < E) st.link_credits[lane] = s_cap[lane] - st.scratch_edge_load[lane];
    if (lane + 32 < E) st.link_credits[lane + 32] = s_cap[lane + 32] - st.scratch_edge_load[lane + 32];
    if (lane < G) {
      long long used = 0;
      #pragma unroll 1
      for (int e = 0; e < E; ++e)
        if ((s_egmask[e] >> lane) & 1u) used += st.scratch_edge_load[e];
      st.group_credits[lane] = s_glim[lane] - used;
    }
    if (lane < kept) {
      const int o = (int)actions[2 * lane], e = (int)actions[2 * lane + 1];
      const int t = edge_tgt[e];
      uint8_t* h = st.holders + (long long)o * V;
      h[t] = 1;
      st.committed[(long long)o * E + e] = 1;
      const int d = st.destinations[o];
      if (t == d && st.residual[o]) {
        atomicAdd(reinterpret_cast<unsigned long long*>(&st.residual_demand[(long long)st.sources[o] * V + d]),
                  ~0ULL);  // -1
        st.residual[o] = 0;
      }
      int best = sched::kInf;
      #pragma unroll 1
      for (int v = 0; v < V; ++v)
        if (h[v] && dist[(long long)v * V + d] < best) best = dist[(long long)v * V + d];
      st.remaining_hops[o] = best;
      if (vm_valid) s_vmc[o] = ordinal_vm(o);  // the actions of one slot have distinct ordinals
    }
  } else {
    #pragma unroll 1
    for (int e = lane; e < E; e += 32) st.link_credits[e] = s_cap[e];
    #pragma unroll 1
    for (int g = lane; g < G; g += 32) st.group_credits[g] = s_glim[g];
    __syncwarp();
    if (accepted && kept > 0) {
      if (lane == 0) cold_apply(plan, st, actions, kept);
      vm_valid = false;  // recompute every mask next trigger
    }
  }
  #pragma unroll 1
  for (int t = lane; t < T; t += 32) st.scratch_selected[t] = 0;
  __syncwarp();
  int* L = p.log + (long long)desc * p.log_stride;
  if (lane == 0) {
    S[kCompleted] = completed; S[kRevealedBits] = revealed_bits; S[kPending] = pending;
    S[kDispatched] = dispatched; S[kStaged] = staged; S[kRevealedCount] = revealed_count;
    S[kVersion] = version; S[kFuture] = future; S[kUnrevealed] = unrevealed; S[kStale] = stale;
    clk[5] = (int)(clock64() - clk0);
    L[0] = n; L[1] = kept; L[2] = accepted ? 1 : 0; L[3] = code;
    L[4] = accepted ? kept : 0; L[5] = (int)version; L[6] = revealed; L[7] = gate_ok ? 1 : 0;
  }
  // ---- log and state write-back
  int* sel = L + kLogHeader;
  #pragma unroll 1
  for (int i = lane; i < kept; i += 32) {
    sel[2 * i] = (int)actions[2 * i];
    sel[2 * i + 1] = (int)actions[2 * i + 1];
  }
  int* cl = L + kLogHeader + 2 * T;
  #pragma unroll 1
  for (int i = lane; i < n; i += 32) {
    cl[4 * i] = cand[i].ordinal; cl[4 * i + 1] = cand[i].edge;
    cl[4 * i + 2] = cand[i].before; cl[4 * i + 3] = cand[i].after;
  }
  __syncwarp();
  if (lane == 0) {
    clk[6] = (int)(clock64() - clk0);
    for (int i = 0; i < 7; ++i) L[8 + i] = clk[i];
    L[15] = 1;  // warp-path marker
  }
  __syncwarp();
  }  // trigger loop
}

}  // namespace ctl
}  // namespace raiccl
