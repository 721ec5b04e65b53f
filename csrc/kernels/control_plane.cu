// Device-resident control plane of the progressive MoE layer.
//
// At each scheduler trigger (one per descriptor) a single CTA, stream-ordered
// after the router chunk(s) it consumes, runs the steps the reference runs on
// the host per revealed chunk (scripts/run_r4_a0_c0_full_moe.py:419-580):
//   complete  — mark the chunk completed and stage its control tokens
//               (the first ctl_per_chunk router assignments, source =
//               position mod ctl_nodes, destination = expert mod ctl_nodes)
//               as pending (invisible to the binder and guard);
//   reveal    — activate pending chunks strictly in ordinal order;
//   schedule  — FastBinder enumerate/select + DynamicGuard check/apply with
//               scheduler semantics (csrc/include/sched_core.h, the same code
//               the host C++ core runs);
//   pack gate — the descriptor's chunks must be completed, revealed and not yet
//               dispatched (future / unrevealed / stale counters otherwise);
// and publishes permit[desc] = epoch only when the guard accepted and the
// packing gate passed.  The dispatch kernel refuses to move a byte without it.
// Every step is logged for the host's post-hoc differential replay.
//
// The scheduler itself is sequential; to keep its dependent accesses at
// shared-memory latency the CTA stages the compiled plan and the state in
// shared memory, one thread runs the trigger, and the CTA writes the state
// back.
#include <cstdint>

#include "launchers.h"
#include "moe_kernels.h"
#include "sm100_ptx.cuh"

namespace raiccl {

namespace {
enum Scalar : int {
  kStaged = 0, kRevealedCount = 1, kVersion = 2, kCompleted = 3, kRevealedBits = 4,
  kDispatched = 5, kFuture = 6, kUnrevealed = 7, kDuplicate = 8, kStale = 9, kPending = 10,
  kChunkStarts = 11
};
constexpr int kLogHeader = 8;

struct Carver {
  uint8_t* base;
  size_t off;
  template <typename T>
  __device__ T* take(long long n) {
    off = (off + 15) & ~(size_t)15;
    T* p = reinterpret_cast<T*>(base + off);
    off += (size_t)(n > 0 ? n : 1) * sizeof(T);
    return p;
  }
};

template <typename T>
__device__ void copy_arr(T* dst, const T* src, long long n) {
  for (long long i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}
}  // namespace

// Shared-memory bytes the kernel carves (mirrors the Carver sequence below).
size_t control_smem_bytes(const ControlParams& p) {
  size_t off = 0;
  auto take = [&](long long n, size_t elem) {
    off = (off + 15) & ~(size_t)15;
    off += (size_t)(n > 0 ? n : 1) * elem;
  };
  const int E = p.plan.E, G = p.plan.G, V = p.plan.V, T = p.st.max_tokens;
  take(E, 4); take(E, 4); take(E, 8); take(G, 8); take(G + 1, 4); take(p.n_group_members, 4);
  take(E + 1, 4); take(p.n_edge_group_members, 4); take((long long)V * V, 4); take(V + 1, 4);
  take(p.n_tmpl, 4); take(p.n_tmpl, 4); take(p.n_tmpl, 4); take(p.n_tmpl, 4);
  take(T, 4); take(T, 4); take((long long)T * V, 1); take(T, 1); take((long long)T * E, 1); take(T, 1);
  take(T, 4); take((long long)V * V, 8); take(E, 8); take(G, 8); take(T, 1); take(T, 1); take(E, 8);
  take(p.max_cands, sizeof(sched::Cand)); take(p.max_cands, 4); take(2LL * T, 8);
  take(kChunkStarts + 2LL * p.chunks, 8);
  return off + 16;
}

__global__ void __launch_bounds__(256) moe_control_kernel(ControlParams p) {
  extern __shared__ __align__(16) uint8_t csm[];
  Carver cv{csm, 0};
  const int E = p.plan.E, G = p.plan.G, V = p.plan.V, T = p.st.max_tokens, C = p.chunks;
  // ---- plan -> shared
  sched::PlanView plan = p.plan;
  int32_t* s_edge_src = cv.take<int32_t>(E);
  int32_t* s_edge_tgt = cv.take<int32_t>(E);
  int64_t* s_cap = cv.take<int64_t>(E);
  int64_t* s_glim = cv.take<int64_t>(G);
  int32_t* s_gptr = cv.take<int32_t>(G + 1);
  int32_t* s_gmem = cv.take<int32_t>(p.n_group_members);
  int32_t* s_egptr = cv.take<int32_t>(E + 1);
  int32_t* s_egmem = cv.take<int32_t>(p.n_edge_group_members);
  int32_t* s_dist = cv.take<int32_t>((long long)V * V);
  int32_t* s_tptr = cv.take<int32_t>(V + 1);
  int32_t* s_tedge = cv.take<int32_t>(p.n_tmpl);
  int32_t* s_tsrc = cv.take<int32_t>(p.n_tmpl);
  int32_t* s_ttgt = cv.take<int32_t>(p.n_tmpl);
  int32_t* s_ttd = cv.take<int32_t>(p.n_tmpl);
  copy_arr(s_edge_src, p.plan.edge_src, E);
  copy_arr(s_edge_tgt, p.plan.edge_tgt, E);
  copy_arr(s_cap, p.plan.cap_units, E);
  if (G) { copy_arr(s_glim, p.plan.group_limits, G); copy_arr(s_gmem, p.plan.group_members, p.n_group_members); }
  copy_arr(s_gptr, p.plan.group_ptr, G + 1);
  copy_arr(s_egptr, p.plan.edge_group_ptr, E + 1);
  if (p.n_edge_group_members) copy_arr(s_egmem, p.plan.edge_group_members, p.n_edge_group_members);
  copy_arr(s_dist, p.plan.distances, (long long)V * V);
  copy_arr(s_tptr, p.plan.tmpl_ptr, V + 1);
  if (p.n_tmpl) {
    copy_arr(s_tedge, p.plan.tmpl_edge, p.n_tmpl); copy_arr(s_tsrc, p.plan.tmpl_src, p.n_tmpl);
    copy_arr(s_ttgt, p.plan.tmpl_tgt, p.n_tmpl); copy_arr(s_ttd, p.plan.tmpl_tdist, p.n_tmpl);
  }
  plan.edge_src = s_edge_src; plan.edge_tgt = s_edge_tgt; plan.cap_units = s_cap;
  plan.group_limits = s_glim; plan.group_ptr = s_gptr; plan.group_members = s_gmem;
  plan.edge_group_ptr = s_egptr; plan.edge_group_members = s_egmem; plan.distances = s_dist;
  plan.tmpl_ptr = s_tptr; plan.tmpl_edge = s_tedge; plan.tmpl_src = s_tsrc; plan.tmpl_tgt = s_ttgt;
  plan.tmpl_tdist = s_ttd;
  // ---- state -> shared (reset at the first trigger of a call)
  sched::StateView st;
  st.max_tokens = T;
  st.sources = cv.take<int32_t>(T);
  st.destinations = cv.take<int32_t>(T);
  st.holders = cv.take<uint8_t>((long long)T * V);
  st.ready = cv.take<uint8_t>(T);
  st.committed = cv.take<uint8_t>((long long)T * E);
  st.residual = cv.take<uint8_t>(T);
  st.remaining_hops = cv.take<int32_t>(T);
  st.residual_demand = cv.take<int64_t>((long long)V * V);
  st.link_credits = cv.take<int64_t>(E);
  st.group_credits = cv.take<int64_t>(G);
  st.scratch_selected = cv.take<uint8_t>(T);
  st.scratch_seen = cv.take<uint8_t>(T);
  st.scratch_edge_load = cv.take<int64_t>(E);
  sched::Cand* cand = cv.take<sched::Cand>(p.max_cands);
  int* keep = cv.take<int>(p.max_cands);
  int64_t* actions = cv.take<int64_t>(2LL * T);
  long long* S = cv.take<long long>(kChunkStarts + 2LL * C);
  const sched::StateView& gs = p.st;
  if (p.desc == 0) {
    for (int i = threadIdx.x; i < T; i += blockDim.x) {
      st.sources[i] = -1; st.destinations[i] = -1; st.ready[i] = 0; st.residual[i] = 0;
      st.remaining_hops[i] = sched::kInf; st.scratch_selected[i] = 0; st.scratch_seen[i] = 0;
    }
    for (long long i = threadIdx.x; i < (long long)T * V; i += blockDim.x) st.holders[i] = 0;
    for (long long i = threadIdx.x; i < (long long)T * E; i += blockDim.x) st.committed[i] = 0;
    for (int i = threadIdx.x; i < V * V; i += blockDim.x) st.residual_demand[i] = 0;
    for (int i = threadIdx.x; i < E; i += blockDim.x) { st.link_credits[i] = s_cap[i]; st.scratch_edge_load[i] = 0; }
    for (int i = threadIdx.x; i < G; i += blockDim.x) st.group_credits[i] = s_glim[i];
    for (int i = threadIdx.x; i < kChunkStarts + 2 * C; i += blockDim.x)
      S[i] = (i >= kChunkStarts && i < kChunkStarts + C) ? -1 : 0;
  } else {
    copy_arr(st.sources, gs.sources, T); copy_arr(st.destinations, gs.destinations, T);
    copy_arr(st.holders, gs.holders, (long long)T * V); copy_arr(st.ready, gs.ready, T);
    copy_arr(st.committed, gs.committed, (long long)T * E); copy_arr(st.residual, gs.residual, T);
    copy_arr(st.remaining_hops, gs.remaining_hops, T);
    copy_arr(st.residual_demand, gs.residual_demand, (long long)V * V);
    copy_arr(st.link_credits, gs.link_credits, E);
    if (G) copy_arr(st.group_credits, gs.group_credits, G);
    copy_arr(st.scratch_selected, gs.scratch_selected, T); copy_arr(st.scratch_seen, gs.scratch_seen, T);
    copy_arr(st.scratch_edge_load, gs.scratch_edge_load, E);
    copy_arr(S, p.scalars, kChunkStarts + 2LL * C);
  }
  __syncthreads();

  __shared__ int s_n, s_kept;
  if (threadIdx.x == 0) {
    const int P = p.partial_chunks;
    const bool final_trigger = p.desc >= P;
    const int c_lo = final_trigger ? P : p.desc;
    const int c_hi = final_trigger ? C - 1 : p.desc;
    long long* starts = S + kChunkStarts;
    long long* counts = S + kChunkStarts + C;
    bool gate_ok = true;
    // complete: stage control tokens of each newly completed chunk
    for (int c = c_lo; c <= c_hi; ++c) {
      const long long bit = 1LL << c;
      if (S[kCompleted] & bit) { gate_ok = false; continue; }  // completed-chunk replay
      S[kCompleted] |= bit;
      const int off = p.chunk_offsets[c];
      const int size = p.chunk_offsets[c + 1] - off;
      const int limit = size < p.ctl_per_chunk ? size : p.ctl_per_chunk;
      const long long start = S[kStaged];
      int n = 0;
      for (int i = 0; i < limit; ++i) {
        const int pos = off + i;
        const int src = pos % p.ctl_nodes;
        const int dst = p.expert_ids[(long long)pos * p.top_k] % p.ctl_nodes;
        if (src == dst) continue;
        if (start + n >= T) {
          record_status(p.status, kBoundsViolation, 60, start + n, T);
          gate_ok = false;
          break;
        }
        sched::write_token(plan, st, (int)(start + n), src, dst);
        ++n;
      }
      starts[c] = start;
      counts[c] = n;
      S[kStaged] = start + n;
      S[kPending] |= bit;
    }
    // reveal: activate pending chunks in ordinal order
    for (int c = c_lo; c <= c_hi; ++c) {
      const long long bit = 1LL << c;
      if (!(S[kCompleted] & bit)) { S[kFuture] += 1; gate_ok = false; continue; }
      if (S[kRevealedBits] & bit) { gate_ok = false; continue; }  // revealed-chunk replay
      if (!(S[kPending] & bit) || starts[c] != S[kRevealedCount]) { gate_ok = false; continue; }
      S[kRevealedBits] |= bit;
      sched::activate_range(plan, st, (int)starts[c], (int)counts[c]);
      S[kRevealedCount] += counts[c];
      S[kPending] &= ~bit;
    }
    // schedule: enumerate -> select -> guard check -> apply
    const int revealed = (int)S[kRevealedCount];
    int n = sched::enumerate(plan, st, revealed, cand, p.max_cands);
    if (n > p.max_cands) {
      record_status(p.status, kBoundsViolation, 61, n, p.max_cands);
      n = p.max_cands;
      gate_ok = false;
    }
    const int kept = sched::select(plan, st, cand, n, revealed, keep);
    for (int i = 0; i < kept; ++i) {
      actions[2 * i] = cand[keep[i]].ordinal;
      actions[2 * i + 1] = cand[keep[i]].edge;
    }
    const int code = sched::check(plan, st, actions, kept, revealed, true);
    const bool accepted = code == sched::kAccept;
    if (accepted && kept > 0) {
      sched::apply(plan, st, actions, kept);
      S[kVersion] += 1;
    }
    // packing gate over the descriptor's chunks
    for (int c = c_lo; c <= c_hi; ++c) {
      const long long bit = 1LL << c;
      if (!(S[kCompleted] & bit)) { S[kFuture] += 1; gate_ok = false; }
      else if (!(S[kRevealedBits] & bit)) { S[kUnrevealed] += 1; gate_ok = false; }
      else if (S[kDispatched] & bit) { S[kStale] += 1; gate_ok = false; }
    }
    if (gate_ok)
      for (int c = c_lo; c <= c_hi; ++c) S[kDispatched] |= 1LL << c;
    p.permit[p.desc] = (accepted && gate_ok) ? *p.epoch : 0ULL;
    if (!(accepted && gate_ok)) record_status(p.status, kTimeoutPermit, 62, p.desc, code);
    int* L = p.log + (long long)p.desc * p.log_stride;
    L[0] = n; L[1] = kept; L[2] = accepted ? 1 : 0; L[3] = code;
    L[4] = accepted ? kept : 0; L[5] = (int)S[kVersion]; L[6] = revealed; L[7] = gate_ok ? 1 : 0;
    s_n = n;
    s_kept = kept;
  }
  __syncthreads();
  // ---- log (parallel) and state write-back
  {
    int* L = p.log + (long long)p.desc * p.log_stride;
    int* sel = L + kLogHeader;
    for (int i = threadIdx.x; i < s_kept; i += blockDim.x) {
      sel[2 * i] = (int)actions[2 * i];
      sel[2 * i + 1] = (int)actions[2 * i + 1];
    }
    int* cl = L + kLogHeader + 2 * T;
    for (int i = threadIdx.x; i < s_n; i += blockDim.x) {
      cl[4 * i] = cand[i].ordinal; cl[4 * i + 1] = cand[i].edge;
      cl[4 * i + 2] = cand[i].before; cl[4 * i + 3] = cand[i].after;
    }
  }
  copy_arr(gs.sources, st.sources, T); copy_arr(gs.destinations, st.destinations, T);
  copy_arr(gs.holders, st.holders, (long long)T * V); copy_arr(gs.ready, st.ready, T);
  copy_arr(gs.committed, st.committed, (long long)T * E); copy_arr(gs.residual, st.residual, T);
  copy_arr(gs.remaining_hops, st.remaining_hops, T);
  copy_arr(gs.residual_demand, st.residual_demand, (long long)V * V);
  copy_arr(gs.link_credits, st.link_credits, E);
  if (G) copy_arr(gs.group_credits, st.group_credits, G);
  copy_arr(gs.scratch_selected, st.scratch_selected, T); copy_arr(gs.scratch_seen, st.scratch_seen, T);
  copy_arr(gs.scratch_edge_load, st.scratch_edge_load, E);
  copy_arr(p.scalars, S, kChunkStarts + 2LL * C);
}

void launch_control(const ControlParams& p, cudaStream_t s) {
  const size_t smem = control_smem_bytes(p);
  static size_t configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    cudaFuncSetAttribute(moe_control_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured = smem;
  }
  moe_control_kernel<<<1, 256, smem, s>>>(p);
}

}  // namespace raiccl
