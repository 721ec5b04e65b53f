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
}  // namespace

__global__ void __launch_bounds__(256) moe_control_kernel(ControlParams p) {
  sched::StateView st = p.st;
  const sched::PlanView& plan = p.plan;
  long long* S = p.scalars;
  const int C = p.chunks;
  if (p.desc == 0) {
    const int T = st.max_tokens;
    for (int i = threadIdx.x; i < T; i += blockDim.x) {
      st.sources[i] = -1; st.destinations[i] = -1; st.ready[i] = 0; st.residual[i] = 0;
      st.remaining_hops[i] = sched::kInf; st.scratch_selected[i] = 0; st.scratch_seen[i] = 0;
    }
    for (long long i = threadIdx.x; i < (long long)T * plan.V; i += blockDim.x) st.holders[i] = 0;
    for (long long i = threadIdx.x; i < (long long)T * plan.E; i += blockDim.x) st.committed[i] = 0;
    for (int i = threadIdx.x; i < plan.V * plan.V; i += blockDim.x) st.residual_demand[i] = 0;
    for (int i = threadIdx.x; i < plan.E; i += blockDim.x) { st.link_credits[i] = plan.cap_units[i]; st.scratch_edge_load[i] = 0; }
    for (int i = threadIdx.x; i < plan.G; i += blockDim.x) st.group_credits[i] = plan.group_limits[i];
    for (int i = threadIdx.x; i < kChunkStarts + 2 * C; i += blockDim.x)
      S[i] = (i >= kChunkStarts && i < kChunkStarts + C) ? -1 : 0;
    __syncthreads();
  }
  if (threadIdx.x != 0) return;

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
      if (start + n >= st.max_tokens) {
        record_status(p.status, kBoundsViolation, 60, start + n, st.max_tokens);
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
  int n = sched::enumerate(plan, st, revealed, p.cand_buf, p.max_cands);
  if (n > p.max_cands) {
    record_status(p.status, kBoundsViolation, 61, n, p.max_cands);
    n = p.max_cands;
    gate_ok = false;
  }
  const int kept = sched::select(plan, st, p.cand_buf, n, revealed, p.keep_buf);
  for (int i = 0; i < kept; ++i) {
    p.action_buf[2 * i] = p.cand_buf[p.keep_buf[i]].ordinal;
    p.action_buf[2 * i + 1] = p.cand_buf[p.keep_buf[i]].edge;
  }
  const int code = sched::check(plan, st, p.action_buf, kept, revealed, true);
  const bool accepted = code == sched::kAccept;
  if (accepted && kept > 0) {
    sched::apply(plan, st, p.action_buf, kept);
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

  // log
  int* L = p.log + (long long)p.desc * p.log_stride;
  L[0] = n; L[1] = kept; L[2] = accepted ? 1 : 0; L[3] = code;
  L[4] = accepted ? kept : 0; L[5] = (int)S[kVersion]; L[6] = revealed; L[7] = gate_ok ? 1 : 0;
  int* sel = L + kLogHeader;
  for (int i = 0; i < kept; ++i) { sel[2 * i] = (int)p.action_buf[2 * i]; sel[2 * i + 1] = (int)p.action_buf[2 * i + 1]; }
  int* cand = L + kLogHeader + 2 * st.max_tokens;
  for (int i = 0; i < n; ++i) {
    cand[4 * i] = p.cand_buf[i].ordinal; cand[4 * i + 1] = p.cand_buf[i].edge;
    cand[4 * i + 2] = p.cand_buf[i].before; cand[4 * i + 3] = p.cand_buf[i].after;
  }
}

void launch_control(const ControlParams& p, cudaStream_t s) {
  moe_control_kernel<<<1, 256, 0, s>>>(p);
}

}  // namespace raiccl
