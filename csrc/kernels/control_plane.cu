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
// The CTA stages the compiled plan and the state in shared memory; the resets
// and the per-ordinal candidate enumeration run across the CTA, and only the
// order-dependent steps (staging, greedy selection, guard check, apply) run
// on one thread, at shared-memory latency.  The CTA writes the state back.
#include <cstdint>

#include "launchers.h"
#include "moe_kernels.h"
#include "control_warp.cuh"
#include "sm100_ptx.cuh"

namespace raiccl {

namespace {
using namespace ctl;

ControlDims dims_of(const ControlParams& p) {
  return ControlDims{p.plan.E, p.plan.G, p.plan.V, p.st.max_tokens, p.n_group_members,
                     p.n_edge_group_members, p.n_tmpl, p.max_cands, p.chunks};
}
}  // namespace

// Shared-memory bytes of the kernel: the whole blob.
size_t control_smem_bytes(const ControlParams& p) { return (size_t)control_layout(dims_of(p)).total; }
ControlDims control_dims(const ControlParams& p) { return dims_of(p); }

__global__ void __launch_bounds__(256) moe_control_kernel(ControlParams p, ControlDims dims) {
  TraceScope trace_scope(p.trace);
  extern __shared__ __align__(16) uint8_t csm[];
  __shared__ int s_clk[8];  // SM cycles since kernel start at each phase end (thread 0)
  const long long clk0 = clock64();
  const ControlLayout Lt = control_layout(dims);
  const int E = dims.E, G = dims.G, V = dims.V, T = dims.T, C = dims.chunks;
  // ---- stage plan + state into shared memory: one vector copy
  // the whole persistent part, also at the first trigger (whose reset then
  // overwrites every array), so alignment padding round-trips unchanged
  const long long stage_bytes = Lt.state_end;
  copy16(reinterpret_cast<uint4*>(csm), reinterpret_cast<const uint4*>(p.blob), stage_bytes / 16);
  // control-token destinations of the trigger's chunks, fetched in parallel
  __shared__ int s_dst[kCtlStageMax];
  __shared__ int s_coff[kCtlMaxChunks + 1];
  const int P = p.partial_chunks;
  const bool final_trigger = p.desc >= P;
  const int c_lo = final_trigger ? P : p.desc;
  const int c_hi = final_trigger ? C - 1 : p.desc;
  const int cpc = p.ctl_per_chunk;
  const int n_stage = (c_hi - c_lo + 1) * cpc;
  const bool staged = n_stage <= kCtlStageMax && C <= kCtlMaxChunks;
  if (staged) {
    for (int c = threadIdx.x; c <= C; c += blockDim.x) s_coff[c] = p.chunk_offsets[c];
    for (int i = threadIdx.x; i < n_stage; i += blockDim.x) {
      const int c = c_lo + i / cpc, j = i % cpc;
      const int off = p.chunk_offsets[c];
      const int size = p.chunk_offsets[c + 1] - off;
      s_dst[i] = j < size ? p.expert_ids[(long long)(off + j) * p.top_k] % p.ctl_nodes : -1;
    }
  }
  auto at = [&](int a) { return csm + Lt.off[a]; };
  sched::PlanView plan = p.plan;
  int64_t* s_cap = reinterpret_cast<int64_t*>(at(kCtlCap));
  int64_t* s_glim = reinterpret_cast<int64_t*>(at(kCtlGroupLimits));
  plan.edge_src = reinterpret_cast<const int32_t*>(at(kCtlEdgeSrc));
  plan.edge_tgt = reinterpret_cast<const int32_t*>(at(kCtlEdgeTgt));
  plan.cap_units = s_cap;
  plan.group_limits = s_glim;
  plan.group_ptr = reinterpret_cast<const int32_t*>(at(kCtlGroupPtr));
  plan.group_members = reinterpret_cast<const int32_t*>(at(kCtlGroupMembers));
  plan.edge_group_ptr = reinterpret_cast<const int32_t*>(at(kCtlEdgeGroupPtr));
  plan.edge_group_members = reinterpret_cast<const int32_t*>(at(kCtlEdgeGroupMembers));
  plan.distances = reinterpret_cast<const int32_t*>(at(kCtlDistances));
  plan.tmpl_ptr = reinterpret_cast<const int32_t*>(at(kCtlTmplPtr));
  plan.tmpl_edge = reinterpret_cast<const int32_t*>(at(kCtlTmplEdge));
  plan.tmpl_src = reinterpret_cast<const int32_t*>(at(kCtlTmplSrc));
  plan.tmpl_tgt = reinterpret_cast<const int32_t*>(at(kCtlTmplTgt));
  plan.tmpl_tdist = reinterpret_cast<const int32_t*>(at(kCtlTmplTdist));
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
  __syncthreads();
  if (p.desc == 0) {  // first trigger of a layer call: fresh state
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
  }
  __syncthreads();
  __shared__ int s_n, s_kept, s_revealed, s_gate, s_accepted, s_code;
  int* cnt = keep;  // per-ordinal candidate counts reuse the keep buffer before selection
  if (threadIdx.x == 0) s_clk[0] = (int)(clock64() - clk0);
  // ---- phase A (one thread): complete + reveal
  if (threadIdx.x == 0) {
    long long* starts = S + kChunkStarts;
    long long* counts = S + kChunkStarts + C;
    bool gate_ok = true;
    for (int c = c_lo; c <= c_hi; ++c) {
      const long long bit = 1LL << c;
      if (S[kCompleted] & bit) { gate_ok = false; continue; }  // completed-chunk replay
      S[kCompleted] |= bit;
      const int off = staged ? s_coff[c] : p.chunk_offsets[c];
      const int size = (staged ? s_coff[c + 1] : p.chunk_offsets[c + 1]) - off;
      const int limit = size < cpc ? size : cpc;
      const long long start = S[kStaged];
      int n = 0;
      for (int i = 0; i < limit; ++i) {
        const int pos = off + i;
        const int src = pos % p.ctl_nodes;
        const int dst = staged ? s_dst[(c - c_lo) * cpc + i]
                               : p.expert_ids[(long long)pos * p.top_k] % p.ctl_nodes;
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
    s_revealed = (int)S[kRevealedCount];
    s_gate = gate_ok ? 1 : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) s_clk[1] = (int)(clock64() - clk0);
  // ---- phase B (CTA): slot-credit reset + per-ordinal candidate enumeration
  const int revealed = s_revealed;
  for (int e = threadIdx.x; e < E; e += blockDim.x) st.link_credits[e] = s_cap[e];
  for (int g = threadIdx.x; g < G; g += blockDim.x) st.group_credits[g] = s_glim[g];
  for (int t = threadIdx.x; t < T; t += blockDim.x) st.scratch_selected[t] = 0;
  for (int o = threadIdx.x; o < revealed; o += blockDim.x) cnt[o] = sched::enumerate_one(plan, st, o, nullptr, 0);
  __syncthreads();
  if (threadIdx.x == 0) {  // exclusive prefix over ordinals: candidate order = (ordinal, template)
    int run = 0;
    for (int o = 0; o < revealed; ++o) { const int c0 = cnt[o]; cnt[o] = run; run += c0; }
    s_n = run;
  }
  __syncthreads();
  for (int o = threadIdx.x; o < revealed; o += blockDim.x) {
    const int base = cnt[o];
    if (base < p.max_cands) sched::enumerate_one(plan, st, o, cand + base, p.max_cands - base);
  }
  __syncthreads();
  if (threadIdx.x == 0) s_clk[2] = (int)(clock64() - clk0);
  // ---- phase C (one thread): greedy selection in candidate order
  if (threadIdx.x == 0) {
    int n = s_n;
    if (n > p.max_cands) {
      record_status(p.status, kBoundsViolation, 61, n, p.max_cands);
      n = p.max_cands;
      s_gate = 0;
    }
    s_n = n;
    const int kept = sched::select(plan, st, cand, n, revealed, keep, true);
    for (int i = 0; i < kept; ++i) {
      actions[2 * i] = cand[keep[i]].ordinal;
      actions[2 * i + 1] = cand[keep[i]].edge;
    }
    s_kept = kept;
  }
  __syncthreads();
  if (threadIdx.x == 0) s_clk[3] = (int)(clock64() - clk0);
  // ---- phase D (CTA): guard scratch reset; phase E (one thread): guard check
  for (int t = threadIdx.x; t < T; t += blockDim.x) st.scratch_seen[t] = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) st.scratch_edge_load[e] = 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    s_code = sched::check(plan, st, actions, s_kept, revealed, true, true);
    s_accepted = s_code == sched::kAccept ? 1 : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) s_clk[4] = (int)(clock64() - clk0);
  // ---- phase F (CTA): credit reset for apply; phase G (one thread): apply, gate, permit
  for (int e = threadIdx.x; e < E; e += blockDim.x) st.link_credits[e] = s_cap[e];
  for (int g = threadIdx.x; g < G; g += blockDim.x) st.group_credits[g] = s_glim[g];
  for (int t = threadIdx.x; t < T; t += blockDim.x) st.scratch_selected[t] = 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool accepted = s_accepted != 0;
    const int kept = s_kept;
    bool gate_ok = s_gate != 0;
    if (accepted && kept > 0) {
      sched::apply(plan, st, actions, kept, true);
      S[kVersion] += 1;
    }
    for (int c = c_lo; c <= c_hi; ++c) {
      const long long bit = 1LL << c;
      if (!(S[kCompleted] & bit)) { S[kFuture] += 1; gate_ok = false; }
      else if (!(S[kRevealedBits] & bit)) { S[kUnrevealed] += 1; gate_ok = false; }
      else if (S[kDispatched] & bit) { S[kStale] += 1; gate_ok = false; }
    }
    if (gate_ok)
      for (int c = c_lo; c <= c_hi; ++c) S[kDispatched] |= 1LL << c;
    p.permit[p.desc] = (accepted && gate_ok) ? *p.epoch : 0ULL;
    if (!(accepted && gate_ok)) record_status(p.status, kTimeoutPermit, 62, p.desc, s_code);
    int* L = p.log + (long long)p.desc * p.log_stride;
    s_clk[5] = (int)(clock64() - clk0);
    L[0] = s_n; L[1] = kept; L[2] = accepted ? 1 : 0; L[3] = s_code;
    L[4] = accepted ? kept : 0; L[5] = (int)S[kVersion]; L[6] = revealed; L[7] = gate_ok ? 1 : 0;
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
  __syncthreads();
  if (threadIdx.x == 0) {
    s_clk[6] = (int)(clock64() - clk0);
    s_clk[7] = 0;
    int* L = p.log + (long long)p.desc * p.log_stride;
    for (int i = 0; i < 8; ++i) L[8 + i] = s_clk[i];
  }
  // ---- state back to the blob: one vector copy (scratch stays in shared memory;
  // the trigger's candidates and selection are in its log row)
  copy16(reinterpret_cast<uint4*>(p.blob + Lt.state_begin), reinterpret_cast<const uint4*>(csm + Lt.state_begin),
         (Lt.state_end - Lt.state_begin) / 16);
}

__global__ void __launch_bounds__(32) moe_control_warp_kernel(ControlParams p, ControlDims dims) {
  TraceScope trace_scope(p.trace);
  extern __shared__ __align__(16) uint8_t csm[];
  __shared__ int s_dst[ctl::kCtlStageMax];
  __shared__ int s_coff[ctl::kCtlMaxChunks + 1];
  __shared__ uint32_t s_egmask[ctl::kWarpMaxE];
  const ControlLayout Lt = control_layout(dims);
  // the whole persistent part, also at the first trigger (whose reset then
  // overwrites every array), so alignment padding round-trips unchanged
  ctl::copy16(reinterpret_cast<uint4*>(csm), reinterpret_cast<const uint4*>(p.blob), Lt.state_end / 16);
  __syncwarp();
  ctl::NoHooks hooks;
  ctl::control_warp_run(p, dims, csm, s_dst, s_coff, s_egmask, p.desc, p.desc + 1, p.desc == 0, hooks);
  __syncwarp();
  ctl::copy16(reinterpret_cast<uint4*>(p.blob + Lt.state_begin), reinterpret_cast<const uint4*>(csm + Lt.state_begin),
              (Lt.state_end - Lt.state_begin) / 16);
}

bool control_warp_path_ok(const ControlParams& p) {
  // s_dst holds every chunk's control tokens (chunks x ctl_per_chunk entries)
  return p.plan.E <= kWarpMaxE && p.plan.G <= kWarpMaxG && p.max_tmpl <= kWarpMaxTmpl &&
         p.ctl_per_chunk <= kWarpMaxPerChunk && p.chunks <= kCtlMaxChunks &&
         p.chunks * p.ctl_per_chunk <= kCtlStageMax;
}

void launch_control(const ControlParams& p, cudaStream_t s) {
  const size_t smem = control_smem_bytes(p);
  if (!p.force_serial && control_warp_path_ok(p)) {
    static size_t configured_w = 0;
    if (smem > 48 * 1024 && smem > configured_w) {
      cudaFuncSetAttribute(moe_control_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      configured_w = smem;
    }
    moe_control_warp_kernel<<<1, 32, smem, s>>>(p, dims_of(p));
    return;
  }
  static size_t configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    cudaFuncSetAttribute(moe_control_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured = smem;
  }
  moe_control_kernel<<<1, 256, smem, s>>>(p, dims_of(p));
}

}  // namespace raiccl
