// Packed single-warp control plane: the front end's path whenever the plan
// has at most 32 nodes, 64 edges and 32 bandwidth groups, and no edge lists a
// group twice.
//
// Same decisions, scheduler state and log rows as control_warp_run (the
// layer tests compare the final state and every log row with the step
// pipeline, and the host replays every trigger), but the per-ordinal state a
// trigger touches is held packed, one word per field, in shared memory:
//
//   hold[o]  holders of ordinal o as a node bitmask
//   comm[o]  committed edges of o as an edge bitmask
//   meta[o]  source | destination << 8 | ready << 16 | residual << 17
//   hops[o]  remaining hops (kInf when none)
//   vm[o]    template mask of o (the candidate templates of its destination,
//            kept up to date whenever o's state changes)
//   act[o]   the edge selected for o in this trigger, or -1
//
// and the route templates are turned, once per call, into bitmask tables per
// destination d (bit j = template j of d):
//
//   src_m[d V + v]  templates whose source is v
//   tgt_m[d V + v]  templates whose target is v
//   td_m [d V + t]  templates whose target is t hops from d
//   edge [d 32 + j] the edge of template j
//
// so an ordinal's template mask is (OR of src_m over its holders) &
// ~(OR of tgt_m over its holders) & td_m[remaining hops - 1]: a few table
// reads instead of a dependent pass over every template of the destination.
// Every lane owns the ordinals o = 32 i + lane; the greedy selection still
// walks ordinals in order (one warp step per ordinal with a viable
// candidate), and the guard checks each action on its owner lane.  The
// byte-per-entry state arrays of the blob are written once, at the end of the
// call.  A selection holds at most one action per ordinal, so the guard's
// duplicate-in-slot check cannot fire here.
#pragma once

#include <cstdint>

#include "control_warp.cuh"

namespace raiccl {
namespace ctl {

constexpr uint32_t kMetaReady = 1u << 16;
constexpr uint32_t kMetaResidual = 1u << 17;

// Shared bytes of the packed path after the blob: tables, then the packed
// per-ordinal arrays (T ordinals), then per-trigger edge / group loads.
CTL_HD long long packed_smem_bytes(const ControlDims& d) {
  const long long V = d.V, T = d.T;
  const long long tables = (3 * V * V + 32 * V) * 4;
  const long long per_ord = T * (4 + 8 + 4 + 4 + 4 + 4 + 4);
  return ((tables + 15) & ~15LL) + ((per_ord + 15) & ~15LL) + (64 + 32) * 4 + 16;
}

CTL_HD bool packed_path_ok(const ControlDims& d) { return d.V <= 32 && d.E <= 64 && d.G <= 32; }

struct PackedView {
  uint32_t* src_m;
  uint32_t* tgt_m;
  uint32_t* td_m;
  int32_t* tedge;
  uint64_t* comm;
  uint32_t* hold;
  uint32_t* meta;
  int32_t* hops;
  uint32_t* vm;
  int32_t* act;
  int32_t* base;
  int32_t* eload;  // [64]
  int32_t* gload;  // [32]
};

__device__ __forceinline__ PackedView packed_view(uint8_t* p, const ControlDims& d) {
  const long long V = d.V, T = d.T;
  PackedView v;
  v.src_m = reinterpret_cast<uint32_t*>(p);
  v.tgt_m = v.src_m + V * V;
  v.td_m = v.tgt_m + V * V;
  v.tedge = reinterpret_cast<int32_t*>(v.td_m + V * V);
  uint8_t* q = p + (((3 * V * V + 32 * V) * 4 + 15) & ~15LL);
  v.comm = reinterpret_cast<uint64_t*>(q);
  v.hold = reinterpret_cast<uint32_t*>(v.comm + T);
  v.meta = v.hold + T;
  v.hops = reinterpret_cast<int32_t*>(v.meta + T);
  v.vm = reinterpret_cast<uint32_t*>(v.hops + T);
  v.act = reinterpret_cast<int32_t*>(v.vm + T);
  v.base = v.act + T;
  v.eload = reinterpret_cast<int32_t*>(q + ((T * 32 + 15) & ~15LL));
  v.gload = v.eload + 64;
  return v;
}

// Template tables from the staged blob; collective over the CTA (the caller
// synchronises before and after).
__device__ inline void build_packed_tables(const uint8_t* csm, const ControlDims& dims, PackedView pv) {
  const ControlLayout Lt = control_layout(dims);
  const int V = dims.V;
  const int32_t* tptr = reinterpret_cast<const int32_t*>(csm + Lt.off[kCtlTmplPtr]);
  const int32_t* tedge = reinterpret_cast<const int32_t*>(csm + Lt.off[kCtlTmplEdge]);
  const int32_t* tsrc = reinterpret_cast<const int32_t*>(csm + Lt.off[kCtlTmplSrc]);
  const int32_t* ttgt = reinterpret_cast<const int32_t*>(csm + Lt.off[kCtlTmplTgt]);
  const int32_t* ttd = reinterpret_cast<const int32_t*>(csm + Lt.off[kCtlTmplTdist]);
  for (int i = threadIdx.x; i < 3 * V * V; i += blockDim.x) pv.src_m[i] = 0;
  for (int i = threadIdx.x; i < 32 * V; i += blockDim.x) pv.tedge[i] = -1;
  __syncthreads();
  for (int k = threadIdx.x; k < dims.n_tmpl; k += blockDim.x) {
    int d = 0;
    while (d + 1 < V && tptr[d + 1] <= k) ++d;
    const int j = k - tptr[d];
    if (j < 0 || j >= 32) continue;  // (the warp path allows 32 templates per destination)
    const uint32_t b = 1u << j;
    atomicOr(&pv.src_m[d * V + tsrc[k]], b);
    atomicOr(&pv.tgt_m[d * V + ttgt[k]], b);
    if (ttd[k] >= 0 && ttd[k] < V) atomicOr(&pv.td_m[d * V + ttd[k]], b);
    pv.tedge[d * 32 + j] = tedge[k];
  }
}

template <class Hooks>
__device__ void control_warp_run_packed(const ControlParams& p, const ControlDims& dims, uint8_t* csm, int* s_dst,
                                        int* s_coff, const uint32_t* s_egmask, PackedView pv, int q0, int q1,
                                        Hooks& hooks) {
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
  const int64_t* s_cap = reinterpret_cast<const int64_t*>(at(kCtlCap));
  const int64_t* s_glim = reinterpret_cast<const int64_t*>(at(kCtlGroupLimits));
  const int32_t* edge_src = reinterpret_cast<const int32_t*>(at(kCtlEdgeSrc));
  const int32_t* edge_tgt = reinterpret_cast<const int32_t*>(at(kCtlEdgeTgt));
  const int32_t* dist = reinterpret_cast<const int32_t*>(at(kCtlDistances));
  int64_t* resdem = reinterpret_cast<int64_t*>(at(kCtlResidualDemand));
  long long* S = reinterpret_cast<long long*>(at(kCtlScalars));
  sched::Cand* cand = reinterpret_cast<sched::Cand*>(at(kCtlCands));
  int64_t* actions = reinterpret_cast<int64_t*>(at(kCtlActions));
  uint32_t* const hold = pv.hold;
  uint64_t* const comm = pv.comm;
  uint32_t* const meta = pv.meta;
  int32_t* const hops = pv.hops;
  uint32_t* const vm = pv.vm;
  int32_t* const act = pv.act;
  int32_t* const cbase = pv.base;

  // remaining hops of a holder set towards d, and the template mask of an ordinal
  auto hops_of = [&](uint32_t h, int d) -> int {
    int best = sched::kInf;
    #pragma unroll 1
    for (uint32_t m = h; m; m &= m - 1) {
      const int x = dist[(__ffs(m) - 1) * V + d];
      best = x < best ? x : best;
    }
    return best;
  };
  auto vm_of = [&](uint32_t mt, uint32_t h, int before) -> uint32_t {
    if ((mt & (kMetaReady | kMetaResidual)) != (kMetaReady | kMetaResidual)) return 0u;
    if (before <= 0 || before >= sched::kInf || before - 1 >= V) return 0u;
    const int d = (mt >> 8) & 0xff;
    uint32_t sa = 0, ta = 0;
    #pragma unroll 1
    for (uint32_t m = h; m; m &= m - 1) {
      const int v = __ffs(m) - 1;
      sa |= pv.src_m[d * V + v];
      ta |= pv.tgt_m[d * V + v];
    }
    return sa & ~ta & pv.td_m[d * V + before - 1];
  };

  // fresh call: per-ordinal state, residual demand, trigger scalars
  #pragma unroll 1
  for (int o = lane; o < T; o += 32) {
    hold[o] = 0; comm[o] = 0; meta[o] = 0; hops[o] = sched::kInf; vm[o] = 0; act[o] = -1;
  }
  #pragma unroll 1
  for (int i = lane; i < V * V; i += 32) resdem[i] = 0;
  #pragma unroll 1
  for (int i = lane; i < kChunkStarts + 2 * C; i += 32) S[i] = (i >= kChunkStarts && i < kChunkStarts + C) ? -1 : 0;
  // edges e = lane and lane + 32, group g = lane
  const bool elo = lane < E, ehi = lane + 32 < E, gl = lane < G;
  const long long cap_lo = elo ? s_cap[lane] : 0, cap_hi = ehi ? s_cap[lane + 32] : 0;
  const long long glim = gl ? s_glim[lane] : 0;
  const uint32_t eg_lo = elo ? s_egmask[lane] : 0u, eg_hi = ehi ? s_egmask[lane + 32] : 0u;
  long long lc_lo = cap_lo, lc_hi = cap_hi, gc = glim;  // credits after the last applied slot
  int el_lo = 0, el_hi = 0;                             // edge loads of the last guard check
  bool pa_ok = false;                                   // the last guard's per-action checks passed
  __syncwarp();

  #pragma unroll 1
  for (int desc = q0; desc < q1; ++desc) {
    if (!hooks.before(desc)) break;
    const long long clk0 = clock64();
    int clk[7] = {0, 0, 0, 0, 0, 0, 0};
    const bool final_trigger = desc >= P;
    const int c_lo = final_trigger ? P : desc;
    const int c_hi = final_trigger ? C - 1 : desc;
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
      if (completed & bit) { gate_ok = false; continue; }
      completed |= bit;
      const int off = s_coff[c];
      const int size = s_coff[c + 1] - off;
      const int limit = size < cpc ? size : cpc;
      const long long start = staged;
      const int src = (off + lane) % p.ctl_nodes;
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
        meta[o] = (uint32_t)src | ((uint32_t)dst << 8);
        hold[o] = 1u << src;
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
      if (revealed_bits & bit) { gate_ok = false; continue; }
      const long long s0 = starts[c], cn = counts[c];
      if (!(pending & bit) || s0 != revealed_count) { gate_ok = false; continue; }
      revealed_bits |= bit;
      #pragma unroll 1
      for (long long o = s0 + lane; o < s0 + cn; o += 32) {
        uint32_t mt = meta[o];
        const int s = mt & 0xff, d = (mt >> 8) & 0xff;
        const uint32_t h = hold[o];
        mt |= kMetaReady;
        if (!((h >> d) & 1u)) {
          mt |= kMetaResidual;
          atomicAdd(reinterpret_cast<unsigned long long*>(&resdem[s * V + d]), 1ULL);
        }
        const int hp = hops_of(h, d);
        meta[o] = mt;
        hops[o] = hp;
        vm[o] = vm_of(mt, h, hp);
      }
      revealed_count += cn;
      pending &= ~bit;
      __syncwarp();
    }
    const int revealed = (int)revealed_count;
    if (lane == 0) clk[1] = (int)(clock64() - clk0);

    // ---- enumerate: candidate prefix per ordinal; the candidate list (for the log)
    int carry = 0;
    #pragma unroll 1
    for (int o0 = 0; o0 < revealed; o0 += 32) {
      const int o = o0 + lane;
      const uint32_t m0 = o < revealed ? vm[o] : 0u;
      const int cnt = __popc(m0);
      int incl = cnt;
      #pragma unroll
      for (int s = 1; s < 32; s <<= 1) {
        const int v = __shfl_up_sync(FULL, incl, s);
        if (lane >= s) incl += v;
      }
      const int base = carry + incl - cnt;
      if (o < revealed) {
        cbase[o] = base;
        if (m0) {
          const int d = (meta[o] >> 8) & 0xff;
          const int before = hops[o];
          int i = base;
          #pragma unroll 1
          for (uint32_t m = m0; m; m &= m - 1, ++i)
            if (i < p.max_cands) cand[i] = sched::Cand{o, pv.tedge[d * 32 + __ffs(m) - 1], before, before - 1};
        }
      }
      carry += __shfl_sync(FULL, incl, 31);
    }
    int n = carry;
    if (n > p.max_cands) {
      if (lane == 0) cold_status(p.status, kBoundsViolation, 61, n, p.max_cands);
      n = p.max_cands;
      gate_ok = false;
    }
    __syncwarp();
    if (lane == 0) clk[2] = (int)(clock64() - clk0);

    // ---- select: greedy over ordinals in order, each taking its first
    // template whose edge has link credit and credit in all of its groups
    int kept = 0;
    {
      long long cred_lo = cap_lo, cred_hi = cap_hi, gcred = glim;
      uint32_t lack_grp = __ballot_sync(FULL, gl && gcred < 1);
      auto usable_edges = [&]() -> unsigned long long {
        const bool ulo = elo && cred_lo >= 1 && !(eg_lo & lack_grp);
        const bool uhi = ehi && cred_hi >= 1 && !(eg_hi & lack_grp);
        return (unsigned long long)__ballot_sync(FULL, ulo) | ((unsigned long long)__ballot_sync(FULL, uhi) << 32);
      };
      unsigned long long usable = usable_edges();
      #pragma unroll 1
      for (int o0 = 0; o0 < T; o0 += 32)
        if (o0 + lane < T) act[o0 + lane] = -1;
      #pragma unroll 1
      for (int o0 = 0; o0 < revealed && usable != 0ull; o0 += 32) {
        const int o = o0 + lane;
        const uint32_t my_vm = o < revealed ? vm[o] : 0u;
        const int my_base = o < revealed ? cbase[o] : 0;
        const int d = o < revealed ? (int)((meta[o] >> 8) & 0xff) : 0;
        unsigned long long my_edges = 0;  // edges of this ordinal's candidates inside the bound n
        {
          int i = my_base;
          #pragma unroll 1
          for (uint32_t m = my_vm; m && i < n; m &= m - 1, ++i) my_edges |= 1ull << pv.tedge[d * 32 + __ffs(m) - 1];
        }
        uint32_t todo = __ballot_sync(FULL, (my_edges & usable) != 0ull);
        #pragma unroll 1
        while (todo) {
          const int src_lane = __ffs(todo) - 1;
          int es = -1;
          if (lane == src_lane) {  // the owner takes its first viable template
            int i = my_base;
            #pragma unroll 1
            for (uint32_t m = my_vm; m && i < n; m &= m - 1, ++i) {
              const int e = pv.tedge[d * 32 + __ffs(m) - 1];
              if ((usable >> e) & 1ull) { es = e; break; }
            }
            act[o] = es;
          }
          es = __shfl_sync(FULL, es, src_lane);
          const uint32_t later = ~((2u << src_lane) - 1u);  // lanes after src_lane
          if (es < 0) { todo &= later; continue; }
          if (lane == 0) {
            actions[2 * kept] = o0 + src_lane;
            actions[2 * kept + 1] = es;
          }
          ++kept;
          if (lane == (es & 31)) { if (es < 32) cred_lo -= 1; else cred_hi -= 1; }
          const uint32_t egs = __shfl_sync(FULL, es < 32 ? eg_lo : eg_hi, es & 31);
          if (gl && ((egs >> lane) & 1u)) gcred -= 1;
          lack_grp = __ballot_sync(FULL, gl && gcred < 1);
          usable = usable_edges();
          todo = __ballot_sync(FULL, (my_edges & usable) != 0ull) & later;
        }
      }
    }
    __syncwarp();
    if (lane == 0) clk[3] = (int)(clock64() - clk0);

    // ---- guard check, each action on its owner lane (actions are in ordinal order)
    if (elo) pv.eload[lane] = 0;
    if (ehi) pv.eload[lane + 32] = 0;
    if (gl) pv.gload[lane] = 0;
    __syncwarp();
    int code = sched::kAccept;
    #pragma unroll 1
    for (int o0 = 0; o0 < revealed && code == sched::kAccept; o0 += 32) {
      const int o = o0 + lane;
      const int e = o < revealed ? act[o] : -1;
      int reason = 0;
      if (e >= 0) {
        const uint32_t mt = meta[o], h = hold[o];
        if (!(mt & kMetaReady)) {
          reason = sched::kUnrevealed;
        } else if (e >= E) {
          reason = sched::kEdgeRange;
        } else {
          const int es = edge_src[e], et = edge_tgt[e];
          if (!((h >> es) & 1u)) reason = sched::kSourceHolder;
          else if (((h >> et) & 1u) || ((comm[o] >> e) & 1ull)) reason = sched::kDupCommit;
          else {
            const int d = (mt >> 8) & 0xff, before = hops[o];
            if (!(mt & kMetaResidual) || before <= 0 || dist[et * V + d] != before - 1) reason = sched::kResidual;
          }
        }
      }
      const unsigned fb = __ballot_sync(FULL, reason != 0);
      if (fb) code = __shfl_sync(FULL, reason, __ffs(fb) - 1);
    }
    pa_ok = code == sched::kAccept;
    if (pa_ok) {
      #pragma unroll 1
      for (int o0 = 0; o0 < revealed; o0 += 32) {
        const int o = o0 + lane;
        const int e = o < revealed ? act[o] : -1;
        if (e >= 0) {
          atomicAdd(&pv.eload[e], 1);
          #pragma unroll 1
          for (uint32_t m = s_egmask[e]; m; m &= m - 1) atomicAdd(&pv.gload[__ffs(m) - 1], 1);
        }
      }
      __syncwarp();
      el_lo = elo ? pv.eload[lane] : 0;
      el_hi = ehi ? pv.eload[lane + 32] : 0;
      const bool over = (elo && el_lo > cap_lo) || (ehi && el_hi > cap_hi);
      if (__ballot_sync(FULL, over)) code = sched::kEdgeCap;
      else if (__ballot_sync(FULL, gl && pv.gload[lane] > glim)) code = sched::kGroup;
    } else {
      el_lo = el_hi = 0;
    }
    const bool accepted = code == sched::kAccept;
    __syncwarp();
    if (lane == 0) clk[4] = (int)(clock64() - clk0);

    // ---- packing gate and permit, then the release (the state update below
    // does not touch anything the descriptor's dispatch reads)
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

    // ---- apply the accepted actions
    if (accepted && kept > 0) {
      lc_lo = cap_lo - el_lo;
      lc_hi = cap_hi - el_hi;
      gc = gl ? glim - pv.gload[lane] : 0;
      #pragma unroll 1
      for (int o0 = 0; o0 < revealed; o0 += 32) {
        const int o = o0 + lane;
        const int e = o < revealed ? act[o] : -1;
        if (e >= 0) {
          const int t = edge_tgt[e];
          uint32_t mt = meta[o];
          const uint32_t h = hold[o] | (1u << t);
          const int s = mt & 0xff, d = (mt >> 8) & 0xff;
          hold[o] = h;
          comm[o] |= 1ull << e;
          if (t == d && (mt & kMetaResidual)) {
            atomicAdd(reinterpret_cast<unsigned long long*>(&resdem[s * V + d]), ~0ULL);  // -1
            mt &= ~kMetaResidual;
            meta[o] = mt;
          }
          const int hp = hops_of(h, d);
          hops[o] = hp;
          vm[o] = vm_of(mt, h, hp);
        }
      }
    } else {
      lc_lo = cap_lo; lc_hi = cap_hi; gc = glim;
    }
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
    // ---- log
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
      L[15] = 2;  // packed-path marker
    }
    __syncwarp();
  }  // trigger loop

  // ---- the blob's state arrays, as the byte-per-entry path leaves them
  const long long staged = S[kStaged];
  int32_t* sources = reinterpret_cast<int32_t*>(at(kCtlSources));
  int32_t* destinations = reinterpret_cast<int32_t*>(at(kCtlDestinations));
  uint8_t* holders = at(kCtlHolders);
  uint8_t* ready = at(kCtlReady);
  uint8_t* committed = at(kCtlCommitted);
  uint8_t* residual = at(kCtlResidual);
  int32_t* rhops = reinterpret_cast<int32_t*>(at(kCtlRemainingHops));
  uint8_t* sel_scr = at(kCtlScratchSelected);
  uint8_t* seen = at(kCtlScratchSeen);
  #pragma unroll 1
  for (int o = lane; o < T; o += 32) {
    const bool st = o < staged;
    const uint32_t mt = meta[o], h = hold[o];
    const uint64_t cm = comm[o];
    sources[o] = st ? (int)(mt & 0xff) : -1;
    destinations[o] = st ? (int)((mt >> 8) & 0xff) : -1;
    ready[o] = (mt & kMetaReady) ? 1 : 0;
    residual[o] = (mt & kMetaResidual) ? 1 : 0;
    rhops[o] = hops[o];
    sel_scr[o] = 0;
    seen[o] = (pa_ok && act[o] >= 0) ? 1 : 0;
    #pragma unroll 1
    for (int v = 0; v < V; ++v) holders[(long long)o * V + v] = (h >> v) & 1u;
    #pragma unroll 1
    for (int e = 0; e < E; ++e) committed[(long long)o * E + e] = (cm >> e) & 1ull;
  }
  int64_t* lcred = reinterpret_cast<int64_t*>(at(kCtlLinkCredits));
  int64_t* gcred_arr = reinterpret_cast<int64_t*>(at(kCtlGroupCredits));
  int64_t* eload_arr = reinterpret_cast<int64_t*>(at(kCtlScratchEdgeLoad));
  if (elo) { lcred[lane] = lc_lo; eload_arr[lane] = el_lo; }
  if (ehi) { lcred[lane + 32] = lc_hi; eload_arr[lane + 32] = el_hi; }
  if (gl) gcred_arr[lane] = gc;
  __syncwarp();
}

}  // namespace ctl
}  // namespace raiccl
