// Persistent progressive front end of the MoE layer: router + device control
// plane + revealed-only dispatch in ONE cooperative launch per layer call.
//
// The one-launch-per-step pipeline (moe_router_kernel per chunk on a router
// stream, moe_control_*_kernel per trigger, moe_dispatch_kernel per
// descriptor, joined by events) pays a launch, a cross-stream hop and a cold
// instruction cache on every step, and the control kernel re-stages its state
// from global memory at every trigger.  Here the grid (one CTA per SM) stays
// resident for the whole front end:
//
//   CTA 0, warp 0 — the control plane (control_warp_packed.cuh, or
//       control_warp.cuh when the plan does not fit the packed path) for
//       triggers 0..n_desc-1.  Plan and scheduler state stay in shared memory
//       across triggers.  Before trigger q it waits (bounded) until the router
//       chunks q depends on are routed.  After it, it hands the decision to
//       warp 1, which turns the chunks' per-expert router counts into the
//       descriptor's receive bases and counts, writes the permit and releases
//       desc_ready[q] = epoch while warp 0 goes on with the next trigger.
//   CTAs 1..W — workers.  For each router chunk: route a share of its tokens
//       (groups of tokens per CTA, or one warp per token for more than 32
//       experts), add the per-expert counts, and add the routed units to
//       chunk_done[c] (a worker with no units in a chunk skips it).  A resident
//       batch is streamed into shared memory by bulk copies ahead of the routing
//       and routed chunk after chunk without interruption; a streamed batch is
//       routed as its chunks land, and while
//       a worker waits for the next chunk (early arm) it dispatches every
//       descriptor already released.  After the last chunk a worker dispatches
//       the rest, waiting (bounded) for each release.  In the delayed arm nothing is
//       dispatched before the final trigger.  Each worker packs and stores its
//       token share of a descriptor (dispatch_rows).  The last worker to finish
//       a descriptor publishes the counts and the per-destination ready words.
//
// All waits are between CTAs of this one launch, whose co-residency the
// cooperative launch guarantees, and every wait has a %globaltimer deadline
// after which the waiter records a status and returns.  Cross-GPU traffic is
// the same P2P stores and release words as the step kernels (no TMA).
// Decisions, rows, counts and flags are identical to the step pipeline's,
// which the layer tests check against each other.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdint>
#include <type_traits>

#include "control_warp.cuh"
#include "control_warp_packed.cuh"
#include "launchers.h"
#include "moe_device.cuh"
#include "router_tc.cuh"
#include "moe_kernels.h"
#include "sm100_ptx.cuh"

namespace raiccl {
namespace {

constexpr int kFrontThreads = 256;
constexpr int kFrontKernelId = 70;

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void trace_begin(TraceSlot* s) {
  if (s) atomicMin(&s->t_start, (unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void trace_end(TraceSlot* s) {
  if (s) {
    atomicMax(&s->t_end, (unsigned long long)globaltimer_ns());
    atomicAdd(&s->ctas, 1);
  }
}

// Per-CTA timeline (diagnostics): stamp k of this CTA, thread 0 only.
constexpr int kCtaClockSlots = 128;  // stamps per CTA in FrontendParams::cta_clock
__device__ __forceinline__ void cta_stamp(const FrontendParams& f, int k) {
  if (f.cta_clock != nullptr && threadIdx.x == 0) f.cta_clock[(long long)blockIdx.x * kCtaClockSlots + k] = globaltimer_ns();
}

// Routing work is dealt out over the workers as one sequence across chunks:
// unit u of chunk c (a token group, or a token for the warp-per-token router)
// goes to worker (units of chunks before c + u) mod n.  A chunk with fewer
// units than workers therefore leaves the next workers free for the next
// chunk, so consecutive chunks are routed side by side.  Returns this
// worker's first unit index in the chunk.
__device__ __forceinline__ int first_share(int worker, int units_before, int n) {
  const int g = worker - units_before % n;
  return g < 0 ? g + n : g;
}

// Units of a share that starts at unit `first` and takes every n-th of `units`.
__device__ __forceinline__ int share_count(int first, int units, int n) {
  return first < units ? (units - first + n - 1) / n : 0;
}

// Routing units of chunk c: token groups of `unit` tokens (1: single tokens).
// chunk_done[c] counts the units routed so far; the chunk is complete when it
// reaches this number.
__device__ __forceinline__ int chunk_units(const int* s_coff, int c, int unit) {
  return (s_coff[c + 1] - s_coff[c] + unit - 1) / unit;
}

__device__ __forceinline__ int trigger_first_chunk(int q, int P) { return q < P ? q : P; }
__device__ __forceinline__ int trigger_last_chunk(int q, int P, int C) { return q < P ? q : C - 1; }

__device__ __forceinline__ void st_release_cta_shared_s32(int* p, int v) {
  asm volatile("st.release.cta.shared.s32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta_shared_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

// Hand-off words from the control warp to the publisher warp, one per descriptor.
constexpr int kPubNone = 0, kPubPermitted = 1, kPubDenied = 2, kPubStop = 3;

// Control-warp hooks.  before(q): wait (bounded) for the router chunks trigger q
// needs, then, in one round trip, fetch the control-token destinations and the
// per-expert router counts of EVERY chunk complete by now into shared memory,
// so later triggers usually read no global memory.  after(q): hand the
// decision to the publisher warp (publish_descriptors), which writes the
// permit, the descriptor's receive bases and counts and releases it, so the
// release's memory fence is not on the control warp's chain of triggers.
struct FrontHooks {
  static constexpr bool kFetchesTokens = true;
  static constexpr bool kPublishesPermit = true;
  const FrontendParams* f;
  int workers, P, C, E;
  unsigned long long epoch;
  int* s_sent;         // [E] rows already assigned per expert (shared)
  int* s_dst;          // [C * cpc] control-token destinations (shared)
  const int* s_coff;   // [C + 1] chunk offsets (shared)
  int* s_ccount;       // [C * E] router counts per (chunk, expert) (shared)
  int cpc;
  int chunks_ready;    // chunks [0, chunks_ready) complete and fetched
  int unit;            // tokens per routing unit
  int* s_pub;          // [n_desc] hand-off words to the publisher warp (shared)

  __device__ bool before(int q) {
    const int lane = threadIdx.x & 31;
    const int need = trigger_last_chunk(q, P, C) + 1;
    if (chunks_ready >= need) {  // fetched with an earlier trigger: no global traffic
      if (lane == 0 && f->phase_trace) trace_begin(&f->phase_trace[C + q]);
      if (q < 16) cta_stamp(*f, 2 + 2 * q);
      return true;
    }
    int ok = 1;
    if (lane == 0) {
      const unsigned long long deadline = globaltimer_ns() + f->timeout_ns;
      #pragma unroll 1
      for (int c = chunks_ready; c < need && ok; ++c) {
        const int need_units = chunk_units(s_coff, c, unit);
        int got;
        #pragma unroll 1
        while ((got = ld_acquire_gpu_s32(&f->chunk_done[c])) < need_units) {
          if (globaltimer_ns() > deadline) {
            // index: the chunk; bound: how many of its routing units had been routed
            record_status(f->dp.status, kTimeoutChunkFlag, kFrontKernelId, c, got);
            ok = 0;
            break;
          }
        }
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return false;
    // every further chunk that is already complete (one parallel poll)
    int hi = need;
    #pragma unroll 1
    for (int base = need; base < C; base += 32) {
      const int c = base + lane;
      const bool done = c < C && ld_acquire_gpu_s32(&f->chunk_done[c]) >= chunk_units(s_coff, c, unit);
      const unsigned notdone = __ballot_sync(0xffffffffu, !done);
      const int run = notdone ? __ffs(notdone) - 1 : 32;
      hi = base + run;
      if (run < 32) break;
    }
    if (hi > C) hi = C;
    __threadfence();
    __syncwarp();
    const int lo = chunks_ready;
    const int nd = (hi - lo) * cpc, nt = nd + (hi - lo) * E;
    #pragma unroll 1
    for (int i = lane; i < nt; i += 32) {  // destinations and counts in one pass (loads overlap)
      if (i < nd) {
        const int c = lo + i / cpc, j = i % cpc;
        const int off = s_coff[c];
        const int size = s_coff[c + 1] - off;
        s_dst[c * cpc + j] = j < size ? f->cp.expert_ids[(long long)(off + j) * f->cp.top_k] % f->cp.ctl_nodes : -1;
      } else {
        s_ccount[lo * E + (i - nd)] = f->chunk_counts[(long long)lo * E + (i - nd)];
      }
    }
    chunks_ready = hi;
    __syncwarp();
    if (lane == 0 && f->phase_trace) trace_begin(&f->phase_trace[C + q]);
    if (q < 16) cta_stamp(*f, 2 + 2 * q);
    return true;
  }

  __device__ void after(int q, bool permitted) {
    const int lane = threadIdx.x & 31;
    if (q < 16) cta_stamp(*f, 3 + 2 * q);
    if (lane == 0) {
      if (f->phase_trace) trace_end(&f->phase_trace[C + q]);
      // the warp barrier before after() ordered every lane's shared-memory
      // writes (router counts fetched by before()); the release makes them
      // visible to the publisher warp with the decision
      st_release_cta_shared_s32(&s_pub[q], permitted ? kPubPermitted : kPubDenied);
    }
    __syncwarp();
  }
};

// Publisher warp of the control CTA: for each descriptor in order, wait
// (bounded) for the control warp's decision, then write the permit word, the
// descriptor's receive bases and per-expert counts, and release desc_ready[q].
// s_sent (rows already assigned per expert) is this warp's alone.
__device__ void publish_descriptors(const FrontendParams& f, int P, int C, int E, int n_desc, unsigned long long epoch,
                                    const int* s_pub, int* s_sent, const int* s_ccount) {
  const int lane = threadIdx.x & 31;
  #pragma unroll 1
  for (int q = 0; q < n_desc; ++q) {
    int st = kPubNone;
    if (lane == 0) {
      const uint64_t deadline = globaltimer_ns() + f.timeout_ns;
      #pragma unroll 1
      while ((st = ld_acquire_cta_shared_s32(&s_pub[q])) == kPubNone) {
        if (globaltimer_ns() > deadline) {
          record_status(f.dp.status, kTimeoutPermit, kFrontKernelId + 3, q, 0);
          st = kPubStop;
          break;
        }
      }
    }
    st = __shfl_sync(0xffffffffu, st, 0);
    __syncwarp();  // lane 0's acquire orders the other lanes' reads below
    if (st == kPubStop) return;
    const bool permitted = st == kPubPermitted;
    const int c_lo = trigger_first_chunk(q, P), c_hi = trigger_last_chunk(q, P, C);
    #pragma unroll 1
    for (int e = lane; e < E; e += 32) {
      int cnt = 0;
      #pragma unroll 1
      for (int c = c_lo; c <= c_hi; ++c) cnt += s_ccount[c * E + e];
      const int base = s_sent[e];
      f.disp_base[(long long)q * E + e] = base;
      f.dp.desc_counts[(long long)q * E + e] = permitted ? cnt : 0;
      if (permitted) s_sent[e] = base + cnt;
    }
    if (lane == 0) f.cp.permit[q] = permitted ? epoch : 0ULL;
    __syncwarp();
    // the warp barrier orders every lane's stores (permit, bases, counts)
    // before this release, which publishes them at gpu scope
    if (lane == 0) st_release_gpu_u64(&f.desc_ready[q], epoch);
    __syncwarp();
  }
}

// One worker's share of descriptor q (collective over the CTA).
template <typename T>
__device__ void worker_dispatch(const FrontendParams& f, int q, int w, int W, unsigned long long epoch,
                                int* hist, int* run, int* item_pos, int* s_base, const int* s_coff, int nc,
                                int* s_flag, bool streamed, bool indexed = false,
                                const DispatchStage* stage = nullptr, bool ids_ready = false) {
  const MoEDims& d = f.dp.dims;
  const int P = f.cp.partial_chunks, C = d.chunks, E = d.experts, k = d.top_k;
  const int t0 = s_coff[trigger_first_chunk(q, P)];
  const int t1 = s_coff[trigger_last_chunk(q, P, C) + 1];
  TraceSlot* slot = f.phase_trace ? &f.phase_trace[C + d.n_desc + q] : nullptr;
  if (threadIdx.x == 0) trace_begin(slot);
  cta_stamp(f, 24 + 2 * q);
  const int ntok = t1 - t0;
  const int per = (ntok + W - 1) / W;
  const int a = t0 + min(ntok, w * per);
  const int b = t0 + min(ntok, (w + 1) * per);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    if (!indexed) {
      hist[e] = 0;
      run[e] = 0;
    }
    s_base[e] = f.disp_base[(long long)q * E + e];
  }
  if (threadIdx.x == 0) *s_flag = (f.dp.permit[q] == epoch) ? 1 : 0;
  __syncthreads();
  const bool permitted = *s_flag != 0;
  if (!permitted && threadIdx.x == 0 && w == 0) record_status(f.dp.status, kTimeoutPermit, 20, q, (long long)epoch);
  if (permitted && (long long)(b - a) * k > kDispatchMaxItems) {
    if (threadIdx.x == 0) record_status(f.dp.status, kBadConfig, 22, (long long)(b - a) * k, kDispatchMaxItems);
  } else if (permitted && a < b) {
    // diagnostics: descriptor q's phases in stamps 68 + 4 q .. (q < 8)
    unsigned long long* dbg =
        (f.cta_clock != nullptr && q < 8) ? f.cta_clock + (long long)blockIdx.x * kCtaClockSlots + 68 + 4 * q : nullptr;
    dispatch_rows<T>(f.dp, t0, a, b, s_base, hist, run, item_pos, s_coff, nc, streamed, indexed, stage, dbg,
                     ids_ready);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atom_add_acq_rel_gpu(&f.dp.done_counter[q], 1);
    *s_flag = (prev == W - 1) ? 1 : 0;
  }
  __syncthreads();
  cta_stamp(f, 44 + q);
  if (*s_flag) dispatch_publish(f.dp, q, q == f.fault_skip_desc, epoch, false);
  if (threadIdx.x == 0) trace_end(slot);
  cta_stamp(f, 25 + 2 * q);
  __syncthreads();
}

// This worker's index part of descriptor q (dispatch_index), computed while
// the release is still pending; worker_dispatch(..., indexed = true) then
// only loads the bases and copies.  Collective over the CTA.
__device__ bool worker_index(const FrontendParams& f, int q, int w, int W, int* hist, int* run, int* item_pos,
                             const int* s_coff, const DispatchStage* stage) {
  const MoEDims& d = f.dp.dims;
  const int P = f.cp.partial_chunks, C = d.chunks, E = d.experts;
  const int t0 = s_coff[trigger_first_chunk(q, P)];
  const int t1 = s_coff[trigger_last_chunk(q, P, C) + 1];
  const int ntok = t1 - t0;
  const int per = (ntok + W - 1) / W;
  const int a = t0 + min(ntok, w * per);
  const int b = t0 + min(ntok, (w + 1) * per);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    hist[e] = 0;
    run[e] = 0;
  }
  __syncthreads();
  if (a < b && (long long)(b - a) * d.top_k <= kDispatchMaxItems) dispatch_index(f.dp, t0, a, b, hist, run, item_pos);
  __syncthreads();
  // the share's identity inputs too (staging memory is free once routing is done)
  return a < b && (long long)(b - a) * d.top_k <= kDispatchMaxItems && dispatch_stage_ids(f.dp, a, b, stage);
}

// Whether every router chunk of descriptor q is complete (all its routing
// units routed); a non-blocking poll, collective over the CTA.
__device__ bool chunks_complete(const FrontendParams& f, int q, const int* s_coff, int unit, int* s_flag) {
  const int P = f.cp.partial_chunks, C = f.dp.dims.chunks;
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int c = trigger_first_chunk(q, P); c <= trigger_last_chunk(q, P, C) && ok; ++c)
      ok = ld_acquire_gpu_s32(&f.chunk_done[c]) >= chunk_units(s_coff, c, unit) ? 1 : 0;
    if (ok) __threadfence();
    *s_flag = ok;
  }
  __syncthreads();
  const bool v = *s_flag != 0;
  __syncthreads();
  return v;
}

// Whether descriptor q was released: 1 yes, 0 not yet (non-blocking poll),
// -1 the bounded wait ran out (status recorded).  Collective over the CTA.
__device__ int wait_released(const FrontendParams& f, int q, unsigned long long epoch, int* s_flag, bool block) {
  if (threadIdx.x == 0) {
    int ok = ld_acquire_gpu_u64(&f.desc_ready[q]) == epoch ? 1 : 0;
    if (!ok && block) {
      const unsigned long long deadline = globaltimer_ns() + f.timeout_ns;
      while (ok == 0) {
        ok = ld_acquire_gpu_u64(&f.desc_ready[q]) == epoch ? 1 : 0;
        if (ok == 0 && globaltimer_ns() > deadline) {
          record_status(f.dp.status, kTimeoutPermit, kFrontKernelId + 1, q, (long long)epoch);
          ok = -1;
        }
      }
    }
    if (ok == 1) __threadfence();
    *s_flag = ok;
  }
  __syncthreads();
  const int v = *s_flag;
  __syncthreads();
  return v;
}

// Routing: a worker routes units of kUnitTokens consecutive tokens, one token
// per warp (router_token, up to EMAX experts), from the shared-memory ring
// (resident batch) or from global memory; the step pipeline's router kernel
// runs the same per-token code, so both route identically.  With the
// tensor-core router (bf16, f.tc_router) a unit is kTcRows tokens, one MMA
// tile (router_tc.cuh).
constexpr int kUnitTokens = 8;

template <typename T, int EMAX>
__global__ void __launch_bounds__(kFrontThreads, 1) moe_frontend_kernel(const __grid_constant__ FrontendParams f) {
  // tokens per routing unit (the control CTA counts chunk completion in the same units)
  const bool tc = std::is_same<T, __nv_bfloat16>::value && f.tc_router != 0;
  const int NT = tc ? kTcRows : kUnitTokens;
  extern __shared__ __align__(16) uint8_t fsm[];
  __shared__ int hist[kMaxExperts];
  __shared__ int run[kMaxExperts];
  __shared__ int s_base[kMaxExperts];
  __shared__ int item_pos[kDispatchMaxItems];
  __shared__ int s_coff[kDispatchMaxChunks + 1];
  __shared__ int s_flag;
  TraceScope trace_scope(f.trace);
  const MoEDims& d = f.dp.dims;
  const int C = d.chunks, E = d.experts, n_desc = d.n_desc;
  const int W = (int)gridDim.x - 1;  // worker CTAs
  const int w = (int)blockIdx.x - 1;  // this CTA's worker index
  const unsigned long long epoch = *f.dp.epoch;
  const int nc = min(C, kDispatchMaxChunks);
  for (int c = threadIdx.x; c <= nc; c += blockDim.x) s_coff[c] = f.dp.chunk_offsets[c];
  // the progressive expert planner (next launch) may start now: it waits on
  // the ready words itself (workers signal it once their TMEM columns, if
  // any, are allocated, so a dependent CTA never holds TMEM before them)
  if (f.early_dependents && blockIdx.x == 0) griddep_launch_dependents();

  if (blockIdx.x == 0) {
    // ---------------- control CTA
    __shared__ int s_dst[ctl::kCtlStageMax];
    __shared__ int s_ccoff[ctl::kCtlMaxChunks + 1];
    __shared__ uint32_t s_egmask[ctl::kWarpMaxE];
    __shared__ uint32_t s_vmc[ctl::kCtlStageMax];
    const ControlDims dims{f.cp.plan.E, f.cp.plan.G, f.cp.plan.V, f.cp.st.max_tokens, f.cp.n_group_members,
                           f.cp.n_edge_group_members, f.cp.n_tmpl, f.cp.max_cands, f.cp.chunks};
    const ControlLayout Lt = control_layout(dims);
    ctl::copy16(reinterpret_cast<uint4*>(fsm), reinterpret_cast<const uint4*>(f.cp.blob), Lt.state_end / 16);
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;  // s_sent of the hooks
    __syncthreads();
    // packed control path: template tables (whole CTA) and the edge -> group
    // masks; an edge that lists a group twice keeps the byte-per-entry path
    __shared__ int s_dup;
    const bool packed = f.ctl_packed_off > 0;
    ctl::PackedView pv = ctl::packed_view(fsm + f.ctl_packed_off, dims);
    if (packed) {
      ctl::build_packed_tables(fsm, dims, pv);
      if (threadIdx.x < 32)
        s_dup = ctl::edge_group_masks(reinterpret_cast<const int32_t*>(fsm + Lt.off[kCtlEdgeGroupPtr]),
                                      reinterpret_cast<const int32_t*>(fsm + Lt.off[kCtlEdgeGroupMembers]),
                                      dims.E, s_egmask);
      __syncthreads();
    }
    __shared__ int s_pub[ctl::kCtlMaxChunks];
    for (int q = threadIdx.x; q < ctl::kCtlMaxChunks; q += blockDim.x) s_pub[q] = kPubNone;
    __syncthreads();
    int* s_ccount = reinterpret_cast<int*>(fsm + ((Lt.total + 15) & ~15LL));
    if (threadIdx.x < 32) {
      FrontHooks hooks{&f, W, f.cp.partial_chunks, C, E, epoch, hist, s_dst, s_ccoff, s_ccount,
                       f.cp.ctl_per_chunk, 0, NT, s_pub};
      if (packed && !s_dup)
        ctl::control_warp_run_packed(f.cp, dims, fsm, s_dst, s_ccoff, s_egmask, pv, 0, n_desc, hooks);
      else
        ctl::control_warp_run(f.cp, dims, fsm, s_dst, s_ccoff, s_egmask, 0, n_desc, true, hooks, s_vmc);
      __syncwarp();
      // descriptors the control warp did not reach (a wait ran out) release nothing
      if (threadIdx.x == 0)
        for (int q = 0; q < n_desc; ++q)
          if (ld_acquire_cta_shared_s32(&s_pub[q]) == kPubNone) st_release_cta_shared_s32(&s_pub[q], kPubStop);
    } else if (threadIdx.x < 64) {
      publish_descriptors(f, f.cp.partial_chunks, C, E, n_desc, epoch, s_pub, hist, s_ccount);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) f.dp.sent_base[e] = hist[e];
    ctl::copy16(reinterpret_cast<uint4*>(f.cp.blob + Lt.state_begin),
                reinterpret_cast<const uint4*>(fsm + Lt.state_begin), (Lt.state_end - Lt.state_begin) / 16);
    return;
  }

  // ---------------- worker CTAs
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // workers [0, Wd) dispatch; the others only route and then leave
  const int Wd = f.dispatch_ctas > 0 ? min(W, f.dispatch_ctas) : W;
  const bool dispatcher = w < Wd;
  // router weights: a shared-memory copy when the launch made room for one
  const bool w_smem = f.w_off > 0;
  const T* wts = w_smem ? reinterpret_cast<const T*>(fsm + f.w_off) : (const T*)f.rp.weight;
  __shared__ __align__(8) uint64_t s_wbar;
  // the per-chunk router bias rows in shared memory (behind the blob area)
  float* s_cbias = reinterpret_cast<float*>(fsm);
  if (f.rp.chunk_bias)
    for (int i = threadIdx.x; i < C * E; i += blockDim.x) s_cbias[i] = f.rp.chunk_bias[i];
  // inputs resident at launch (not streamed in by the copy engine during this call)
  const unsigned long long ready_all = f.tok_ready == nullptr ? ~0ULL : ld_acquire_gpu_u64(f.tok_ready_all);
  const bool resident = ready_all >= epoch;
  if (f.cta_clock != nullptr && threadIdx.x == 0) {  // diagnostics: what this CTA saw at its start
    unsigned int smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    unsigned long long* row = f.cta_clock + (long long)blockIdx.x * kCtaClockSlots;
    row[18] = smid;
    row[19] = ready_all;
    row[20] = epoch;
  }
  const int row_bytes = f.rp.hidden * (int)sizeof(T);
  // bulk-copy ring (resident batch): this worker's routing units stream into
  // shared memory ring_slots units ahead of the routing
  constexpr int kRingMax = 8;
  __shared__ __align__(8) uint64_t s_rbar[kRingMax];
  const bool ring = resident && f.ring_slots >= 2 && f.ring_slots <= kRingMax;
  const int R = ring ? f.ring_slots : 1;
  const long long unit_bytes = (long long)NT * row_bytes;
  uint8_t* ring_base = fsm + f.ring_off;
  int pc = 0, pg = 0, pcum = 0;          // producer (thread 0): next group to copy, chunk / group / units before
  long long issued = 0, consumed = 0;    // groups copied / routed
  auto unit_norm = [&]() {
    #pragma unroll 1
    while (pc < C) {
      const int ng = chunk_units(s_coff, pc, NT);
      if (pg < ng) return;
      pcum += ng;
      if (++pc < C) pg = first_share(w, pcum, W);
    }
  };
  auto issue_next = [&]() {  // thread 0: copy the next group into its slot
    if (pc >= C) return;
    const int slot = (int)(issued % R);
    const int tf = s_coff[pc] + pg * NT, nt = min(NT, s_coff[pc + 1] - tf);
    const uint32_t bytes = (uint32_t)((long long)nt * row_bytes);
    mbar_arrive_expect_tx(&s_rbar[slot], bytes);
    bulk_load_g2s(ring_base + slot * unit_bytes, (const char*)f.rp.tokens + (long long)tf * row_bytes, bytes,
                  &s_rbar[slot]);
    ++issued;
    pg += W;
    unit_norm();
  };
  // dispatch staging: the ring's memory, free once routing is done (or never
  // used by a streamed batch), holds the rows of a dispatch share
  __shared__ __align__(8) uint64_t s_dbar[2];
  __shared__ uint32_t s_duses[2];
  // tensor-core router: stages at the first 1024-byte boundary of the ring memory
  uint8_t* tc_base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ring_base) + 1023) & ~(uintptr_t)1023);
  const DispatchStage dstage{tc ? tc_base : ring_base, f.ring_bytes, s_dbar, s_duses, f.timeout_ns};
  const DispatchStage* stage = f.ring_bytes > 0 ? &dstage : nullptr;
  __shared__ __align__(8) uint64_t s_tcbar[2 * kTcMaxStages + 1];
  __shared__ uint32_t s_tmem;
  TcRouter tcr{};
  if (tc) {
    tcr.stages = tc_base;
    tcr.npad = f.tc_npad;
    tcr.n_stages = f.tc_stages;
    tcr.kblocks = f.rp.hidden / kTcBK;
    tcr.lg = reinterpret_cast<float*>(tc_base + (long long)f.tc_stages * tcr.stage_bytes());
    tcr.sel = tcr.lg + f.tc_npad * kTcRows;  // 8-byte aligned: npad * kTcRows words is even
    tcr.full = s_tcbar;
    tcr.empty = s_tcbar + kTcMaxStages;
    tcr.done = s_tcbar + 2 * kTcMaxStages;
    if (threadIdx.x == 0) {
      for (int i = 0; i < f.tc_stages; ++i) {
        mbar_init(&tcr.full[i], 1);
        mbar_init(&tcr.empty[i], 1);
      }
      mbar_init(tcr.done, 1);
      fence_mbarrier_init();
      tma_prefetch_desc(&f.tmap_x);
      tma_prefetch_desc(&f.tmap_w);
    }
    // the accumulator's TMEM columns (a power of two >= 32), held while routing
    if (warp == 4) {
      tmem_alloc(&s_tmem, f.tc_npad <= 32 ? 32u : 64u);
      tmem_relinquish();
    }
    tc_fence_before_sync();
  }
  if (threadIdx.x == 0) {
    mbar_init(&s_dbar[0], 1);
    mbar_init(&s_dbar[1], 1);
    s_duses[0] = s_duses[1] = 0;
    fence_mbarrier_init();
  }
  __syncthreads();  // the chunk offsets in shared memory are complete before thread 0 walks them
  if (w_smem && threadIdx.x == 0) {  // weights first: every routing unit needs them
    mbar_init(&s_wbar, 1);
    fence_mbarrier_init();
    fence_proxy_async_smem();
    const uint32_t wb = (uint32_t)((long long)E * row_bytes);
    mbar_arrive_expect_tx(&s_wbar, wb);
    bulk_load_g2s(fsm + f.w_off, f.rp.weight, wb, &s_wbar);
  }
  if (ring && threadIdx.x == 0) {
    for (int i = 0; i < R; ++i) mbar_init(&s_rbar[i], 1);
    fence_mbarrier_init();
    fence_proxy_async_smem();
    pg = first_share(w, 0, W);
    unit_norm();
    for (int i = 0; i < R; ++i) issue_next();
  }
  cta_stamp(f, 0);
  __syncthreads();
  if (tc) {
    tc_fence_after_sync();
    tcr.tmem = s_tmem;
  }
  if (f.early_dependents) griddep_launch_dependents();
  cta_stamp(f, 1);
  // Descriptors this worker dispatches.  When every partial descriptor can
  // have workers of its own, the partial descriptors get disjoint worker
  // groups (in proportion to their tokens), so released descriptors are
  // dispatched side by side, and the workers of every group but the last then
  // also take a share of the final descriptor, the one the layer waits for
  // after the last trigger (the last partial descriptor is released just
  // before it, so its group is still busy when the final one is released).
  // Otherwise every worker takes a share of every descriptor in turn.
  const bool grouped = f.dispatch_groups && n_desc >= 2 && n_desc - 1 <= Wd && dispatcher;
  int qa = 0, wia = w, wna = Wd;  // grouped: this worker's partial descriptor, its index and group size
  int fin_n = Wd;                 // grouped: workers [0, fin_n) share the final descriptor
  if (grouped) {
    const int P = f.cp.partial_chunks;
    const int np = n_desc - 1;
    const long long total = s_coff[trigger_first_chunk(np, P)] - s_coff[0];
    long long cum = 0;
    int lo = 0;
    for (int q = 0; q < np; ++q) {
      cum += s_coff[trigger_last_chunk(q, P, C) + 1] - s_coff[trigger_first_chunk(q, P)];
      int hi = total > 0 ? (int)((long long)Wd * cum / total) : lo + 1;
      hi = max(hi, lo + 1);
      hi = min(hi, Wd - (np - 1 - q));
      if (q == np - 1) {
        hi = Wd;
        if (np >= 2 && lo >= 1) fin_n = lo;
      }
      if (w >= lo && w < hi) { qa = q; wia = w - lo; wna = hi - lo; }
      lo = hi;
    }
  }
  // cursor over this worker's descriptors: the descriptor, the worker's share
  // index in it and the number of workers sharing it (n_desc: no more)
  int k_cur = 0;
  auto cq = [&]() {
    return grouped ? (k_cur == 0 ? qa : k_cur == 1 && w < fin_n ? n_desc - 1 : n_desc) : k_cur;
  };
  auto cwi = [&]() { return grouped && k_cur == 0 ? wia : w; };
  auto cwn = [&]() { return grouped ? (k_cur == 0 ? wna : fin_n) : Wd; };
  int cum_units = 0;  // routing units (token groups, or tokens) of the chunks before c
  bool w_wait = w_smem;  // the weights' copy has not been waited for yet
  for (int c = 0; c < C; ++c) {
    // this worker's routing units in chunk c (token groups, or tokens over its warps)
    const int my_units = share_count(first_share(w, cum_units, W), chunk_units(s_coff, c, NT), W);
    if (resident && my_units == 0) {  // nothing to route or to report for this chunk
      if (c < 8) { cta_stamp(f, 2 + 2 * c); cta_stamp(f, 52 + c); cta_stamp(f, 3 + 2 * c); }
      cum_units += chunk_units(s_coff, c, NT);
      continue;
    }
    TraceSlot* rslot = f.phase_trace ? &f.phase_trace[c] : nullptr;
    if (threadIdx.x == 0) trace_begin(rslot);
    if (c < 8) cta_stamp(f, 2 + 2 * c);
    // early arm: this chunk's poll of the next release is a relaxed load issued
    // before the routing work and read after it (a fence makes it an acquire
    // when it saw the release)
    unsigned long long early_v = 0;
    if (threadIdx.x == 0 && !f.delayed && cq() < n_desc) early_v = ld_relaxed_gpu_u64(&f.desc_ready[cq()]);
    for (int e = threadIdx.x; e < E; e += blockDim.x) run[e] = 0;  // per-chunk expert counts
    if (!resident) {
      // streamed: wait for this chunk's rows; early arm: dispatch every
      // descriptor the control warp releases meanwhile
      const unsigned long long deadline = globaltimer_ns() + f.timeout_ns;
      for (;;) {
        if (threadIdx.x == 0) {
          int st = 0;
          while (st == 0) {
            if (ld_acquire_sys_u64(reinterpret_cast<const uint64_t*>(&f.tok_ready[c])) >= epoch ||
                ld_acquire_sys_u64(reinterpret_cast<const uint64_t*>(f.tok_ready_all)) >= epoch) {
              st = 1;
            } else if (dispatcher && !f.delayed && cq() < n_desc &&
                       ld_relaxed_gpu_u64(&f.desc_ready[cq()]) == epoch) {
              __threadfence();  // acquire the release seen by the relaxed poll
              st = 2;
            } else if (globaltimer_ns() > deadline) {
              record_status(f.dp.status, kTimeoutInput, kFrontKernelId, c, (long long)epoch);
              st = 1;  // route what is there; the status fails the call
            } else {
              __nanosleep(100);
            }
          }
          s_flag = st;
        }
        __syncthreads();
        const int st = s_flag;
        __syncthreads();
        if (st == 1) break;
        worker_dispatch<T>(f, cq(), cwi(), cwn(), epoch, hist, run, item_pos, s_base, s_coff, nc, &s_flag, true, false,
                           stage);
        ++k_cur;
      }
      if (threadIdx.x == 0 && !f.delayed && cq() < n_desc) early_v = ld_relaxed_gpu_u64(&f.desc_ready[cq()]);
      for (int e = threadIdx.x; e < E; e += blockDim.x) run[e] = 0;  // worker_dispatch used it
    }
    __syncthreads();
    const float* cbias = f.rp.chunk_bias ? s_cbias + (long long)c * E : nullptr;
    const int t0 = s_coff[c], t1 = s_coff[c + 1];
    // streamed batches: the workers digest the rows they route (feature digest
    // + checksum base); a resident batch had them computed when it was loaded
    const bool digest = !resident && f.digest_out != nullptr;
    const int ngroups = chunk_units(s_coff, c, NT);
    for (int g = first_share(w, cum_units, W); g < ngroups; g += W) {
      const int tf = t0 + g * NT, nt = min(NT, t1 - tf);
      if (tc) {
        // tensor-core unit: thread 128 (warp 4) issues the loads and MMAs,
        // then two threads finish each token; diagnostics of the first two units
        // in stamps 40.. and 64.. (issue, MMAs done, finish, barrier)
        unsigned long long* tdbg = (f.cta_clock != nullptr && tcr.n_units < 2)
                                       ? f.cta_clock + (long long)blockIdx.x * kCtaClockSlots +
                                             (tcr.n_units == 0 ? 40 : 64)
                                       : nullptr;
        if (tdbg != nullptr && threadIdx.x == 0) tdbg[0] = globaltimer_ns();
        if (threadIdx.x == 128)
          tc_router_issue(tcr, &f.tmap_x, &f.tmap_w, tf, f.dp.status, kFrontKernelId + 5, f.timeout_ns);
        tc_router_finish<EMAX>(f.rp, cbias, tcr, tf, nt, run, f.dp.status, kFrontKernelId + 5, f.timeout_ns,
                               tdbg != nullptr ? tdbg + 1 : nullptr);
        if (tdbg != nullptr && threadIdx.x == 0) tdbg[2] = globaltimer_ns();
        tc_fence_before_sync();
        __syncthreads();
        tc_fence_after_sync();
        ++tcr.n_units;
        if (digest) {  // streamed rows: feature digest and checksum base, one warp per token
          for (int i = warp; i < nt; i += kFrontThreads / 32) {
            const int t = tf + i;
            const long long dg =
                warp_row_digest((const uint4*)((const T*)f.rp.tokens + (long long)t * f.rp.hidden), row_bytes / 16);
            if (lane == 0) {
              f.digest_out[t] = dg;
              f.csbase_out[t] = token_checksum_base(f.dp.token_ids[t], f.dp.dims.rank, c, t - t0, t, dg);
            }
          }
          __syncthreads();
        }
        if (tdbg != nullptr && threadIdx.x == 0) tdbg[3] = globaltimer_ns();
        continue;
      }
      const T* srows = nullptr;
      if (ring) {
        const int slot = (int)(consumed % R);
        // a wait that runs out records the status (the call fails) and routes what is there
        mbar_wait_bounded(&s_rbar[slot], (uint32_t)((consumed / R) & 1), f.dp.status, kFrontKernelId + 2,
                          f.timeout_ns);
        srows = reinterpret_cast<const T*>(ring_base + slot * unit_bytes);
        if (consumed == 0) cta_stamp(f, 21);  // first unit in shared memory
      }
      // diagnostics: the first two units' phases (landed, warp 0's products,
      // its finish, the CTA barrier) in stamps 40.. and 64..
      unsigned long long* udbg = (f.cta_clock != nullptr && consumed < 2)
                                     ? f.cta_clock + (long long)blockIdx.x * kCtaClockSlots + (consumed == 0 ? 40 : 64)
                                     : nullptr;
      if (udbg != nullptr && threadIdx.x == 0) udbg[0] = globaltimer_ns();
      if (w_wait) {  // the weights' copy, once (a wait that runs out fails the call)
        mbar_wait_bounded(&s_wbar, 0, f.dp.status, kFrontKernelId + 4, f.timeout_ns);
        w_wait = false;
      }
      if (warp < nt) {  // token tf + warp, one warp each
        const int t = tf + warp;
        const T* x = srows ? srows + (long long)warp * f.rp.hidden : (const T*)f.rp.tokens + (long long)t * f.rp.hidden;
        unsigned long long* tdbg = (udbg != nullptr && warp == 0) ? udbg + 1 : nullptr;
        if (w_smem) router_token<T, EMAX, true>(f.rp, cbias, t, x, srows != nullptr, wts, run, tdbg);
        else router_token<T, EMAX, false>(f.rp, cbias, t, x, srows != nullptr, wts, run, tdbg);
        if (digest) {
          const long long dg = warp_row_digest((const uint4*)x, row_bytes / 16);
          if (lane == 0) {
            f.digest_out[t] = dg;
            f.csbase_out[t] = token_checksum_base(f.dp.token_ids[t], f.dp.dims.rank, c, t - t0, t, dg);
          }
        }
      }
      __syncthreads();  // every warp is done with the unit's rows
      if (udbg != nullptr && threadIdx.x == 0) udbg[3] = globaltimer_ns();
      if (ring) {
        if (consumed == 0) cta_stamp(f, 22);  // first unit routed
        if (threadIdx.x == 0) issue_next();
        ++consumed;
      }
    }
    cum_units += ngroups;
    if (c < 8) cta_stamp(f, 52 + c);
    __syncthreads();
    if (c < 4) cta_stamp(f, 60 + c);
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (run[e]) atomicAdd(&f.chunk_counts[(long long)c * E + e], run[e]);
    __syncthreads();
    if (threadIdx.x == 0) {
      // the CTA barrier above ordered every thread's expert ids, gates and
      // counts before this release
      if (my_units > 0) red_add_release_gpu(&f.chunk_done[c], my_units);
      trace_end(rslot);
    }
    if (c < 8) cta_stamp(f, 3 + 2 * c);
    // early arm, streamed batch: dispatch every descriptor already released
    // (never waits).  A resident batch routes every chunk first: routing is
    // then a few microseconds per chunk and the scheduler chain, which needs
    // each chunk, is not held back by dispatch work queued between chunks.
    if (dispatcher && !f.delayed && !resident) {
      if (threadIdx.x == 0) {
        if (early_v == epoch) __threadfence();
        s_flag = early_v == epoch ? 1 : 0;
      }
      __syncthreads();
      bool ready = s_flag == 1;
      __syncthreads();
      while (cq() < n_desc && ready) {
        worker_dispatch<T>(f, cq(), cwi(), cwn(), epoch, hist, run, item_pos, s_base, s_coff, nc, &s_flag, !resident,
                           false, stage);
        ++k_cur;
        ready = cq() < n_desc && wait_released(f, cq(), epoch, &s_flag, false) == 1;
      }
    }
  }
  if (ring && threadIdx.x == 0) {
    // every copy issued was routed; after a failed wait, let any copy still in
    // flight land before the CTA moves on (bounded)
    #pragma unroll 1
    for (; consumed < issued; ++consumed)
      mbar_wait_bounded(&s_rbar[(int)(consumed % R)], (uint32_t)((consumed / R) & 1), f.dp.status,
                        kFrontKernelId + 2, f.timeout_ns);
  }
  // a worker that routed nothing still lets the weights' copy land before
  // its shared memory is reused or released
  if (w_wait) mbar_wait_bounded(&s_wbar, 0, f.dp.status, kFrontKernelId + 4, f.timeout_ns);
  if (tc) {  // every unit's MMAs completed and were read: give the TMEM columns back
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    if (warp == 4) tmem_dealloc(tcr.tmem, f.tc_npad <= 32 ? 32u : 64u);
  }
  if (!dispatcher) return;  // routing done: this SM is free for the expert side
  if (f.delayed && wait_released(f, n_desc - 1, epoch, &s_flag, true) != 1) return;
  int n_indexed = 0;  // descriptors whose index part ran before their release (diagnostics)
  while (cq() < n_desc) {
    const int next = cq();
    // a descriptor not yet released whose chunks are routed: compute its
    // index part (prefix counts and ranks, from the expert ids only) while
    // the control warp works, so the release is followed by the copy alone
    const int rel = wait_released(f, next, epoch, &s_flag, false);
    bool indexed = false, ids_ready = false;
    if (rel == 0 && chunks_complete(f, next, s_coff, NT, &s_flag)) {
      ids_ready = worker_index(f, next, cwi(), cwn(), hist, run, item_pos, s_coff, stage);
      indexed = true;
      ++n_indexed;
    }
    if (rel != 1 && wait_released(f, next, epoch, &s_flag, true) != 1) return;
    worker_dispatch<T>(f, next, cwi(), cwn(), epoch, hist, run, item_pos, s_base, s_coff, nc, &s_flag, !resident,
                       indexed, stage, ids_ready);
    ++k_cur;
  }
  if (f.cta_clock != nullptr && threadIdx.x == 0) f.cta_clock[(long long)blockIdx.x * kCtaClockSlots + 23] = 1 + n_indexed;
}

template <typename T, int EMAX>
bool launch_one_frontend(const FrontendParams& f, int sms, size_t smem, cudaStream_t s) {
  auto kern = moe_frontend_kernel<T, EMAX>;
  static size_t configured = 0;
  if (smem > configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return false;
    configured = smem;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFrontThreads, smem) != cudaSuccess ||
      per_sm < 1)
    return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kFrontThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, f) == cudaSuccess;
}

}  // namespace

bool launch_frontend(const FrontendParams& f, bool bf16, int sms, cudaStream_t s, int* tc_used) {
  const int E = f.rp.experts;
  if (sms < 2 || !control_warp_path_ok(f.cp) || E > 64 || f.rp.top_k > 8 || f.dp.dims.chunks > kDispatchMaxChunks ||
      (f.rp.hidden * (bf16 ? 2 : 4)) % 16 != 0)
    return false;
  // dynamic shared memory: the control blob (CTA 0); the workers' per-chunk
  // bias rows and then the ring of routing units (two to eight units of
  // kUnitTokens rows within kRingBudget bytes)
  const size_t cwords = (size_t)f.dp.dims.chunks * f.dp.dims.experts * sizeof(int);
  FrontendParams g = f;
  // Workers: [bias rows][router weights, when they fit][ring].  The weights
  // (at most kWeightBudget bytes) come out of the ring's share of
  // kSmemBudget, as long as the ring keeps two slots; kSmemBudget leaves room
  // for the kernel's static shared memory (about 31 KB) under the 227 KB limit.
  const size_t w_bytes = (size_t)E * f.rp.hidden * (bf16 ? 2 : 4);
  constexpr size_t kSmemBudget = 196 * 1024, kWeightBudget = 64 * 1024, kRingMaxBudget = 160 * 1024;
  const size_t w_off = (cwords + 127) & ~(size_t)127;
  const size_t unit = (size_t)kUnitTokens * f.rp.hidden * (bf16 ? 2 : 4);
  auto ring_slots_from = [&](size_t off) {
    const size_t budget = off < kSmemBudget ? std::min(kRingMaxBudget, kSmemBudget - off) : 0;
    const int n = (int)std::min<size_t>(8, budget / unit);
    return n >= 2 ? n : 0;
  };
  const size_t w_end = (w_off + w_bytes + 127) & ~(size_t)127;
  const bool w_smem = f.ring_slots != 0 && f.w_off != 0 && w_bytes <= kWeightBudget && ring_slots_from(w_end) > 0;
  const size_t ring_off = w_smem ? w_end : w_off;
  g.ring_slots = f.ring_slots ? ring_slots_from(ring_off) : 0;
  g.ring_off = (int)ring_off;
  g.w_off = w_smem ? (int)w_off : 0;
  g.ring_bytes = g.ring_slots * (int)unit;
  size_t worker_bytes = g.ring_slots ? ring_off + g.ring_slots * unit : cwords;
  // Tensor-core router (bf16): TMA stages in place of the ring and the weight
  // copy, at a 1024-byte boundary, then the finish's logit scratch.
  g.tc_router = 0;
  if (bf16 && f.tc_router && f.rp.hidden % kTcBK == 0 && f.rp.top_k <= kTcSelStride) {
    const int npad = std::max(16, (E + 15) / 16 * 16);
    const size_t stage = (size_t)kTcRows * 128 + (size_t)npad * 128;
    const size_t sel = (size_t)tc_router_scratch_bytes(npad);
    const size_t avail = kSmemBudget > w_off + 1024 + sel ? kSmemBudget - w_off - 1024 - sel : 0;
    const int stages = (int)std::min<size_t>(kTcMaxStages, avail / stage);
    if (stages >= 2) {
      g.tc_router = 1;
      g.tc_stages = stages;
      g.tc_npad = npad;
      g.ring_slots = 0;
      g.w_off = 0;
      g.ring_off = (int)w_off;
      g.ring_bytes = (int)(stages * stage);
      worker_bytes = w_off + 1024 + stages * stage + sel;
    }
  }
  // control CTA: blob, per-(chunk, expert) router counts, then the packed
  // control path's tables and per-ordinal words when the plan fits it
  const size_t ctl_base = ((control_smem_bytes(f.cp) + 15) & ~(size_t)15) + ((cwords + 15) & ~(size_t)15);
  const ControlDims cd = control_dims(f.cp);
  g.ctl_packed_off = ctl::packed_path_ok(cd) ? (int)ctl_base : 0;
  const size_t ctl_bytes = ctl_base + (g.ctl_packed_off ? (size_t)ctl::packed_smem_bytes(cd) : 0);
  const size_t smem = std::max(ctl_bytes, worker_bytes);
  if (tc_used != nullptr) *tc_used = g.tc_router;
  if (E <= 8) return bf16 ? launch_one_frontend<__nv_bfloat16, 8>(g, sms, smem, s)
                          : launch_one_frontend<float, 8>(g, sms, smem, s);
  if (E <= 16) return bf16 ? launch_one_frontend<__nv_bfloat16, 16>(g, sms, smem, s)
                           : launch_one_frontend<float, 16>(g, sms, smem, s);
  return bf16 ? launch_one_frontend<__nv_bfloat16, 64>(g, sms, smem, s) : launch_one_frontend<float, 64>(g, sms, smem, s);
}

}  // namespace raiccl
