// Launch parameter records of the MoE data-plane and control-plane kernels
// (plain data shared by the host bindings and the .cu launch units).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "moe_layout.h"
#include "control_layout.h"
#include "sched_core.h"
#include "types.h"

namespace raiccl {

struct RouterParams {
  const void* tokens;       // [T, D] fp32 or bf16
  const void* weight;       // [E, D] same dtype
  const float* bias;        // [E]
  const float* chunk_bias;  // [E] additive bias of this chunk, or nullptr
  const uint8_t* block_mask;  // [E] 1 = this rank may not route there, or nullptr
  int row0, row1;           // rows routed by this launch (one router chunk)
  int hidden, experts, top_k, gate_mode, mask_mode, pad;
  int32_t* expert_ids;      // [T, k]
  float* gates;             // [T, k]
  TraceSlot* trace;
};

struct DispatchParams {
  MoEDims dims;
  SymLayout layout;
  PeerBases peers;
  const void* tokens;
  const int32_t* expert_ids;
  const float* gates;
  const long long* token_ids;
  const long long* feat_digest;
  const long long* checksum_base;
  const int32_t* chunk_offsets;
  int desc, t0, t1;
  int fault_skip_signal;    // test hook set by the host: 1 = publish no ready flag for this descriptor
  int32_t* sent_base;       // [E] rows already sent to (e, this rank) in earlier descriptors
  int32_t* desc_counts;     // [n_desc, E]
  int32_t* done_counter;    // [n_desc]
  const unsigned long long* permit;  // [n_desc] == epoch when the guard committed the descriptor
  const unsigned long long* epoch;   // device word holding this call's sequence number
  DeviceStatus* status;
  TraceSlot* trace;
  unsigned long long* peer_counters;  // [world][kPeerCounterFields] or nullptr
};

struct PlanParams {
  MoEDims dims;
  SymLayout layout;
  PeerBases peers;
  GemmSegment* segs;        // [E_slot * W]
  int32_t* rows_out;        // [E_slot * W]
  const unsigned long long* epoch;
  unsigned long long timeout_ns;
  DeviceStatus* status;
  TraceSlot* trace;
  // Optional GEMM tile tables ([E_slot * W + 1] each): prefix[s] counts the
  // tiles of segments < s, a segment holding ceil(rows / bm) * nblocks tiles.
  // Both are skipped when prefix1 is null.
  int32_t* prefix1;
  int32_t* prefix2;
  int nblocks1, nblocks2;
  int bm1, bm2;
  // Swapped tail tiles (CTA-pair GEMMs at BN = 256): when swap1 > 0, a
  // segment's last 256-row tile of at most swap1 rows is left out of prefix1
  // and counted in tail1 instead (nblocks1 tiles); likewise swap2 / tail2.
  int32_t* tail1;
  int32_t* tail2;
  int swap1, swap2;
  unsigned long long* peer_counters;  // [world][kPeerCounterFields] or nullptr
  // Progressive planning (launch_expert_plan_progressive): GEMM-1's tiles in
  // arrival order, published descriptor by descriptor in tile_word.
  int32_t* tile_list;               // [max_tiles1][4]
  unsigned long long* tile_word;
  int max_tiles1;
};

struct ReturnMetaParams {
  MoEDims dims;
  SymLayout layout;
  PeerBases peers;
  const GemmSegment* segs;
  DeviceStatus* status;
  TraceSlot* trace;
  // Optional return-signal handoff (see CombineParams::ret_sync): when set,
  // the grid's last CTA reports the metadata part done.
  const unsigned long long* epoch;
  unsigned long long* ret_sync;
};

struct CombineParams {
  MoEDims dims;
  SymLayout layout;
  PeerBases peers;
  void* out;                // [T, Dout]
  const unsigned long long* epoch;
  unsigned long long timeout_ns;
  DeviceStatus* status;
  TraceSlot* trace;
  // Return-signal handoff words, zero at creation and only ever increased:
  // [0] the epoch of the last call whose combine elected its reporting CTA,
  // [1] return parts reported (two per call: the metadata grid and the
  //     combine, which follows GEMM-2 in stream order), [2] metadata CTAs
  //     finished.  The second part of a call to report publishes this rank's
  //     return signal, so neither part waits for the other.  Null: the
  //     combine publishes the signal itself.
  unsigned long long* ret_sync;
};

struct BarrierParams {
  MoEDims dims;
  SymLayout layout;
  PeerBases peers;
  unsigned long long* counter;  // this rank's barrier sequence (device word)
  unsigned long long timeout_ns;
  DeviceStatus* status;
  TraceSlot* trace;
};

// Device-resident compiled-scheduler control plane (one CTA).
struct ControlParams {
  // Working set as one blob laid out by control_layout(); plan/st below are
  // typed views of the same memory (the kernel stages the blob instead).
  uint8_t* blob;
  sched::PlanView plan;
  sched::StateView st;
  const int32_t* expert_ids;   // [T, k]
  const int32_t* chunk_offsets;  // [C + 1]
  int top_k, chunks, partial_chunks, desc;
  int ctl_per_chunk, ctl_nodes, max_cands, log_stride;
  int n_group_members, n_edge_group_members, n_tmpl, max_tmpl;  // max_tmpl: templates per destination
  int force_serial;  // 1: always the CTA control kernel (the single-warp one otherwise, where it fits)
  // scalars kept across triggers of one layer call:
  // [0] staged_count [1] revealed_count [2] state_version [3] completed bitmap
  // [4] revealed bitmap [5] dispatched bitmap [6] future_access [7] unrevealed_execution
  // [8] duplicate_dispatch [9] stale_dispatch [10] pending bitmap [11..11+C) chunk starts
  // [11+C..11+2C) chunk counts
  long long* scalars;
  sched::Cand* cand_buf;       // [max_cands]
  int* keep_buf;               // [max_cands]
  int64_t* action_buf;         // [2 * max_tokens]
  int* log;                    // [n_desc, log_stride]
  unsigned long long* permit;  // [n_desc]
  const unsigned long long* epoch;
  DeviceStatus* status;
  TraceSlot* trace;
};

// Persistent progressive front end (one cooperative launch per layer call):
// CTA 0's first warp runs the control plane for every trigger, keeping the
// compiled plan and scheduler state in shared memory; every other CTA routes
// its share of each router chunk and, as descriptors are released, packs and
// stores its share of their rows into the owners' receive regions.
struct FrontendParams {
  RouterParams rp;          // rp.chunk_bias: [C, E] base (row c per chunk) or nullptr
  ControlParams cp;
  DispatchParams dp;        // desc / t0 / t1 / fault_skip_signal are set per descriptor
  int* chunk_done;          // [C] routing units (token groups or tokens) of chunk c routed so far (zeroed per call)
  int* chunk_counts;        // [C, E] router assignments per (chunk, expert) (zeroed per call)
  int* disp_base;           // [n_desc, E] first receive row of (descriptor, expert)
  unsigned long long* desc_ready;  // [n_desc] == epoch once the control warp released q
  int delayed;              // 1: dispatch only after the final trigger
  int fault_skip_desc;      // test hook: descriptor whose ready flags are withheld (-1: none)
  unsigned long long timeout_ns;
  TraceSlot* phase_trace;   // [C + 2 n_desc]: router c, control q, dispatch q; or nullptr
  TraceSlot* trace;         // the launch
  unsigned long long* cta_clock;  // [grid, 128] per-CTA %globaltimer stamps (diagnostics), or nullptr
  // Per-token feature digests and checksum bases written by the workers while
  // they route (null: precomputed by the digest / checksum-base kernels).
  long long* digest_out;    // [T]
  long long* csbase_out;    // [T]
  // Streamed inputs: router chunk c is read only once tok_ready[c] or
  // tok_ready_all has reached this call's epoch (null: tokens resident).
  const unsigned long long* tok_ready;      // [C], written by the copy stream after chunk c's rows
  const unsigned long long* tok_ready_all;  // set by the layer reset when the batch was resident
  // Progressive expert side: the next launch (the expert planner) may start
  // as soon as this grid is resident, and only the first dispatch_ctas
  // workers dispatch; the others leave after routing, so their SMs take
  // GEMM-1 tiles while the scheduler chain runs (0: every worker dispatches).
  int early_dependents;
  int dispatch_ctas;
  // Resident batches: each worker streams its token groups into a ring of
  // ring_slots group-sized slots at byte ring_off of its dynamic shared
  // memory with bulk copies, issued ring_slots groups ahead of the routing
  // (the caller passes ring_slots = 1 to ask for the ring, 0 to read every
  // group from global memory; launch_frontend sizes it).
  int ring_off;
  int ring_slots;
  // Control CTA: byte offset of the packed control path's tables and
  // per-ordinal words in dynamic shared memory (set by launch_frontend when
  // the plan fits that path; 0: the byte-per-entry path).
  int ctl_packed_off;
  // 1: each descriptor is dispatched by its own group of workers (when there
  // are at least as many dispatching workers as descriptors); 0: every
  // worker takes a share of every descriptor.
  int dispatch_groups;
  // Router weights [E, D] copied into each worker's dynamic shared memory at
  // byte w_off by one bulk copy at the start (the caller passes 1 to ask for
  // the copy, 0 to read the weights from global memory; launch_frontend
  // places them when they fit and sets 0 otherwise).
  int w_off;
  // Tensor-core router (bf16 batches, E <= 64, D a multiple of 64): workers
  // route units of 128 tokens as one tcgen05 MMA tile (M = 128 tokens, N =
  // tc_npad = E rounded up to 16) from tc_stages TMA stages carved from the
  // ring memory (set by launch_frontend; the caller passes tc_router = 1 to
  // ask for it).  tmap_x / tmap_w: the token matrix [T, D] and the router
  // weights [E, D] as 2-D tensor maps with 64 x 128 and 64 x tc_npad boxes,
  // 128-byte swizzle (built once by the caller).
  int tc_router;
  int tc_stages;
  int tc_npad;
  // Bytes of the ring memory (routing ring or tensor-core stages) that the
  // dispatch stages rows through once routing is done (0: no staging).
  int ring_bytes;
  CUtensorMap tmap_x;
  CUtensorMap tmap_w;
};

// Returns false (nothing launched) when the device cannot co-schedule the grid.
// tc_used (optional): 1 when the launch routes on the tensor cores.
bool launch_frontend(const FrontendParams& f, bool bf16, int sms, cudaStream_t s, int* tc_used = nullptr);
size_t control_smem_bytes(const ControlParams& p);
ControlDims control_dims(const ControlParams& p);
bool control_warp_path_ok(const ControlParams& p);

void launch_feature_digest(const void* rows, long long row_bytes, int nrows, long long* digest,
                           cudaStream_t s);
void launch_checksum_base(const long long* token_ids, const long long* digest, const int* chunk_offsets,
                          int chunks, int rank, int n, long long* base, cudaStream_t s);
void launch_router(const RouterParams& p, bool bf16, cudaStream_t s);
void launch_dispatch(const DispatchParams& p, bool bf16, int grid, cudaStream_t s);
void launch_expert_plan(const PlanParams& p, cudaStream_t s, bool pdl = false);
// One-warp planner of the progressive expert side (a programmatic dependent
// of the front end that starts at once): per descriptor, waits for every
// source's ready word, appends the newly complete 256-row GEMM-1 tiles to
// p.tile_list and publishes their count; after the last, the remaining and
// swapped tail tiles, the segments, rows_out and GEMM-2's tile tables.
void launch_expert_plan_progressive(const PlanParams& p, cudaStream_t s);
void launch_return_meta(const ReturnMetaParams& p, int grid, cudaStream_t s);
void launch_combine(const CombineParams& p, bool bf16, int grid, cudaStream_t s, bool pdl = false);
void launch_host_flag_signal(unsigned long long* flag, unsigned long long value, unsigned long long delay_ns,
                             cudaStream_t s);
void launch_layer_reset(int* sent_base, int experts, int* desc_counts, int n_desc, int* done_counter,
                        unsigned long long* epoch, TraceSlot* trace, int n_trace, int* chunk_words,
                        int n_chunk_words, unsigned long long* tok_ready_all, unsigned long long* stream_pending,
                        cudaStream_t s, unsigned int* ticket_counter = nullptr);
void launch_control(const ControlParams& p, cudaStream_t s);
void launch_device_barrier(const BarrierParams& p, cudaStream_t s);

}  // namespace raiccl
