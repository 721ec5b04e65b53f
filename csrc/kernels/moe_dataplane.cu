// Progressive MoE data plane for sm_100a: router top-k, revealed-only
// dispatch straight into peers' receive buffers over NVLink, expert plan,
// return identity rows, return/ready signalling and the device combine.
//
// Reference call sites replaced (rlccl / scripts):
//   router_topk (rlccl/transport/reference_router.py:15-25)          -> moe_router_kernel
//   FastProgressiveDataPrep.mark_completed/build_delta_payload + the
//     count all_to_all_single + the two payload all_to_all_single
//     (scripts/run_r4_a0_c0_full_moe.py:104-207)                      -> moe_dispatch_kernel
//   pack_return_payload + return all_to_all_single (:628-695)          -> moe_return_meta_kernel
//                                                                        + grouped GEMM-2 epilogue
//   NumPy position scatter combine (:833-838)                          -> moe_combine_kernel
//
// Every cross-GPU wait is bounded (globaltimer deadline) and reports through
// DeviceStatus; there is no __trap and no intra-GPU wait on another kernel.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>

#include "launchers.h"
#include "moe_kernels.h"
#include "moe_device.cuh"
#include "sm100_ptx.cuh"

namespace raiccl {

// ---------------------------------------------------------------------------
// Row digest: (sum_i splitmix64((i << 32) | w_i)) mod 2^64, masked to 62 bits,
// over the row's 32-bit words.  One warp per row.
// ---------------------------------------------------------------------------
__global__ void moe_feature_digest_kernel(const uint32_t* rows, long long words_per_row, int nrows,
                                          long long* digest) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= nrows) return;
  const uint32_t* r = rows + (long long)row * words_per_row;
  uint64_t acc = 0;
  for (long long i = lane; i < words_per_row; i += 32)
    acc += splitmix64(((uint64_t)i << 32) | (uint64_t)__ldg(r + i));
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) digest[row] = (long long)(acc & ((1ULL << 62) - 1));
}

// Checksum base of every token (token_checksum_base) from precomputed digests.
__global__ void moe_checksum_base_kernel(const long long* token_ids, const long long* digest,
                                         const int* chunk_offsets, int chunks, int rank, int n,
                                         long long* base) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  int c = 0;
  while (c + 1 < chunks && chunk_offsets[c + 1] <= t) ++c;
  base[t] = token_checksum_base(token_ids[t], rank, c, t - chunk_offsets[c], t, digest[t]);
}

// ---------------------------------------------------------------------------
// Router: logits = x @ W^T + b (+ chunk bias), masks, stable top-k (ties pick
// the smaller expert id), gates.  One warp per token row, fp32 accumulation
// (exact fp32 for fp32 inputs).  W is [E, D] in the token dtype.
// ---------------------------------------------------------------------------
// Router rows are streamed with UNROLL independent 16-byte loads in flight per
// lane (the kernel is HBM-bound for small E); W is staged once per CTA in
// shared memory when it fits (SMEM_W), else read through the read-only cache.
template <typename T, int EMAX, bool SMEM_W>
__global__ void __launch_bounds__(256) moe_router_kernel(RouterParams p) {
  TraceScope trace_scope(p.trace);
  extern __shared__ __align__(16) uint8_t router_smem[];
  const T* __restrict__ w = (const T*)p.weight;
  if constexpr (SMEM_W) {
    uint4* ws = (uint4*)router_smem;
    const uint4* wg = (const uint4*)p.weight;
    const int nvec = p.experts * p.hidden * (int)sizeof(T) / 16;
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) ws[i] = __ldg(wg + i);
    __syncthreads();
    w = (const T*)router_smem;
  }
  const int warps = blockDim.x >> 5;
  const int t = p.row0 + blockIdx.x * warps + (threadIdx.x >> 5);
  if (t >= p.row1) return;
  router_token<T, EMAX, SMEM_W>(p, p.chunk_bias, t, (const T*)p.tokens + (long long)t * p.hidden, false, w,
                                nullptr);
}

// ---------------------------------------------------------------------------
// Dispatch of one revealed descriptor (a run of router chunks) straight into
// the owners' receive regions.  Rows keep the reference's deterministic order
// inside every (expert, source) region: descriptor order, then token order.
// The last CTA publishes per-expert counts into each owner's header and then
// one release store of the sequence number per destination rank (sent even
// for zero rows, like the reference's header-only zero-payload slot).
// ---------------------------------------------------------------------------
constexpr int kDispatchThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kDispatchThreads) moe_dispatch_kernel(DispatchParams p) {
  TraceScope trace_scope(p.trace);
  const MoEDims& d = p.dims;
  __shared__ int hist[kMaxExperts];
  __shared__ int run[kMaxExperts];
  __shared__ int item_pos[kDispatchMaxItems];
  __shared__ int s_last;
  __shared__ int s_permitted;
  __shared__ int s_sent[kMaxExperts];
  __shared__ int s_coff[kDispatchMaxChunks + 1];
  const int k = d.top_k;
  const int E = d.experts;
  const int ntok = p.t1 - p.t0;
  const int per = (ntok + gridDim.x - 1) / gridDim.x;
  const int a = p.t0 + min(ntok, (int)blockIdx.x * per);
  const int b = p.t0 + min(ntok, (int)(blockIdx.x + 1) * per);

  for (int e = threadIdx.x; e < E; e += blockDim.x) { hist[e] = 0; run[e] = 0; s_sent[e] = p.sent_base[e]; }
  const int nc = min(d.chunks, kDispatchMaxChunks);
  for (int c = threadIdx.x; c <= nc; c += blockDim.x) s_coff[c] = p.chunk_offsets[c];
  const unsigned long long epoch = *p.epoch;
  if (threadIdx.x == 0) s_permitted = (p.permit[p.desc] == epoch) ? 1 : 0;
  __syncthreads();
  const bool permitted = s_permitted != 0;
  if (!permitted && threadIdx.x == 0 && blockIdx.x == 0)
    record_status(p.status, kTimeoutPermit, 20, p.desc, (long long)epoch);

  if (permitted && (long long)(b - a) * k > kDispatchMaxItems) {
    if (threadIdx.x == 0) record_status(p.status, kBadConfig, 22, (long long)(b - a) * k, kDispatchMaxItems);
  } else if (permitted && a < b) {
    dispatch_rows<T>(p, p.t0, a, b, s_sent, hist, run, item_pos, s_coff, nc);
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (run[e]) atomicAdd(&p.desc_counts[(long long)p.desc * E + e], run[e]);
  }

  // completion: the last CTA of the launch publishes counts and signals
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atom_add_acq_rel_gpu(&p.done_counter[p.desc], 1);
    s_last = (prev == (int)gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;
  dispatch_publish(p, p.desc, p.fault_skip_signal != 0, epoch, true);
}

// ---------------------------------------------------------------------------
// Expert plan: wait (bounded) for every (source, descriptor) ready signal,
// then emit one grouped-GEMM segment per (local expert slot, source).
// ---------------------------------------------------------------------------
// Tiles of one segment in a GEMM tile table: ceil(rows / bm) row tiles times
// nblocks column tiles.  With swap > 0 a last row tile of at most swap rows
// is counted apart (tail = nblocks) for the swapped-operand tail pass.
__device__ __forceinline__ void plan_tiles(int rows, int bm, int nblocks, int swap, int& full, int& tail) {
  const int mt = (rows + bm - 1) / bm;
  const bool sw = swap > 0 && mt > 0 && rows - (mt - 1) * bm <= swap;
  full = (mt - (sw ? 1 : 0)) * nblocks;
  tail = sw ? nblocks : 0;
}

// Traffic counters of the expert side: one ready word waited for per (source,
// descriptor), and per source rank the return bytes (output rows and return
// identity rows of every row received from it) and one return signal.
__device__ __forceinline__ void plan_count_traffic(const PlanParams& p) {
  if (p.peer_counters == nullptr || threadIdx.x != 0) return;
  const MoEDims& d = p.dims;
  const unsigned long long row_bytes = (unsigned long long)d.out_dim * d.out_bytes + kRetMetaFields * 8;
  for (int src = 0; src < d.world; ++src) {
    unsigned long long rows = 0;
    for (int s = 0; s < d.expert_slots; ++s) rows += (unsigned long long)p.rows_out[s * d.world + src];
    unsigned long long* pc = p.peer_counters + (long long)src * kPeerCounterFields;
    atomicAdd(pc + kPcWaits, (unsigned long long)d.n_desc);
    atomicAdd(pc + kPcReturnBytes, rows * row_bytes);
    atomicAdd(pc + kPcReturnSignals, 1ULL);
  }
}

__global__ void moe_expert_plan_kernel(PlanParams p) {
  griddep_wait();  // programmatic dependent of the front end (no-op otherwise)
  griddep_launch_dependents();
  TraceScope trace_scope(p.trace);
  const MoEDims& d = p.dims;
  const uint8_t* mine = (const uint8_t*)p.peers.base[d.rank];
  const uint64_t* flags = (const uint64_t*)(mine + p.layout.recv_flag);
  __shared__ int s_ok;
  const unsigned long long epoch = *p.epoch;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  for (int i = threadIdx.x; i < d.world * d.n_desc; i += blockDim.x) {
    if (!wait_flag_geq_sys(flags + i, epoch, p.status, kTimeoutPeerSignal, 30, i, p.timeout_ns))
      s_ok = 0;
  }
  __syncthreads();
  const int* counts = (const int*)(mine + p.layout.recv_count);
  // Each thread owns a contiguous run of segments, so the GEMM tile tables
  // (exclusive prefixes of plan_tiles counts per segment, for both GEMMs)
  // come out of one block scan in this same launch.
  const int S = d.expert_slots * d.world;
  const int per = (S + blockDim.x - 1) / blockDim.x;
  const int s0 = threadIdx.x * per;
  const int s1 = min(S, s0 + per);
  int local[4] = {0, 0, 0, 0};  // full tiles of GEMM 1, its swapped tails, and the same for GEMM 2
  for (int s = s0; s < s1; ++s) {
    int rows = 0;
    if (s_ok) {
      for (int q = 0; q < d.n_desc; ++q) rows += counts[(long long)s * d.n_desc + q];
      if (rows > d.cap) { record_status(p.status, kBoundsViolation, 31, rows, d.cap); rows = 0; }
    }
    GemmSegment seg;
    seg.a_row0 = (int)((long long)s * d.cap);
    seg.rows = rows;
    seg.expert = s / d.world;
    seg.out_slot = s % d.world;
    seg.out_row0 = seg.a_row0;
    seg.pad0 = seg.pad1 = seg.pad2 = 0;
    p.segs[s] = seg;
    p.rows_out[s] = rows;
    if (p.prefix1 != nullptr) {
      int f, tl;
      plan_tiles(rows, p.bm1, p.nblocks1, p.swap1, f, tl);
      local[0] += f; local[1] += tl;
      plan_tiles(rows, p.bm2, p.nblocks2, p.swap2, f, tl);
      local[2] += f; local[3] += tl;
    }
  }
  __syncthreads();  // rows_out of every segment written
  plan_count_traffic(p);
  if (p.prefix1 == nullptr) return;
  __shared__ int s_scan[4][256];
#pragma unroll
  for (int a = 0; a < 4; ++a) s_scan[a][threadIdx.x] = local[a];
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    int v[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) v[a] = threadIdx.x >= off ? s_scan[a][threadIdx.x - off] : 0;
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; ++a) s_scan[a][threadIdx.x] += v[a];
    __syncthreads();
  }
  int run[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) run[a] = s_scan[a][threadIdx.x] - local[a];
  int32_t* out[4] = {p.prefix1, p.tail1, p.prefix2, p.tail2};
  for (int s = s0; s < s1; ++s) {
    const int rows = p.rows_out[s];
    int c[4];
    plan_tiles(rows, p.bm1, p.nblocks1, p.swap1, c[0], c[1]);
    plan_tiles(rows, p.bm2, p.nblocks2, p.swap2, c[2], c[3]);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      if (out[a] != nullptr) out[a][s] = run[a];
      run[a] += c[a];
    }
  }
  if (threadIdx.x == blockDim.x - 1) {
#pragma unroll
    for (int a = 0; a < 4; ++a)
      if (out[a] != nullptr) out[a][S] = s_scan[a][threadIdx.x];
  }
}

// ---------------------------------------------------------------------------
// Progressive expert plan: one warp, a programmatic dependent of the front
// end that lets it start as soon as the front end is resident.  Descriptor
// by descriptor (in order), it waits (bounded) for every source's ready
// word, adds the descriptor's rows to each (local expert slot, source)
// segment, appends the 256-row GEMM-1 tiles that are now complete (all
// column blocks of each) to the tile list and publishes the list's length
// with a release store; the GEMM-1 CTA pairs take tiles as they appear.
// After the last descriptor it appends each segment's remaining tiles and
// then the swapped tail tiles (the order of the non-progressive plan), and
// writes the segments, rows_out and GEMM-2's tile tables before the final
// publish.  Segment row counts only grow, so a tile never reads a row count
// below its own rows.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void publish_tiles(unsigned long long* word, unsigned long long epoch, int count,
                                              bool final) {
  __threadfence();
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(word),
               "l"(((epoch & 0xffffffffULL) << 32) | (final ? 0x80000000ULL : 0ULL) | (unsigned long long)count)
               : "memory");
}

__global__ void __launch_bounds__(32) moe_expert_plan_progressive_kernel(PlanParams p) {
  griddep_launch_dependents();  // the progressive GEMM-1 may launch now
  TraceScope trace_scope(p.trace);
  const unsigned FULL = 0xffffffffu;
  const MoEDims& d = p.dims;
  const int lane = threadIdx.x;
  const uint8_t* mine = (const uint8_t*)p.peers.base[d.rank];
  const uint64_t* flags = (const uint64_t*)(mine + p.layout.recv_flag);
  const int* counts = (const int*)(mine + p.layout.recv_count);
  const unsigned long long epoch = *p.epoch;
  const int S = d.expert_slots * d.world;
  extern __shared__ int psm[];
  int* cum = psm;       // [S] rows received so far
  int* done = psm + S;  // [S] row tiles already listed
  for (int s = lane; s < S; s += 32) {
    cum[s] = 0;
    done[s] = 0;
    GemmSegment seg;
    seg.a_row0 = (int)((long long)s * d.cap);
    seg.rows = 0;
    seg.expert = s / d.world;
    seg.out_slot = s % d.world;
    seg.out_row0 = seg.a_row0;
    seg.pad0 = seg.pad1 = seg.pad2 = 0;
    p.segs[s] = seg;
  }
  __syncwarp();
  const int bm = 256, nb1 = p.nblocks1;
  int listed = 0;
  bool ok = true;
  for (int q = 0; q < d.n_desc; ++q) {
    const bool final = q == d.n_desc - 1;
    bool got = true;
    for (int src = lane; src < d.world && ok; src += 32)
      got = wait_flag_geq_sys(flags + (long long)src * d.n_desc + q, epoch, p.status, kTimeoutPeerSignal, 33,
                              (long long)src * d.n_desc + q, p.timeout_ns) && got;
    ok = __all_sync(FULL, got) && ok;  // (the warp barrier orders every lane's acquire before the reads below)
    for (int s = lane; s < S && ok; s += 32) {
      int v = cum[s] + counts[(long long)s * d.n_desc + q];
      if (v > d.cap) {
        record_status(p.status, kBoundsViolation, 31, v, d.cap);
        v = cum[s];
      }
      cum[s] = v;
      p.segs[s].rows = v;
    }
    __syncwarp();
    // pass 0: complete row tiles (every remaining one after the last
    // descriptor); pass 1 (last descriptor): swapped tail tiles
    for (int pass = 0; pass < (final ? 2 : 1) && ok; ++pass) {
      for (int s0 = 0; s0 < S; s0 += 32) {
        const int s = s0 + lane;
        int first = 0, n = 0, nsw = 0;
        if (s < S) {
          const int rows = cum[s];
          if (!final) {
            first = done[s];
            n = rows / bm - first;
          } else {
            const int mt = (rows + bm - 1) / bm;
            const bool sw = p.swap1 > 0 && mt > 0 && rows - (mt - 1) * bm <= p.swap1;
            if (pass == 0) {
              first = done[s];
              n = mt - (sw ? 1 : 0) - first;
            } else if (sw) {
              first = mt - 1;
              n = 1;
              nsw = (rows - first * bm + 15) & ~15;
            }
          }
          if (n < 0) n = 0;
        }
        const int cnt = n * nb1;
        int incl = cnt;
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(FULL, incl, o);
          if (lane >= o) incl += v;
        }
        const int base = listed + incl - cnt;
        if (cnt > 0 && base + cnt <= p.max_tiles1) {
          for (int i = 0; i < cnt; ++i) {
            int4 e;
            e.x = s; e.y = first + i / nb1; e.z = i % nb1; e.w = nsw;
            reinterpret_cast<int4*>(p.tile_list)[base + i] = e;
          }
        } else if (cnt > 0) {
          record_status(p.status, kBoundsViolation, 34, base + cnt, p.max_tiles1);
        }
        if (s < S && pass == 0) done[s] = first + n;
        listed += __shfl_sync(FULL, incl, 31);
      }
    }
    if (listed > p.max_tiles1) listed = p.max_tiles1;
    if (final || !ok) break;
    __syncwarp();
    if (lane == 0) publish_tiles(p.tile_word, epoch, listed, false);
  }
  // final segment rows (all zero rows after a failed wait), rows_out and GEMM-2's tile tables
  const int S2 = S;
  int run2 = 0, runt = 0;
  for (int s0 = 0; s0 < S2; s0 += 32) {
    const int s = s0 + lane;
    int f = 0, tl = 0;
    if (s < S2) {
      const int rows = ok ? cum[s] : 0;
      p.segs[s].rows = rows;
      p.rows_out[s] = rows;
      plan_tiles(rows, p.bm2, p.nblocks2, p.swap2, f, tl);
    }
    int a = f, b = tl;
    for (int o = 1; o < 32; o <<= 1) {
      const int va = __shfl_up_sync(FULL, a, o), vb = __shfl_up_sync(FULL, b, o);
      if (lane >= o) { a += va; b += vb; }
    }
    if (s < S2) {
      if (p.prefix2 != nullptr) p.prefix2[s] = run2 + a - f;
      if (p.tail2 != nullptr) p.tail2[s] = runt + b - tl;
    }
    run2 += __shfl_sync(FULL, a, 31);
    runt += __shfl_sync(FULL, b, 31);
  }
  if (lane == 0) {
    if (p.prefix2 != nullptr) p.prefix2[S2] = run2;
    if (p.tail2 != nullptr) p.tail2[S2] = runt;
  }
  __syncwarp();
  plan_count_traffic(p);
  __syncwarp();
  if (lane == 0) publish_tiles(p.tile_word, epoch, listed, true);
}

// Publish this rank's return sequence number at every source rank.
__device__ void publish_return_signal(const MoEDims& d, const SymLayout& L, const PeerBases& P,
                                      unsigned long long epoch) {
  __threadfence_system();
  for (int r = 0; r < d.world; ++r)
    st_release_sys_u64((uint64_t*)((uint8_t*)P.base[r] + L.ret_flag) + d.rank, epoch);
}

// One of the two return parts of a call is complete (its stores fenced at
// system scope): the second to report publishes the return signal.
__device__ void return_part_done(const MoEDims& d, const SymLayout& L, const PeerBases& P,
                                 unsigned long long epoch, unsigned long long* ret_sync) {
  __threadfence_system();
  if (atomicAdd(ret_sync + 1, 1ULL) & 1ULL) publish_return_signal(d, L, P, epoch);
}

// Return identity rows to the token's source rank, at row (position * k + j)
// of its return region (rlccl/transport/reference_full_moe.py:143-182 order:
// token, source, expert rank, expert, original position, chunk, chunk offset,
// checksum).
__global__ void moe_return_meta_kernel(ReturnMetaParams p) {
  TraceScope trace_scope(p.trace);
  const MoEDims& d = p.dims;
  const uint8_t* mine = (const uint8_t*)p.peers.base[d.rank];
  const long long* meta = (const long long*)(mine + p.layout.recv_meta);
  const int* retrow = (const int*)(mine + p.layout.recv_retrow);
  const long long total = (long long)d.expert_slots * d.world * d.cap;
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
    const int s = (int)(g / d.cap);
    const long long r = g % d.cap;
    if (r >= p.segs[s].rows) continue;
    const int src = s % d.world;
    const long long* m = meta + g * kFwdMetaFields;
    const uint64_t f[7] = {(uint64_t)m[0], (uint64_t)src, (uint64_t)d.rank, (uint64_t)m[3],
                           (uint64_t)m[6], (uint64_t)m[4], (uint64_t)m[5]};
    uint64_t cs = 0;
#pragma unroll
    for (int i = 0; i < 7; ++i) cs = addmod(cs, mulmod_coeff(f[i], c_checksum_coeff[i]));
    const long long dst_row = retrow[g];
    if (dst_row < 0 || dst_row >= (long long)d.tokens * d.top_k) {
      record_status(p.status, kBoundsViolation, 40, dst_row, (long long)d.tokens * d.top_k);
      continue;
    }
    long long* out = (long long*)((uint8_t*)p.peers.base[src] + p.layout.ret_meta) + dst_row * kRetMetaFields;
#pragma unroll
    for (int i = 0; i < 7; ++i) out[i] = (long long)f[i];
    out[7] = (long long)cs;
  }
  if (p.ret_sync == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    // every call adds gridDim.x, so the CTA completing a multiple is the last
    if ((atomicAdd(p.ret_sync + 2, 1ULL) + 1ULL) % gridDim.x == 0)
      return_part_done(d, p.layout, p.peers, *p.epoch, p.ret_sync);
  }
}

// Combine: wait (bounded) for every expert rank's return signal, then
// out[t] = sum_j ret_out[t * k + j] (rows already carry their gate weight).
template <typename OutT>
__global__ void moe_combine_kernel(CombineParams p) {
  griddep_wait();  // the return rows of GEMM-2 (previous launch) are complete and visible
  TraceScope trace_scope(p.trace);
  const MoEDims& d = p.dims;
  const uint8_t* mine = (const uint8_t*)p.peers.base[d.rank];
  __shared__ int s_ok;
  const unsigned long long epoch = *p.epoch;
  if (threadIdx.x == 0) {
    s_ok = 1;
    // Whichever CTA runs first reports the return rows (written by the
    // GEMM-2 launch before this one), so the signal never waits on the
    // scheduling of a particular CTA.
    if (p.ret_sync == nullptr) {
      if (blockIdx.x == 0) publish_return_signal(d, p.layout, p.peers, epoch);
    } else if (atomicMax(p.ret_sync, epoch) < epoch) {
      return_part_done(d, p.layout, p.peers, epoch, p.ret_sync);
    }
  }
  __syncthreads();
  // This rank's own rows come from the GEMM-2 launch that precedes this one
  // in the stream; only the other ranks' signals need waiting for.
  if (threadIdx.x < d.world && threadIdx.x != d.rank) {
    const uint64_t* f = (const uint64_t*)(mine + p.layout.ret_flag) + threadIdx.x;
    if (!wait_flag_geq_sys(f, epoch, p.status, kTimeoutPeerSignal, 50, threadIdx.x, p.timeout_ns))
      s_ok = 0;
  }
  __syncthreads();
  if (!s_ok) return;
  const OutT* ret = (const OutT*)(mine + p.layout.ret_out);
  OutT* out = (OutT*)p.out;
  const int k = d.top_k, n = d.out_dim;
  constexpr int VEC = 16 / sizeof(OutT);  // elements per 16-byte vector
  constexpr int U = 4;                    // vectors in flight per lane
  if (n % VEC == 0) {
    // one warp per token row, lanes over 16-byte column vectors; the k return
    // rows of a token are adjacent (row t * k + j), so each load is coalesced
    const int nv = n / VEC;
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < d.tokens; t += warps) {
      const uint4* src = reinterpret_cast<const uint4*>(ret + (long long)t * k * n);
      uint4* dst = reinterpret_cast<uint4*>(out + (long long)t * n);
      for (int v0 = lane; v0 < nv; v0 += 32 * U) {
        float acc[U][VEC];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[u][e] = 0.f;
        for (int j = 0; j < k; ++j) {
          uint4 x[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int v = v0 + 32 * u;
            if (v < nv) x[u] = src[(long long)j * nv + v];
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const OutT* xe = reinterpret_cast<const OutT*>(&x[u]);
            if (v0 + 32 * u < nv)
#pragma unroll
              for (int e = 0; e < VEC; ++e) acc[u][e] += to_f(xe[e]);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int v = v0 + 32 * u;
          if (v >= nv) continue;
          uint4 y;
          OutT* ye = reinterpret_cast<OutT*>(&y);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            if constexpr (sizeof(OutT) == 4) ye[e] = acc[u][e];
            else ye[e] = __float2bfloat16(acc[u][e]);
          }
          dst[v] = y;
        }
      }
    }
    return;
  }
  const long long total = (long long)d.tokens * n;  // ragged widths: one element per thread
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
    const long long t = g / n, c = g % n;
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += to_f(ret[(t * k + j) * n + c]);
    if constexpr (sizeof(OutT) == 4) out[g] = acc;
    else out[g] = __float2bfloat16(acc);
  }
}

// Cross-GPU barrier: publish this rank's barrier sequence at every peer, then
// wait (bounded) until every peer's sequence arrived here.  Used to align the
// ranks before a timed layer call without a host round-trip.
__global__ void moe_device_barrier_kernel(BarrierParams p) {
  TraceScope trace_scope(p.trace);
  const MoEDims& d = p.dims;
  __shared__ unsigned long long seq;
  if (threadIdx.x == 0) {
    seq = *p.counter + 1;
    *p.counter = seq;
    __threadfence_system();
    for (int r = 0; r < d.world; ++r)
      st_release_sys_u64((uint64_t*)((uint8_t*)p.peers.base[r] + p.layout.bar_flag) + d.rank, seq);
  }
  __syncthreads();
  if (threadIdx.x < d.world) {
    const uint64_t* f = (const uint64_t*)((const uint8_t*)p.peers.base[d.rank] + p.layout.bar_flag) + threadIdx.x;
    wait_flag_geq_sys(f, seq, p.status, kTimeoutPeerSignal, 70, threadIdx.x, p.timeout_ns);
  }
}

void launch_device_barrier(const BarrierParams& p, cudaStream_t s) {
  moe_device_barrier_kernel<<<1, 32, 0, s>>>(p);
}

// Per-call reset of the dispatch cursors and counters; advances the call's
// sequence number (the value every ready / return / permit word is compared to).
// Start of a layer call: next epoch, zeroed per-call counters and trace slots.
// Inputs: when the host announced a streamed call (*stream_pending != 0) the
// copy stream publishes each chunk's arrival itself; otherwise the batch is
// resident and tok_ready_all takes the new epoch.
__global__ void moe_layer_reset_kernel(int* sent_base, int experts, int* desc_counts, int n_desc,
                                       int* done_counter, unsigned long long* epoch, TraceSlot* trace,
                                       int n_trace, int* chunk_words, int n_chunk_words,
                                       unsigned long long* tok_ready_all, unsigned long long* stream_pending,
                                       unsigned int* ticket_counter) {
  if (threadIdx.x == 0) {
    if (ticket_counter != nullptr) *ticket_counter = 0;
    const unsigned long long e = *epoch + 1;
    *epoch = e;
    if (tok_ready_all != nullptr) {
      if (*stream_pending != 0) *stream_pending = 0;
      else *tok_ready_all = e;
    }
  }
  for (int i = threadIdx.x; i < n_chunk_words; i += blockDim.x) chunk_words[i] = 0;
  for (int i = threadIdx.x; i < n_trace; i += blockDim.x) {
    trace[i].t_start = ~0ULL;
    trace[i].t_end = 0;
    trace[i].ctas = 0;
  }
  for (int i = threadIdx.x; i < experts; i += blockDim.x) sent_base[i] = 0;
  for (int i = threadIdx.x; i < experts * n_desc; i += blockDim.x) desc_counts[i] = 0;
  for (int i = threadIdx.x; i < n_desc; i += blockDim.x) done_counter[i] = 0;
}

// One thread: hold the stream for delay_ns (a fixed-length busy loop on
// %globaltimer, capped at 10 ms), then publish value to a host-mapped word with
// a system-scope release — the device side of the event bridge's flag slots.
__global__ void host_flag_signal_kernel(unsigned long long* flag, unsigned long long value,
                                        unsigned long long delay_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (delay_ns > 10000000ULL) delay_ns = 10000000ULL;
  const unsigned long long t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < delay_ns) {
  }
  __threadfence_system();
  st_release_sys_u64(reinterpret_cast<uint64_t*>(flag), value);
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
void launch_feature_digest(const void* rows, long long row_bytes, int nrows, long long* digest,
                           cudaStream_t s) {
  const int warps = 8;
  moe_feature_digest_kernel<<<(nrows + warps - 1) / warps, warps * 32, 0, s>>>(
      (const uint32_t*)rows, row_bytes / 4, nrows, digest);
}

void launch_checksum_base(const long long* token_ids, const long long* digest, const int* chunk_offsets,
                          int chunks, int rank, int n, long long* base, cudaStream_t s) {
  moe_checksum_base_kernel<<<(n + 255) / 256, 256, 0, s>>>(token_ids, digest, chunk_offsets, chunks,
                                                            rank, n, base);
}

void launch_router(const RouterParams& p, bool bf16, cudaStream_t s) {
  const int rows = p.row1 - p.row0;
  if (rows <= 0) return;
  if (p.experts > 64) throw std::invalid_argument("the router handles at most 64 experts");
  const int warps = 8;
  const dim3 grid((rows + warps - 1) / warps);
  const long long wbytes = (long long)p.experts * p.hidden * (bf16 ? 2 : 4);
  const bool smem_w = wbytes <= 96 * 1024;
  const int smem = smem_w ? (int)wbytes : 0;
#define RAICCL_ROUTER(T, EM)                                                                    \
  do {                                                                                          \
    if (smem_w) {                                                                               \
      static bool attr = false;                                                                 \
      if (!attr) {                                                                              \
        cudaFuncSetAttribute(moe_router_kernel<T, EM, true>,                                    \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);           \
        attr = true;                                                                            \
      }                                                                                         \
      moe_router_kernel<T, EM, true><<<grid, warps * 32, smem, s>>>(p);                         \
    } else {                                                                                    \
      moe_router_kernel<T, EM, false><<<grid, warps * 32, 0, s>>>(p);                           \
    }                                                                                           \
  } while (0)
  if (p.experts <= 8) {
    if (bf16) RAICCL_ROUTER(__nv_bfloat16, 8); else RAICCL_ROUTER(float, 8);
  } else if (p.experts <= 16) {
    if (bf16) RAICCL_ROUTER(__nv_bfloat16, 16); else RAICCL_ROUTER(float, 16);
  } else {
    if (bf16) RAICCL_ROUTER(__nv_bfloat16, 64); else RAICCL_ROUTER(float, 64);
  }
#undef RAICCL_ROUTER
}

void launch_dispatch(const DispatchParams& p, bool bf16, int grid, cudaStream_t s) {
  if (bf16) moe_dispatch_kernel<__nv_bfloat16><<<grid, kDispatchThreads, 0, s>>>(p);
  else moe_dispatch_kernel<float><<<grid, kDispatchThreads, 0, s>>>(p);
}

void launch_expert_plan(const PlanParams& p, cudaStream_t s, bool pdl) {
  launch_with_pdl(moe_expert_plan_kernel, dim3(1), dim3(256), 0, s, pdl, p);
}

void launch_expert_plan_progressive(const PlanParams& p, cudaStream_t s) {
  const size_t smem = 2 * sizeof(int) * (size_t)p.dims.expert_slots * p.dims.world;
  launch_with_pdl(moe_expert_plan_progressive_kernel, dim3(1), dim3(32), smem, s, true, p);
}

void launch_return_meta(const ReturnMetaParams& p, int grid, cudaStream_t s) {
  moe_return_meta_kernel<<<grid, 256, 0, s>>>(p);
}

void launch_combine(const CombineParams& p, bool bf16, int grid, cudaStream_t s, bool pdl) {
  // enough warps for one token row each (capped at 8 CTAs per SM)
  const int rows_grid = (p.dims.tokens + 7) / 8;
  const int g = std::max(1, std::min(rows_grid, 8 * grid));
  if (bf16) launch_with_pdl(moe_combine_kernel<__nv_bfloat16>, dim3(g), dim3(256), 0, s, pdl, p);
  else launch_with_pdl(moe_combine_kernel<float>, dim3(g), dim3(256), 0, s, pdl, p);
}

void launch_host_flag_signal(unsigned long long* flag, unsigned long long value, unsigned long long delay_ns,
                             cudaStream_t s) {
  host_flag_signal_kernel<<<1, 32, 0, s>>>(flag, value, delay_ns);
}

void launch_layer_reset(int* sent_base, int experts, int* desc_counts, int n_desc, int* done_counter,
                        unsigned long long* epoch, TraceSlot* trace, int n_trace, int* chunk_words,
                        int n_chunk_words, unsigned long long* tok_ready_all, unsigned long long* stream_pending,
                        cudaStream_t s, unsigned int* ticket_counter) {
  moe_layer_reset_kernel<<<1, 256, 0, s>>>(sent_base, experts, desc_counts, n_desc, done_counter, epoch, trace,
                                           trace ? n_trace : 0, chunk_words, chunk_words ? n_chunk_words : 0,
                                           tok_ready_all, stream_pending, ticket_counter);
}

}  // namespace raiccl
