// CTA-pair variant of the grouped GEMM (tcgen05 cta_group::2, clusters of 2).
//
// Same math, segments, epilogues and outputs as grouped_gemm_kernel, with a
// 256 x BN output tile per CTA pair instead of 128 x BN per CTA:
//   * each CTA stages ITS 128 rows of A and HALF (BN/2 rows) of the B tile;
//   * the pair leader (cluster rank 0) issues tcgen05.mma.cta_group::2 with
//     M = 256, which reads A and B from both CTAs' shared memory and writes
//     each CTA's 128 x BN accumulator into that CTA's TMEM;
//   * both CTAs' TMA loads complete on the leader's stage barrier; the
//     leader's MMA completion is committed to the stage-free barriers of both
//     CTAs and to both CTAs' accumulator-ready barriers; both CTAs' epilogue
//     warps report a drained accumulator to the leader's barrier.
// Per CTA and K step this moves 128 + BN/2 operand rows instead of 128 + BN,
// i.e. a third fewer bytes from L2 per FLOP at BN = 256.
//
// tile_prefix must count 256-row tiles (launch_tile_plan(..., bm = 256)).
// Every wait is bounded; on a timeout each role stops and all threads still
// meet at the final cluster barrier before the pair frees its TMEM, so no CTA
// leaves while its partner may still address its shared memory.
// All loads read this GPU's own memory (activations and weights); none uses
// multicast.
#pragma once

#include "grouped_gemm.cuh"

namespace raiccl {

// Tile t of the pair kernel.  Full tiles come first, in segment order, then
// the swapped tail tiles (GroupedGemmParams::tail_prefix); nsw is 0 for a full
// tile and the tail's row count rounded up to 16 for a swapped one.
struct PairTile {
  int s, mb, nb, nsw;
};

__device__ __forceinline__ PairTile pair_tile(const GroupedGemmParams& p, int t, int total_full, int nblocks) {
  PairTile r;
  if (t < total_full) {
    r.s = find_segment(p.tile_prefix, p.num_segs, t);
    const int local = t - p.tile_prefix[r.s];
    r.mb = local / nblocks;
    r.nb = local % nblocks;
    r.nsw = 0;
  } else {
    const int u = t - total_full;
    r.s = find_segment(p.tail_prefix, p.num_segs, u);
    r.nb = u - p.tail_prefix[r.s];
    const int rows = p.segs[r.s].rows;
    r.mb = (rows - 1) / 256;
    r.nsw = (rows - r.mb * 256 + 15) & ~15;
  }
  return r;
}

// ---------------------------------------------------------------------------
// Progressive tile source (GroupedGemmParams::progressive).
//
// The pair leader's producer owns the schedule.  It draws ticket T for its
// next tile from the per-call counter one tile ahead (the atomic's latency
// hides behind the current tile's loads), waits (bounded) until the
// planner's published tile count passes T, reads the tile from the list and
// posts it, fully resolved, in the pair's ring slot for that iteration
// (two 64-bit words: the packed tile, then a release store of the epoch /
// iteration tag with T; T = kNoTicket ends the pair's loop).  The partner's
// producer and both CTAs' epilogue warps read the ring (one acquire load
// when the slot is already posted); the leader's MMA warp reads the tile
// from a shared-memory slot the producer writes before the tile's first
// stage barrier, so its scheduling costs no global round trip.
// ---------------------------------------------------------------------------
constexpr unsigned int kNoTicket = 0xfffffu;
constexpr int kTileSlots = 16;  // shared-memory tile slots of the leader (>= stages + 1)

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64_gg(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ring_tag(unsigned long long epoch, int k) {
  return ((epoch & 0xffffffULL) << 40) | ((unsigned long long)(k & 0xfffff) << 20);
}

__device__ __forceinline__ unsigned long long pack_tile(const PairTile& t) {
  return (unsigned long long)(t.s & 0xffff) | ((unsigned long long)(t.mb & 0xffff) << 16) |
         ((unsigned long long)(t.nb & 0xffff) << 32) | ((unsigned long long)(t.nsw & 0xffff) << 48);
}

__device__ __forceinline__ PairTile unpack_tile(unsigned long long v) {
  PairTile t;
  t.s = (int)(v & 0xffff);
  t.mb = (int)((v >> 16) & 0xffff);
  t.nb = (int)((v >> 32) & 0xffff);
  t.nsw = (int)((v >> 48) & 0xffff);
  return t;
}

// Leader producer: the tile of ticket T once published.  1: tile in pt;
// 0: the planner finished without it; -1: the wait ran out (status recorded).
__device__ __forceinline__ int resolve_ticket(const GroupedGemmParams& p, unsigned int T, unsigned long long epoch,
                                              PairTile& pt, int kernel_id, int pair) {
  const unsigned long long want = (epoch & 0xffffffffULL) << 32;
  const uint64_t start = globaltimer_ns();
  for (uint32_t polls = 1;; ++polls) {
    const unsigned long long w = ld_acquire_gpu_u64_gg(p.tile_word);
    if ((w & 0xffffffff00000000ULL) == want) {
      if (T < (unsigned int)(w & 0x7fffffffULL)) break;
      if (w & 0x80000000ULL) return 0;
    }
    __nanosleep(64);
    if ((polls & 63u) == 0) {
      if (globaltimer_ns() - start > p.timeout_ns) {
        record_status(p.status, kTimeoutPeerSignal, kernel_id, (long long)T, pair);
        return -1;
      }
      if (status_failed(p.status)) return -1;
    }
  }
  const int4 e = reinterpret_cast<const int4*>(p.tile_list)[T];
  pt.s = e.x; pt.mb = e.y; pt.nb = e.z; pt.nsw = e.w;
  return 1;
}

__device__ __forceinline__ void post_ticket(const GroupedGemmParams& p, int pair, int k, unsigned long long epoch,
                                            bool has_tile, const PairTile& pt) {
  unsigned long long* slot = p.pair_tickets + 2LL * ((long long)pair * kPairTicketRing + (k & (kPairTicketRing - 1)));
  if (has_tile) slot[1] = pack_tile(pt);
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(slot),
               "l"(ring_tag(epoch, k) | (has_tile ? 0ULL : (unsigned long long)kNoTicket)) : "memory");
}

// Partner producer / epilogue: tile k of the pair from the ring.  1: tile in
// pt; 0: no more tiles; -1: the wait ran out (status recorded).
__device__ __forceinline__ int read_ticket(const GroupedGemmParams& p, int pair, int k, unsigned long long epoch,
                                           PairTile& pt, int kernel_id) {
  const unsigned long long* slot =
      p.pair_tickets + 2LL * ((long long)pair * kPairTicketRing + (k & (kPairTicketRing - 1)));
  const unsigned long long tag = ring_tag(epoch, k);
  const uint64_t start = globaltimer_ns();
  for (uint32_t polls = 1;; ++polls) {
    const unsigned long long v = ld_acquire_gpu_u64_gg(slot);
    if ((v & ~0xfffffULL) == tag) {
      if ((unsigned int)(v & 0xfffffULL) == kNoTicket) return 0;
      pt = unpack_tile(slot[1]);
      return 1;
    }
    __nanosleep(32);
    if ((polls & 63u) == 0) {
      if (globaltimer_ns() - start > p.timeout_ns) {
        record_status(p.status, kTimeoutPipeline, kernel_id, k, pair);
        return -1;
      }
      if (status_failed(p.status)) return -1;
    }
  }
}

__device__ __forceinline__ void store1(float* dst, float v) { *dst = v; }
__device__ __forceinline__ void store1(__nv_bfloat16* dst, float v) { *dst = __float2bfloat16_rn(v); }

// Epilogue of a swapped tail tile.  The accumulator holds output features in
// TMEM lanes (this CTA's 128 of the tile's 256: column nb * BN + feat for the
// calling thread) and the tail's tokens in TMEM columns [0, nsw).  Warps ew
// and ew + 4 split the token columns; for each token the warp's 32 lanes store
// 32 consecutive features of that token's output row.
template <int BN, Act ACT, typename OutT>
__device__ __forceinline__ void gemm_epilogue_swapped(const GroupedGemmParams& p, const GemmSegment& seg,
                                                      const PairTile& pt, int feat, uint32_t t_row, int ew) {
  const int lane = threadIdx.x & 31;
  int c0, c1;
  epi_columns(ew, pt.nsw, c0, c1);
  const int row0 = pt.mb * 256;       // first segment row of the tail tile
  const int rem = seg.rows - row0;    // its valid tokens
  OutT* out = (OutT*)p.out_ptrs[seg.out_slot];
  const int col = pt.nb * BN + feat;
  const float b = p.bias ? __ldg(p.bias + (long long)seg.expert * p.N + col) : 0.f;
#pragma unroll 1
  for (int c = c0; c < c1; c += 16) {
    uint32_t r[16];
    tmem_ld16(t_row + c, r);
    // lanes 0..15 fetch the output row and scale of tokens c .. c + 15
    const int tok = c + (lane & 15);
    long long orow = 0;
    float sc = 1.f;
    if (tok < rem) {
      const int arow = seg.a_row0 + row0 + tok;
      orow = p.row_map ? (long long)__ldg(p.row_map + arow) : (long long)(seg.out_row0 + row0 + tok);
      if (p.row_scale) sc = __ldg(p.row_scale + arow);
    }
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const long long o = __shfl_sync(0xffffffffu, orow, j);
      const float sj = __shfl_sync(0xffffffffu, sc, j);
      if (c + j < rem) store1(out + o * p.ldo + col, apply_act(__uint_as_float(r[j]) + b, ACT) * sj);
    }
  }
}

template <int BN, bool TF32, typename OutT = float>
struct PairCfg {
  static constexpr int BM = 128;                  // rows per CTA; the pair's tile has 256
  static constexpr int BNH = BN / 2;              // B rows staged per CTA
  static constexpr int ELEM = TF32 ? 4 : 2;
  static constexpr int BK = 128 / ELEM;
  static constexpr int UK = 32 / ELEM;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BNH * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // staging tiles of the eight epilogue warps (coalesced stores), behind the ring
  static constexpr int EPI_BYTES = kEpiWarps * EpiTile<OutT>::BYTES;
  static constexpr int SMEM_BUDGET = 224 * 1024 - EPI_BYTES;
  static constexpr int STAGES_RAW = SMEM_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int TMEM_COLS = (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64 : (2 * BN) <= 128 ? 128 : (2 * BN) <= 256 ? 256 : 512;
  static constexpr uint32_t IDESC = umma_idesc(TF32 ? 2u : 1u, 256, BN);
  static constexpr int SMEM_TOTAL = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + 256 + 256;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "pair tile: BN/2 rows of B per CTA, N <= 256");
  static_assert(STAGES >= 2, "pipeline needs two stages");
};

template <int BN, bool TF32, Act ACT, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_a8,
                         const __grid_constant__ CUtensorMap tmap_b, GroupedGemmParams p) {
  using C = PairCfg<BN, TF32, OutT>;
  constexpr int kKernelId = 300 + BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* stage_base = smem;
  uint8_t* epi_base = smem + C::STAGES * C::STAGE_BYTES;  // epilogue staging tiles
  uint64_t* bars = (uint64_t*)(epi_base + C::EPI_BYTES);
  uint64_t* full_bar = bars;                   // used in the leader only
  uint64_t* empty_bar = bars + C::STAGES;      // per CTA: stage free again
  uint64_t* tfull_bar = bars + 2 * C::STAGES;  // per CTA: accumulator ready
  uint64_t* tempty_bar = tfull_bar + 2;        // leader: accumulator drained by both CTAs
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = (uint32_t*)(drain_bar + 1);
  // progressive: the leader producer's tile slots for its MMA warp (16 bytes each, 256 bytes in all)
  int4* tile_slot = (int4*)(epi_base + C::EPI_BYTES + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full_bar[s], 1); mbar_init(&empty_bar[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull_bar[a], 1); mbar_init(&tempty_bar[a], 2 * kEpiWarps); }
    mbar_init(drain_bar, 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (p.tail_prefix != nullptr) tma_prefetch_desc(&tmap_a8);
  }
  if (warp == 1) { tmem_alloc_pair(tmem_slot, C::TMEM_COLS); tmem_relinquish_pair(); }
  tc_fence_before_sync();
  cluster_sync_all();  // barrier inits and the TMEM allocation are visible to the partner
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // Prologue: shared memory, TMEM and the partner only; the tile table,
  // segments and A rows come from the previous launch.  A progressive GEMM
  // does not wait for the planner to finish: it takes tiles as they are
  // published (the ticket protocol above).
  const bool progressive = p.progressive != 0;
  if (!progressive) griddep_wait();
  griddep_launch_dependents();
  if (p.trace != nullptr && threadIdx.x == 0) atomicMin(&p.trace->t_start, (unsigned long long)globaltimer_ns());
  const unsigned long long epoch = progressive ? *p.epoch : 0ULL;

  // Swapped tail tiles need the weights to fill the 256-row operand: BN = 256.
  const bool swapping = BN == 256 && ACT != Act::kSwiGLU && (p.tail_prefix != nullptr || progressive);
  const int total_full = progressive ? 0 : p.tile_prefix[p.num_segs];
  const int total_tiles = progressive ? 0 : total_full + (swapping ? p.tail_prefix[p.num_segs] : 0);
  const int nblocks = p.N / BN;
  const int kblocks = (p.K + C::BK - 1) / C::BK;
  const uint64_t lim = p.timeout_ns;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one_sync()) {
      int stage = 0; uint32_t phase = 0;
      // progressive leader: the current tile (resolved) and the ticket drawn for the next one
      PairTile cur{0, 0, 0, 0};
      int have = 0;
      if (progressive && rank == 0) {
        const unsigned int T0 = atomicAdd(p.ticket_counter, 1u) & 0xfffffu;
        have = resolve_ticket(p, T0, epoch, cur, kKernelId, pair);
        post_ticket(p, pair, 0, epoch, have > 0, cur);
      }
      for (int t = pair, k = 0;; t += npairs, ++k) {
        PairTile pt;
        unsigned int next_ticket = 0;
        if (progressive) {
          if (rank == 0) {
            if (have <= 0) {
              // no more tiles: complete the next stage's phase without data so the
              // MMA warp, which reads the tile slot behind that barrier, learns it
              tile_slot[k & (kTileSlots - 1)] = make_int4(0, 0, 0, -1);
              if (mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.status, kKernelId, lim))
                mbar_arrive(&full_bar[stage]);
              break;
            }
            pt = cur;
            next_ticket = atomicAdd(p.ticket_counter, 1u) & 0xfffffu;  // drawn a tile ahead
          } else if (read_ticket(p, pair, k, epoch, pt, kKernelId) <= 0) {
            break;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");  // rows landed by generic stores, read by TMA
        } else {
          if (t >= total_tiles) break;
          pt = pair_tile(p, t, total_full, nblocks);
        }
        const GemmSegment seg = p.segs[pt.s];
        // a swapped tile's tokens are the N operand: each CTA stages half of them
        const int arow = seg.a_row0 + pt.mb * 2 * C::BM + (int)rank * (pt.nsw ? pt.nsw / 2 : C::BM);
        const int brow = seg.expert * p.N + pt.nb * BN + (int)rank * C::BNH;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.status, kKernelId, lim)) { ok = false; break; }
          uint8_t* sa = stage_base + stage * C::STAGE_BYTES;
          // a swapped tile stages only its nsw / 2 token rows per CTA (8-row boxes,
          // each one 1024-byte swizzle atom)
          if (rank == 0) {
            // the MMA warp reads the tile behind the first stage's barrier (its arrive releases the slot)
            if (progressive && kb == 0) tile_slot[k & (kTileSlots - 1)] = make_int4(pt.s, pt.mb, pt.nb, pt.nsw);
            mbar_arrive_expect_tx(&full_bar[stage], pt.nsw ? 2 * C::B_BYTES + pt.nsw * 128 : 2 * C::STAGE_BYTES);
          }
          const uint32_t leader_full = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (pt.nsw) {
            for (int j = 0; j < pt.nsw / 16; ++j)
              tma_load_2d_pair(sa + j * 1024, &tmap_a8, leader_full, kb * C::BK, arow + j * 8);
          } else {
            tma_load_2d_pair(sa, &tmap_a, leader_full, kb * C::BK, arow);
          }
          tma_load_2d_pair(sa + C::A_BYTES, &tmap_b, leader_full, kb * C::BK, brow);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (progressive && rank == 0) {
          // resolve the ticket drawn above while this tile's loads are in flight
          have = ok ? resolve_ticket(p, next_ticket, epoch, cur, kKernelId, pair) : -1;
          post_ticket(p, pair, k + 1, epoch, have > 0, cur);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && elect_one_sync()) {
      int stage = 0; uint32_t phase = 0; int iter = 0;
      for (int t = pair;; t += npairs, ++iter) {
        int nsw = 0;
        if (progressive) {
          // the tile's first stage (or an empty phase at the end) carries its slot
          if (!mbar_wait_bounded(&full_bar[stage], phase, p.status, kKernelId, lim)) break;
          const int4 ts = tile_slot[iter & (kTileSlots - 1)];
          if (ts.w < 0) break;
          nsw = ts.w;
        } else {
          if (t >= total_tiles) break;
          nsw = t < total_full ? 0 : pair_tile(p, t, total_full, nblocks).nsw;
        }
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1u, p.status, kKernelId, lim)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        // swapped tail: weights (the B stage) are the M = 256 operand, tokens N = nsw
        const uint32_t idesc = nsw ? umma_idesc(TF32 ? 2u : 1u, 256, (uint32_t)nsw) : C::IDESC;
        const uint32_t swap_off = nsw ? (uint32_t)C::A_BYTES : 0u;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, p.status, kKernelId, lim)) { ok = false; break; }
          tc_fence_after_sync();
          const uint32_t stage_addr = smem_u32(stage_base + stage * C::STAGE_BYTES);
          const uint32_t a_addr = stage_addr + swap_off;
          const uint32_t b_addr = stage_addr + (C::A_BYTES - swap_off);
#pragma unroll
          for (int k = 0; k < C::BK / C::UK; ++k) {
            const uint64_t ad = umma_desc_k_sw128(a_addr + k * 32);
            const uint64_t bd = umma_desc_k_sw128(b_addr + k * 32);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (TF32) umma_tf32_pair(d_tmem, ad, bd, idesc, accum);
            else umma_f16_pair(d_tmem, ad, bd, idesc, accum);
          }
          const uint32_t eb = smem_u32(&empty_bar[stage]);
          umma_commit_pair(mapa_shared(eb, 0));
          umma_commit_pair(mapa_shared(eb, 1));
          if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        const uint32_t tb = smem_u32(&tfull_bar[acc]);
        umma_commit_pair(mapa_shared(tb, 0));
        umma_commit_pair(mapa_shared(tb, 1));
      }
      // Drain: every MMA issued above has completed before TMEM is freed.
      umma_commit_pair(mapa_shared(smem_u32(drain_bar), 0));
      mbar_wait_bounded(drain_bar, 0, p.status, kKernelId, lim);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int c0, c1;
    epi_columns(warp - 2, ACT == Act::kSwiGLU ? BN / 2 : BN, c0, c1);
    int iter = 0;
    for (int t = pair;; t += npairs, ++iter) {
      PairTile pt;
      if (progressive) {
        int r = 0;
        if (lane == 0) r = read_ticket(p, pair, iter, epoch, pt, kKernelId);
        r = __shfl_sync(0xffffffffu, r, 0);
        if (r <= 0) break;
        pt.s = __shfl_sync(0xffffffffu, pt.s, 0);
        pt.mb = __shfl_sync(0xffffffffu, pt.mb, 0);
        pt.nb = __shfl_sync(0xffffffffu, pt.nb, 0);
        pt.nsw = __shfl_sync(0xffffffffu, pt.nsw, 0);
        __syncwarp();  // orders lane 0's acquire before every lane's reads of the segment
      } else {
        if (t >= total_tiles) break;
        pt = pair_tile(p, t, total_full, nblocks);
      }
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      const GemmSegment seg = p.segs[pt.s];
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, p.status, kKernelId, lim)) break;
      tc_fence_after_sync();
      const int r_local = pt.mb * 2 * C::BM + (int)rank * C::BM + row_in_tile;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if constexpr (ACT == Act::kSwiGLU) {
        gemm_epilogue_row<BN, ACT, OutT>(p, seg, pt.nb, r_local, t_row, c0, c1);
      } else {
        if (pt.nsw)
          gemm_epilogue_swapped<BN, ACT, OutT>(p, seg, pt, (int)rank * C::BNH + row_in_tile, t_row, warp - 2);
        else
          gemm_epilogue_staged<BN, ACT, OutT>(p, seg, pt.nb, r_local, t_row, c0, c1,
                                              epi_base + (warp - 2) * EpiTile<OutT>::BYTES);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0));
    }
  }

  tc_fence_before_sync();
  cluster_sync_all();  // both CTAs finished every role before the pair frees TMEM or exits
  tc_fence_after_sync();
  if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  if (p.trace != nullptr && threadIdx.x == 0) {
    atomicMax(&p.trace->t_end, (unsigned long long)globaltimer_ns());
    atomicAdd(&p.trace->ctas, 1);
  }
}

template <int BN, bool TF32, Act ACT, typename OutT>
inline void launch_one_pair(const CUtensorMap& ta, const CUtensorMap& ta8, const CUtensorMap& tb,
                            const GroupedGemmParams& p, int grid, cudaStream_t stream) {
  using C = PairCfg<BN, TF32, OutT>;
  auto kern = grouped_gemm_pair_kernel<BN, TF32, ACT, OutT>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_TOTAL);
    configured = true;
  }
  const int g = grid & ~1;  // whole pairs
  launch_with_pdl(kern, dim3(g < 2 ? 2 : g), dim3(kGemmThreads), C::SMEM_TOTAL, stream, p.pdl != 0, ta, ta8, tb, p);
}

template <bool TF32, Act ACT, typename OutT>
inline void dispatch_bn_pair(int bn, const CUtensorMap& ta, const CUtensorMap& ta8, const CUtensorMap& tb,
                             const GroupedGemmParams& p, int grid, cudaStream_t stream) {
  switch (bn) {
    case 64: launch_one_pair<64, TF32, ACT, OutT>(ta, ta8, tb, p, grid, stream); return;
    case 128: launch_one_pair<128, TF32, ACT, OutT>(ta, ta8, tb, p, grid, stream); return;
    case 256: launch_one_pair<256, TF32, ACT, OutT>(ta, ta8, tb, p, grid, stream); return;
    default: break;
  }
  throw std::runtime_error("grouped_gemm (pair): unsupported BN " + std::to_string(bn));
}

template <bool TF32, typename OutT>
inline void dispatch_act_pair(int act, int bn, const CUtensorMap& ta, const CUtensorMap& ta8, const CUtensorMap& tb,
                              const GroupedGemmParams& p, int grid, cudaStream_t stream) {
  switch ((Act)act) {
    case Act::kNone: dispatch_bn_pair<TF32, Act::kNone, OutT>(bn, ta, ta8, tb, p, grid, stream); return;
    case Act::kRelu: dispatch_bn_pair<TF32, Act::kRelu, OutT>(bn, ta, ta8, tb, p, grid, stream); return;
    case Act::kGelu: dispatch_bn_pair<TF32, Act::kGelu, OutT>(bn, ta, ta8, tb, p, grid, stream); return;
    case Act::kSilu: dispatch_bn_pair<TF32, Act::kSilu, OutT>(bn, ta, ta8, tb, p, grid, stream); return;
    case Act::kSwiGLU: dispatch_bn_pair<TF32, Act::kSwiGLU, OutT>(bn, ta, ta8, tb, p, grid, stream); return;
  }
  throw std::runtime_error("grouped_gemm (pair): unknown activation");
}

}  // namespace raiccl
