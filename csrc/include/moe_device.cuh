// Device building blocks of the progressive MoE data plane, shared by the
// one-launch-per-step kernels (csrc/kernels/moe_dataplane.cu) and the
// persistent front-end kernel (csrc/kernels/moe_frontend.cu):
//   * identity-checksum arithmetic mod 2^63 - 25;
//   * router_token  — one warp routes one token (logits, mask, stable top-k, gates,
//                     the finish lane-parallel over experts);
//   * dispatch_rows — one CTA packs and stores its share of a revealed
//                     descriptor's rows into the owners' receive regions;
//   * dispatch_publish — the last CTA of a descriptor publishes its per-expert
//                     counts and the per-destination ready words.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "moe_kernels.h"
#include "sm100_ptx.cuh"

namespace raiccl {

// Identity checksum coefficients c_0..c_7 (the reference's RouterAssignment
// checksum, rlccl/transport/reference_a2av.py:20-29); one copy per unit.
static __constant__ unsigned long long c_checksum_coeff[8] = {1000003ULL, 1000033ULL, 1000037ULL, 1000081ULL,
                                                             1000099ULL, 1000117ULL, 1000121ULL, 1000133ULL};

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

// splitmix64 finaliser (Steele, Lea & Flood 2014 / Vigna), used as the word
// mixer of the order-dependent row digest.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t addmod(uint64_t a, uint64_t b) {
  uint64_t s = a + b;  // a, b < M < 2^63: no overflow
  return s >= kChecksumModulus ? s - kChecksumModulus : s;
}

// x mod M for M = 2^63 - 25 and any 64-bit x, from 2^63 = M + 25:
// x = h * 2^63 + l (h <= 1) is congruent to l + 25 h < 2M.
__device__ __forceinline__ uint64_t mod_m(uint64_t x) {
  const uint64_t r = (x & ((1ULL << 63) - 1)) + (x >> 63) * 25ULL;
  return r >= kChecksumModulus ? r - kChecksumModulus : r;
}

// (v mod M) * c mod M for a coefficient c < 2^32 (the identity coefficients are
// about 10^6), without 128-bit division: with a = v mod M < 2^63 the product
// a * c = hi * 2^64 + lo has hi < 2^32, and 2^64 = 2M + 50, so it is congruent
// to (lo mod M) + 50 hi < M + 2^38 < 2M.
__device__ __forceinline__ uint64_t mulmod_coeff(uint64_t v, uint64_t c) {
  const uint64_t a = mod_m(v);
  const uint64_t lo = a * c;
  const uint64_t hi = __umul64hi(a, c);
  const uint64_t r = mod_m(lo) + hi * 50ULL;
  return r >= kChecksumModulus ? r - kChecksumModulus : r;
}

// Row digest (sum_i splitmix64((i << 32) | w_i) mod 2^64 over the row's 32-bit
// words, masked to 62 bits); moe_feature_digest_kernel computes the same value.
// Token rows are read through L2 only (ld.global.cg) everywhere in the front
// end: with streamed inputs they land while the launch is running, so the
// non-coherent read-only path must not be used for them.

// Digest terms of the four 32-bit words of 16-byte vector v of a row.
__device__ __forceinline__ uint64_t digest_vec(uint4 x, int v) {
  const uint64_t i = (uint64_t)(4 * v);
  return splitmix64((i << 32) | x.x) + splitmix64(((i + 1) << 32) | x.y) + splitmix64(((i + 2) << 32) | x.z) +
         splitmix64(((i + 3) << 32) | x.w);
}

// The digest of one row of nvec 16-byte vectors, by one warp; every lane returns it.
__device__ __forceinline__ long long warp_row_digest(const uint4* row, int nvec) {
  const int lane = threadIdx.x & 31;
  constexpr int U = 8;  // loads in flight per lane
  uint64_t acc = 0;
  for (int v0 = 0; v0 < nvec; v0 += 32 * U) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = v0 + u * 32 + lane;
      x[u] = v < nvec ? __ldcg(row + v) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = v0 + u * 32 + lane;
      if (v < nvec) acc += digest_vec(x[u], v);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return (long long)(acc & ((1ULL << 62) - 1));
}

// identity_checksum(token, src, 0, 0, chunk, chunk_offset, position, digest):
// the destination and expert terms are added per assignment at dispatch time
// (the checksum is linear in every field).
__device__ __forceinline__ long long token_checksum_base(long long token_id, int rank, int chunk, int chunk_pos,
                                                         int t, long long digest) {
  const uint64_t fields[8] = {(uint64_t)token_id, (uint64_t)rank, 0, 0, (uint64_t)chunk, (uint64_t)chunk_pos,
                              (uint64_t)t, (uint64_t)digest};
  uint64_t acc = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc = addmod(acc, mulmod_coeff(fields[i], c_checksum_coeff[i]));
  return (long long)acc;
}

constexpr int kRouterUnroll = 8;
constexpr int kDispatchMaxItems = 4096;
constexpr int kMaxExperts = 256;
constexpr int kDispatchMaxChunks = 128;  // chunk-offset table staged in shared memory

// Order of the router's top-k candidates: rank 2 (a number) above rank 1
// (NaN) above rank 0 (no candidate: an id >= E, or already chosen); numbers
// by value; equal values, and equal ranks below 2, by the smaller expert id.
__device__ __forceinline__ bool router_better(int ra, float va, int ea, int rb, float vb, int eb) {
  if (ra != rb) return ra > rb;
  if (ra == 2 && va != vb) return va > vb;
  return ea < eb;
}

// Warp-parallel finish of token t; every lane holds every expert's raw dot
// product in acc.  Lane e takes expert e (and e + 32 when EMAX is 64): logit =
// raw + bias + chunk bias, -inf when masked.  Top-k is k rounds of a warp
// arg-max in router_better's order (a strict total order, so every lane of
// the butterfly agrees); lane j keeps choice j and writes its expert id, its
// count in sel_counts (shared, or nullptr) and its gate per gate_mode.
template <int EMAX>
__device__ __forceinline__ void router_finish_warp(const RouterParams& p, const float* chunk_bias, int t,
                                                   const float (&acc)[EMAX], int* sel_counts) {
  constexpr int PER = EMAX > 32 ? 2 : 1;
  const int E = p.experts, k = p.top_k, lane = threadIdx.x & 31;
  const float ninf = -__int_as_float(0x7f800000);
  float v[PER];
  int rank[PER];
#pragma unroll
  for (int h = 0; h < PER; ++h) {
    const int e = lane + 32 * h;
    float raw = 0.f;
#pragma unroll
    for (int i = 32 * h; i < EMAX && i < 32 * h + 32; ++i)
      if (i == e) raw = acc[i];
    if (e < E) {
      const float l = raw + __ldg(p.bias + e) + (chunk_bias ? chunk_bias[e] : 0.f);
      const bool masked = (p.mask_mode == 1 && e == (t % E)) || (p.block_mask && __ldg(p.block_mask + e));
      v[h] = masked ? ninf : l;
      rank[h] = v[h] == v[h] ? 2 : 1;
    } else {
      v[h] = ninf;
      rank[h] = 0;
    }
  }
  float l0 = 0.f, my_l = ninf;
  int my_e = -1;
#pragma unroll 1
  for (int j = 0; j < k; ++j) {
    float bv = v[0];
    int br = rank[0], be = lane;
    if (PER == 2 && router_better(rank[PER - 1], v[PER - 1], lane + 32, br, bv, be)) {
      bv = v[PER - 1];
      br = rank[PER - 1];
      be = lane + 32;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int orank = __shfl_xor_sync(0xffffffffu, br, o), oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (router_better(orank, ov, oe, br, bv, be)) {
        bv = ov;
        br = orank;
        be = oe;
      }
    }
    if ((be & 31) == lane) rank[be >> 5] = 0;  // chosen: out of the later rounds
    if (lane == j) {
      my_e = be;
      my_l = bv;
    }
    if (j == 0) l0 = bv;
  }
  float sum = 1.f;
  if (p.gate_mode != 0) {
    float part = 0.f;
    if (p.gate_mode == 1) {
      if (lane < k) part = __expf(my_l - l0);
    } else {
#pragma unroll
      for (int h = 0; h < PER; ++h)
        if (lane + 32 * h < E && v[h] != ninf) part += __expf(v[h] - l0);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    sum = part;
  }
  if (lane < k) {
    p.expert_ids[(long long)t * k + lane] = my_e;
    if (sel_counts) atomicAdd(&sel_counts[my_e], 1);
    p.gates[(long long)t * k + lane] = p.gate_mode == 0 ? 1.f : __expf(my_l - l0) / sum;
  }
}

// ---------------------------------------------------------------------------
// Router of one token (warp collective): logits = x_t . W_e + b_e (+ chunk
// bias), masked experts -inf, stable descending top-k (the smaller expert id
// wins ties), gates per gate_mode; writes expert_ids / gates of row t and
// counts the choices in sel_counts (shared, or nullptr).  x: the token's row,
// in shared memory (x_shared) or in global memory.  SMEM_W: w points at a
// shared-memory copy of the weights.  Every lane sums its vectors in row
// order, then a butterfly adds the lanes (every lane ends with the same sums):
// the same order wherever the row comes from.
// ---------------------------------------------------------------------------
template <typename T, int EMAX, bool SMEM_W>
__device__ __forceinline__ void router_token(const RouterParams& p, const float* chunk_bias, int t, const T* x,
                                             bool x_shared, const T* __restrict__ w, int* sel_counts,
                                             unsigned long long* dbg = nullptr) {
  const int D = p.hidden, E = p.experts;
  const int lane = threadIdx.x & 31;
  constexpr int VEC = 16 / sizeof(T);
  float acc[EMAX];
#pragma unroll
  for (int e = 0; e < EMAX; ++e) acc[e] = 0.f;
  constexpr int STEP = 32 * VEC * kRouterUnroll;
  for (int base0 = 0; base0 < D; base0 += STEP) {
    uint4 xr[kRouterUnroll];
#pragma unroll
    for (int u = 0; u < kRouterUnroll; ++u) {
      const int base = base0 + (u * 32 + lane) * VEC;
      // a row in shared memory, or in global memory read through L2 only
      // (streamed rows land while the launch runs)
      xr[u] = base >= D  ? make_uint4(0, 0, 0, 0)
              : x_shared ? *(const uint4*)(x + base)
                         : __ldcg((const uint4*)(x + base));
    }
#pragma unroll
    for (int u = 0; u < kRouterUnroll; ++u) {
      const int base = base0 + (u * 32 + lane) * VEC;
      if (base >= D) break;
      const T* xv = (const T*)&xr[u];
#pragma unroll
      for (int e = 0; e < EMAX; ++e) {
        if (e < E) {
          uint4 wr;
          if constexpr (SMEM_W) wr = *(const uint4*)(w + (long long)e * D + base);
          else wr = __ldg((const uint4*)(w + (long long)e * D + base));
          const T* wv = (const T*)&wr;
          float s = 0.f;
#pragma unroll
          for (int v = 0; v < VEC; ++v) s = fmaf(to_f(xv[v]), to_f(wv[v]), s);
          acc[e] += s;
        }
      }
    }
  }
  // dbg (diagnostics, lane 0): %globaltimer after the products and after the finish
  if (dbg != nullptr && lane == 0) dbg[0] = globaltimer_ns();
#pragma unroll
  for (int e = 0; e < EMAX; ++e) {
    if (e < E) {
      float v = acc[e];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[e] = v;
    }
  }
  router_finish_warp<EMAX>(p, chunk_bias, t, acc, sel_counts);
  if (dbg != nullptr && lane == 0) dbg[1] = globaltimer_ns();
}

// ---------------------------------------------------------------------------
// One CTA's share [a, b) of a descriptor whose tokens start at t0: rows keep
// the reference's deterministic order inside every (expert, source) region,
// descriptor order then token order, so the row of item i (token t, choice j,
// expert e) is base[e] + (items of expert e in [t0, a)) + (its in-order
// rank inside [a, b)).  hist / run must be zero on entry (E entries); on
// return run[e] holds this share's item count per expert.  Collective over the
// CTA (contains __syncthreads); the caller checks (b - a) * k <= kDispatchMaxItems.
// ---------------------------------------------------------------------------
// Index part of dispatch_rows: hist[e] = items of expert e in [t0, a), and
// item_pos[i - a k] = (in-order rank within its expert in [a, b)) | expert << 24.
// Reads only the routed expert ids, so it may run before the descriptor is
// released once its chunks are complete.  hist / run zero on entry.
__device__ inline void dispatch_index(const DispatchParams& p, int t0, int a, int b, int* hist, int* run, int* item_pos) {
  const MoEDims& d = p.dims;
  const int k = d.top_k;
  const int E = d.experts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  // rows of earlier tokens of this descriptor per expert: lanes holding the
  // same expert elect one leader that adds the group's size (one shared-memory
  // atomic per distinct expert per warp instead of one per item)
  {
    // UH independent loads in flight per lane before the matches (the scan is
    // latency-bound: one round trip per UH x 32 items per warp)
    // warps 1.. scan while warp 0 ranks the share's own items below
    constexpr int UH = 8;
    const long long i_end = (long long)a * k;
    const int hw = nwarps > 1 ? nwarps - 1 : 1, hwarp = nwarps > 1 ? warp - 1 : warp;
    const long long stride = (long long)hw * 32;
    for (long long i0 = (long long)t0 * k + (long long)hwarp * 32; hwarp >= 0 && i0 < i_end; i0 += stride * UH) {
      int ev[UH];
#pragma unroll
      for (int u = 0; u < UH; ++u) {
        const long long i = i0 + u * stride + lane;
        ev[u] = i < i_end ? p.expert_ids[i] : E;  // sentinel groups the tail lanes
      }
#pragma unroll
      for (int u = 0; u < UH; ++u) {
        const unsigned peers = __match_any_sync(0xffffffffu, ev[u]);
        if (ev[u] < E && lane == __ffs(peers) - 1) atomicAdd(&hist[ev[u]], __popc(peers));
      }
    }
  }
  // in-order rank of every item of this share within its expert (run is
  // this share's own counter, so it does not race with the scan above)
  if (warp == 0) {
    const long long i0 = (long long)a * k, i1 = (long long)b * k;
    for (long long base = i0; base < i1; base += 32) {
      const long long i = base + lane;
      const bool valid = i < i1;
      const int e = valid ? p.expert_ids[i] : E;  // sentinel groups the tail lanes
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank_in = __popc(peers & ((1u << lane) - 1u));
      const int prev = valid ? run[e] : 0;
      if (valid) item_pos[i - i0] = (prev + rank_in) | (e << 24);  // rank (< 2^24 rows) and expert (< 256)
      __syncwarp();
      if (valid && lane == __ffs(peers) - 1) run[e] = prev + __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
}

// Staging area for dispatch_rows: the share's token rows come into shared
// memory by bulk copies (two halves, double-buffered), so all of a half's
// bytes are in flight at once, and go out with plain 16-byte stores.
struct DispatchStage {
  uint8_t* buf;      // shared memory, 16-byte aligned
  int bytes;         // size of buf (two halves)
  uint64_t* bar;     // [2] mbarriers, initialised with count 1
  uint32_t* uses;    // [2] completed phases of each barrier (shared)
  unsigned long long timeout_ns;  // bound of each wait for a half
};

// Identity inputs of share [a, b) (token id, digest and checksum base per
// token, the gate per item) into the head of the staging buffer, when they
// fit a quarter of it; returns whether they were staged.  Reads only what the
// router wrote, so it may run before the descriptor is released once its
// chunks are complete.  Collective over the CTA (ends with a barrier).
__device__ inline bool dispatch_stage_ids(const DispatchParams& p, int a, int b, const DispatchStage* stage) {
  const int k = p.dims.top_k;
  const long long ntok = b > a ? b - a : 0, nitems = ntok * k;
  const long long id_bytes = (ntok * 24 + nitems * 4 + 15) & ~15LL;
  if (stage == nullptr || ntok == 0 || id_bytes > stage->bytes / 4) return false;
  long long* s_tid = reinterpret_cast<long long*>(stage->buf);
  long long* s_dig = s_tid + ntok;
  long long* s_csb = s_dig + ntok;
  float* s_gate = reinterpret_cast<float*>(s_csb + ntok);
  for (long long i = threadIdx.x; i < ntok; i += blockDim.x) {
    s_tid[i] = p.token_ids[a + i];
    s_dig[i] = p.feat_digest[a + i];
    s_csb[i] = p.checksum_base[a + i];
  }
  if (p.dims.gate_mode)
    for (long long i = threadIdx.x; i < nitems; i += blockDim.x) s_gate[i] = p.gates[(long long)a * k + i];
  __syncthreads();
  return true;
}

// indexed: hist / run / item_pos already hold dispatch_index's result.
// stage (optional): stage rows through shared memory (see DispatchStage).
// ids_ready: dispatch_stage_ids already staged the identity inputs.
template <typename T>
__device__ void dispatch_rows(const DispatchParams& p, int t0, int a, int b, const int* base_e, int* hist, int* run,
                              int* item_pos, const int* s_coff, int nc, bool streamed = false, bool indexed = false,
                              const DispatchStage* stage = nullptr, unsigned long long* dbg = nullptr,
                              bool ids_ready = false) {
  // dbg (diagnostics, thread 0): %globaltimer after the index part, the
  // identity rows and the staged feature rows
  auto stamp = [&](int i) {
    if (dbg != nullptr && threadIdx.x == 0) dbg[i] = globaltimer_ns();
  };
  const MoEDims& d = p.dims;
  const int k = d.top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  if (!indexed) dispatch_index(p, t0, a, b, hist, run, item_pos);
  stamp(0);
  const long long nitems = (long long)(b - a) * k;
  const long long row_bytes = (long long)d.hidden * d.feat_bytes;
  const int vec_per_row = (int)(row_bytes / 16);
  // staging layout: the share's identity inputs (token id, digest and
  // checksum base per token, the gate per item) when they fit a quarter of
  // the buffer, then two halves of token rows; the first half's copy is
  // issued before the identity rows so that it is in flight while they are
  // written
  const long long ntok = b > a ? b - a : 0;
  const long long id_bytes = (ntok * 24 + nitems * 4 + 15) & ~15LL;
  const bool stage_ids = stage != nullptr && ntok > 0 && id_bytes <= stage->bytes / 4;
  long long* s_tid = stage_ids ? reinterpret_cast<long long*>(stage->buf) : nullptr;
  long long* s_dig = s_tid + ntok;
  long long* s_csb = s_dig + ntok;
  float* s_gate = reinterpret_cast<float*>(s_csb + ntok);
  uint8_t* rows_buf = stage ? stage->buf + (stage_ids ? id_bytes : 0) : nullptr;
  const int half_rows = stage ? (int)(((stage->bytes - (stage_ids ? id_bytes : 0)) / 2) / row_bytes) : 0;
  const bool staged = half_rows > 0 && b > a;
  auto issue_half = [&](int h, int tb) {  // thread 0: tokens [tb, tb + rows) into half h
    const int rows = min(half_rows, b - tb);
    const uint32_t bytes = (uint32_t)(rows * row_bytes);
    fence_proxy_async_global();  // rows written by generic stores or the copy engine, read by the bulk copy
    mbar_arrive_expect_tx(&stage->bar[h], bytes);
    bulk_load_g2s(rows_buf + (long long)h * half_rows * row_bytes,
                  (const uint8_t*)p.tokens + (long long)tb * row_bytes, bytes, &stage->bar[h]);
  };
  if (staged && threadIdx.x == 0) {
    issue_half(0, a);
    if (a + half_rows < b) issue_half(1, a + half_rows);
  }
  if (stage_ids && !ids_ready) dispatch_stage_ids(p, a, b, stage);  // one round trip for every item's inputs
  stamp(3);
  // identity rows, one thread per item: its nine metadata words, its
  // return-row index and its gate (an item whose row falls outside the
  // receive region records the status here and is skipped below).  A thread
  // works out the item's destination and chunk once, so the items of a share
  // are written side by side instead of one item per warp in turn.
  for (int li = threadIdx.x; li < (int)nitems; li += blockDim.x) {  // nitems <= kDispatchMaxItems
    const int t = a + li / k, j = li % k;
    const int packed = item_pos[li];
    const int e = (int)((unsigned)packed >> 24);
    const int r = expert_owner(d, e), le = expert_slot(d, e);
    const long long row = (long long)base_e[e] + hist[e] + (packed & 0xFFFFFF);
    if (row >= d.cap || r >= d.world || le >= d.expert_slots) {
      record_status(p.status, kBoundsViolation, 21, row, d.cap);
      continue;
    }
    const long long grow = ((long long)le * d.world + d.rank) * d.cap + row;
    uint8_t* base = (uint8_t*)p.peers.base[r];
    const long long tid = stage_ids ? s_tid[t - a] : p.token_ids[t];
    const long long dig = stage_ids ? s_dig[t - a] : p.feat_digest[t];
    const long long csb = stage_ids ? s_csb[t - a] : p.checksum_base[t];
    const float gate = !d.gate_mode ? 1.f : stage_ids ? s_gate[li] : p.gates[(long long)a * k + li];
    // chunk of token t: the last c with offset[c] <= t, by bisection of the
    // staged offsets [0, nc]; global offsets only past the staged table
    int c = 0;
    for (int hi = nc; c < hi;) {
      const int mid = (c + hi + 1) >> 1;
      if (s_coff[mid] <= t) c = mid;
      else hi = mid - 1;
    }
    if (c == nc)
      while (c + 1 < d.chunks && p.chunk_offsets[c + 1] <= t) ++c;
    const int c_off = c <= nc ? s_coff[c] : p.chunk_offsets[c];
    uint64_t cs = (uint64_t)csb;
    cs = addmod(cs, mulmod_coeff((uint64_t)r, c_checksum_coeff[2]));
    cs = addmod(cs, mulmod_coeff((uint64_t)e, c_checksum_coeff[3]));
    long long* m = (long long*)(base + p.layout.recv_meta) + grow * kFwdMetaFields;
    m[0] = tid;
    m[1] = d.rank;
    m[2] = r;
    m[3] = e;
    m[4] = c;
    m[5] = t - c_off;
    m[6] = t;
    m[7] = dig;
    m[8] = (long long)cs;
    ((int*)(base + p.layout.recv_retrow))[grow] = t * k + j;
    ((float*)(base + p.layout.recv_gate))[grow] = gate;
  }
  stamp(1);
  if (staged) {
    // feature rows from shared memory: batch n holds tokens [a + n half_rows, ...)
    // in half n % 2; a warp stores one item (token, choice) at a time
    int n = 0;
    for (int tb = a; tb < b; tb += half_rows, ++n) {
      const int h = n & 1;
      const int rows = min(half_rows, b - tb);
      mbar_wait_bounded(&stage->bar[h], stage->uses[h] & 1u, p.status, 23, stage->timeout_ns);
      const uint4* sbase = (const uint4*)(rows_buf + (long long)h * half_rows * row_bytes);
      for (int li_b = warp; li_b < rows * k; li_b += nwarps) {
        const long long li = (long long)(tb - a) * k + li_b;
        const int packed = item_pos[li];
        const int e = (int)((unsigned)packed >> 24);
        const int r = expert_owner(d, e), le = expert_slot(d, e);
        const long long row = (long long)base_e[e] + hist[e] + (packed & 0xFFFFFF);
        if (row >= d.cap || r >= d.world || le >= d.expert_slots) continue;  // recorded above
        const long long grow = ((long long)le * d.world + d.rank) * d.cap + row;
        uint4* dst = (uint4*)((uint8_t*)p.peers.base[r] + p.layout.recv_feat + grow * row_bytes);
        const uint4* src = sbase + (long long)(li_b / k) * vec_per_row;
        for (int v = lane; v < vec_per_row; v += 32) dst[v] = src[v];
      }
      __syncthreads();  // every warp is done with this half
      if (threadIdx.x == 0) {
        stage->uses[h] += 1;
        if (tb + 2 * half_rows < b) issue_half(h, tb + 2 * half_rows);
      }
      __syncthreads();
    }
    stamp(2);
    return;
  }
  // feature rows: each warp copies two items at a time, eight 16-byte loads
  // per lane and item in flight before their stores (the item's source and
  // destination rows are worked out once per item, not per vector)
  constexpr int U = 8;
  auto row_ptrs = [&](long long li, const uint4*& src, uint4*& dst) -> bool {
    const long long i = (long long)a * k + li;
    const int t = (int)(i / k);
    const int packed = item_pos[li];
    const int e = (int)((unsigned)packed >> 24);
    const int r = expert_owner(d, e), le = expert_slot(d, e);
    const long long row = (long long)base_e[e] + hist[e] + (packed & 0xFFFFFF);
    if (row >= d.cap || r >= d.world || le >= d.expert_slots) return false;
    const long long grow = ((long long)le * d.world + d.rank) * d.cap + row;
    dst = (uint4*)((uint8_t*)p.peers.base[r] + p.layout.recv_feat + grow * row_bytes);
    src = (const uint4*)((const uint8_t*)p.tokens + (long long)t * row_bytes);
    return true;
  };
  for (long long la = warp; la < nitems; la += 2LL * nwarps) {
    const long long lb = la + nwarps;
    const uint4* sa = nullptr;
    const uint4* sb = nullptr;
    uint4* da = nullptr;
    uint4* db = nullptr;
    const bool oka = row_ptrs(la, sa, da);
    const bool okb = lb < nitems && row_ptrs(lb, sb, db);
    for (int v0 = 0; v0 < vec_per_row; v0 += 32 * U) {
      uint4 ra[U], rb[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * 32 + lane;
        // rows streamed in during the launch are read through L2 only; resident
        // rows through the read-only path (the second choice of a token hits L1)
        if (oka && v < vec_per_row) ra[u] = streamed ? __ldcg(sa + v) : __ldg(sa + v);
        if (okb && v < vec_per_row) rb[u] = streamed ? __ldcg(sb + v) : __ldg(sb + v);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * 32 + lane;
        if (oka && v < vec_per_row) da[v] = ra[u];
        if (okb && v < vec_per_row) db[v] = rb[u];
      }
    }
  }
}

// Last CTA of a descriptor: per-expert counts into every owner's header
// (optionally advancing sent_base), then one release store of the call's
// sequence number per destination rank (sent for zero rows too).  Ordering:
// every share's stores -> bar.sync -> the CTA's acq_rel increment of the
// descriptor counter; the last CTA's acquiring increment sees them all and
// its st.release.sys is cumulative, so a peer that acquires the ready word
// sees every row.
__device__ __forceinline__ void dispatch_publish(const DispatchParams& p, int desc, bool skip_signal,
                                                 unsigned long long epoch, bool update_sent_base) {
  const MoEDims& d = p.dims;
  const int E = d.experts;
  // bytes one forward row moves: features, identity row, return-row index, gate
  const unsigned long long row_bytes = (unsigned long long)d.hidden * d.feat_bytes + kFwdMetaFields * 8 + 4 + 4;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int cnt = atomicAdd(&p.desc_counts[(long long)desc * E + e], 0);
    const int r = expert_owner(d, e), le = expert_slot(d, e);
    uint8_t* base = (uint8_t*)p.peers.base[r];
    ((int*)(base + p.layout.recv_count))[((long long)le * d.world + d.rank) * d.n_desc + desc] = cnt;
    if (update_sent_base) p.sent_base[e] += cnt;
    if (p.peer_counters != nullptr)
      atomicAdd(p.peer_counters + (long long)r * kPeerCounterFields + kPcBytes, (unsigned long long)cnt * row_bytes + 4);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int r = 0; r < d.world && !skip_signal; ++r) {
      uint8_t* base = (uint8_t*)p.peers.base[r];
      st_release_sys_u64((uint64_t*)(base + p.layout.recv_flag) + (long long)d.rank * d.n_desc + desc, epoch);
    }
    if (p.peer_counters != nullptr)
      for (int r = 0; r < d.world; ++r) {
        unsigned long long* pc = p.peer_counters + (long long)r * kPeerCounterFields;
        atomicAdd(pc + kPcPutCalls, 1ULL);
        if (!skip_signal) atomicAdd(pc + kPcSignals, 1ULL);
      }
    p.done_counter[desc] = 0;
  }
}

}  // namespace raiccl
