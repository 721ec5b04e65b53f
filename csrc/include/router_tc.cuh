// Tensor-core router unit of the persistent front end (bf16 tokens and
// weights): the logits of up to 128 consecutive tokens of one router chunk
// against E <= 64 experts are one tcgen05 MMA tile, M = 128 tokens, N = E
// rounded up to 16, K = D in steps of 64 elements (one 128-byte swizzle row).
// TMA brings each K step's token tile (128 x 128 B) and weight tile
// (N x 128 B) into a ring of stages; one thread issues the loads and the
// MMAs; the fp32 accumulator stays in TMEM until the first four warps read it
// back, one thread per token, and finish the token: bias, chunk bias, mask,
// stable top-k and gates, the contract of the warp router (router_token) in
// moe_device.cuh.
//
// The reference's router is a dense fp32 matmul + top-k
// (rlccl/transport/reference_router.py:15-25); bf16 products are exact in
// fp32 and the MMA accumulates in fp32, so the routing differs from the warp
// router's only in the order of the fp32 additions.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "moe_device.cuh"
#include "moe_kernels.h"
#include "sm100_ptx.cuh"

namespace raiccl {

constexpr int kTcRows = 128;       // tokens per unit (the MMA's M)
constexpr int kTcBK = 64;          // bf16 elements per K step: one 128-byte swizzle row
constexpr int kTcMaxStages = 8;
constexpr int kTcSelStride = 8;    // candidates kept per token and half (top_k <= 8)
constexpr int kTcMaxE = 64;        // experts at most

// Per-CTA state.  n_load / n_mma count K steps over every unit this CTA
// routed (the issuing thread's copy is the one that matters); n_units counts
// units (every thread keeps the same count).
struct TcRouter {
  uint8_t* stages;     // 1024-aligned shared memory: n_stages x [tokens 128 x 128 B | weights npad x 128 B]
  float* lg;           // [npad, kTcRows] shared: the unit's logits, expert-major
  float* sel;          // shared: the finish's bias row, candidate lists and choices (tc_router_scratch_bytes)
  uint64_t* full;      // [n_stages] TMA bytes landed
  uint64_t* empty;     // [n_stages] the stage's MMAs completed
  uint64_t* done;      // the unit's MMAs completed
  uint32_t tmem;       // accumulator: 128 lanes x npad fp32 columns
  int n_stages, npad, kblocks;
  uint32_t n_load, n_mma, n_units;

  __device__ int stage_bytes() const { return kTcRows * 128 + npad * 128; }
};

// One thread: the TMA loads and MMAs of the unit whose first token row is
// row0; arrives on `done` once every MMA completed.  A stage is refilled one
// K step after its MMAs were committed, so the loads stay n_stages - 1 steps
// ahead without waiting on the MMAs just issued.  Bounded waits record the
// status and go on (the call then fails).
__device__ inline void tc_router_issue(TcRouter& s, const CUtensorMap* tx, const CUtensorMap* tw, int row0,
                                       DeviceStatus* st, int kid, unsigned long long lim) {
  const int S = s.n_stages, KB = s.kblocks;
  const uint32_t bytes = (uint32_t)s.stage_bytes();
  const uint32_t idesc = umma_idesc(1, kTcRows, (uint32_t)s.npad);
  fence_proxy_async_global();  // token rows published to this thread before the async-proxy reads
  fence_proxy_async_smem();    // stage memory last read by generic loads (dispatch staging)
  auto load = [&](int kb) {
    const uint32_t n = s.n_load++;
    const int stg = (int)(n % (uint32_t)S);
    const uint32_t use = n / (uint32_t)S;
    if (use > 0) mbar_wait_bounded(&s.empty[stg], (use - 1) & 1u, st, kid, lim);
    uint8_t* a = s.stages + stg * bytes;
    mbar_arrive_expect_tx(&s.full[stg], bytes);
    tma_load_2d(a, tx, &s.full[stg], kb * kTcBK, row0);
    tma_load_2d(a + kTcRows * 128, tw, &s.full[stg], kb * kTcBK, 0);
  };
  const int pre = KB < S ? KB : S;
#pragma unroll 1
  for (int kb = 0; kb < pre; ++kb) load(kb);
#pragma unroll 1
  for (int kb = 0; kb < KB; ++kb) {
    const uint32_t n = s.n_mma++;
    const int stg = (int)(n % (uint32_t)S);
    mbar_wait_bounded(&s.full[stg], (n / (uint32_t)S) & 1u, st, kid, lim);
    tc_fence_after_sync();
    const uint32_t a = smem_u32(s.stages + stg * bytes), b = a + kTcRows * 128;
#pragma unroll
    for (int k = 0; k < kTcBK / 16; ++k)
      umma_f16(s.tmem, umma_desc_k_sw128(a + k * 32), umma_desc_k_sw128(b + k * 32), idesc,
               (kb > 0 || k > 0) ? 1u : 0u);
    umma_commit(&s.empty[stg]);
    if (kb >= 1 && kb - 1 + S < KB) load(kb - 1 + S);
  }
  umma_commit(s.done);
}

// Sort key of a router candidate, larger = preferred: rank 2 (a number) above
// rank 1 (NaN) above 0 (no candidate); numbers by value (an order-preserving
// map of the float bits, -0 taken as +0); then the smaller expert id.  The
// same order as router_better, in one 64-bit compare.
__device__ __forceinline__ unsigned long long tc_router_key(float v, int e) {
  if (v != v) return (1ull << 40) | (unsigned long long)(255 - e);
  const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
  const uint32_t u = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (2ull << 40) | ((unsigned long long)u << 8) | (unsigned long long)(255 - e);
}

// Finish of the unit's tokens, every thread of the CTA: token r = threadIdx.x
// % 128 (warps w and w + 4 share TMEM lane quarter w % 4), half h =
// threadIdx.x / 128.  (1) The unit's bias row (bias + chunk bias, and the
// block mask) goes to shared memory; half h reads the 16-column groups c with
// c % 2 == h of its tokens' accumulator rows and stores the logits
// expert-major in shared memory (-inf when masked).  (2) Half h keeps the
// best k of the experts [h Eh, (h + 1) Eh), Eh = ceil(E / 2), as a sorted
// list of tc_router_key values, and its sum of exp(logit - its best) for
// softmax-over-all gates.  (3) Half 0 merges the two lists and writes the
// choices, their counts in sel_counts and the gates.  Rows >= nt belong to
// later tokens (or lie past the matrix) and are dropped.  This code runs a
// few times per launch, mostly from a cold instruction cache, so its loops
// stay rolled wherever the body is not a fixed-size register array.
template <int EMAX>
__device__ __noinline__ void tc_router_finish(const RouterParams& p, const float* chunk_bias, TcRouter& s, int tf,
                                              int nt, int* sel_counts, DeviceStatus* st, int kid,
                                              unsigned long long lim, unsigned long long* dbg = nullptr) {
  const int r = threadIdx.x & (kTcRows - 1), h = threadIdx.x >> 7;
  const int t = tf + r, E = p.experts, k = p.top_k;
  const bool valid = r < nt;
  const float ninf = -__int_as_float(0x7f800000);
  float* sb = s.sel;                                       // [E] bias + chunk bias
  int* sbm = reinterpret_cast<int*>(s.sel + kTcMaxE);      // [E] 1: masked for every token
  unsigned long long* lst = reinterpret_cast<unsigned long long*>(s.sel + 2 * kTcMaxE);  // [2][k][kTcRows]
  int* chosen = reinterpret_cast<int*>(lst + 2 * kTcSelStride * kTcRows);                 // [k][kTcRows]
  float* prt = reinterpret_cast<float*>(chosen + kTcSelStride * kTcRows);                 // [kTcRows]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    sb[e] = p.bias[e] + (chunk_bias ? chunk_bias[e] : 0.f);
    sbm[e] = p.block_mask ? (int)p.block_mask[e] : 0;
  }
  mbar_wait_bounded(s.done, s.n_units & 1u, st, kid, lim);
  __syncwarp();
  tc_fence_after_sync();
  if (dbg != nullptr && threadIdx.x == 0) *dbg = globaltimer_ns();  // diagnostics: the unit's MMAs completed
  __syncthreads();  // the bias row is in shared memory
  float* lg = s.lg + r;  // lg[e * kTcRows]: expert e's logit of token r
  const uint32_t taddr = s.tmem + ((uint32_t)(((threadIdx.x >> 5) & 3) * 32) << 16);
  const int tm = p.mask_mode == 1 ? t % E : -1;
#pragma unroll 1
  for (int c = h; c * 16 < s.npad; c += 2) {
    uint32_t raw[16];
    tmem_ld16(taddr + c * 16, raw);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int e = c * 16 + i;
      if (e < E && valid) lg[e * kTcRows] = (e == tm || sbm[e]) ? ninf : __uint_as_float(raw[i]) + sb[e];
    }
  }
  tc_fence_before_sync();
  __syncthreads();  // every logit of the unit is in shared memory
  const int eh = (E + 1) >> 1, e0 = h * eh, e1 = min(E, e0 + eh);
  unsigned long long key[kTcSelStride];
#pragma unroll
  for (int q = 0; q < kTcSelStride; ++q) key[q] = 0ull;
  float part = 0.f;
  if (valid) {
#pragma unroll 1
    for (int e = e0; e < e1; ++e) {
      const unsigned long long x = tc_router_key(lg[e * kTcRows], e);
      // insert x into the sorted list of the best k (slots >= k stay empty)
#pragma unroll
      for (int q = kTcSelStride - 1; q >= 0; --q) {
        if (q < k && x > key[q]) {
          if (q > 0) key[q] = x > key[q - 1] ? key[q - 1] : x;
          else key[q] = x;
        }
      }
    }
    if (p.gate_mode == 2 && key[0] != 0ull) {  // this half's softmax terms, relative to its best
      const float m = lg[(255 - (int)(key[0] & 0xFF)) * kTcRows];
#pragma unroll 1
      for (int e = e0; e < e1; ++e)
        if (lg[e * kTcRows] != ninf) part += __expf(lg[e * kTcRows] - m);
    }
    unsigned long long* mine = lst + h * kTcSelStride * kTcRows + r;
#pragma unroll
    for (int q = 0; q < kTcSelStride; ++q)
      if (q < k) mine[q * kTcRows] = key[q];
    if (h == 1) prt[r] = part;
  }
  __syncthreads();
  if (h != 0 || !valid) return;
  const unsigned long long* la = lst + r;
  const unsigned long long* lb = lst + kTcSelStride * kTcRows + r;
  const int nb = min(k, E - eh);  // entries of half 1's list
  int ia = 0, ib = 0;
  float l0 = 0.f, gsum = 0.f;
#pragma unroll 1
  for (int j = 0; j < k; ++j) {
    const unsigned long long a = ia < k ? la[ia * kTcRows] : 0ull;
    const unsigned long long b = ib < nb ? lb[ib * kTcRows] : 0ull;
    const unsigned long long x = a > b ? a : b;
    if (a > b) ++ia;
    else ++ib;
    const int e = 255 - (int)(x & 0xFF);
    const float v = lg[e * kTcRows];
    if (j == 0) l0 = v;
    chosen[j * kTcRows + r] = e;
    p.expert_ids[(long long)t * k + j] = e;
    if (sel_counts) atomicAdd(&sel_counts[e], 1);
    if (p.gate_mode == 1) gsum += __expf(v - l0);
  }
  if (p.gate_mode == 2) {  // both halves' parts, each rescaled from its own best to l0
    const unsigned long long k1 = nb > 0 ? lb[0] : 0ull;
    const float m0 = key[0] != 0ull ? lg[(255 - (int)(key[0] & 0xFF)) * kTcRows] : ninf;
    const float m1 = k1 != 0ull ? lg[(255 - (int)(k1 & 0xFF)) * kTcRows] : ninf;
    gsum = (m0 != ninf ? part * __expf(m0 - l0) : 0.f) + (m1 != ninf ? prt[r] * __expf(m1 - l0) : 0.f);
  }
#pragma unroll 1
  for (int j = 0; j < k; ++j)
    p.gates[(long long)t * k + j] =
        p.gate_mode == 0 ? 1.f : __expf(lg[chosen[j * kTcRows + r] * kTcRows] - l0) / gsum;
}

// Shared scratch of tc_router_finish: logits [npad, kTcRows], then the bias
// row and mask [kTcMaxE] each, both halves' lists [2, kTcSelStride, kTcRows]
// (64-bit keys), the choices [kTcSelStride, kTcRows] and half 1's softmax
// parts [kTcRows].
__host__ __device__ constexpr int tc_router_scratch_bytes(int npad) {
  return npad * kTcRows * 4 + 2 * kTcMaxE * 4 + 2 * kTcSelStride * kTcRows * 8 + kTcSelStride * kTcRows * 4 +
         kTcRows * 4;
}

}  // namespace raiccl
