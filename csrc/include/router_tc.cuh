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
constexpr int kTcSelStride = 8;    // selected logits kept per token (top_k <= 8)

// Per-CTA state.  n_load / n_mma count K steps over every unit this CTA
// routed (the issuing thread's copy is the one that matters); n_units counts
// units (every thread keeps the same count).
struct TcRouter {
  uint8_t* stages;     // 1024-aligned shared memory: n_stages x [tokens 128 x 128 B | weights npad x 128 B]
  float* lg;           // [npad, kTcRows] shared: the unit's logits, expert-major
  float* sel;          // [kTcSelStride, kTcRows] shared: each token's chosen logits
  uint64_t* full;      // [n_stages] TMA bytes landed
  uint64_t* empty;     // [n_stages] the stage's MMAs completed
  uint64_t* done;      // the unit's MMAs completed
  uint32_t tmem;       // accumulator: 128 lanes x npad fp32 columns
  int n_stages, npad, kblocks;
  uint32_t n_load, n_mma, n_units;

  __device__ int stage_bytes() const { return kTcRows * 128 + npad * 128; }
};

// Shared scratch of tc_router_finish: logits [npad, kTcRows] and choices [kTcSelStride, kTcRows].
__host__ __device__ constexpr int tc_router_scratch_bytes(int npad) {
  return (npad + kTcSelStride) * kTcRows * 4;
}

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

// Threads 0..127 (warps 0-3, one TMEM lane quarter each): wait for the unit's
// MMAs, read token row threadIdx.x's logits into shared memory (expert-major,
// so the lanes of a warp touch consecutive words) and finish the token (rows
// < nt only; the tile's other rows belong to later tokens and are dropped).
// Same order as router_finish_warp: the larger logit, then the smaller expert
// id; NaN below every number.  The loops stay rolled (small code, few live
// registers in a kernel that is at its register limit).
template <int EMAX>
__device__ inline void tc_router_finish(const RouterParams& p, const float* chunk_bias, TcRouter& s, int tf, int nt,
                                        int* sel_counts, DeviceStatus* st, int kid, unsigned long long lim,
                                        unsigned long long* dbg = nullptr) {
  constexpr int EP = EMAX < 16 ? 16 : EMAX;  // TMEM columns read (multiple of 16)
  const int r = threadIdx.x, t = tf + r, E = p.experts, k = p.top_k;
  const float ninf = -__int_as_float(0x7f800000);
  mbar_wait_bounded(s.done, s.n_units & 1u, st, kid, lim);
  tc_fence_after_sync();
  if (dbg != nullptr && r == 0) *dbg = globaltimer_ns();  // diagnostics: the unit's MMAs completed
  float* lg = s.lg + r;  // lg[e * kTcRows]: expert e's logit of this token
  const uint32_t taddr = s.tmem + ((uint32_t)((r >> 5) * 32) << 16);
#pragma unroll
  for (int c = 0; c < EP / 16; ++c) {
    if (c * 16 < s.npad) {
      uint32_t raw[16];
      tmem_ld16(taddr + c * 16, raw);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int e = c * 16 + i;
        if (e < E && r < nt) {
          const float l = __uint_as_float(raw[i]) + __ldg(p.bias + e) + (chunk_bias ? chunk_bias[e] : 0.f);
          const bool masked = (p.mask_mode == 1 && e == (t % E)) || (p.block_mask && __ldg(p.block_mask + e));
          lg[e * kTcRows] = masked ? ninf : l;
        }
      }
    }
  }
  if (r >= nt) return;
  float* sel = s.sel + r;  // sel[j * kTcRows]: choice j's logit
  unsigned long long taken = 0;
  float l0 = 0.f;
#pragma unroll 1
  for (int j = 0; j < k; ++j) {
    int best = -1, br = 0;
    float bv = ninf;
#pragma unroll 1
    for (int e = 0; e < E; ++e) {
      if ((taken >> e) & 1ull) continue;
      const float v = lg[e * kTcRows];
      const int re = v == v ? 2 : 1;
      if (best < 0 || router_better(re, v, e, br, bv, best)) {
        best = e;
        bv = v;
        br = re;
      }
    }
    taken |= 1ull << best;
    sel[j * kTcRows] = bv;
    if (j == 0) l0 = bv;
    p.expert_ids[(long long)t * k + j] = best;
    if (sel_counts) atomicAdd(&sel_counts[best], 1);
  }
  float sum = 1.f;
  if (p.gate_mode == 1) {
    sum = 0.f;
#pragma unroll 1
    for (int j = 0; j < k; ++j) sum += __expf(sel[j * kTcRows] - l0);
  } else if (p.gate_mode == 2) {
    sum = 0.f;
#pragma unroll 1
    for (int e = 0; e < E; ++e)
      if (lg[e * kTcRows] != ninf) sum += __expf(lg[e * kTcRows] - l0);
  }
#pragma unroll 1
  for (int j = 0; j < k; ++j)
    p.gates[(long long)t * k + j] = p.gate_mode == 0 ? 1.f : __expf(sel[j * kTcRows] - l0) / sum;
}

}  // namespace raiccl
