// Device-visible description of one progressive MoE layer instance on one
// rank: problem dimensions, expert placement, and the byte layout of the
// symmetric (peer-mapped) region every rank allocates identically.
//
// Symmetric region (offsets identical on every rank, 256-byte aligned):
//   recv_feat   [E_slot][W][cap][D]     forward features written by source ranks
//   recv_meta   [E_slot][W][cap][9]     int64 forward identity rows
//   recv_retrow [E_slot][W][cap]        int32 row of the source's return buffer
//   recv_gate   [E_slot][W][cap]        fp32 combine weight of the row
//   recv_count  [E_slot][W][n_desc]     int32 rows per (local expert, source, descriptor)
//   recv_flag   [W][n_desc]             uint64 ready sequence per (source, descriptor)
//   ret_out     [T*k][Dout]             expert outputs written back by expert ranks
//   ret_meta    [T*k][8]                int64 return identity rows
//   ret_flag    [W]                     uint64 return sequence per expert rank
//   bar_flag    [W]                     uint64 device-barrier sequence per rank
// cap = T (a token contributes at most one row to any one expert).
#pragma once

#include <cstdint>

namespace raiccl {

constexpr int kMaxRanks = 8;

// Per-peer traffic counters of one rank (int64 words, [world][kPeerCounterFields],
// monotonic across calls): forward descriptors put to the peer, forward bytes
// (feature rows, identity rows, return-row and gate words, count header),
// ready signals sent to it, ready words waited for from it, return bytes sent
// to it (output rows + return identity rows) and return signals sent to it.
enum PeerCounter : int {
  kPcPutCalls = 0, kPcBytes = 1, kPcSignals = 2, kPcWaits = 3, kPcReturnBytes = 4, kPcReturnSignals = 5,
  kPeerCounterFields = 8
};
constexpr int kFwdMetaFields = 9;
constexpr int kRetMetaFields = 8;

struct MoEDims {
  int world;
  int rank;
  int tokens;         // T: tokens on this rank
  int hidden;         // D: token / expert-input width
  int out_dim;        // Dout: expert output width
  int experts;        // E: total experts
  int expert_slots;   // E_slot: local expert capacity per rank
  int top_k;
  int chunks;
  int n_desc;
  int feat_bytes;     // bytes per feature element (4 fp32, 2 bf16)
  int out_bytes;      // bytes per return output element
  int placement;      // 0: owner = e % W, slot = e / W; 1: owner = e / E_slot, slot = e % E_slot
  int gate_mode;      // 0: weight 1; 1: softmax over the selected top-k; 2: softmax over all experts
  int mask_mode;      // 0: none; 1: exclude expert (position % E) ("topology source" mask)
  int ctl_per_chunk;  // control-projection tokens per chunk
  int ctl_nodes;      // node count of the control topology
  int pad0;
  long long cap;      // rows per (slot, source) region
};

// Every array of the region is followed by a guard band of kGuardBytes that
// no kernel writes: the host fills the bands with a canary pattern when the
// region is created and the checker verifies them after a call, so a store
// past the end of any receive or return array is caught.
constexpr int kSymArrays = 10;
constexpr long long kGuardBytes = 256;

struct SymLayout {
  long long recv_feat, recv_meta, recv_retrow, recv_gate, recv_count, recv_flag;
  long long ret_out, ret_meta, ret_flag, bar_flag;
  long long guard[kSymArrays];  // offset of the guard band after each array, in the order above
  long long total;
};

inline long long align256(long long x) { return (x + 255) / 256 * 256; }

inline SymLayout make_sym_layout(const MoEDims& d) {
  SymLayout L;
  long long off = 0;
  int g = 0;
  auto place = [&](long long& at, long long bytes) {
    at = off;
    off = align256(off + bytes);
    L.guard[g++] = off;
    off += kGuardBytes;
  };
  const long long rows = (long long)d.expert_slots * d.world * d.cap;
  const long long ret_rows = (long long)d.tokens * d.top_k;
  place(L.recv_feat, rows * d.hidden * d.feat_bytes);
  place(L.recv_meta, rows * kFwdMetaFields * 8);
  place(L.recv_retrow, rows * 4);
  place(L.recv_gate, rows * 4);
  place(L.recv_count, (long long)d.expert_slots * d.world * d.n_desc * 4);
  place(L.recv_flag, (long long)d.world * d.n_desc * 8);
  place(L.ret_out, ret_rows * d.out_dim * d.out_bytes);
  place(L.ret_meta, ret_rows * kRetMetaFields * 8);
  place(L.ret_flag, (long long)d.world * 8);
  place(L.bar_flag, (long long)d.world * 8);
  L.total = off;
  return L;
}

#if defined(__CUDACC__)
#define MOE_HD __host__ __device__ __forceinline__
#else
#define MOE_HD inline
#endif

MOE_HD int expert_owner(const MoEDims& d, int e) {
  return d.placement == 0 ? e % d.world : e / d.expert_slots;
}

MOE_HD int expert_slot(const MoEDims& d, int e) {
  return d.placement == 0 ? e / d.world : e % d.expert_slots;
}

// Peer base pointers of the symmetric regions (index = rank; own rank included).
struct PeerBases {
  unsigned long long base[kMaxRanks];
};

// Identity checksum of the reference payload rows: sum_i (v_i mod M) * c_i mod M
// with M = 2^63 - 25 (rlccl/transport/reference_full_moe.py:19-32).
constexpr unsigned long long kChecksumModulus = 9223372036854775783ULL;  // 2^63 - 25
constexpr unsigned long long kChecksumCoeff[8] = {1000003ULL, 1000033ULL, 1000037ULL, 1000081ULL,
                                                   1000099ULL, 1000117ULL, 1000121ULL, 1000133ULL};

}  // namespace raiccl
