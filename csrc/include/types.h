// Plain data types shared by device code and host C++ (no CUDA builtins here).
#pragma once

#include <cstdint>

namespace raiccl {

// ---------------------------------------------------------------------------
// Status / error reporting (no __trap, no device assert anywhere).
// ---------------------------------------------------------------------------
enum StatusCode : int {
  kOk = 0,
  kTimeoutPipeline = 1,     // an intra-CTA mbarrier wait ran out (a bug)
  kTimeoutPeerSignal = 2,   // a peer's ready/return signal never arrived
  kTimeoutChunkFlag = 3,    // a router chunk flag never arrived
  kBoundsViolation = 4,     // an index failed its capacity check
  kBadConfig = 5,           // launch parameters inconsistent
  kTimeoutPermit = 6,       // the scheduler permit for a descriptor never arrived
  kSeqMismatch = 7,         // a signal carried an unexpected sequence number
  kTimeoutInput = 8,        // a streamed input chunk never landed
};

struct DeviceStatus {
  int code;        // first error code recorded (0 = ok)
  int kernel_id;   // which kernel recorded it
  int block;       // blockIdx.x of the recorder
  int thread;      // threadIdx.x of the recorder
  long long index; // offending index / waited-on slot
  long long bound; // capacity or expected value
};

// Device trace ring entry: one per kernel launch of a layer call.  Every CTA
// folds its first and last %globaltimer reading into the slot (min / max), so
// the slot holds the launch's device span; `ctas` counts the CTAs that ran.
struct TraceSlot {
  unsigned long long t_start;  // ~0 until a CTA started (reset per call)
  unsigned long long t_end;
  int ctas;
  int pad0;
  long long pad1;
};

enum class Act : int { kNone = 0, kRelu = 1, kGelu = 2, kSilu = 3, kSwiGLU = 4 };

struct GemmSegment {
  int a_row0;    // first A row of the segment
  int rows;      // valid rows in the segment (may be 0)
  int expert;    // weight slice index into B / bias
  int out_slot;  // index into GroupedGemmParams::out_ptrs (local or peer buffer)
  int out_row0;  // first output row when no row map is given
  int pad0, pad1, pad2;
};

struct GroupedGemmParams {
  const GemmSegment* segs;   // [num_segs]
  const int* tile_prefix;    // [num_segs + 1] cumulative tile counts (device computed)
  int num_segs;
  int N;                     // GEMM N (for SwiGLU: 2 * output width, interleaved per BN tile)
  int K;
  const float* bias;         // [E, N] or nullptr
  const int* row_map;        // [rows_total] output row of each A row, or nullptr
  const float* row_scale;    // [rows_total] multiplier applied after activation, or nullptr
  void* const* out_ptrs;     // output base pointers (device or peer)
  long long ldo;             // output row stride in elements
  DeviceStatus* status;
  unsigned long long timeout_ns;
  TraceSlot* trace;          // launch trace slot or nullptr
  int pair;                  // 1: CTA-pair kernel (256-row tiles in tile_prefix), 0: one CTA per 128-row tile
  int pdl;                   // 1: launch as a programmatic dependent of the previous kernel in the stream
  // CTA-pair kernel at BN = 256 only: [num_segs + 1] cumulative counts of
  // swapped tail tiles, or nullptr.  When given, tile_prefix counts every
  // segment's 256-row tiles except a last tile of at most swap_max rows; that
  // tail tile is computed with the operands swapped (weights as the 256-row
  // operand, the tail's tokens as N = rows rounded up to 16) and is ordered
  // after all full tiles.
  const int* tail_prefix;
  int swap_max;
  // Progressive tile source (CTA-pair kernel, progressive != 0): tiles are
  // taken in arrival order from tile_list as the expert planner publishes
  // them in tile_word ((call epoch low 32 bits) << 32 | final << 31 | count);
  // each pair's leader draws tickets from ticket_counter (zeroed per call) and
  // passes them to its partner and its other roles through its
  // kPairTicketRing slots of pair_tickets.  tile_prefix / tail_prefix unused.
  int progressive;
  const int* tile_list;                 // [max] 4 ints per tile: segment, row tile, column block, nsw
  const unsigned long long* tile_word;
  unsigned int* ticket_counter;
  unsigned long long* pair_tickets;     // [pairs][kPairTicketRing][2]: tag | ticket, packed tile
  const unsigned long long* epoch;      // this call's sequence number
  // Split K (one-CTA kernel, activations other than SwiGLU): when the tiles
  // are few and K is long, each tile's K range is split over up to ksplit_max
  // CTAs (chosen on the device from the tile count: one (tile, split) per CTA,
  // at least kSplitMinKBlocks K blocks per split, at most ksplit_entries
  // partial tiles).  Each split stores its fp32 partial tile in
  // ksplit_partial [entries, 128, BN]; the tile's last split (ksplit_ticket
  // [tiles], zeroed per call) adds the partials in split order and runs the
  // epilogue, so results do not depend on arrival order.  nullptr: no split.
  float* ksplit_partial;
  int* ksplit_ticket;
  int ksplit_entries;
  int ksplit_max;
};

constexpr int kPairTicketRing = 32;

}  // namespace raiccl
