// Byte layout of the device control plane's working set (compiled plan,
// scheduler state, trigger scalars, scratch) as ONE contiguous blob.
//
// The same layout is used in global memory (one device allocation; the
// Python layer takes typed views of it at these offsets) and in the control
// kernel's shared memory, so staging the working set in or out is a single
// 16-byte vector copy instead of one dependent round trip per array.
// Every array starts on a 16-byte boundary; empty arrays take 16 bytes.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define CTL_HD __host__ __device__ __forceinline__
#else
#define CTL_HD inline
#endif

namespace raiccl {

struct ControlDims {
  int E, G, V, T;                  // plan edges, bandwidth groups, nodes, control-token capacity
  int n_gm, n_egm, n_tmpl;         // group members, edge->group members, route templates
  int max_cands, chunks;
};

enum CtlArray : int {
  // compiled plan (read-only)
  kCtlEdgeSrc, kCtlEdgeTgt, kCtlCap, kCtlGroupLimits, kCtlGroupPtr, kCtlGroupMembers,
  kCtlEdgeGroupPtr, kCtlEdgeGroupMembers, kCtlDistances, kCtlTmplPtr, kCtlTmplEdge,
  kCtlTmplSrc, kCtlTmplTgt, kCtlTmplTdist,
  // scheduler state (persists across the triggers of one layer call)
  kCtlSources, kCtlDestinations, kCtlHolders, kCtlReady, kCtlCommitted, kCtlResidual,
  kCtlRemainingHops, kCtlResidualDemand, kCtlLinkCredits, kCtlGroupCredits,
  kCtlScratchSelected, kCtlScratchSeen, kCtlScratchEdgeLoad, kCtlScalars,
  // per-trigger scratch
  kCtlCands, kCtlKeep, kCtlActions,
  kCtlArrays
};

constexpr int kCtlFirstState = kCtlSources;
constexpr int kCtlFirstScratch = kCtlCands;
constexpr int kCtlScalarHeader = 11;  // scalars: 11 words, then chunk starts [C], chunk counts [C]

struct ControlLayout {
  long long off[kCtlArrays];
  long long count[kCtlArrays];
  int elem[kCtlArrays];
  long long state_begin, state_end, total;  // all multiples of 16
};

CTL_HD ControlLayout control_layout(const ControlDims& d) {
  ControlLayout L{};
  const long long E = d.E, G = d.G, V = d.V, T = d.T;
  const long long counts[kCtlArrays] = {
      E, E, E, G, G + 1, d.n_gm, E + 1, d.n_egm, V * V, V + 1, d.n_tmpl, d.n_tmpl, d.n_tmpl, d.n_tmpl,
      T, T, T * V, T, T * E, T, T, V * V, E, G, T, T, E, kCtlScalarHeader + 2LL * d.chunks,
      4LL * d.max_cands, d.max_cands, 2 * T};
  const int elems[kCtlArrays] = {4, 4, 8, 8, 4, 4, 4, 4, 4, 4, 4, 4, 4, 4,
                                 4, 4, 1, 1, 1, 1, 4, 8, 8, 8, 1, 1, 8, 8,
                                 4, 4, 8};
  long long off = 0;
  for (int i = 0; i < kCtlArrays; ++i) {
    if (i == kCtlFirstState) L.state_begin = off;
    if (i == kCtlFirstScratch) L.state_end = off;
    L.off[i] = off;
    L.count[i] = counts[i];
    L.elem[i] = elems[i];
    const long long bytes = (counts[i] > 0 ? counts[i] : 1) * elems[i];
    off += (bytes + 15) & ~15LL;
  }
  L.total = off;
  return L;
}

}  // namespace raiccl
