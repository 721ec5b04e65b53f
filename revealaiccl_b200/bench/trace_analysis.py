"""Fail-closed analysis of a layer call's device trace: the control plane's
ready -> release -> dispatch latencies and the dispatch / routing overlap.

The reference measures these with host stamps and profiler traces: the time
from a Router chunk's completion event becoming host-visible to the NCCL
submit returning (scripts/run_r2_f0_integrated.py, report
docs/phase_r2/R2_F0_REPORT.md), and the device overlap of early NCCL
kernels with the Router (scripts/run_r2_o0_profiled.py and its analyzer
scripts/analyze_r2_o0_traces.py: the share of early transfers that start on
the GPU before the final Router chunk ends, and the share that coexists
with Router work).  Here the whole chain is on the device, so the trace ring
of one call (``ProgressiveMoELayer(trace=True).trace_events()``) holds every
stamp; per descriptor q with last router chunk c(q):

* ``ready_to_release_us`` = end of control trigger q - end of router chunk c(q)
  (the scheduler's latency from the chunk being complete to the descriptor
  being released);
* ``ready_to_dispatch_us`` = start of dispatch q - end of router chunk c(q)
  (ready -> first byte on the wire);
* ``dispatch_us`` = duration of dispatch q;

and per call ``early_start_share`` (descriptors whose dispatch starts before
the final router chunk ends, among the early ones) and ``coexist_share``
(the part of dispatch time that overlaps router time).

Fail-closed: a missing phase, a dispatch that starts before its release or a
release before its chunk is complete raises ``TraceError`` (the analyzer
never reports numbers from an inconsistent trace).

    python -m revealaiccl_b200.bench.trace_analysis trace_events.json [--partial-chunks P]
"""

from __future__ import annotations

import argparse
import json
import statistics
from typing import Any, Mapping, Sequence


class TraceError(ValueError):
    pass


def _intervals_overlap(a: list[tuple[int, int]], b: list[tuple[int, int]]) -> int:
    """Total length of the intersection of two interval sets (ns)."""
    def merge(xs):
        out: list[list[int]] = []
        for s, e in sorted(xs):
            if out and s <= out[-1][1]:
                out[-1][1] = max(out[-1][1], e)
            else:
                out.append([s, e])
        return out
    A, B = merge(a), merge(b)
    i = j = total = 0
    while i < len(A) and j < len(B):
        lo, hi = max(A[i][0], B[j][0]), min(A[i][1], B[j][1])
        total += max(0, hi - lo)
        if A[i][1] < B[j][1]:
            i += 1
        else:
            j += 1
    return total


def analyze_rank(events: Sequence[Mapping[str, Any]], *, partial_chunks: int, chunks: int,
                 slack_ns: int = 0) -> dict[str, Any]:
    """One rank's events of one call.  ``partial_chunks``: descriptors 0..P-1
    are chunks 0..P-1, descriptor P holds chunks P..C-1.  ``slack_ns``
    tolerates the trace's timer granularity in the ordering checks."""
    by = {}
    for e in events:
        by.setdefault(e["kind"], {})[int(e["arg"])] = e
    for kind in ("router", "control", "dispatch"):
        if kind not in by:
            raise TraceError(f"no {kind} phases in the trace (layer built with trace=True, persistent front end?)")
    n_desc = partial_chunks + (1 if partial_chunks < chunks else 0)
    rows = []
    for q in range(n_desc):
        last_chunk = q if q < partial_chunks else chunks - 1
        try:
            r, c, d = by["router"][last_chunk], by["control"][q], by["dispatch"][q]
        except KeyError as exc:
            raise TraceError(f"descriptor {q}: missing phase {exc}") from None
        if c["end_ns"] + slack_ns < r["end_ns"]:
            raise TraceError(f"descriptor {q} released before router chunk {last_chunk} completed")
        if d["start_ns"] + slack_ns < c["end_ns"]:
            raise TraceError(f"descriptor {q} dispatched before its release")
        rows.append({"desc": q, "ready_to_release_us": (c["end_ns"] - r["end_ns"]) / 1e3,
                     "ready_to_dispatch_us": (d["start_ns"] - r["end_ns"]) / 1e3,
                     "dispatch_us": (d["end_ns"] - d["start_ns"]) / 1e3})
    final_router_end = max(e["end_ns"] for e in by["router"].values())
    early = [by["dispatch"][q] for q in range(min(partial_chunks, n_desc))]
    router_iv = [(e["start_ns"], e["end_ns"]) for e in by["router"].values()]
    disp_iv = [(e["start_ns"], e["end_ns"]) for e in by["dispatch"].values()]
    disp_total = sum(e - s for s, e in disp_iv)
    med = lambda k: statistics.median(r[k] for r in rows)
    return {
        "descriptors": rows,
        "ready_to_release_us_p50": med("ready_to_release_us"),
        "ready_to_dispatch_us_p50": med("ready_to_dispatch_us"),
        "dispatch_us_p50": med("dispatch_us"),
        "early_start_share": (sum(1 for e in early if e["start_ns"] < final_router_end) / len(early)) if early else 0.0,
        "coexist_share": (_intervals_overlap(router_iv, disp_iv) / disp_total) if disp_total else 0.0,
    }


def analyze(events: Sequence[Mapping[str, Any]], *, partial_chunks: int, chunks: int,
            slack_ns: int = 0) -> dict[str, Any]:
    """Every rank of one call (events carry ``rank``); medians are per rank."""
    ranks: dict[int, list[Mapping[str, Any]]] = {}
    for e in events:
        ranks.setdefault(int(e.get("rank", 0)), []).append(e)
    if not ranks:
        raise TraceError("empty trace")
    return {"ranks": {r: analyze_rank(evs, partial_chunks=partial_chunks, chunks=chunks, slack_ns=slack_ns)
                      for r, evs in sorted(ranks.items())}}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("events", help="JSON list of trace events (kind, arg, start_ns, end_ns, rank)")
    ap.add_argument("--chunks", type=int, default=8)
    ap.add_argument("--partial-chunks", type=int, default=6)
    ap.add_argument("--slack-ns", type=int, default=0)
    args = ap.parse_args(argv)
    with open(args.events, encoding="utf-8") as f:
        events = json.load(f)
    print(json.dumps(analyze(events, partial_chunks=args.partial_chunks, chunks=args.chunks,
                             slack_ns=args.slack_ns), indent=1))


__all__ = ["TraceError", "analyze", "analyze_rank", "main"]

if __name__ == "__main__":
    main()
