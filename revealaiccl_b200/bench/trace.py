"""Device trace of a layer call: per-launch %globaltimer spans from the trace
ring (``ProgressiveMoELayer(trace=True).trace_events()``), gathered over ranks,
summarised and written as a Chrome / Perfetto trace.

The reference traces with host ``perf_counter_ns`` stamps, CUDA-event
durations and Kineto ``record_function`` labels of the form
``R5P4|kind=...|arm=...|item=...`` (scripts/run_r4_a0_c0_full_moe.py:151-152,
339-342).  Here the device writes the timestamps itself, so a span is the
kernel's own first-CTA-start to last-CTA-end on the GPU's global timer, and
labels keep the ``key=value|...`` schema: ``kind=dispatch|arg=3|rank=1|arm=early``.

    python -m revealaiccl_b200.bench.layer_probe --config full_tf32 --trace trace.json
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Iterable, Mapping, Sequence

# Chrome-trace thread rows: one per pipeline role
_ROWS = {"layer_reset": 0, "router": 1, "control": 2, "dispatch": 3, "expert_plan": 4,
         "gemm1": 5, "gemm2_return": 5, "return_meta": 6, "combine": 7}


def label(ev: Mapping[str, Any], arm: str | None = None) -> str:
    parts = [f"kind={ev['kind']}", f"arg={ev['arg']}", f"rank={ev.get('rank', 0)}"]
    if arm:
        parts.append(f"arm={arm}")
    return "|".join(parts)


def gather(events: list[dict[str, Any]], group=None) -> list[dict[str, Any]]:
    """All ranks' events on every rank (collective when a process group is up)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return list(events)
    out: list[Any] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, events, group=group)
    return [e for rank_events in out for e in rank_events]


def summarize(events: Sequence[Mapping[str, Any]]) -> dict[str, Any]:
    """Device makespan per rank (first router start -> combine end) and busy
    time per kind; ``makespan_ms`` is the max over ranks."""
    by_rank: dict[int, list[Mapping[str, Any]]] = {}
    for e in events:
        by_rank.setdefault(int(e.get("rank", 0)), []).append(e)
    ranks = {}
    for r, evs in sorted(by_rank.items()):
        starts = [e["start_ns"] for e in evs if e["kind"] == "router"] or [e["start_ns"] for e in evs]
        ends = [e["end_ns"] for e in evs if e["kind"] == "combine"] or [e["end_ns"] for e in evs]
        kinds: dict[str, dict[str, float]] = {}
        for e in evs:
            k = kinds.setdefault(e["kind"], {"launches": 0, "busy_us": 0.0})
            k["launches"] += 1
            k["busy_us"] += (e["end_ns"] - e["start_ns"]) / 1e3
        ranks[r] = {"makespan_ms": (max(ends) - min(starts)) / 1e6, "kinds": kinds}
    return {"ranks": ranks, "makespan_ms": max((v["makespan_ms"] for v in ranks.values()), default=0.0)}


def to_chrome(events: Iterable[Mapping[str, Any]], arm: str | None = None) -> dict[str, Any]:
    evs = list(events)
    t0 = min((e["start_ns"] for e in evs), default=0)
    out = []
    for e in evs:
        out.append({"name": e["kind"] + (f"[{e['arg']}]" if e["arg"] >= 0 else ""), "cat": e["kind"], "ph": "X",
                    "ts": (e["start_ns"] - t0) / 1e3, "dur": max(0.0, (e["end_ns"] - e["start_ns"]) / 1e3),
                    "pid": int(e.get("rank", 0)), "tid": _ROWS.get(e["kind"], 9),
                    "args": {"label": label(e, arm), "ctas": e.get("ctas", 0)}})
    return {"traceEvents": out, "displayTimeUnit": "ns"}


def write_chrome(events: Iterable[Mapping[str, Any]], path: str | Path, arm: str | None = None) -> Path:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(json.dumps(to_chrome(events, arm)), encoding="utf-8")
    return p


__all__ = ["gather", "label", "summarize", "to_chrome", "write_chrome"]
