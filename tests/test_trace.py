"""Trace summarisation / Chrome export (CPU) and the device trace ring (GPU)."""

import json

import pytest

from revealaiccl_b200.bench import trace


def _evs():
    return [
        {"kind": "router", "arg": 0, "start_ns": 1000, "end_ns": 3000, "ctas": 64, "rank": 0},
        {"kind": "control", "arg": 0, "start_ns": 3500, "end_ns": 9000, "ctas": 1, "rank": 0},
        {"kind": "combine", "arg": -1, "start_ns": 20000, "end_ns": 26000, "ctas": 148, "rank": 0},
        {"kind": "router", "arg": 0, "start_ns": 1500, "end_ns": 3200, "ctas": 64, "rank": 1},
        {"kind": "combine", "arg": -1, "start_ns": 21000, "end_ns": 31500, "ctas": 148, "rank": 1},
    ]


def test_summary_is_max_over_ranks(tmp_path):
    s = trace.summarize(_evs())
    assert s["ranks"][0]["makespan_ms"] == pytest.approx(0.025)
    assert s["ranks"][1]["makespan_ms"] == pytest.approx(0.03)
    assert s["makespan_ms"] == pytest.approx(0.03)
    assert s["ranks"][0]["kinds"]["control"]["launches"] == 1
    p = trace.write_chrome(_evs(), tmp_path / "t.json", arm="early")
    doc = json.loads(p.read_text())
    assert len(doc["traceEvents"]) == 5
    first = doc["traceEvents"][0]
    assert first["ph"] == "X" and first["ts"] == 0.0 and first["args"]["label"] == "kind=router|arg=0|rank=0|arm=early"


@pytest.mark.gpu
def test_device_trace_ring_spans():
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    layer = ProgressiveMoELayer(preset("r4_reference"), timeout_s=5.0, trace=True)
    try:
        for arm in ("early", "delayed"):
            layer.forward(arm)
            evs = layer.trace_events()
            kinds = [e["kind"] for e in evs]
            assert kinds.count("router") == 8 and kinds.count("control") == 7 and kinds.count("dispatch") == 7
            for k in ("gemm1", "gemm2_return", "combine", "expert_plan"):
                assert k in kinds
            assert all(e["end_ns"] >= e["start_ns"] > 0 for e in evs)
            by = {(e["kind"], e["arg"]): e for e in evs}
            for q in range(7):  # stream order: control q before dispatch q, dispatch before the expert side
                assert by[("control", q)]["end_ns"] <= by[("dispatch", q)]["start_ns"]
                assert by[("dispatch", q)]["end_ns"] <= by[("expert_plan", -1)]["start_ns"]
            assert by[("gemm1", -1)]["end_ns"] <= by[("gemm2_return", -1)]["start_ns"]
            assert trace.summarize(evs)["makespan_ms"] > 0
    finally:
        layer.close()


def _ev(kind, arg, s, e, rank=0):
    return {"kind": kind, "arg": arg, "start_ns": s, "end_ns": e, "rank": rank, "ctas": 1}


def _call(shift=0, rank=0):
    evs = []
    for c in range(8):
        evs.append(_ev("router", c, 1000 * c + shift, 1000 * c + 900 + shift, rank))
    for q in range(7):
        last = q if q < 6 else 7
        r_end = 1000 * last + 900 + shift
        evs.append(_ev("control", q, r_end + 100, r_end + 600, rank))
        evs.append(_ev("dispatch", q, r_end + 700, r_end + 1500, rank))
    return evs


def test_trace_analysis_latencies_overlap_and_fail_closed():
    from revealaiccl_b200.bench.trace_analysis import TraceError, analyze

    rep = analyze(_call() + _call(rank=1), partial_chunks=6, chunks=8)
    r0 = rep["ranks"][0]
    assert r0["ready_to_release_us_p50"] == 0.6 and r0["ready_to_dispatch_us_p50"] == 0.7
    assert r0["dispatch_us_p50"] == 0.8 and len(r0["descriptors"]) == 7
    assert r0["early_start_share"] == 1.0 and 0.0 < r0["coexist_share"] < 1.0
    bad = _call()
    for e in bad:
        if e["kind"] == "dispatch" and e["arg"] == 3:
            e["start_ns"] -= 1000  # starts before its release
    with pytest.raises(TraceError, match="before its release"):
        analyze(bad, partial_chunks=6, chunks=8)
    with pytest.raises(TraceError, match="missing"):
        analyze([e for e in _call() if not (e["kind"] == "control" and e["arg"] == 2)], partial_chunks=6, chunks=8)
