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
