"""Completion -> host-visible latency of the completion bridge
(scripts/run_r2_e0_event_bridge.py).

Each trial launches a kernel that holds the stream for --delay-us and then
(a) records a CUDA event after it and (b) publishes a mapped host flag from
inside it; both slots are armed before the launch.  Reported per source: the
bridge's conservative upper bound (hit time - start of the last missed poll),
the poll count and the host wall time from launch to READY.

    python -m revealaiccl_b200.bench.event_latency --trials 200
"""

from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch

from ..runtime import CompletionBridge, HostFlag


def _dist(v) -> dict:
    a = np.asarray(v, dtype=np.float64)
    return {"count": int(a.size), "p50": float(np.percentile(a, 50)), "p95": float(np.percentile(a, 95)),
            "p99": float(np.percentile(a, 99)), "max": float(a.max())} if a.size else {"count": 0}


def run(trials: int = 200, delay_us: float = 20.0, cpu_core: int = -1, device: int = 0) -> dict:
    torch.cuda.set_device(device)
    flag = HostFlag()
    out = {"event": {"upper_bound_ns": [], "wall_ns": [], "polls": []},
           "flag": {"upper_bound_ns": [], "wall_ns": [], "polls": []}}
    with CompletionBridge(2, cpu_core=cpu_core, device=device) as br:
        for i in range(1, trials + 1):
            ev = torch.cuda.Event()
            br.reset_all()
            br.arm_flag(1, flag, i)
            t0 = time.perf_counter_ns()
            flag.signal_from_device(i, int(delay_us * 1e3))
            ev.record()
            br.arm_event(0, ev)
            br.wait_all(5.0)
            snap = br.snapshot()
            for idx, key in ((0, "event"), (1, "flag")):
                s = snap[idx]
                if s["upper_bound_valid"]:
                    out[key]["upper_bound_ns"].append(s["visibility_upper_bound_ns"])
                out[key]["wall_ns"].append(s["ready_ns"] - t0 if s["ready_ns"] >= t0 else 0)
                out[key]["polls"].append(s["poll_count"])
        torch.cuda.synchronize()
    flag.close()
    return {"trials": trials, "delay_us": delay_us,
            **{k: {m: _dist(v) for m, v in d.items()} for k, d in out.items()}}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="completion bridge latency")
    ap.add_argument("--trials", type=int, default=200)
    ap.add_argument("--delay-us", type=float, default=20.0)
    ap.add_argument("--cpu-core", type=int, default=-1)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    rep = run(a.trials, a.delay_us, a.cpu_core)
    if a.out:
        with open(a.out, "w") as fh:
            json.dump(rep, fh, indent=2)
    print(json.dumps({k: rep[k]["upper_bound_ns"] for k in ("event", "flag")}))


if __name__ == "__main__":
    main()
