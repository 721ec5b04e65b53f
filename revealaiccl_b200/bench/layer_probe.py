"""Small-case driver of one MoE layer for kernel profiling.

    python -m revealaiccl_b200.bench.layer_probe --config r4_reference --calls 4 [--graph] [--trace t.json]

Builds one layer on cuda:0, runs ``--calls`` layer calls (eager launches, or
replays of a captured graph with ``--graph``), verifies the last one and
prints the per-call device time.  Meant to be wrapped by ``ncu -k ... -c ...``
so that a capture sees only a handful of launches of the kernel of interest.
"""

from __future__ import annotations

import argparse
import json


def main() -> None:
    import torch

    from ..moe.config import preset
    from ..moe.layer import ProgressiveMoELayer

    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="r4_reference")
    ap.add_argument("--calls", type=int, default=4)
    ap.add_argument("--arm", default="early", choices=("early", "delayed"))
    ap.add_argument("--graph", action="store_true")
    ap.add_argument("--tokens", type=int, default=0, help="override tokens per rank (uniform chunks)")
    ap.add_argument("--trace", default=None, help="write a Chrome trace of the last call to this path")
    ap.add_argument("--frontend", default="persistent", choices=("persistent", "steps"),
                    help="one cooperative front-end launch, or one launch per router chunk / trigger / descriptor")
    args = ap.parse_args()
    cfg = preset(args.config)
    if args.tokens:
        n = cfg.chunks
        cfg = cfg.with_overrides(tokens_per_rank=args.tokens, chunk_sizes=(args.tokens // n,) * n)
    layer = ProgressiveMoELayer(cfg, device=torch.device("cuda", 0), timeout_s=10.0, trace=bool(args.trace),
                                frontend=args.frontend)
    try:
        layer.forward(args.arm)
        if args.graph:
            layer.capture(args.arm)
        times = []
        for _ in range(args.calls):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(layer.comm_stream)
            layer.replay(args.arm) if args.graph else layer.forward(args.arm)
            e.record(layer.comm_stream)
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        rep = layer.verify()
        rec = {"config": cfg.name, "arm": args.arm, "graph": args.graph, "ms": times,
               "pass": rep["pass"], "launches_per_call": layer.launches_per_call}
        if args.trace:
            from .trace import summarize, write_chrome

            evs = layer.trace_events()
            write_chrome(evs, args.trace, arm=args.arm)
            rec["trace"] = summarize(evs)
        print(json.dumps(rec))
    finally:
        layer.close()


if __name__ == "__main__":
    main()
