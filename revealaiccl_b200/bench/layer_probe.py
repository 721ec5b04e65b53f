"""Small-case driver of one MoE layer for kernel profiling.

    python -m revealaiccl_b200.bench.layer_probe --config r4_reference --calls 4 [--graph] [--trace t.json]
        [--control-clocks] [--streamed]

Builds one layer on cuda:0, runs ``--calls`` layer calls (eager launches, or
replays of a captured graph with ``--graph``), verifies the last one and
prints the per-call device time.  Meant to be wrapped by ``ncu -k ... -c ...``
so that a capture sees only a handful of launches of the kernel of interest.
``--control-clocks`` adds, per scheduler trigger of the last call, the SM
clock (cumulative cycles) at the end of each control phase (stage, reveal,
enumerate, select, guard, apply, log) from the control log rows.
``--streamed`` times end-to-end calls instead (pinned host batch streamed in
chunk by chunk, combined output copied back).
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
    ap.add_argument("--control-clocks", action="store_true", help="per-trigger control phase clocks")
    ap.add_argument("--cta-clocks", action="store_true",
                    help="per-CTA front-end timeline of the last call: router chunks, triggers, dispatches")
    ap.add_argument("--streamed", action="store_true", help="end-to-end calls with a streamed host batch")
    ap.add_argument("--gemm-swap-max", type=int, default=128,
                    help="swapped-operand tail tiles of at most this many rows (0: off)")
    args = ap.parse_args()
    cfg = preset(args.config)
    if args.tokens:
        n = cfg.chunks
        cfg = cfg.with_overrides(tokens_per_rank=args.tokens, chunk_sizes=(args.tokens // n,) * n)
    layer = ProgressiveMoELayer(cfg, device=torch.device("cuda", 0), timeout_s=10.0, trace=bool(args.trace),
                                frontend=args.frontend, gemm_swap_max=args.gemm_swap_max)
    try:
        if args.cta_clocks:
            sms = torch.cuda.get_device_properties(layer.device).multi_processor_count
            layer.tensors["fe_clock"] = torch.zeros(sms * 64, dtype=torch.int64, device=layer.device)
        layer.forward(args.arm)
        if args.graph:
            layer.capture(args.arm)
        times = []
        if args.streamed:
            host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
            host_in.copy_(layer.inputs.tokens.cpu())
            host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
        for _ in range(args.calls):
            cur = torch.cuda.current_stream()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if args.streamed:
                s.record(cur)
                layer(host_in, host_out, arm=args.arm)
                e.record(cur)
            else:
                s.record(layer.comm_stream)
                layer.replay(args.arm) if args.graph else layer.forward(args.arm)
                e.record(layer.comm_stream)
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        rep = layer.verify()
        rec = {"config": cfg.name, "arm": args.arm, "graph": args.graph, "ms": times,
               "pass": rep["pass"], "launches_per_call": layer.launches_per_call}
        if args.control_clocks:
            from ..moe.layer import LOG_HEADER  # noqa: F401  (log row layout lives with the layer)
            log = layer.tensors["ctl_log"].cpu().view(layer.cfg.n_desc, layer.log_stride)
            rec["control_clocks"] = [{"trigger": q, "candidates": int(log[q, 0]), "kept": int(log[q, 1]),
                                      "revealed": int(log[q, 6]), "cycles": [int(x) for x in log[q, 8:15]]}
                                     for q in range(layer.cfg.n_desc)]
        if args.cta_clocks:
            rec["cta_clocks"] = _cta_clocks(layer)
        if args.trace:
            from .trace import summarize, write_chrome

            evs = layer.trace_events()
            write_chrome(evs, args.trace, arm=args.arm)
            rec["trace"] = summarize(evs)
        print(json.dumps(rec))
    finally:
        layer.close()


def _cta_clocks(layer) -> dict:
    """Summarise the front end's per-CTA %globaltimer stamps (us from the first
    worker's start): row 0 is the control CTA (trigger q begin / end at slots
    2 + 2q / 3 + 2q), rows 1.. the workers (chunk c begin / end at 2 + 2c /
    3 + 2c, descriptor q begin / rows done / end at 24 + 2q / 44 + q / 25 + 2q)."""
    import numpy as np

    clk = layer.tensors["fe_clock"].cpu().numpy().reshape(-1, 64).astype(np.float64)
    t0 = clk[1:, 0][clk[1:, 0] > 0].min()
    wk = (clk[1:] - t0) / 1e3
    wk[clk[1:] == 0] = np.nan
    r = lambda x: round(float(x), 2)
    out = {"chunks": [], "descriptors": [], "triggers": []}
    for c in range(min(8, layer.cfg.chunks)):
        b, e = wk[:, 2 + 2 * c], wk[:, 3 + 2 * c]
        out["chunks"].append({"chunk": c, "begin_med": r(np.nanmedian(b)), "dur_med": r(np.nanmedian(e - b)),
                              "end_max": r(np.nanmax(e))})
    for q in range(min(8, layer.cfg.n_desc)):
        b, mid, e = wk[:, 24 + 2 * q], wk[:, 44 + q], wk[:, 25 + 2 * q]
        out["descriptors"].append({"desc": q, "begin_min": r(np.nanmin(b)), "begin_med": r(np.nanmedian(b)),
                                   "rows_med": r(np.nanmedian(mid - b)), "publish_max": r(np.nanmax(e - mid)),
                                   "end_max": r(np.nanmax(e))})
    c0 = (clk[0] - t0) / 1e3
    for q in range(min(7, layer.cfg.n_desc)):
        out["triggers"].append({"trigger": q, "begin": r(c0[2 + 2 * q]), "end": r(c0[3 + 2 * q])})
    return out


if __name__ == "__main__":
    main()
