"""Small-case driver of one MoE layer for kernel profiling.

    python -m revealaiccl_b200.bench.layer_probe --config r4_reference --calls 4 [--graph] [--trace t.json]
        [--control-clocks] [--streamed]

Builds one layer per rank (run it under ``torch.distributed.run`` for
several GPUs; one GPU otherwise), runs ``--calls`` layer calls (eager
launches, or replays of a captured graph with ``--graph``), verifies the
last one and prints, on rank 0, the per-call device time (max over ranks).  Meant to be wrapped by ``ncu -k ... -c ...``
so that a capture sees only a handful of launches of the kernel of interest.
``--control-clocks`` adds, per scheduler trigger of the last call, the SM
clock (cumulative cycles) at the end of each control phase (stage, reveal,
enumerate, select, guard, apply, log) from the control log rows.
``--streamed`` times end-to-end calls instead (pinned host batch streamed in
chunk by chunk, combined output copied back).
``--roofline`` (with ``--trace``) adds, per rank, achieved fractions of the
fused paths against their rooflines: the front end's dispatch (the bytes this
rank put to its peers, from the device traffic counters, over the dispatch
span, against the measured peer-copy bandwidth per direction), each grouped
GEMM (its FLOPs over its span against the measured tensor peak) and GEMM-2
with its fused return (the slower of its FLOPs at the tensor peak and its
return bytes at the link bandwidth, over its span).
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
    ap.add_argument("--roofline", action="store_true", help="achieved fractions of the fused paths (needs --trace)")
    ap.add_argument("--progressive", type=int, default=0, choices=(0, 1),
                    help="GEMM-1 takes tiles as descriptors arrive (1) or after the whole batch (0)")
    ap.add_argument("--dispatch-ctas", type=int, default=0, help="front-end workers that dispatch (0: all)")
    ap.add_argument("--router-ring", type=int, default=1, choices=(0, 1),
                    help="resident batches reach shared memory by bulk copies (routing and dispatch staging)")
    ap.add_argument("--dispatch-groups", type=int, default=1, choices=(0, 1),
                    help="one worker group per partial descriptor, dispatched side by side")
    ap.add_argument("--router-wsmem", type=int, default=1, choices=(0, 1),
                    help="router weights copied into each front-end worker's shared memory")
    ap.add_argument("--router-tc", type=int, default=1, choices=(0, 1),
                    help="bf16 batches: 128-token router units on the tensor cores")
    args = ap.parse_args()
    import os

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rank = dist.get_rank() if world > 1 else 0
    cfg = preset(args.config)
    if args.tokens:
        n = cfg.chunks
        cfg = cfg.with_overrides(tokens_per_rank=args.tokens, chunk_sizes=(args.tokens // n,) * n)
    layer = ProgressiveMoELayer(cfg, device=dev, timeout_s=10.0, trace=bool(args.trace or args.roofline),
                                frontend=args.frontend, gemm_swap_max=args.gemm_swap_max,
                                progressive=bool(args.progressive), dispatch_ctas=args.dispatch_ctas,
                                router_ring=bool(args.router_ring), dispatch_groups=bool(args.dispatch_groups),
                                router_wsmem=bool(args.router_wsmem), router_tc=bool(args.router_tc))
    try:
        if args.cta_clocks:
            sms = torch.cuda.get_device_properties(layer.device).multi_processor_count
            layer.tensors["fe_clock"] = torch.zeros(sms * FE_CLOCK_SLOTS, dtype=torch.int64, device=layer.device)
        layer.forward(args.arm)
        if args.graph:
            layer.capture(args.arm)
        times = []
        if args.streamed:
            host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
            host_in.copy_(layer.inputs.tokens.cpu())
            host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
        counters_before = None
        for i in range(args.calls):
            if i == args.calls - 1:
                torch.cuda.synchronize()
                counters_before = layer.channel.peer_counters()
                if world > 1:
                    layer.device_barrier()
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
        counters_after = layer.channel.peer_counters()
        rep = layer.verify()
        if world > 1:
            t = torch.tensor(times, dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times = t.tolist()
        rec = {"config": cfg.name, "world": world, "arm": args.arm, "graph": args.graph, "ms": times,
               "pass": rep["pass"], "launches_per_call": layer.launches_per_call}
        if args.control_clocks:
            from ..moe.layer import LOG_HEADER  # noqa: F401  (log row layout lives with the layer)
            log = layer.tensors["ctl_log"].cpu().view(layer.cfg.n_desc, layer.log_stride)
            rec["control_clocks"] = [{"trigger": q, "candidates": int(log[q, 0]), "kept": int(log[q, 1]),
                                      "revealed": int(log[q, 6]), "cycles": [int(x) for x in log[q, 8:15]]}
                                     for q in range(layer.cfg.n_desc)]
        if args.cta_clocks:
            rec["cta_clocks"] = _cta_clocks(layer)
        if args.trace or args.roofline:
            from .trace import summarize, write_chrome

            evs = layer.trace_events()
            roof = _roofline(layer, evs, counters_before, counters_after) if args.roofline else None
            if world > 1:
                every = [None] * world
                dist.all_gather_object(every, (evs, roof))
                evs = [e for part, _ in every for e in part]
                roofs = [r for _, r in every]
            else:
                roofs = [roof]
            if args.trace and rank == 0:
                write_chrome(evs, args.trace, arm=args.arm)
            rec["trace"] = summarize(evs)
            if layer.runner.persistent_frontend():
                from .trace_analysis import TraceError, analyze

                try:  # fail closed: an inconsistent trace reports its error, never numbers
                    rep = analyze(evs, partial_chunks=cfg.progressive_chunks, chunks=cfg.chunks, slack_ns=1024)
                    rec["control_chain"] = {r: {k: v for k, v in x.items() if k != "descriptors"}
                                            for r, x in rep["ranks"].items()}
                except TraceError as exc:
                    rec["control_chain"] = {"error": str(exc)}
            if args.roofline:
                rec["roofline"] = roofs
        if rank == 0:
            print(json.dumps(rec))
    finally:
        layer.close()
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


def _peaks() -> dict:
    """Measured denominators: HBM copy bandwidth and bf16 tensor throughput
    (MEASURED_PEAKS.json beside the repository when present, else an earlier
    measurement on B200) and the measured NVLink peer-copy bandwidth per
    direction.  tf32 tensor throughput is taken as half of bf16's."""
    import os
    from pathlib import Path

    peaks = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "nvlink_gbs": 770.0, "source": "fallback"}
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        peaks.update(hbm_gbs=float(d.get("hbm_gbs", peaks["hbm_gbs"])),
                     bf16_tflops=float(d.get("bf16_tflops", peaks["bf16_tflops"])), source="measured")
    peaks["nvlink_gbs"] = float(os.environ.get("RAICCL_NVLINK_GBS", peaks["nvlink_gbs"]))
    return peaks


def _roofline(layer, evs, before, after) -> dict:
    """Achieved fraction of each fused path of this rank's last call."""
    cfg, W, r = layer.cfg, layer.world, layer.rank
    pk = _peaks()
    tensor_tflops = pk["bf16_tflops"] * (0.5 if cfg.dtype == "fp32" else 1.0)
    delta = [{k: after[p][k] - before[p][k] for k in after[p]} for p in range(W)]
    out_bytes = sum(delta[p]["bytes_transferred"] for p in range(W) if p != r)
    ret_bytes = sum(delta[p]["return_bytes"] for p in range(W) if p != r)
    # per kind: the sum of its launches' (or phases') spans, and the wall
    # time from the first start to the last end; descriptors are dispatched
    # side by side, so the dispatch is measured over its wall time
    us: dict[str, float] = {}
    first: dict[str, int] = {}
    last: dict[str, int] = {}
    for e in evs:
        k = e["kind"]
        us[k] = us.get(k, 0.0) + (e["end_ns"] - e["start_ns"]) / 1e3
        first[k] = min(first.get(k, e["start_ns"]), e["start_ns"])
        last[k] = max(last.get(k, e["end_ns"]), e["end_ns"])
    wall = {k: (last[k] - first[k]) / 1e3 for k in us}
    rows = int(layer.rows_out.sum().item())
    f1 = 2.0 * rows * cfg.hidden * cfg.gemm1_n
    f2 = 2.0 * rows * cfg.ffn_hidden * cfg.out_dim

    def frac(target_us, span):
        return round(target_us / span, 3) if span and span > 0 else None

    res = {"rank": r, "peaks": pk, "rows": rows}
    if "dispatch" in us:
        tgt = out_bytes / (pk["nvlink_gbs"] * 1e3)
        span = wall["dispatch"]
        res["dispatch"] = {"nvlink_bytes": out_bytes, "span_us": round(span, 2), "busy_us": round(us["dispatch"], 2),
                           "achieved_gbs": round(out_bytes / (span * 1e3), 1) if span else None,
                           "roofline_us": round(tgt, 2), "fraction": frac(tgt, span)}
    if "gemm1" in us:
        tgt = f1 / (tensor_tflops * 1e6)
        res["gemm1"] = {"gflop": round(f1 / 1e9, 2), "span_us": round(us["gemm1"], 2),
                        "tflops": round(f1 / (us["gemm1"] * 1e6), 1), "roofline_us": round(tgt, 2),
                        "fraction": frac(tgt, us["gemm1"])}
    if "gemm2_return" in us:
        tgt = max(f2 / (tensor_tflops * 1e6), ret_bytes / (pk["nvlink_gbs"] * 1e3))
        res["gemm2_return"] = {"gflop": round(f2 / 1e9, 2), "nvlink_bytes": ret_bytes,
                               "span_us": round(us["gemm2_return"], 2), "roofline_us": round(tgt, 2),
                               "fraction": frac(tgt, us["gemm2_return"])}
    return res


FE_CLOCK_SLOTS = 128  # per-CTA stamps of the front end (kCtaClockSlots in csrc/kernels/moe_frontend.cu)


def _cta_clocks(layer) -> dict:
    """Summarise the front end's per-CTA %globaltimer stamps (us from the first
    worker's start): row 0 is the control CTA (trigger q begin / end at slots
    2 + 2q / 3 + 2q), rows 1.. the workers (chunk c begin / end at 2 + 2c /
    3 + 2c, descriptor q begin / rows done / end at 24 + 2q / 44 + q / 25 + 2q)."""
    import numpy as np

    clk = layer.tensors["fe_clock"].cpu().numpy().reshape(-1, FE_CLOCK_SLOTS).astype(np.float64)
    t0 = clk[1:, 0][clk[1:, 0] > 0].min()
    wk = (clk[1:] - t0) / 1e3
    wk[clk[1:] == 0] = np.nan
    r = lambda x: round(float(x), 2)
    first = ~np.isnan(wk[:, 21]) & ~np.isnan(wk[:, 22]) & (wk[:, 21] >= wk[:, 0])
    out = {"chunks": [], "descriptors": [], "triggers": [],
           "worker_start": {"med": r(np.nanmedian(wk[:, 0])), "max": r(np.nanmax(wk[:, 0]))},
           # resident batches: first token group in shared memory / routed (workers with a group)
           "first_group": ({"landed_med": r(np.median(wk[first, 21])), "landed_max": r(np.max(wk[first, 21])),
                            "routed_med": r(np.median(wk[first, 22])), "routed_max": r(np.max(wk[first, 22]))}
                           if first.any() else None)}
    # the first two units' phases (stamps 40.. and 64..: landed, warp 0's
    # products, its top-k finish, the CTA barrier), medians in us
    for name, b in (("unit0", 40), ("unit1", 64)):
        ok = ~np.isnan(wk[:, b]) & ~np.isnan(wk[:, b + 3]) & (wk[:, b] >= wk[:, 0])
        if ok.any():
            d = lambda i, j: r(np.median(wk[ok, b + j] - wk[ok, b + i]))
            out[name] = {"landed_med": r(np.median(wk[ok, b])), "products": d(0, 1), "finish": d(1, 2),
                         "barrier": d(2, 3), "workers": int(ok.sum())}
    for c in range(min(8, layer.cfg.chunks)):
        b, e, routed = wk[:, 2 + 2 * c], wk[:, 3 + 2 * c], wk[:, 52 + c]
        out["chunks"].append({"chunk": c, "begin_med": r(np.nanmedian(b)), "dur_med": r(np.nanmedian(e - b)),
                              "route_med": r(np.nanmedian(routed - b)), "publish_med": r(np.nanmedian(e - routed)),
                              "end_p50": r(np.nanmedian(e)), "end_p90": r(np.nanpercentile(e, 90)),
                              "end_max": r(np.nanmax(e))})
    for q in range(min(8, layer.cfg.n_desc)):
        b, mid, e = wk[:, 24 + 2 * q], wk[:, 44 + q], wk[:, 25 + 2 * q]
        ix, idn, rw, ids = wk[:, 68 + 4 * q], wk[:, 69 + 4 * q], wk[:, 70 + 4 * q], wk[:, 71 + 4 * q]
        ok = (ix >= b) & (rw <= mid) & (ids >= ix)  # this call's stamps (staged rows only)
        phase = ({"index_med": r(np.median(ix[ok] - b[ok])), "id_inputs_med": r(np.median(ids[ok] - ix[ok])),
                  "identity_med": r(np.median(idn[ok] - ids[ok])),
                  "rows_med": r(np.median(rw[ok] - idn[ok]))} if ok.any() else None)
        out["descriptors"].append({"desc": q, "begin_min": r(np.nanmin(b)), "begin_med": r(np.nanmedian(b)),
                                   "rows_med": r(np.nanmedian(mid - b)), "publish_max": r(np.nanmax(e - mid)),
                                   "end_max": r(np.nanmax(e)), "phases": phase})
    c0 = (clk[0] - t0) / 1e3
    for q in range(min(7, layer.cfg.n_desc)):
        out["triggers"].append({"trigger": q, "begin": r(c0[2 + 2 * q]), "end": r(c0[3 + 2 * q])})
    return out


if __name__ == "__main__":
    main()
