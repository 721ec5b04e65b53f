#!/usr/bin/env python
"""Full progressive MoE layer benchmark (one rank per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config full_tf32|r4_reference|...]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W
    python bench.py --impl reference ...     (the unmodified reference build)
    python bench.py --impl nccl ...          (PyTorch + NCCL baseline layer, same preset and N)

Metric: full MoE layer p50 latency (first Router launch -> combined output),
device-timed with CUDA events on the layer's stream, max over ranks per step,
plus the progressive gain Delta = T_delayed - T_early (paired per step).
Every step of both arms starts after an L2 flush (a 256 MiB write) and a
device-side cross-GPU barrier; the flush and barrier are outside the step's
events.  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Published reference number of this metric: the full-MoE primary makespan
# p50 of the early arm on the reference's R4 layer (4096 tokens/rank, D=2048,
# 4 experts top-1, 2048->32 ReLU->16 experts, 8 x 512 chunks), 2 x V100
# (docs/phase_r4/R4_F0_REPORT.md:62).  It is quoted on that one configuration,
# so vs_baseline is reported only for it (and is null for the others).
PUBLISHED_P50_MS = {"r4_reference": 480.265}
PUBLISHED_NOTE = "reference published p50 of the same R4 config on 2x V100 (other hardware)"
METRIC = "full MoE layer p50 ms + Delta=T_delayed-T_early"
DEFAULT_CONFIG = "r4_reference"


def vs_baseline(config: str, p50_ms: float):
    ref = PUBLISHED_P50_MS.get(config)
    return None if ref is None else round(p50_ms / ref, 6)


def _env_world() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons of the given PCI bus ids."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_ids: list[str]):
        self.bus_ids = {str(b).lower()[-7:] for b in bus_ids}
        self.rows: list[list[str]] = []
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 10 and parts[1].lower()[-7:] in self.bus_ids:
                        self.rows.append(parts)
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=10)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in self.rows if r[3].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[6:10]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def _max_over_ranks(values, world: int, device):
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.cpu().tolist()


def run_product(args) -> dict | None:
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from revealaiccl_b200.bench.paired import bootstrap_median
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.layer import ProgressiveMoELayer

    rank, world, local = _env_world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if local >= torch.cuda.device_count():
        # one rank per GPU: ranks that wait on each other must never share a GPU
        raise SystemExit(f"LOCAL_RANK={local} but only {torch.cuda.device_count()} GPU(s) on this node")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cfg = preset(args.config)
    layer = ProgressiveMoELayer(cfg, device=dev, timeout_s=10.0, progressive=bool(args.progressive),
                                dispatch_ctas=args.dispatch_ctas)
    try:
        # correctness gate (untimed): both arms verified, outputs identical
        layer.forward("early")
        layer.verify()
        ref_out = layer.out.clone()
        layer.forward("delayed")
        layer.verify()
        if not torch.equal(ref_out, layer.out):
            raise RuntimeError("early and delayed arms produced different outputs")
        launches = {"early": layer.capture("early"), "delayed": layer.capture("delayed")}
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        cs = layer.comm_stream

        def step(arm):
            with torch.cuda.stream(cs):
                flush.zero_()
            layer.device_barrier()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(cs)
            layer.replay(arm)
            e.record(cs)
            return s, e

        for _ in range(args.warmup):
            step("early")
            step("delayed")
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        props = torch.cuda.get_device_properties(dev)
        bus = (f"{int(props.pci_bus_id):02X}:{int(props.pci_device_id):02X}.0"
               if hasattr(props, "pci_bus_id") and hasattr(props, "pci_device_id") else None)
        bus_ids = [bus] if bus else []
        if world > 1:
            gathered = [None] * world
            dist.all_gather_object(gathered, bus)
            bus_ids = [b for b in gathered if b]
        sampler = ClockSampler(bus_ids) if rank == 0 else None
        if sampler:
            sampler.__enter__()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t_begin = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_begin.record(cs)
        events = []
        for _ in range(args.steps):
            events.append((step("early"), step("delayed")))
        t_end.record(cs)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        if sampler:
            sampler.__exit__(None, None, None)
        layer.check_status()
        early = [a[0].elapsed_time(a[1]) for a, _ in events]
        delayed = [b[0].elapsed_time(b[1]) for _, b in events]
        bracket = t_begin.elapsed_time(t_end)
        early = _max_over_ranks(early, world, dev)
        delayed = _max_over_ranks(delayed, world, dev)
        bracket = _max_over_ranks([bracket], world, dev)[0]
        deltas = [d - e for e, d in zip(early, delayed)]
        layer.verify()  # the timed replays left a checkable last call

        # end-to-end through the public call: pinned H2D of the step's tokens,
        # digests, the layer (captured graph), D2H of the combined output
        host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
        host_in.copy_(layer.inputs.tokens.cpu())
        host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
        e2e = []
        for i in range(args.warmup + args.steps):
            with torch.cuda.stream(cs):
                flush.zero_()
            layer.device_barrier()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(cs)
            layer(host_in, host_out, arm="early")
            e.record(cs)
            if i >= args.warmup:
                e2e.append((s, e))
        torch.cuda.synchronize(dev)
        e2e_ms = _max_over_ranks([s.elapsed_time(e) for s, e in e2e], world, dev)
        clocks = sampler.summary() if sampler else None
        if rank != 0:
            return None
        p50 = statistics.median(early)
        ci = bootstrap_median(deltas)  # paired median CI, 10k resamples
        tokens_total = cfg.tokens_per_rank * world
        return {
            "metric": METRIC, "value": round(p50, 4), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(statistics.fmean(early), 4),
            "higher_is_better": False, "scaling": "weak",
            "vs_baseline": vs_baseline(args.config, p50), "vs_baseline_note": PUBLISHED_NOTE,
            "dtype": "fp32-tf32" if cfg.dtype == "fp32" else "bf16",
            "data": "synthetic (reference seeded token/router/expert recipes; random-init weights)",
            "config": {"model": f"{cfg.name}: {cfg.experts} experts top-{cfg.top_k}, D={cfg.hidden}, "
                                f"expert {cfg.hidden}->{cfg.ffn_hidden} {cfg.activation}->{cfg.out_dim}",
                       "global_batch": tokens_total, "seq_len": cfg.tokens_per_rank,
                       "tokens_per_rank": cfg.tokens_per_rank, "chunks": cfg.chunks,
                       "parallelism": f"ep{world}", "l2": "256 MiB flush before every timed step",
                       "progressive_gemm1": bool(layer.runner.progressive()),
                       "dispatch_ctas": args.dispatch_ctas},
            "p50_early_ms": round(p50, 4), "p50_delayed_ms": round(statistics.median(delayed), 4),
            "delta_ms": round(statistics.median(deltas), 4),
            "delta_ci95_ms": [round(ci["ci95_lower"], 4), round(ci["ci95_upper"], 4)],
            "p95_early_ms": round(sorted(early)[max(0, int(0.95 * len(early)) - 1)], 4),
            "tokens_per_s": round(tokens_total / (p50 / 1e3), 1),
            "bracket_ms": round(bracket, 3),
            "e2e": {"value": round(statistics.median(e2e_ms), 4), "unit": "ms",
                    "h2d_bytes_per_step": int(layer.inputs.tokens.numel() * layer.inputs.tokens.element_size()),
                    "d2h_bytes_per_step": int(layer.out.numel() * layer.out.element_size())},
            "gpu_launches": int((launches["early"] + launches["delayed"]) * args.steps),
            "clocks": clocks, "verified": True,
        }
    finally:
        try:
            layer.close()
        except Exception:
            pass
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


def run_nccl(args) -> dict | None:
    """The PyTorch + NCCL baseline layer (transport/nccl_baseline.py) at the
    same preset and GPU count: router per chunk, per-descriptor count exchange
    and uneven all_to_all_single, PyTorch experts, NCCL return, scatter-add
    combine.  Device-timed with CUDA events around each call (which synchronises
    with the host inside, as the reference's driver does), max over ranks."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from revealaiccl_b200.bench.paired import bootstrap_median
    from revealaiccl_b200.moe.config import preset
    from revealaiccl_b200.moe.oracle import layer_reference
    from revealaiccl_b200.transport.nccl_baseline import NcclMoELayer

    rank, world, local = _env_world()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    cfg = preset(args.config)
    try:
        layer = NcclMoELayer(cfg, device=dev)
        out_e = layer.forward("early").clone()
        ref, _ = layer_reference(cfg, layer.inputs.tokens, layer.weights, layer.ids.int(), layer.gates)
        tol = 2e-2 if cfg.dtype == "bf16" else 5e-3
        if not torch.allclose(out_e, ref, atol=tol, rtol=tol):
            raise RuntimeError("NCCL baseline output differs from the fp32 oracle")
        if not torch.equal(out_e, layer.forward("delayed")):
            raise RuntimeError("NCCL baseline early and delayed arms differ")
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        cur = torch.cuda.current_stream(dev)

        def step(arm, host_in=None, host_out=None):
            flush.zero_()
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(cur)
            if host_in is not None:
                layer.inputs.tokens.copy_(host_in, non_blocking=True)
            out = layer.forward(arm)
            if host_out is not None:
                host_out.copy_(out, non_blocking=True)
            e.record(cur)
            torch.cuda.synchronize(dev)
            return s.elapsed_time(e)

        for _ in range(args.warmup):
            step("early")
            step("delayed")
        early, delayed = [], []
        for _ in range(args.steps):
            early.append(step("early"))
            delayed.append(step("delayed"))
        host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
        host_in.copy_(layer.inputs.tokens.cpu())
        host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
        e2e = [step("early", host_in, host_out) for _ in range(args.steps)]
        early = _max_over_ranks(early, world, dev)
        delayed = _max_over_ranks(delayed, world, dev)
        e2e = _max_over_ranks(e2e, world, dev)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
    if rank != 0:
        return None
    p50 = statistics.median(early)
    deltas = [d - e for e, d in zip(early, delayed)]
    ci = bootstrap_median(deltas)
    return {
        "impl": "nccl", "metric": METRIC, "value": round(p50, 4), "unit": "ms", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(statistics.fmean(early), 4),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": vs_baseline(args.config, p50),
        "dtype": "fp32-tf32" if cfg.dtype == "fp32" else "bf16",
        "data": "synthetic (the product layer's seeded inputs and weights)",
        "config": {"model": f"{cfg.name}: {cfg.experts} experts top-{cfg.top_k}, D={cfg.hidden}, "
                            f"expert {cfg.hidden}->{cfg.ffn_hidden} {cfg.activation}->{cfg.out_dim}",
                   "global_batch": cfg.tokens_per_rank * world, "seq_len": cfg.tokens_per_rank,
                   "parallelism": f"ep{world}", "l2": "256 MiB flush before every timed step",
                   "path": "PyTorch router/experts + NCCL all_to_all_single per descriptor"},
        "p50_early_ms": round(p50, 4), "p50_delayed_ms": round(statistics.median(delayed), 4),
        "delta_ms": round(statistics.median(deltas), 4),
        "delta_ci95_ms": [round(ci["ci95_lower"], 4), round(ci["ci95_upper"], 4)],
        "e2e": {"value": round(statistics.median(e2e), 4), "unit": "ms",
                "h2d_bytes_per_step": int(host_in.numel() * host_in.element_size()),
                "d2h_bytes_per_step": int(host_out.numel() * host_out.element_size())},
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    # r4_reference (default): the reference's own full-MoE layer, the one configuration
    # its stock driver runs, so both arms measure the same shape (4096 tokens/rank,
    # D=2048, 4 experts top-1, 2048->32 ReLU->16, fp32, 8 x 512 chunks).  full_tf32,
    # skewed_bf16, mixtral_8x7b and deepseek_v2_lite are explicit runs.
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--impl", choices=("product", "reference", "nccl"), default="product")
    # expert side: GEMM-1 takes 256-row tiles as descriptors arrive (1) or after the
    # whole batch (0); front-end workers that keep dispatching (0: all of them)
    ap.add_argument("--progressive", type=int, default=0, choices=(0, 1))
    ap.add_argument("--dispatch-ctas", type=int, default=0)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        from baseline.reference_arm import run_reference

        out = run_reference(args, ClockSampler)
    elif args.impl == "nccl":
        out = run_nccl(args)
    else:
        out = run_product(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
