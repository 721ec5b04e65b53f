"""Reference arm of bench.py: the unmodified reference build, stock code path.

The reference source tree has no packaging metadata, so ``pip install
--target baseline/_ref`` refuses it; ``baseline/_ref`` holds a verbatim copy of
the tree instead and nothing in it is edited.  This module only performs
what the reference's own driver ``scripts/run_r4_a0_c0_full_moe.py::main``
does before calling ``_run_arm`` (topology load, static plan compile, JIT
build of its C++ event bridge, seeded router and expert weights, case
inputs, streams) and then calls the reference's ``_run_arm`` for the early
("C") and delayed ("D") arms, paired per step.  The reported latency is the
reference's own full-MoE primary makespan (first Router launch -> combined
output, ``timing.primary_makespan_us``), max over ranks.

The reference driver hard-codes a world size of two (``main`` raises on any
other size, and ``_run_arm`` builds its packing state with ``world_size=2``),
so every other GPU count prints an ``unavailable`` line.

End to end: before each early-arm call the case's tokens are copied from
pinned host memory into the device tensor the reference reads
(``tokens_device``), on the current stream, which ``_run_arm`` synchronises
before its first Router launch.  The reference's combined output is a host
array when ``primary_done_host_ns`` is taken, so the end-to-end time is that
stamp minus the host clock read just before the copy (same monotonic clock).
"""

from __future__ import annotations

import json
import os
from pathlib import Path
import statistics
import sys
import time

REF_ROOT = Path(__file__).resolve().parent / "_ref"


def _unavailable(why: str) -> dict:
    return {"impl": "reference", "unavailable": why}


def run_reference(args, clock_sampler=None) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not (REF_ROOT / "scripts" / "run_r4_a0_c0_full_moe.py").exists():
        return _unavailable("reference tree not present under baseline/_ref") if rank == 0 else None
    if args.config != "r4_reference":
        return _unavailable(
            "the reference's full-MoE path runs only its R4 shape: its driver hard-codes D=2048, 4 experts, "
            "top-1 and a 2048->32->16 expert (scripts/run_r2_f0_integrated.py:59-66, "
            "scripts/run_r4_a0_c0_full_moe.py:50-51, one expert per token in scripts/run_r3_a0_c0.py:155-161) "
            "and its expert MLP is ReLU-only (rlccl/transport/reference_full_moe.py:263-281), so "
            f"{args.config} (top-k > 1, GELU/SwiGLU experts) has no stock reference path") if rank == 0 else None
    if args.gpus != 2 or world != 2:
        return _unavailable("the reference full-MoE driver requires exactly two ranks "
                            "(scripts/run_r4_a0_c0_full_moe.py:1062)") if rank == 0 else None
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    sys.path.insert(0, str(REF_ROOT))
    from scripts import run_r4_a0_c0_full_moe as r4  # noqa: E402  (reference module, unmodified)

    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist.init_process_group("nccl", init_method="env://", timeout=timedelta(seconds=300))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    try:
        topology, _ = r4._load_rear4_topology(REF_ROOT)
        plan = r4.StaticPlanCompiler().compile(topology)
        build = Path("/tmp") / f"raiccl_reference_bridge_rank{rank}"
        ext = r4._load_bridge_extension(build)
        allowed = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else [-1]
        bridge = ext.IntegratedEventBridge(r4.CHUNKS, allowed[-(rank + 1)], rank)
        router_stream = torch.cuda.Stream(device=device)
        comm_stream = torch.cuda.Stream(device=device)
        rw_cpu, rb_cpu = r4.seed_router_params(r4.D, r4.EXPERTS, r4.ROUTER_SEED)
        router_weight = rw_cpu.to(device)
        expert_weights = tuple(v.to(device) for v in r4.seed_reference_experts(
            r4.D, r4.EXPERT_HIDDEN, r4.EXPERT_OUTPUT, r4.EXPERTS, r4.EXPERT_SEED))
        case = "balanced"
        case_data = r4._case_inputs(case, rank)
        tokens = torch.from_numpy(case_data["tokens"]).to(device)
        bias = (rb_cpu + torch.from_numpy(case_data["bias_delta"])).to(device)
        T = r4.TOTAL_TOKENS
        mask = torch.zeros((T, r4.EXPERTS), dtype=torch.bool, device=device)
        mask[torch.arange(T, device=device), torch.from_numpy(case_data["topology_sources"]).to(device)] = True
        chunks = tuple(tokens.narrow(0, case_data["chunk_offsets"][i], case_data["chunk_sizes"][i])
                       for i in range(r4.CHUNKS))
        masks = tuple(mask.narrow(0, case_data["chunk_offsets"][i], case_data["chunk_sizes"][i])
                      for i in range(r4.CHUNKS))

        host_tokens = torch.from_numpy(case_data["tokens"]).pin_memory()

        def arm(name: str, copy_in: bool = False) -> tuple[float, float]:
            dist.barrier()
            t0 = time.monotonic_ns()
            if copy_in:
                tokens.copy_(host_tokens, non_blocking=True)
            res = r4._run_arm(
                arm=name, case_name=case, rank=rank, topology=topology, plan=plan, bridge=bridge,
                case_data=case_data, tokens_device=tokens, token_chunks=chunks, mask_chunks=masks,
                router_weight=router_weight, router_bias=bias, expert_weights=expert_weights,
                router_stream=router_stream, comm_stream=comm_stream)
            timing = res["timing"]
            return (float(timing["primary_makespan_us"]) / 1e3,
                    (int(timing["primary_done_host_ns"]) - t0) / 1e6)

        for _ in range(args.warmup):
            arm("C", copy_in=True)
            arm("D")
        bus = None
        props = torch.cuda.get_device_properties(device)
        if hasattr(props, "pci_bus_id") and hasattr(props, "pci_device_id"):
            bus = f"{int(props.pci_bus_id):02X}:{int(props.pci_device_id):02X}.0"
        gathered = [None] * world
        dist.all_gather_object(gathered, bus)
        sampler = clock_sampler([b for b in gathered if b]) if (clock_sampler and rank == 0) else None
        if sampler:
            sampler.__enter__()
        early, delayed, e2e = [], [], []
        for _ in range(args.steps):
            ms, e2e_ms = arm("C", copy_in=True)
            early.append(ms)
            e2e.append(e2e_ms)
            delayed.append(arm("D")[0])
        if sampler:
            sampler.__exit__(None, None, None)
        t = torch.tensor([early, delayed, e2e], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        early, delayed, e2e = t[0].tolist(), t[1].tolist(), t[2].tolist()
        bridge.stop()
    finally:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    p50 = statistics.median(early)
    return {
        "impl": "reference", "metric": "full MoE layer p50 ms + Delta=T_delayed-T_early", "value": round(p50, 4),
        "unit": "ms", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.fmean(early), 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": round(p50 / 480.265, 6),
        "vs_baseline_note": "reference published p50 of the same R4 config on 2x V100 (other hardware)",
        "dtype": "fp32",
        "data": "synthetic (reference balanced case; seeded reference weights)",
        "config": {"model": "r4_reference: 4 experts top-1, D=2048, expert 2048->32 relu->16",
                   "global_batch": r4.TOTAL_TOKENS * world, "seq_len": r4.TOTAL_TOKENS, "parallelism": f"ep{world}",
                   "timing": "reference primary makespan (host monotonic ns), max over ranks"},
        "p50_early_ms": round(p50, 4), "p50_delayed_ms": round(statistics.median(delayed), 4),
        "delta_ms": round(statistics.median([d - e for e, d in zip(early, delayed)]), 4),
        "e2e": {"value": round(statistics.median(e2e), 4), "unit": "ms",
                "h2d_bytes_per_step": int(host_tokens.numel() * host_tokens.element_size()),
                "d2h_bytes_per_step": int(r4.TOTAL_TOKENS * r4.EXPERT_OUTPUT * 4),
                "timing": "pinned H2D of the case tokens + the reference primary path, whose combined "
                          "output is a host array (host monotonic ns), max over ranks"},
        "clocks": sampler.summary() if sampler else None,
    }


if __name__ == "__main__":  # pragma: no cover
    print(json.dumps(_unavailable("run through bench.py --impl reference")))
