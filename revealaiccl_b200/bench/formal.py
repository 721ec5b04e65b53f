"""Paired Early-vs-Delayed corpus of the full MoE layer (one process per GPU).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m revealaiccl_b200.bench.formal --config r4_reference --seeds 0 1 2 --jobs 10 \\
        --output-dir runs/formal

The device-driven counterpart of the reference's formal R4 study
(scripts/run_r4_f0_full_moe.py, scripts/analyze_r4_f0_full_moe.py): for every
seed x case family x job it runs one early and one delayed layer call (order
alternating per job), each after an L2 flush and a cross-GPU device barrier,
times each call with CUDA events on the layer's stream, takes the max over
ranks, and records Delta = T_delayed - T_early together with output
equivalence.  The first pair of every (seed, family) is also verified by the
fail-closed checker.  Rank 0 writes the corpus and its paired analysis
(``paired.analyze_pairs``: bootstrap median CI, per-seed / per-family
summaries, the progressive-gain gate).
"""

from __future__ import annotations

import argparse
from datetime import timedelta
import json
import os
from pathlib import Path


def main(argv=None) -> None:
    import torch
    import torch.distributed as dist

    from ..moe.config import CASE_ORDER, preset, r4_case
    from ..moe.layer import ProgressiveMoELayer
    from .paired import analyze_pairs, sha256_file, write_report

    ap = argparse.ArgumentParser(prog="revealaiccl_b200.bench.formal")
    ap.add_argument("--config", default="r4_reference")
    ap.add_argument("--families", nargs="*", default=None,
                    help="case families (default: the 7 reference families for r4_reference, else 'balanced')")
    ap.add_argument("--seeds", nargs="+", type=int, default=[0, 1, 2])
    ap.add_argument("--jobs", type=int, default=10, help="pairs per (seed, family)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--graph", action="store_true", help="replay captured graphs of both arms")
    ap.add_argument("--output-dir", type=Path, required=True)
    args = ap.parse_args(argv)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=timedelta(seconds=120), device_id=dev)
    families = args.families or (list(CASE_ORDER) if args.config == "r4_reference" else ["balanced"])
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    pairs, verified = [], []
    try:
        for seed in args.seeds:
            for fam in families:
                cfg = r4_case(fam) if args.config == "r4_reference" else preset(args.config)
                layer = ProgressiveMoELayer(cfg, device=dev, timeout_s=10.0, seed=seed)
                try:
                    for arm in ("early", "delayed"):
                        layer.forward(arm)
                        verified.append(bool(layer.verify()["pass"]))
                    if args.graph:
                        for arm in ("early", "delayed"):
                            layer.forward(arm)
                            layer.capture(arm)

                    def call(arm: str) -> float:
                        flush.zero_()
                        layer.device_barrier()
                        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        s.record(layer.comm_stream)
                        layer.replay(arm) if args.graph else layer.forward(arm)
                        e.record(layer.comm_stream)
                        torch.cuda.synchronize(dev)
                        return max_over_ranks(s.elapsed_time(e))

                    for _ in range(args.warmup):
                        call("early"), call("delayed")
                    for job in range(args.jobs):
                        order = ("early", "delayed") if job % 2 == 0 else ("delayed", "early")
                        t, outs = {}, {}
                        for arm in order:
                            t[arm] = call(arm)
                            outs[arm] = layer.out.clone()
                        same = torch.tensor([0 if torch.equal(outs["early"], outs["delayed"]) else 1],
                                            dtype=torch.int32, device=dev)
                        if world > 1:
                            dist.all_reduce(same)
                        pairs.append({"seed": seed, "family": fam, "job": job, "early_ms": t["early"],
                                      "delayed_ms": t["delayed"], "delta_ms": t["delayed"] - t["early"],
                                      "pass": int(same.item()) == 0})
                finally:
                    layer.close()
        if rank == 0:
            corr = {"checker_pass_100pct": all(verified), "paired_equivalence_100pct": all(p["pass"] for p in pairs)}
            corpus = {"schema_version": 1, "study": "paired early-vs-delayed full MoE layer",
                      "protocol": {"config": args.config, "seeds": args.seeds, "families": families,
                                   "jobs_per_family": args.jobs, "world": world, "graph": args.graph,
                                   "timing": "CUDA events on the layer stream, max over ranks, L2 flushed"},
                      "correctness": corr, "pairs": pairs}
            args.output_dir.mkdir(parents=True, exist_ok=True)
            src = args.output_dir / "corpus.json"
            src.write_text(json.dumps(corpus, indent=2) + "\n", encoding="utf-8")
            result = analyze_pairs(pairs, key="delta_ms", seeds=args.seeds, families=families, correctness=corr)
            result["source"] = {"path": str(src), "sha256": sha256_file(src)}
            out = write_report(result, args.output_dir)
            print(json.dumps({"output": str(out), "gate": result["gate"], "primary_ms": result["primary_delta"]}),
                  flush=True)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
