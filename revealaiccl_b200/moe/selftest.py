"""Multi-rank correctness run of the progressive MoE layer (one process per GPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m revealaiccl_b200.moe.selftest --configs full_tf32 r4_reference

For every config: one early call and one delayed call, each verified by the
fail-closed checker on every rank (identity rows, lost / duplicate /
wrong-expert / wrong-return rows, expert outputs against the fp32 oracle,
packing counters, differential replay of the device control plane), then the
early and delayed outputs must be bit-identical, and a captured CUDA graph of
the early arm replayed twice must reproduce them.  Rank 0 prints one JSON line
per config; the exit code is non-zero if any rank saw a failure.

This is the multi-GPU form of the reference's R4 correctness gate
(scripts/run_r4_a0_c0_full_moe.py:1080-1143: both arms verified per case,
Early/Delayed output-digest equivalence).
"""

from __future__ import annotations

import argparse
from datetime import timedelta
import json
import os
import sys


def run(configs: list[str], timeout_s: float, tokens: int) -> bool:
    import torch
    import torch.distributed as dist

    from .config import preset
    from .layer import ProgressiveMoELayer

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if local >= torch.cuda.device_count():
        # one rank per GPU: ranks that wait on each other must never share a GPU
        raise SystemExit(f"LOCAL_RANK={local} but only {torch.cuda.device_count()} GPU(s) on this node")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=timedelta(seconds=120),
                                device_id=dev)
    ok_all = True
    try:
        for name in configs:
            cfg = preset(name)
            if tokens:
                n = cfg.chunks
                cfg = cfg.with_overrides(tokens_per_rank=tokens, chunk_sizes=(tokens // n,) * n)
            rec = {"config": name, "world": world, "tokens_per_rank": cfg.tokens_per_rank}
            ok = True
            layer = ProgressiveMoELayer(cfg, device=dev, timeout_s=timeout_s)
            try:
                layer.forward("early")
                rep = layer.verify()
                ok &= bool(rep["pass"])
                early = layer.out.clone()
                layer.forward("delayed")
                ok &= bool(layer.verify()["pass"])
                same = torch.equal(early, layer.out)
                layer.capture("early")
                layer.replay()
                layer.replay()
                torch.cuda.synchronize(dev)
                ok &= bool(layer.verify()["pass"])
                graph_same = torch.equal(early, layer.out)
                ok &= same and graph_same
                # end-to-end calls: the pinned batch streamed into the running front end
                host_in = torch.empty(layer.inputs.tokens.shape, dtype=layer.inputs.tokens.dtype, pin_memory=True)
                host_in.copy_(layer.inputs.tokens.cpu())
                host_out = torch.empty(layer.out.shape, dtype=layer.out.dtype, pin_memory=True)
                stream_same = True
                for _ in range(2):
                    layer.device_barrier()
                    layer(host_in, host_out, arm="early")
                    torch.cuda.synchronize(dev)
                    ok &= bool(layer.verify()["pass"])
                    stream_same &= torch.equal(host_out, early.cpu())
                ok &= stream_same
                rec.update(early_delayed_identical=same, graph_identical=graph_same, streamed_identical=stream_same,
                           launches_per_call=layer.launches_per_call)
            except Exception as exc:  # reported, then the collective error path below
                ok = False
                rec["error"] = f"{type(exc).__name__}: {exc}"
            finally:
                try:
                    layer.close()
                except Exception as exc:
                    ok = False
                    rec.setdefault("error", f"close: {exc}")
            flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
            if world > 1:
                dist.all_reduce(flag)
            rec["pass"] = int(flag.item()) == 0
            ok_all &= rec["pass"]
            if rank == 0:
                print(json.dumps(rec), flush=True)
            elif not ok:
                print(json.dumps({"rank": rank, **rec}), file=sys.stderr, flush=True)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
    return ok_all


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="revealaiccl_b200.moe.selftest")
    ap.add_argument("--configs", nargs="+", default=["full_tf32"])
    ap.add_argument("--timeout", type=float, default=10.0, help="bound of every device-side wait (s)")
    ap.add_argument("--tokens", type=int, default=0, help="override tokens per rank (uniform chunks)")
    args = ap.parse_args(argv)
    sys.exit(0 if run(args.configs, args.timeout, args.tokens) else 1)


if __name__ == "__main__":
    main()
