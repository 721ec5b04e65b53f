"""NVLink peer put bandwidth sweep (one rank per GPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m revealaiccl_b200.bench.peer_bandwidth [--sizes 1M,16M,256M] [--iters 20] [--pattern alltoall|pair]

``alltoall``: every rank puts ``size`` bytes to every other rank at once
(one put per peer, each on its own stream with its share of the SMs), then
waits for all incoming signals.  ``pair``: rank r puts to rank r ^ 1 (both
directions at once).  One iteration is device-timed from before the puts
to after the waits, max over ranks.  Reported per size: the time, the
bytes each GPU sent, ``send_gbs`` = those bytes / time (per GPU, per
direction: the figure the NVLink roofline divides by) and ``busbw_gbs``,
the all-to-all bus bandwidth in NCCL's convention (algbw x (N - 1) / N with
algbw = N x size / time).  This is the bus-GB/s sweep of the dispatch
traffic pattern and the link-bandwidth measurement behind the roofline
fractions of bench/layer_probe.py.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics


def _size(text: str) -> int:
    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    t = text.strip().upper()
    return int(float(t[:-1]) * mult[t[-1]]) if t[-1] in mult else int(t)


def _pattern(rank: int, nbytes: int, dev):
    """The payload rank ``rank`` puts: int32 words (index * 2654435761 + rank) mod 2^31."""
    import torch

    i = torch.arange(nbytes // 4, dtype=torch.int64, device=dev)
    return ((i * 2654435761 + rank) % (1 << 31)).to(torch.int32)


def main(argv=None) -> None:
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from ..parallel.peer_ops import PeerOps

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--sizes", default="64K,1M,4M,16M,64M,256M")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--pattern", default="alltoall", choices=("alltoall", "pair"))
    ap.add_argument("--grid", type=int, default=0, help="CTAs per put (0: SMs / peers)")
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rank = dist.get_rank() if world > 1 else 0
    sizes = [_size(s) for s in args.sizes.split(",")]
    ops = PeerOps(max(sizes), dev, timeout_s=5.0)
    if args.pattern == "pair" and world % 2:
        raise SystemExit("pair pattern needs an even number of ranks")
    peers = [p for p in range(world) if p != rank] if args.pattern == "alltoall" else [rank ^ 1]
    if world == 1:
        peers = [0]  # one GPU: a local put (HBM copy) through the same kernels
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    grid = args.grid or max(1, sms // len(peers))
    streams = [torch.cuda.Stream(device=dev) for _ in peers]
    rows = []
    try:
        for size in sizes:
            src = _pattern(rank, size, dev)
            times = []
            for it in range(args.warmup + args.iters):
                torch.cuda.synchronize(dev)
                if world > 1:
                    dist.barrier()
                cur = torch.cuda.current_stream(dev)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(cur)
                for st, p in zip(streams, peers):
                    st.wait_stream(cur)
                    with torch.cuda.stream(st):
                        ops.put(p, src, grid=grid)
                for st in streams:
                    cur.wait_stream(st)
                for p in peers:
                    ops.expect(p)
                    ops.wait(p)
                e.record(cur)
                torch.cuda.synchronize(dev)
                if it >= args.warmup:
                    times.append(s.elapsed_time(e))
            ops.check_status()
            if world > 1:
                t = torch.tensor(times, dtype=torch.float64, device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                times = t.tolist()
            ms = statistics.median(times)
            sent = size * len(peers)
            row = {"bytes": size, "ms": round(ms, 4), "sent_bytes_per_gpu": sent,
                   "send_gbs": round(sent / (ms * 1e6), 1)}
            if args.pattern == "alltoall" and world > 1:
                algbw = world * size / (ms * 1e6)
                row["busbw_gbs"] = round(algbw * (world - 1) / world, 1)
            rows.append(row)
        # every received slot holds its sender's pattern of the last size
        ok = all(bool(torch.equal(ops.slot(p, size).view(torch.int32), _pattern(p, size, dev))) for p in peers)
        if world > 1:
            flag = torch.tensor([0 if ok else 1], device=dev)
            dist.all_reduce(flag)
            ok = int(flag.item()) == 0
    finally:
        ops.close()
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"pattern": args.pattern, "world": world, "grid_per_put": grid, "data_ok": ok,
                          "counters": ops.counters, "sweep": rows}))


if __name__ == "__main__":
    main()
