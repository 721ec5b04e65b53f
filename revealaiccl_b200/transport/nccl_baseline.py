"""NCCL baseline transport: the reference's two-sided uneven AlltoAllv path.

Reference-equivalent arm (scripts/run_r3_a0_c0.py:260-316,
scripts/run_r4_a0_c0_full_moe.py:104-261) generalised from two ranks to any
world size: host-packed payloads are copied to the device, the per-descriptor
send counts are exchanged with one ``all_to_all_single``, then the identity
rows and the feature rows travel in two uneven ``all_to_all_single`` calls.
This is the baseline the device data plane is measured against, never the
product path.
"""

from __future__ import annotations

from dataclasses import dataclass
import time
from typing import Sequence

import numpy as np
import torch
import torch.distributed as dist


@dataclass
class ExchangeTiming:
    h2d_us: float
    count_exchange_us: float
    payload_us: float
    d2h_us: float


def exchange_counts(sendcounts: Sequence[int], device: torch.device, group=None) -> tuple[int, ...]:
    world = dist.get_world_size(group)
    send = torch.tensor([int(v) for v in sendcounts], dtype=torch.int64, device=device)
    recv = torch.empty(world, dtype=torch.int64, device=device)
    dist.all_to_all_single(recv, send, group=group)
    return tuple(int(v) for v in recv.cpu().tolist())


def exchange_pair(metadata: np.ndarray, values: np.ndarray, sendcounts: Sequence[int], *,
                  meta_width: int, value_width: int, device: torch.device, group=None,
                  value_dtype: torch.dtype = torch.float32) -> tuple[np.ndarray, np.ndarray, tuple[int, ...], ExchangeTiming]:
    """Count exchange + two uneven all_to_all_single (identity rows, values)."""
    t0 = time.perf_counter_ns()
    send_meta = torch.from_numpy(np.ascontiguousarray(metadata.reshape(-1))).to(device)
    send_vals = torch.from_numpy(np.ascontiguousarray(values.reshape(-1))).to(device=device, dtype=value_dtype)
    t1 = time.perf_counter_ns()
    recvcounts = exchange_counts(sendcounts, device, group)
    t2 = time.perf_counter_ns()
    total = sum(recvcounts)
    recv_meta = torch.empty(total * meta_width, dtype=torch.int64, device=device)
    recv_vals = torch.empty(total * value_width, dtype=value_dtype, device=device)
    dist.all_to_all_single(recv_meta, send_meta, output_split_sizes=[c * meta_width for c in recvcounts],
                           input_split_sizes=[int(c) * meta_width for c in sendcounts], group=group)
    dist.all_to_all_single(recv_vals, send_vals, output_split_sizes=[c * value_width for c in recvcounts],
                           input_split_sizes=[int(c) * value_width for c in sendcounts], group=group)
    torch.cuda.synchronize(device)
    t3 = time.perf_counter_ns()
    meta = recv_meta.cpu().numpy().reshape(-1, meta_width).copy()
    vals = recv_vals.float().cpu().numpy().reshape(-1, value_width).copy()
    t4 = time.perf_counter_ns()
    return meta, vals, recvcounts, ExchangeTiming((t1 - t0) / 1e3, (t2 - t1) / 1e3, (t3 - t2) / 1e3,
                                                  (t4 - t3) / 1e3)


def device_alltoallv(send: torch.Tensor, sendcounts: Sequence[int], recvcounts: Sequence[int],
                     row_width: int, group=None) -> torch.Tensor:
    """Uneven AlltoAllv of device rows (no host staging) — the NCCL form of the
    product's dispatch, used for the transport microbenchmark."""
    out = torch.empty(sum(int(c) for c in recvcounts) * row_width, dtype=send.dtype, device=send.device)
    dist.all_to_all_single(out, send.reshape(-1), output_split_sizes=[int(c) * row_width for c in recvcounts],
                           input_split_sizes=[int(c) * row_width for c in sendcounts], group=group)
    return out.reshape(-1, row_width)


__all__ = ["ExchangeTiming", "device_alltoallv", "exchange_counts", "exchange_pair"]
