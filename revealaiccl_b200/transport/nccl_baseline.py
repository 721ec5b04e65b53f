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


# ---------------------------------------------------------------------------
# The whole layer on PyTorch + NCCL (the baseline arm of bench.py)
# ---------------------------------------------------------------------------
_META = 8  # int64 identity fields per forward row: token id, source, destination,
#            expert, position, chunk, choice, descriptor


class NcclMoELayer:
    """The progressive MoE layer built the way the reference builds it, on any
    world size and any preset: a PyTorch router per chunk on its own stream,
    the host waiting for each chunk, then per revealed descriptor a count
    exchange and two uneven ``all_to_all_single`` calls (identity rows and
    feature rows); PyTorch expert MLPs per local expert once every descriptor
    has arrived; the outputs back to their source ranks with one more uneven
    ``all_to_all_single``; and a gate-weighted scatter-add to the original
    positions.  Reference: scripts/run_r4_a0_c0_full_moe.py:104-261 (count and
    payload exchange), rlccl/transport/reference_full_moe.py:249-281 (expert
    loop), scripts/run_r4_a0_c0_full_moe.py:628-838 (return and combine).

    The early arm exchanges descriptor q as soon as its last chunk is routed;
    the delayed arm waits for the final chunk.  Every collective is NCCL; no
    kernel of this repository runs on this path.  Inputs and weights come from
    the same seeded recipes as the product layer, so both compute one layer.
    """

    def __init__(self, cfg, *, device: torch.device, group=None, seed: int = 0) -> None:
        from ..moe.inputs import make_rank_inputs, make_weights

        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.device = device
        self.inputs = make_rank_inputs(cfg, self.rank, self.world, device, seed=seed)
        self.weights = make_weights(cfg, device, seed=seed)
        W, E = self.world, cfg.experts
        self.owner = torch.tensor([cfg.owner(e, W) for e in range(E)], dtype=torch.int64, device=device)
        self.local_experts = [e for e in range(E) if cfg.owner(e, W) == self.rank]
        self.router_stream = torch.cuda.Stream(device=device)
        self.chunk_events = [torch.cuda.Event() for _ in range(cfg.chunks)]
        T, k = cfg.tokens_per_rank, cfg.top_k
        self.ids = torch.zeros((T, k), dtype=torch.int64, device=device)
        self.gates = torch.zeros((T, k), dtype=torch.float32, device=device)
        self.out = torch.zeros((T, cfg.out_dim), dtype=torch.float32, device=device)
        mask = torch.zeros((T, E), dtype=torch.bool, device=device)
        if cfg.mask_mode == "topology_source":
            mask[torch.arange(T, device=device), torch.arange(T, device=device) % E] = True
        if self.inputs.block_mask is not None:
            mask |= self.inputs.block_mask.bool()[None, :]
        self.mask = mask
        self.positions = torch.arange(T, dtype=torch.int64, device=device)

    # ------------------------------------------------------------------ steps
    def _route(self, c: int) -> None:
        cfg = self.cfg
        lo, hi = cfg.chunk_offsets[c], cfg.chunk_offsets[c + 1]
        if hi > lo:
            x = self.inputs.tokens[lo:hi].float()
            logits = x @ self.weights.router_w.float().t() + self.weights.router_b
            if self.inputs.chunk_bias is not None:
                logits = logits + self.inputs.chunk_bias[c]
            logits = logits.masked_fill(self.mask[lo:hi], float("-inf"))
            vals, idx = torch.sort(logits, dim=-1, descending=True, stable=True)
            top = vals[:, :cfg.top_k]
            if cfg.gate_mode == "topk_softmax":
                g = torch.softmax(top, dim=-1)
            elif cfg.gate_mode == "softmax":
                g = torch.softmax(logits, dim=-1).gather(1, idx[:, :cfg.top_k])
            else:
                g = torch.ones_like(top)
            self.ids[lo:hi] = idx[:, :cfg.top_k]
            self.gates[lo:hi] = g
        self.chunk_events[c].record(self.router_stream)

    def _alltoallv(self, send: torch.Tensor, send_counts: list[int], recv_counts: list[int], width: int) -> torch.Tensor:
        if self.world == 1:
            return send.reshape(-1, width).clone()
        return device_alltoallv(send, send_counts, recv_counts, width, group=self.group)

    def _exchange(self, q: int, chunks: tuple[int, ...]) -> dict:
        """Count exchange + identity and feature AlltoAllv of one descriptor."""
        cfg = self.cfg
        lo, hi = cfg.chunk_offsets[chunks[0]], cfg.chunk_offsets[chunks[-1] + 1]
        k = cfg.top_k
        pos = self.positions[lo:hi].repeat_interleave(k)
        choice = torch.arange(k, device=self.device).repeat(hi - lo)
        expert = self.ids[lo:hi].reshape(-1)
        dest = self.owner[expert]
        order = torch.argsort(dest, stable=True)
        pos, choice, expert, dest = pos[order], choice[order], expert[order], dest[order]
        counts = torch.bincount(dest, minlength=self.world)
        chunk = torch.bucketize(pos, torch.tensor(cfg.chunk_offsets[1:], device=self.device), right=True)
        meta = torch.stack([self.inputs.token_ids[pos], torch.full_like(pos, self.rank), dest, expert, pos, chunk,
                            choice, torch.full_like(pos, q)], dim=1)
        if self.world > 1:
            recv = torch.empty_like(counts)
            dist.all_to_all_single(recv, counts, group=self.group)
            both = torch.stack([counts, recv]).cpu()
            send_c, recv_c = both[0].tolist(), both[1].tolist()
        else:
            send_c = recv_c = [int(pos.numel())]
        feats = self.inputs.tokens[pos]
        return {"pos": pos, "choice": choice, "send_counts": send_c, "recv_counts": recv_c,
                "meta": self._alltoallv(meta, send_c, recv_c, _META),
                "feat": self._alltoallv(feats, send_c, recv_c, cfg.hidden)}

    def _experts(self, feat: torch.Tensor, expert: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        w = self.weights
        y = torch.zeros((feat.shape[0], cfg.out_dim), dtype=torch.float32, device=self.device)
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = cfg.dtype == "fp32"  # tf32 tensor cores, as the product
        try:
            for e in self.local_experts:
                sel = (expert == e).nonzero(as_tuple=True)[0]
                if sel.numel() == 0:
                    continue
                x = feat.index_select(0, sel)
                if cfg.activation == "swiglu":
                    F_ = cfg.ffn_hidden
                    h = torch.nn.functional.silu(x @ w.w1[e, :F_].t()) * (x @ w.w1[e, F_:].t())
                else:
                    h = x @ w.w1[e].t()
                    if w.b1 is not None:
                        h = h + w.b1[e].to(h.dtype)
                    h = {"relu": torch.relu, "gelu": torch.nn.functional.gelu,
                         "silu": torch.nn.functional.silu}[cfg.activation](h)
                o = h @ w.w2[e].t()
                if w.b2 is not None:
                    o = o + w.b2[e].to(o.dtype)
                y.index_copy_(0, sel, o.float())
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        return y

    # ------------------------------------------------------------------- call
    def forward(self, arm: str = "early") -> torch.Tensor:
        """One layer call on the current stream (host-synchronising, like the
        reference's driver); returns the combined fp32 output [T, Dout]."""
        if arm not in ("early", "delayed"):
            raise ValueError("arm must be 'early' or 'delayed'")
        cfg = self.cfg
        cur = torch.cuda.current_stream(self.device)
        self.router_stream.wait_stream(cur)
        with torch.cuda.stream(self.router_stream):
            for c in range(cfg.chunks):
                self._route(c)
        groups = cfg.descriptor_groups
        sent = []
        if arm == "delayed":
            self.chunk_events[-1].synchronize()
        for q, chunks in enumerate(groups):
            self.chunk_events[chunks[-1]].synchronize()
            cur.wait_event(self.chunk_events[chunks[-1]])
            sent.append(self._exchange(q, chunks))
        # experts over every received row, then the outputs go back in the same order
        feat = torch.cat([s["feat"] for s in sent])
        meta = torch.cat([s["meta"] for s in sent])
        y = self._experts(feat, meta[:, 3])
        # rows from source r arrive per descriptor; send each source its rows back
        src = meta[:, 1]
        order = torch.argsort(src, stable=True)
        back_counts = [sum(s["recv_counts"][r] for s in sent) for r in range(self.world)]
        ret_y = self._alltoallv(y[order].contiguous(), back_counts,
                                [sum(s["send_counts"][d] for s in sent) for d in range(self.world)], cfg.out_dim)
        ret_meta = self._alltoallv(meta[order][:, [4, 6]].contiguous(), back_counts,
                                   [sum(s["send_counts"][d] for s in sent) for d in range(self.world)], 2)
        pos, choice = ret_meta[:, 0], ret_meta[:, 1]
        # every (position, choice) comes back once: place, then sum the k choices
        # in a fixed order, so both arms give bit-identical outputs
        per = torch.zeros((cfg.tokens_per_rank, cfg.top_k, cfg.out_dim), dtype=torch.float32, device=self.device)
        per[pos, choice] = ret_y * self.gates[pos, choice][:, None]
        torch.sum(per, dim=1, out=self.out)
        return self.out


__all__ += ["NcclMoELayer"]
