"""One-sided peer put with a completion signal, and bounded waits.

``PeerOps`` owns one symmetric region (``PeerChannel``): a receive slot of
``slot_bytes`` per source rank, then one 64-bit signal word per source rank.
``put(peer, tensor)`` copies the tensor into this rank's slot of ``peer``'s
region over NVLink (P2P stores; the own rank is a local copy) and releases
the next sequence number into this rank's signal word there;
``wait(src)`` blocks the stream (bounded) until ``src``'s word reaches the
sequence of its last expected put.  The kernels are in
csrc/kernels/peer_ops.cu; the capability is the MSCCL++ memory-channel
put / signal / wait of extensions/r6_mscclpp/mscclpp_runtime.cu:20-155.

Counters (``counters``): put calls, bytes put, signals sent, waits issued.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import status as _status
from ..ops._native import kernels
from .peer import PeerChannel


class PeerOps:
    def __init__(self, slot_bytes: int, device: torch.device, group=None, timeout_s: float = 5.0) -> None:
        if slot_bytes <= 0 or slot_bytes % 16:
            raise ValueError("slot_bytes must be a positive multiple of 16")
        self.device = torch.device(device)
        self.slot_bytes = int(slot_bytes)
        world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.flags_off = world * self.slot_bytes
        self.channel = PeerChannel(self.flags_off + 8 * world + 256, self.device, group=group)
        self.world, self.rank = self.channel.world, self.channel.rank
        self._k = kernels()
        self.timeout_ns = int(timeout_s * 1e9)
        self.status = _status.new_status(self.device)
        self.waited = torch.zeros(self.world, dtype=torch.int64, device=self.device)
        # one zeroed completion counter per destination (puts to different peers may overlap)
        self._done = torch.zeros(self.world, dtype=torch.int32, device=self.device)
        self.sent_seq = [0] * self.world       # puts issued to each peer
        self.expect_seq = [0] * self.world     # puts expected from each source
        self.counters = {"put_calls": 0, "bytes_transferred": 0, "signals": 0, "waits": 0}
        self.channel.view(self.flags_off, (self.world,), torch.int64).zero_()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=group)

    def slot(self, src: int, nbytes: int | None = None) -> torch.Tensor:
        """This rank's receive slot of source ``src`` as a uint8 tensor view."""
        n = self.slot_bytes if nbytes is None else int(nbytes)
        return self.channel.view(src * self.slot_bytes, (n,), torch.uint8)

    def put(self, peer: int, src: torch.Tensor, *, grid: int = 64) -> int:
        """Enqueue the put of ``src`` into our slot at ``peer`` plus its signal; returns its sequence number."""
        nbytes = src.numel() * src.element_size()
        if nbytes > self.slot_bytes:
            raise ValueError(f"{nbytes} bytes do not fit a {self.slot_bytes}-byte slot")
        self.sent_seq[peer] += 1
        seq = self.sent_seq[peer]
        base = self.channel.bases[peer]
        self._k.peer_put_signal(src.contiguous(), base + self.rank * self.slot_bytes,
                                base + self.flags_off + 8 * self.rank, seq, self._done[peer:peer + 1], grid)
        self.counters["put_calls"] += 1
        self.counters["bytes_transferred"] += int(nbytes)
        self.counters["signals"] += 1
        return seq

    def expect(self, src: int, count: int = 1) -> int:
        """Record that ``count`` more puts from ``src`` are due; returns the sequence to wait for."""
        self.expect_seq[src] += int(count)
        return self.expect_seq[src]

    def wait(self, src: int, seq: int | None = None) -> None:
        """Enqueue a bounded wait for ``src``'s signal to reach ``seq`` (default:
        everything expected so far); a timeout records a status (check_status)."""
        target = self.expect_seq[src] if seq is None else int(seq)
        self._k.peer_wait(self.channel.bases[self.rank] + self.flags_off + 8 * src, target, self.timeout_ns,
                          self.status, self.waited[src:src + 1])
        self.counters["waits"] += 1

    def check_status(self) -> None:
        torch.cuda.synchronize(self.device)
        _status.check(self.status)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        self.channel.close()


__all__ = ["PeerOps"]
