"""Guarded descriptors -> one-sided peer-store actions over a registered layout.

Behaviour of rlccl/transport/mscclpp_backend.py:22-203, generalised from the
frozen two-rank MSCCL++ buffer pair to N ranks of the NVLink peer channel:

* ``RegisteredBufferLayout``: ``[send region | recv region]``, each
  ``max_descriptors x world x peer_stride`` bytes; a slot is an 8-byte
  int64 token-count header followed by fixed-size records.
* ``PeerCommittedAdapter.commit_descriptor`` accepts only a descriptor whose
  scheduling step passed the DynamicGuard and whose chunks are completed and
  revealed; it rejects replays and emits one action per non-empty destination
  — a zero-token *remote* destination still receives the count header (a
  header-only control transfer), an empty local slot needs no action.
* ``HostPeerMemory`` executes actions on host buffers: the CPU stand-in of
  the device put/signal path used by the simulated-ranks harness and tests.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any, Iterable

import numpy as np

from .formats import PAYLOAD_FIELDS, PackedShard

RECORD_BYTES = PAYLOAD_FIELDS * 8
COUNT_HEADER_BYTES = 8


@dataclass(frozen=True, slots=True)
class CommittedAction:
    action_id: int
    descriptor_id: int
    src_rank: int
    dst_rank: int
    src_offset: int
    dst_offset: int
    token_count: int
    bytes: int
    physical_bytes: int
    reveal_ids: tuple[int, ...]

    @property
    def is_remote(self) -> bool:
        return self.src_rank != self.dst_rank


@dataclass(frozen=True, slots=True)
class RegisteredBufferLayout:
    world_size: int
    max_descriptors: int
    max_tokens_per_peer_descriptor: int
    record_bytes: int = RECORD_BYTES
    alignment: int = 8

    def __post_init__(self) -> None:
        if not 1 <= self.world_size <= 8:
            raise ValueError("the peer channel supports 1..8 ranks")
        if self.max_descriptors <= 0 or self.max_tokens_per_peer_descriptor <= 0:
            raise ValueError("buffer capacities must be positive")
        if self.record_bytes <= 0 or self.record_bytes % 8:
            raise ValueError("record_bytes must be a positive multiple of 8")
        if self.alignment < 8 or self.alignment & (self.alignment - 1):
            raise ValueError("alignment must be a power of two and at least 8")

    @property
    def peer_stride(self) -> int:
        raw = COUNT_HEADER_BYTES + self.max_tokens_per_peer_descriptor * self.record_bytes
        return (raw + self.alignment - 1) & ~(self.alignment - 1)

    @property
    def descriptor_stride(self) -> int:
        return self.world_size * self.peer_stride

    @property
    def region_bytes(self) -> int:
        return self.max_descriptors * self.descriptor_stride

    @property
    def capacity_bytes(self) -> int:
        return 2 * self.region_bytes

    def _slot(self, descriptor_id: int, peer: int) -> int:
        if not 0 <= descriptor_id < self.max_descriptors:
            raise ValueError("descriptor exceeds registered buffer capacity")
        if not 0 <= peer < self.world_size:
            raise ValueError("peer rank outside process group")
        return descriptor_id * self.descriptor_stride + peer * self.peer_stride

    def send_offset(self, descriptor_id: int, destination_rank: int) -> int:
        return self._slot(descriptor_id, destination_rank)

    def receive_offset(self, descriptor_id: int, source_rank: int) -> int:
        return self.region_bytes + self._slot(descriptor_id, source_rank)


class PeerCommittedAdapter:
    """Maps guarded delta shards to peer-store actions without rescheduling them."""

    def __init__(self, *, rank: int, layout: RegisteredBufferLayout) -> None:
        if not 0 <= rank < layout.world_size:
            raise ValueError("rank outside process group")
        self.rank = int(rank)
        self.layout = layout
        self._seen: set[int] = set()
        self._next = 0
        self.actions_committed = 0
        self.payload_bytes_committed = 0
        self.physical_bytes_planned = 0
        self.future_access = 0
        self.unrevealed_access = 0
        self.stale_action = 0

    def commit_descriptor(self, packed: PackedShard, *, descriptor_id: int, guard_decision: Any,
                          completed_chunks: Iterable[int], revealed_chunks: Iterable[int]) -> tuple[CommittedAction, ...]:
        d = int(descriptor_id)
        if d in self._seen:
            self.stale_action += 1
            raise ValueError("stale descriptor replay")
        if not bool(getattr(guard_decision, "accepted", False)):
            raise ValueError("peer adapter requires a DynamicGuard PASS")
        if int(getattr(guard_decision, "applied_actions", -1)) < 0:
            raise ValueError("invalid guard decision")
        if packed.source_rank != self.rank:
            raise ValueError("packed shard source rank mismatch")
        chunks = tuple(int(c) for c in packed.chunk_ids)
        if not chunks or len(chunks) != len(set(chunks)):
            raise ValueError("descriptor must name unique revealed chunks")
        completed = set(int(c) for c in completed_chunks)
        revealed = set(int(c) for c in revealed_chunks)
        if any(c not in completed for c in chunks):
            self.future_access += 1
            raise ValueError("future router chunk cannot enter the peer channel")
        if any(c not in revealed for c in chunks):
            self.unrevealed_access += 1
            raise ValueError("unrevealed chunk cannot enter the peer channel")
        W = self.layout.world_size
        if len(packed.sendcounts_tokens) != W or len(packed.offsets_tokens) != W:
            raise ValueError("sendcount/offset cardinality mismatch")
        actions = []
        for dst, (count, poff) in enumerate(zip(packed.sendcounts_tokens, packed.offsets_tokens)):
            count, poff = int(count), int(poff)
            if count < 0 or poff < 0:
                raise ValueError("negative count/offset")
            if count == 0 and dst == self.rank:
                continue
            if count > self.layout.max_tokens_per_peer_descriptor:
                raise ValueError("peer payload exceeds registered slot capacity")
            if poff + count > packed.total_tokens:
                raise ValueError("packed range exceeds descriptor payload")
            payload = count * self.layout.record_bytes
            physical = COUNT_HEADER_BYTES + payload
            base = self.layout.send_offset(d, dst)
            if base + physical > self.layout.capacity_bytes:
                raise ValueError("action exceeds registered buffer")
            actions.append(CommittedAction(self._next, d, self.rank, dst, base,
                                           self.layout.receive_offset(d, self.rank), count, payload,
                                           physical, chunks))
            self._next += 1
        self._seen.add(d)
        self.actions_committed += len(actions)
        self.payload_bytes_committed += sum(a.bytes for a in actions)
        self.physical_bytes_planned += sum(a.physical_bytes for a in actions)
        return tuple(actions)

    def counters(self) -> dict[str, int]:
        return {"committed_actions": self.actions_committed,
                "committed_payload_bytes": self.payload_bytes_committed,
                "planned_physical_bytes": self.physical_bytes_planned,
                "future_access": self.future_access, "unrevealed_access": self.unrevealed_access,
                "stale_action": self.stale_action}


# API-parity alias of the reference's adapter name
MscclppCommittedAdapter = PeerCommittedAdapter


def action_payload(action: CommittedAction) -> dict:
    out = asdict(action)
    out["reveal_ids"] = list(action.reveal_ids)
    return out


class HostPeerMemory:
    """Registered buffers of W simulated ranks in host memory, with the
    put / signal / wait counters of the device channel."""

    def __init__(self, layout: RegisteredBufferLayout) -> None:
        self.layout = layout
        self.buffers = [np.zeros(layout.capacity_bytes, dtype=np.uint8) for _ in range(layout.world_size)]
        self.signals = np.zeros((layout.world_size, layout.world_size, layout.max_descriptors), dtype=np.int64)
        self.counters = {"put_calls": 0, "bytes_transferred": 0, "signals": 0, "waits": 0}

    def stage(self, rank: int, action: CommittedAction, packed: PackedShard, first_token: int) -> None:
        buf = self.buffers[rank]
        recs = np.ascontiguousarray(packed.records[first_token:first_token + action.token_count], dtype=np.int64)
        buf[action.src_offset:action.src_offset + 8] = np.frombuffer(np.int64(action.token_count).tobytes(), np.uint8)
        raw = recs.view(np.uint8).reshape(-1)
        buf[action.src_offset + 8:action.src_offset + 8 + raw.size] = raw

    def stage_bytes(self, rank: int, action: CommittedAction, rows: np.ndarray) -> None:
        """Stage raw fixed-size rows (uint8 [count, record_bytes]) behind the count header."""
        buf = self.buffers[rank]
        raw = np.ascontiguousarray(rows, dtype=np.uint8).reshape(-1)
        if raw.size != action.token_count * self.layout.record_bytes:
            raise ValueError("staged rows do not match the action")
        buf[action.src_offset:action.src_offset + 8] = np.frombuffer(np.int64(action.token_count).tobytes(), np.uint8)
        buf[action.src_offset + 8:action.src_offset + 8 + raw.size] = raw

    def receive_bytes(self, rank: int, source: int, descriptor_id: int) -> np.ndarray:
        off = self.layout.receive_offset(descriptor_id, source)
        buf = self.buffers[rank]
        count = int(np.frombuffer(buf[off:off + 8].tobytes(), dtype=np.int64)[0])
        return buf[off + 8:off + 8 + count * self.layout.record_bytes].reshape(count, self.layout.record_bytes).copy()

    def put_and_signal(self, action: CommittedAction, seq: int = 1) -> None:
        src = self.buffers[action.src_rank][action.src_offset:action.src_offset + action.physical_bytes]
        self.buffers[action.dst_rank][action.dst_offset:action.dst_offset + action.physical_bytes] = src
        self.signals[action.dst_rank, action.src_rank, action.descriptor_id] = seq
        self.counters["put_calls"] += 1
        self.counters["bytes_transferred"] += action.physical_bytes
        self.counters["signals"] += 1

    def wait(self, rank: int, source: int, descriptor_id: int, seq: int = 1) -> bool:
        self.counters["waits"] += 1
        return bool(self.signals[rank, source, descriptor_id] >= seq)

    def receive(self, rank: int, source: int, descriptor_id: int) -> np.ndarray:
        off = self.layout.receive_offset(descriptor_id, source)
        buf = self.buffers[rank]
        count = int(np.frombuffer(buf[off:off + 8].tobytes(), dtype=np.int64)[0])
        raw = buf[off + 8:off + 8 + count * self.layout.record_bytes]
        return np.frombuffer(raw.tobytes(), dtype=np.int64).reshape(count, -1)


__all__ = ["COUNT_HEADER_BYTES", "CommittedAction", "HostPeerMemory", "MscclppCommittedAdapter",
           "PeerCommittedAdapter", "RECORD_BYTES", "RegisteredBufferLayout", "action_payload"]
