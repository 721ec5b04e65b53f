"""Payload identity formats, revealed-only packing state and verifiers.

The host-side (NumPy) form of the data-plane records, used by the CPU
simulated-ranks harness, by the NCCL baseline arm and by the checker:

* A2Av records (rlccl/transport/reference_a2av.py:19-337): 7 identity fields
  ``(token, source, destination, expert, chunk, chunk_offset, payload_word)``
  + checksum ``sum (v mod M) c_i mod M`` (M = 2^63 - 25); fail-closed
  destination layouts; ``ProgressivePackingState`` (completed / revealed /
  dispatched bitmaps with future / unrevealed / stale / duplicate counters);
  receive verifier with a sha256 multiset digest.
* Full-MoE payloads (rlccl/transport/reference_full_moe.py:19-246): forward
  rows ``(token, src, dst, expert, chunk, chunk_offset, position, digest,
  checksum)`` + features; return rows ``(token, src, expert_rank, expert,
  position, chunk, chunk_offset, checksum)`` + outputs; both verifiers.

Row digest: the reference hashes a feature row with blake2b-64 (kept here as
``feature_digest_blake2b`` for host-only paths).  The device data plane uses
``row_digest``: the wrapping 64-bit sum over the row's 32-bit words w_i of
splitmix64((i << 32) | w_i), masked to 62 bits — order dependent, computable
in parallel on the GPU, and recomputed here in NumPy.
"""

from __future__ import annotations

from dataclasses import dataclass
import hashlib
import time
from typing import Iterable, Mapping, Sequence

import numpy as np

PAYLOAD_FIELDS = 8
FORWARD_META_FIELDS = 9
RETURN_META_FIELDS = 8
CHECKSUM_MODULUS = (1 << 63) - 25
CHECKSUM_COEFFICIENTS = (1_000_003, 1_000_033, 1_000_037, 1_000_081, 1_000_099, 1_000_117,
                         1_000_121, 1_000_133)
_DIGEST_MASK = (1 << 62) - 1


def identity_checksum(prefix: Sequence[int]) -> int:
    if len(prefix) > len(CHECKSUM_COEFFICIENTS):
        raise ValueError("identity checksum prefix too long")
    acc = 0
    for v, c in zip(prefix, CHECKSUM_COEFFICIENTS):
        acc = (acc + (int(v) % CHECKSUM_MODULUS) * c) % CHECKSUM_MODULUS
    return int(acc)


def payload_checksum(prefix: Sequence[int]) -> int:
    """Checksum of the seven A2Av identity fields."""
    if len(prefix) != PAYLOAD_FIELDS - 1:
        raise ValueError("payload checksum requires seven fields")
    return identity_checksum(prefix)


def identity_checksum_vec(rows: np.ndarray) -> np.ndarray:
    """Row-wise identity checksum of an int64 [n, m] array (m <= 8)."""
    a = np.asarray(rows, dtype=np.int64)
    if a.ndim != 2:
        raise ValueError("rows must be 2-D")
    obj = a.astype(object)
    acc = np.zeros(a.shape[0], dtype=object)
    for j in range(a.shape[1]):
        acc = (acc + (obj[:, j] % CHECKSUM_MODULUS) * CHECKSUM_COEFFICIENTS[j]) % CHECKSUM_MODULUS
    return acc.astype(np.int64)


def feature_digest_blake2b(row: np.ndarray) -> int:
    values = np.ascontiguousarray(np.asarray(row, dtype=np.float32))
    return int.from_bytes(hashlib.blake2b(values.tobytes(), digest_size=8).digest(), "little") & _DIGEST_MASK


def _splitmix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def row_digest(rows: np.ndarray) -> np.ndarray:
    """Device row digest of each row of a 2-D array (any dtype, row bytes % 4 == 0)."""
    a = np.ascontiguousarray(rows)
    if a.ndim == 1:
        a = a[None, :]
    words = a.view(np.uint32).reshape(a.shape[0], -1).astype(np.uint64)
    idx = (np.arange(words.shape[1], dtype=np.uint64) << np.uint64(32))[None, :]
    with np.errstate(over="ignore"):
        mixed = _splitmix64(idx | words)
        total = mixed.sum(axis=1, dtype=np.uint64)
    return (total & np.uint64(_DIGEST_MASK)).astype(np.int64)


def feature_digest(row: np.ndarray) -> int:
    return int(row_digest(np.asarray(row))[0])


# ---------------------------------------------------------------------------
# A2Av records and revealed-only packing
# ---------------------------------------------------------------------------
@dataclass(frozen=True, slots=True)
class RouterAssignment:
    token_id: int
    source_rank: int
    destination_rank: int
    expert_id: int
    chunk_id: int
    chunk_offset: int
    payload_word: int

    def record(self) -> tuple[int, ...]:
        prefix = (int(self.token_id), int(self.source_rank), int(self.destination_rank), int(self.expert_id),
                  int(self.chunk_id), int(self.chunk_offset), int(self.payload_word))
        return prefix + (payload_checksum(prefix),)


@dataclass(frozen=True, slots=True)
class DestinationLayout:
    source_rank: int
    chunk_ids: tuple[int, ...]
    destination_lists: tuple[tuple[RouterAssignment, ...], ...]
    sendcounts_tokens: tuple[int, ...]
    offsets_tokens: tuple[int, ...]

    @property
    def total_tokens(self) -> int:
        return sum(self.sendcounts_tokens)


@dataclass(frozen=True, slots=True)
class PackedShard:
    source_rank: int
    chunk_ids: tuple[int, ...]
    sendcounts_tokens: tuple[int, ...]
    offsets_tokens: tuple[int, ...]
    records: np.ndarray

    @property
    def sendcounts_elements(self) -> tuple[int, ...]:
        return tuple(v * PAYLOAD_FIELDS for v in self.sendcounts_tokens)

    @property
    def total_tokens(self) -> int:
        return int(self.records.shape[0])

    @property
    def total_bytes(self) -> int:
        return int(self.records.nbytes)


def _exclusive_prefix(counts: Sequence[int]) -> tuple[int, ...]:
    out, cur = [], 0
    for c in counts:
        out.append(cur)
        cur += int(c)
    return tuple(out)


def build_destination_layout(assignments: Iterable[RouterAssignment], *, world_size: int, source_rank: int,
                             chunk_ids: Sequence[int], timing_sink: dict | None = None,
                             destination_of=None) -> DestinationLayout:
    """Per-destination lists, counts and offsets derived only from router
    assignments of the named chunks; fails closed on a wrong source, an
    unrevealed chunk, an out-of-range or non-expert-derived destination and
    duplicate tokens.  ``destination_of(expert)`` defaults to ``expert % W``."""
    t0 = time.perf_counter_ns()
    if world_size <= 0 or not 0 <= source_rank < world_size:
        raise ValueError("invalid world/source rank")
    chunks = tuple(int(c) for c in chunk_ids)
    if len(set(chunks)) != len(chunks):
        raise ValueError("duplicate chunk in descriptor")
    allowed = set(chunks)
    owner = destination_of or (lambda e: e % world_size)
    lists: list[list[RouterAssignment]] = [[] for _ in range(world_size)]
    # one row per token in the reference (top-1) form; one per (token, expert)
    # when a placement function is given (top-k routing)
    seen: set = set()
    for a in assignments:
        if int(a.source_rank) != source_rank:
            raise ValueError("assignment source does not match descriptor source")
        if int(a.chunk_id) not in allowed:
            raise ValueError("assignment belongs to an unrevealed descriptor chunk")
        if not 0 <= int(a.destination_rank) < world_size:
            raise ValueError("assignment destination outside process group")
        if int(a.destination_rank) != owner(int(a.expert_id)):
            raise ValueError("destination rank is not router-expert-derived")
        key = int(a.token_id) if destination_of is None else (int(a.token_id), int(a.expert_id))
        if key in seen:
            raise ValueError("duplicate token in descriptor")
        seen.add(key)
        lists[int(a.destination_rank)].append(a)
    for row in lists:
        row.sort(key=lambda a: (int(a.token_id), int(a.chunk_id), int(a.chunk_offset)))
    counts = tuple(len(v) for v in lists)
    t1 = time.perf_counter_ns()
    offsets = _exclusive_prefix(counts)
    t2 = time.perf_counter_ns()
    if timing_sink is not None:
        timing_sink["count_construction_us"] = (t1 - t0) / 1e3
        timing_sink["offset_construction_us"] = (t2 - t1) / 1e3
    return DestinationLayout(source_rank, chunks, tuple(tuple(v) for v in lists), counts, offsets)


def pack_destination_layout(layout: DestinationLayout) -> PackedShard:
    rows = [a.record() for v in layout.destination_lists for a in v]
    rec = (np.asarray(rows, dtype=np.int64).reshape(-1, PAYLOAD_FIELDS) if rows
           else np.empty((0, PAYLOAD_FIELDS), dtype=np.int64))
    rec = np.ascontiguousarray(rec)
    rec.setflags(write=False)
    return PackedShard(layout.source_rank, layout.chunk_ids, layout.sendcounts_tokens,
                       layout.offsets_tokens, rec)


class ProgressivePackingState:
    """Fail-closed completed / revealed / dispatched state for delta descriptors."""

    def __init__(self, *, world_size: int, source_rank: int, max_chunks: int = 8) -> None:
        if max_chunks <= 0:
            raise ValueError("max_chunks must be positive")
        self.world_size, self.source_rank, self.max_chunks = int(world_size), int(source_rank), int(max_chunks)
        self.completed_bitmap = self.revealed_bitmap = self.dispatched_bitmap = 0
        self._assignments: list[tuple[RouterAssignment, ...] | None] = [None] * self.max_chunks
        self._dispatched: set[tuple[int, int]] = set()
        self.descriptor_count = 0
        self.future_access_attempts = self.unrevealed_execution = 0
        self.duplicate_dispatch = self.stale_dispatch = 0

    def mark_completed(self, chunk: int, assignments: Sequence[RouterAssignment]) -> None:
        i = int(chunk)
        if not 0 <= i < self.max_chunks:
            raise ValueError("chunk outside state")
        if self.completed_bitmap & (1 << i):
            raise ValueError("completed chunk replay")
        vals = tuple(assignments)
        if any(int(a.chunk_id) != i for a in vals):
            raise ValueError("assignment chunk mismatch")
        self._assignments[i] = vals
        self.completed_bitmap |= 1 << i

    def reveal(self, chunk: int) -> None:
        bit = 1 << int(chunk)
        if not self.completed_bitmap & bit:
            self.future_access_attempts += 1
            raise ValueError("cannot reveal incomplete router chunk")
        if self.revealed_bitmap & bit:
            raise ValueError("revealed chunk replay")
        self.revealed_bitmap |= bit

    def build_delta_layout(self, chunk_ids: Sequence[int], *, timing_sink: dict | None = None,
                           destination_of=None) -> DestinationLayout:
        chunks = tuple(int(c) for c in chunk_ids)
        if not chunks:
            raise ValueError("descriptor must name at least one chunk")
        mask = 0
        assigns: list[RouterAssignment] = []
        for i in chunks:
            if not 0 <= i < self.max_chunks:
                raise ValueError("descriptor chunk outside state")
            bit = 1 << i
            mask |= bit
            if not self.completed_bitmap & bit:
                self.future_access_attempts += 1
                raise ValueError("future router chunk access")
            if not self.revealed_bitmap & bit:
                self.unrevealed_execution += 1
                raise ValueError("unrevealed router chunk execution")
            if self.dispatched_bitmap & bit:
                self.stale_dispatch += 1
                raise ValueError("stale chunk dispatch")
            vals = self._assignments[i]
            if vals is None:
                raise RuntimeError("completed chunk has no assignments")
            assigns.extend(vals)
        keys = [(int(a.token_id), int(a.expert_id)) for a in assigns]
        if len(keys) != len(set(keys)) or any(k in self._dispatched for k in keys):
            self.duplicate_dispatch += 1
            raise ValueError("duplicate token dispatch")
        layout = build_destination_layout(assigns, world_size=self.world_size, source_rank=self.source_rank,
                                          chunk_ids=chunks, timing_sink=timing_sink,
                                          destination_of=destination_of)
        self.dispatched_bitmap |= mask
        self._dispatched.update(keys)
        self.descriptor_count += 1
        return layout

    def build_delta(self, chunk_ids: Sequence[int]) -> tuple[DestinationLayout, PackedShard]:
        layout = self.build_delta_layout(chunk_ids)
        return layout, pack_destination_layout(layout)

    @property
    def dispatched_token_count(self) -> int:
        return len(self._dispatched)


def decode_records(records: np.ndarray) -> tuple[tuple[int, ...], ...]:
    v = np.asarray(records, dtype=np.int64)
    if v.ndim != 2 or v.shape[1] != PAYLOAD_FIELDS:
        raise ValueError("invalid payload record shape")
    return tuple(tuple(int(x) for x in row) for row in v.tolist())


def payload_multiset_digest(records: Iterable[Sequence[int]]) -> str:
    h = hashlib.sha256()
    for row in sorted(tuple(int(x) for x in r) for r in records):
        h.update(np.asarray(row, dtype="<i8").tobytes())
    return h.hexdigest()


def verify_received_records(records: np.ndarray, *, destination_rank: int,
                            expected_by_token: Mapping[int, Sequence[int]]) -> dict:
    decoded = decode_records(records)
    seen: set[int] = set()
    dup = wrong = corrupt = unexpected = 0
    for row in decoded:
        tok = int(row[0])
        dup += int(tok in seen)
        seen.add(tok)
        wrong += int(int(row[2]) != int(destination_rank))
        corrupt += int(payload_checksum(row[:7]) != int(row[7]))
        exp = expected_by_token.get(tok)
        if exp is None:
            unexpected += 1
        elif tuple(int(x) for x in exp) != row:
            corrupt += 1
    expected = set(int(t) for t in expected_by_token)
    lost = len(expected - seen)
    unexpected += len(seen - expected)
    return {"pass": not any((lost, dup, wrong, corrupt, unexpected)), "received": len(decoded),
            "expected": len(expected), "lost": lost, "duplicate": dup, "wrong_destination": wrong,
            "corruption": corrupt, "unexpected": unexpected,
            "payload_multiset_digest": payload_multiset_digest(decoded)}


# ---------------------------------------------------------------------------
# Full-MoE forward / return payloads
# ---------------------------------------------------------------------------
@dataclass(frozen=True, slots=True)
class ForwardPayload:
    sendcounts_tokens: tuple[int, ...]
    offsets_tokens: tuple[int, ...]
    metadata: np.ndarray
    features: np.ndarray

    @property
    def total_tokens(self) -> int:
        return int(self.metadata.shape[0])


@dataclass(frozen=True, slots=True)
class ReturnPayload:
    sendcounts_tokens: tuple[int, ...]
    offsets_tokens: tuple[int, ...]
    metadata: np.ndarray
    outputs: np.ndarray

    @property
    def total_tokens(self) -> int:
        return int(self.metadata.shape[0])


def pack_forward_payload(layout: DestinationLayout, *, features_by_token: Mapping[int, np.ndarray],
                         original_position_by_token: Mapping[int, int], digest=feature_digest) -> ForwardPayload:
    rows, feats = [], []
    for lst in layout.destination_lists:
        for a in lst:
            tok = int(a.token_id)
            f = np.asarray(features_by_token[tok], dtype=np.float32)
            prefix = (tok, int(a.source_rank), int(a.destination_rank), int(a.expert_id), int(a.chunk_id),
                      int(a.chunk_offset), int(original_position_by_token[tok]), digest(f))
            rows.append(prefix + (identity_checksum(prefix),))
            feats.append(f)
    meta = np.asarray(rows, dtype=np.int64).reshape(-1, FORWARD_META_FIELDS)
    if feats:
        width = feats[0].shape[0]
        fa = np.asarray(feats, dtype=np.float32).reshape(-1, width)
    else:
        fa = np.empty((0, 0), dtype=np.float32)
    return ForwardPayload(layout.sendcounts_tokens, layout.offsets_tokens, np.ascontiguousarray(meta),
                          np.ascontiguousarray(fa))


def verify_forward_payload(metadata: np.ndarray, features: np.ndarray, *, destination_rank: int, world_size: int,
                           recvcounts_tokens: Sequence[int] | None = None, digest=feature_digest,
                           destination_of=None) -> dict:
    meta = np.asarray(metadata, dtype=np.int64)
    vals = np.asarray(features)
    if meta.ndim != 2 or meta.shape[1] != FORWARD_META_FIELDS:
        raise ValueError("invalid forward metadata shape")
    if vals.ndim != 2 or vals.shape[0] != meta.shape[0]:
        raise ValueError("invalid forward feature shape")
    owner = destination_of or (lambda e: e % world_size)
    sender = None
    if recvcounts_tokens is not None:
        if sum(int(v) for v in recvcounts_tokens) != meta.shape[0]:
            raise ValueError("forward recvcounts mismatch")
        sender = np.repeat(np.arange(len(recvcounts_tokens)), [int(v) for v in recvcounts_tokens])
    seen: set[tuple[int, int]] = set()
    dup = wsrc = wdst = wexp = corrupt = 0
    for i, row in enumerate(meta):
        key = (int(row[0]), int(row[3]))
        dup += int(key in seen)
        seen.add(key)
        if sender is not None:
            wsrc += int(int(row[1]) != int(sender[i]))
        wdst += int(int(row[2]) != destination_rank)
        wexp += int(owner(int(row[3])) != destination_rank)
        corrupt += int(identity_checksum(row[:8]) != int(row[8]))
        corrupt += int(digest(vals[i]) != int(row[7]))
    return {"pass": not any((dup, wsrc, wdst, wexp, corrupt)), "tokens": int(meta.shape[0]), "duplicate": dup,
            "wrong_source": wsrc, "wrong_destination": wdst, "wrong_expert": wexp, "corruption": corrupt}


def pack_return_payload(forward_metadata: np.ndarray, expert_outputs: np.ndarray, *, expert_rank: int,
                        world_size: int) -> ReturnPayload:
    meta = np.asarray(forward_metadata, dtype=np.int64)
    outs = np.asarray(expert_outputs, dtype=np.float32)
    if meta.shape[0] != outs.shape[0]:
        raise ValueError("expert output cardinality mismatch")
    groups: list[list[tuple[np.ndarray, np.ndarray]]] = [[] for _ in range(world_size)]
    for row, o in zip(meta, outs):
        src = int(row[1])
        if not 0 <= src < world_size:
            raise ValueError("invalid original source")
        prefix = (int(row[0]), src, expert_rank, int(row[3]), int(row[6]), int(row[4]), int(row[5]))
        groups[src].append((np.asarray(prefix + (identity_checksum(prefix),), dtype=np.int64), o))
    for g in groups:
        g.sort(key=lambda it: (int(it[0][0]), int(it[0][4])))
    counts = tuple(len(g) for g in groups)
    flat = [it for g in groups for it in g]
    width = outs.shape[1] if outs.ndim == 2 else 0
    return ReturnPayload(counts, _exclusive_prefix(counts),
                         np.ascontiguousarray(np.asarray([it[0] for it in flat], dtype=np.int64).reshape(-1, RETURN_META_FIELDS)),
                         np.ascontiguousarray(np.asarray([it[1] for it in flat], dtype=np.float32).reshape(-1, width)))


def verify_return_and_combine(metadata: np.ndarray, outputs: np.ndarray, *, origin_rank: int,
                              recvcounts_tokens: Sequence[int], expected_expert_by_token: Mapping[int, int],
                              expected_position_by_token: Mapping[int, int],
                              expected_output_by_token: Mapping[int, np.ndarray], total_tokens: int,
                              required_positions: Sequence[int] | None = None, atol: float = 2e-3,
                              rtol: float = 2e-3) -> tuple[np.ndarray, dict]:
    meta = np.asarray(metadata, dtype=np.int64)
    vals = np.asarray(outputs, dtype=np.float32)
    if meta.ndim != 2 or meta.shape[1] != RETURN_META_FIELDS or vals.shape[0] != meta.shape[0]:
        raise ValueError("invalid return payload")
    if sum(int(v) for v in recvcounts_tokens) != meta.shape[0]:
        raise ValueError("return recvcounts mismatch")
    sender = np.repeat(np.arange(len(recvcounts_tokens)), [int(v) for v in recvcounts_tokens])
    width = vals.shape[1] if vals.ndim == 2 else 0
    combined = np.zeros((total_tokens, width), dtype=np.float32)
    filled = np.zeros(total_tokens, dtype=bool)
    seen: set[int] = set()
    dup = wdst = wret = wpos = corrupt = wexp = mism = 0
    for i, row in enumerate(meta):
        tok, pos, exp = int(row[0]), int(row[4]), int(row[3])
        dup += int(tok in seen)
        seen.add(tok)
        wdst += int(int(row[1]) != origin_rank)
        wret += int(int(row[2]) != int(sender[i]))
        wexp += int(expected_expert_by_token.get(tok, -1) != exp)
        wpos += int(pos != expected_position_by_token.get(tok, -1) or not 0 <= pos < total_tokens)
        corrupt += int(identity_checksum(row[:7]) != int(row[7]))
        ref = expected_output_by_token.get(tok)
        if ref is None or not np.allclose(vals[i], ref, atol=atol, rtol=rtol):
            mism += 1
        if 0 <= pos < total_tokens:
            if filled[pos]:
                dup += 1
            combined[pos] = vals[i]
            filled[pos] = True
    expected = set(int(t) for t in expected_expert_by_token)
    required = tuple(int(p) for p in required_positions) if required_positions is not None else tuple(range(total_tokens))
    lost = max(len(expected - seen), sum(not bool(filled[p]) for p in required))
    ok = not any((lost, dup, wdst, wret, wpos, corrupt, wexp, mism))
    return combined, {"pass": ok, "tokens": int(meta.shape[0]), "lost": lost, "duplicate": dup,
                      "wrong_destination": wdst, "wrong_return": wret, "wrong_position": wpos,
                      "wrong_expert": wexp, "corruption": corrupt, "expert_output_mismatch": mism}


__all__ = [
    "CHECKSUM_COEFFICIENTS", "CHECKSUM_MODULUS", "DestinationLayout", "FORWARD_META_FIELDS", "ForwardPayload",
    "PAYLOAD_FIELDS", "PackedShard", "ProgressivePackingState", "RETURN_META_FIELDS", "ReturnPayload",
    "RouterAssignment", "build_destination_layout", "decode_records", "feature_digest",
    "feature_digest_blake2b", "identity_checksum", "identity_checksum_vec", "pack_destination_layout",
    "pack_forward_payload", "pack_return_payload", "payload_checksum", "payload_multiset_digest",
    "row_digest", "verify_forward_payload", "verify_received_records", "verify_return_and_combine",
]
