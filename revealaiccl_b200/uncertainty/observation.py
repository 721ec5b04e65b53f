"""Planner-facing, read-only views of the reveal-aware world.

Mirrors the public boundary of rlccl/uncertainty/observation.py:25-250:

* ``TruthTokenId`` — opaque identity issued only when a real token is revealed;
* ``RevealedDemandToken(token_id, source, destination, holders)``;
* ``PublicTopologyView`` — deep-copied, read-only static topology;
* ``PartialObservationState`` — the only current-demand object an ordinary
  planner may receive (entry/unknown masks, observed matrix, revealed tokens,
  optional totals, state version);
* ``SanitizedHistoryView`` — completed matrices of strictly earlier steps.

All arrays are owned copies with the write flag cleared.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Mapping, Sequence

import numpy as np

from ..traffic.matrix_utils import validate_traffic_matrix


def readonly_array(value: Any, *, dtype: Any | None = None) -> np.ndarray:
    out = np.array(value, dtype=dtype, copy=True)
    out.setflags(write=False)
    return out


def _freeze(values: Mapping[str, Any]) -> Mapping[str, Any]:
    return MappingProxyType(dict(values))


@dataclass(frozen=True, slots=True)
class TruthTokenId:
    opaque_value: str

    def __post_init__(self) -> None:
        if not isinstance(self.opaque_value, str) or not self.opaque_value:
            raise ValueError("TruthTokenId requires a non-empty opaque string")

    def __str__(self) -> str:
        return self.opaque_value


@dataclass(frozen=True, slots=True)
class RevealedDemandToken:
    token_id: TruthTokenId
    source: int
    destination: int
    holders: tuple[int, ...]

    def __post_init__(self) -> None:
        if not isinstance(self.token_id, TruthTokenId):
            raise TypeError("RevealedDemandToken requires a TruthTokenId")
        if self.source < 0 or self.destination < 0 or self.source == self.destination:
            raise ValueError("Invalid revealed demand endpoints")
        holders = tuple(int(h) for h in self.holders)
        if any(h < 0 for h in holders):
            raise ValueError("Holder indices must be nonnegative")
        object.__setattr__(self, "holders", holders)


@dataclass(frozen=True, slots=True)
class PublicTopologyView:
    num_nodes: int
    num_edges: int
    edges: np.ndarray
    capacities: np.ndarray
    shared_constraints: tuple[tuple[tuple[int, ...], float], ...]
    name: str | None = None

    def __post_init__(self) -> None:
        edges = readonly_array(self.edges, dtype=np.int64)
        caps = readonly_array(self.capacities, dtype=np.float64)
        if edges.shape != (self.num_edges, 2):
            raise ValueError("Public topology edge shape mismatch")
        if caps.shape != (self.num_edges,):
            raise ValueError("Public topology capacity shape mismatch")
        groups = tuple((tuple(int(e) for e in idx), float(limit))
                       for idx, limit in self.shared_constraints)
        object.__setattr__(self, "edges", edges)
        object.__setattr__(self, "capacities", caps)
        object.__setattr__(self, "shared_constraints", groups)

    @classmethod
    def from_topology_info(cls, topology: Any) -> "PublicTopologyView":
        return cls(int(topology.V), int(topology.E), np.asarray(topology.edges),
                   np.asarray(topology.capacities), tuple(topology.shared_constraints),
                   getattr(topology, "name", None))

    @property
    def edge_src(self) -> np.ndarray:
        return readonly_array(self.edges[:, 0], dtype=np.int64)

    @property
    def edge_dst(self) -> np.ndarray:
        return readonly_array(self.edges[:, 1], dtype=np.int64)


@dataclass(frozen=True, slots=True)
class PartialObservationState:
    sequence_id: str
    sequence_step: int
    family: str
    mode: str
    stage: int
    ratio: float
    entry_mask: np.ndarray
    observed_matrix: np.ndarray
    unknown_mask: np.ndarray
    revealed_tokens: tuple[RevealedDemandToken, ...]
    source_totals: np.ndarray | None
    destination_totals: np.ndarray | None
    topology: PublicTopologyView
    state_version: int

    def __post_init__(self) -> None:
        entry = readonly_array(self.entry_mask, dtype=bool)
        observed = readonly_array(self.observed_matrix, dtype=np.int64)
        unknown = readonly_array(self.unknown_mask, dtype=bool)
        if observed.ndim != 2 or observed.shape[0] != observed.shape[1]:
            raise ValueError("Observed matrix must be square")
        if entry.shape != observed.shape or unknown.shape != observed.shape:
            raise ValueError("Observation masks must match observed matrix")
        if not np.array_equal(unknown, ~entry):
            raise ValueError("unknown_mask must be the complement of entry_mask")
        if np.any(np.diag(observed) != 0):
            raise ValueError("Observed matrix diagonal must be zero")
        tokens = tuple(self.revealed_tokens)
        if len({t.token_id for t in tokens}) != len(tokens):
            raise ValueError("Revealed token IDs must be unique")
        st = None if self.source_totals is None else readonly_array(self.source_totals, dtype=np.int64)
        dt = None if self.destination_totals is None else readonly_array(self.destination_totals, dtype=np.int64)
        n = observed.shape[0]
        if st is not None and st.shape != (n,):
            raise ValueError("source_totals shape mismatch")
        if dt is not None and dt.shape != (n,):
            raise ValueError("destination_totals shape mismatch")
        for name, value in (("entry_mask", entry), ("observed_matrix", observed),
                            ("unknown_mask", unknown), ("revealed_tokens", tokens),
                            ("source_totals", st), ("destination_totals", dt)):
            object.__setattr__(self, name, value)

    @property
    def executable_token_ids(self) -> tuple[TruthTokenId, ...]:
        return tuple(t.token_id for t in self.revealed_tokens)

    def to_policy_payload(self) -> Mapping[str, Any]:
        topo = _freeze({
            "num_nodes": self.topology.num_nodes, "num_edges": self.topology.num_edges,
            "edges": readonly_array(self.topology.edges),
            "capacities": readonly_array(self.topology.capacities),
            "shared_constraints": self.topology.shared_constraints, "name": self.topology.name,
        })
        return _freeze({
            "sequence_id": self.sequence_id, "sequence_step": self.sequence_step,
            "family": self.family, "mode": self.mode, "stage": self.stage, "ratio": self.ratio,
            "entry_mask": readonly_array(self.entry_mask),
            "observed_matrix": readonly_array(self.observed_matrix),
            "unknown_mask": readonly_array(self.unknown_mask),
            "revealed_tokens": self.revealed_tokens,
            "source_totals": None if self.source_totals is None else readonly_array(self.source_totals),
            "destination_totals": None if self.destination_totals is None else readonly_array(self.destination_totals),
            "topology": topo, "state_version": self.state_version,
        })


@dataclass(frozen=True, slots=True)
class SanitizedHistoryView:
    matrices: tuple[np.ndarray, ...]
    steps: tuple[int, ...]
    sequence_id: str
    current_step: int

    def __post_init__(self) -> None:
        raw = tuple(np.asarray(m) for m in self.matrices)
        for m in raw:
            validate_traffic_matrix(m)
        mats = tuple(readonly_array(m, dtype=np.int64) for m in raw)
        steps = tuple(int(s) for s in self.steps)
        if len(mats) != len(steps):
            raise ValueError("History matrices and steps must have equal lengths")
        if tuple(sorted(steps)) != steps or len(set(steps)) != len(steps):
            raise ValueError("History steps must be strictly increasing")
        if any(s >= self.current_step for s in steps):
            raise ValueError("History steps must be < current step; current/future X is forbidden")
        object.__setattr__(self, "matrices", mats)
        object.__setattr__(self, "steps", steps)

    @classmethod
    def from_completed_matrices(cls, *, matrices: Sequence[np.ndarray], steps: Sequence[int],
                                sequence_id: str, current_step: int) -> "SanitizedHistoryView":
        return cls(tuple(matrices), tuple(steps), str(sequence_id), int(current_step))


__all__ = ["PartialObservationState", "PublicTopologyView", "RevealedDemandToken",
           "SanitizedHistoryView", "TruthTokenId", "readonly_array"]
