"""What an ordinary planner is allowed to see of the reveal-aware world.

The public boundary of rlccl/uncertainty/observation.py:25-250 (class and
field names, the opaque token identity, the rule that only revealed tokens
are listed and that history stops strictly before the current step) with
its own mechanics:

* every array field is frozen by one table-driven pass (``_FROZEN``): an
  owned copy in the field's dtype with the write flag cleared;
* ``to_policy_payload`` is generated from the dataclass fields, so it always
  carries exactly the observation's fields (arrays re-copied read-only, the
  topology as a nested read-only mapping) and nothing evaluator-private.

Types:
* ``TruthTokenId`` — opaque identity issued only when a real token is revealed;
* ``RevealedDemandToken(token_id, source, destination, holders)``;
* ``PublicTopologyView`` — deep-copied, read-only static topology;
* ``PartialObservationState`` — the only current-demand object a planner gets;
* ``SanitizedHistoryView`` — completed matrices of strictly earlier steps.
"""

from __future__ import annotations

from dataclasses import dataclass, fields
from types import MappingProxyType
from typing import Any, Mapping, Sequence

import numpy as np

from ..traffic.matrix_utils import validate_traffic_matrix


def readonly_array(value: Any, *, dtype: Any | None = None) -> np.ndarray:
    """An owned copy of ``value`` that cannot be written through."""
    out = np.array(value, dtype=dtype, copy=True)
    out.setflags(write=False)
    return out


def _freeze_fields(obj: Any, spec: Mapping[str, Any]) -> None:
    """Replace each named array field (None stays None) by a frozen copy."""
    for name, dtype in spec.items():
        value = getattr(obj, name)
        object.__setattr__(obj, name, None if value is None else readonly_array(value, dtype=dtype))


def _publish(value: Any) -> Any:
    """The policy-payload form of one field value."""
    if isinstance(value, np.ndarray):
        return readonly_array(value)
    if isinstance(value, PublicTopologyView):
        return MappingProxyType({f.name: _publish(getattr(value, f.name)) for f in fields(value)})
    return value


@dataclass(frozen=True, slots=True)
class TruthTokenId:
    opaque_value: str

    def __post_init__(self) -> None:
        if not (isinstance(self.opaque_value, str) and self.opaque_value):
            raise ValueError("a truth token id is a non-empty opaque string")

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
            raise TypeError("a revealed token carries a TruthTokenId")
        if min(self.source, self.destination) < 0 or self.source == self.destination:
            raise ValueError("revealed token endpoints must be two distinct nonnegative nodes")
        holders = tuple(map(int, self.holders))
        if holders and min(holders) < 0:
            raise ValueError("holder node indices are nonnegative")
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
        _freeze_fields(self, {"edges": np.int64, "capacities": np.float64})
        if self.edges.shape != (self.num_edges, 2):
            raise ValueError(f"public topology edges must be [{self.num_edges}, 2]")
        if self.capacities.shape != (self.num_edges,):
            raise ValueError(f"public topology capacities must be [{self.num_edges}]")
        object.__setattr__(self, "shared_constraints",
                           tuple((tuple(map(int, members)), float(limit))
                                 for members, limit in self.shared_constraints))

    @classmethod
    def from_topology_info(cls, topology: Any) -> "PublicTopologyView":
        return cls(num_nodes=int(topology.V), num_edges=int(topology.E), edges=np.asarray(topology.edges),
                   capacities=np.asarray(topology.capacities),
                   shared_constraints=tuple(topology.shared_constraints), name=getattr(topology, "name", None))

    @property
    def edge_src(self) -> np.ndarray:
        return readonly_array(self.edges[:, 0], dtype=np.int64)

    @property
    def edge_dst(self) -> np.ndarray:
        return readonly_array(self.edges[:, 1], dtype=np.int64)


_OBSERVATION_ARRAYS = {"entry_mask": bool, "observed_matrix": np.int64, "unknown_mask": bool,
                       "source_totals": np.int64, "destination_totals": np.int64}


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
        _freeze_fields(self, _OBSERVATION_ARRAYS)
        object.__setattr__(self, "revealed_tokens", tuple(self.revealed_tokens))
        obs = self.observed_matrix
        if obs.ndim != 2 or obs.shape[0] != obs.shape[1]:
            raise ValueError("the observed matrix is square")
        n = obs.shape[0]
        if self.entry_mask.shape != obs.shape or self.unknown_mask.shape != obs.shape:
            raise ValueError("entry and unknown masks have the observed matrix's shape")
        if np.any(self.unknown_mask == self.entry_mask):
            raise ValueError("unknown_mask must be exactly the entries entry_mask leaves out")
        if np.diagonal(obs).any():
            raise ValueError("the observed matrix has a zero diagonal")
        ids = [t.token_id for t in self.revealed_tokens]
        if len(set(ids)) != len(ids):
            raise ValueError("a revealed token id is listed twice")
        for name in ("source_totals", "destination_totals"):
            totals = getattr(self, name)
            if totals is not None and totals.shape != (n,):
                raise ValueError(f"{name} must have one entry per node")

    @property
    def executable_token_ids(self) -> tuple[TruthTokenId, ...]:
        return tuple(t.token_id for t in self.revealed_tokens)

    def to_policy_payload(self) -> Mapping[str, Any]:
        """A fresh read-only mapping of this observation's fields."""
        return MappingProxyType({f.name: _publish(getattr(self, f.name)) for f in fields(self)})


@dataclass(frozen=True, slots=True)
class SanitizedHistoryView:
    matrices: tuple[np.ndarray, ...]
    steps: tuple[int, ...]
    sequence_id: str
    current_step: int

    def __post_init__(self) -> None:
        given = [np.asarray(m) for m in self.matrices]
        for m in given:
            validate_traffic_matrix(m)
        steps = np.asarray([int(s) for s in self.steps], dtype=np.int64)
        if len(given) != steps.size:
            raise ValueError("history needs one step number per matrix")
        if steps.size > 1 and np.any(np.diff(steps) <= 0):
            raise ValueError("history step numbers must strictly increase")
        if steps.size and int(steps.max()) >= self.current_step:
            raise ValueError("history may only hold steps before the current one (no current or future matrix)")
        object.__setattr__(self, "matrices", tuple(readonly_array(m, dtype=np.int64) for m in given))
        object.__setattr__(self, "steps", tuple(steps.tolist()))

    @classmethod
    def from_completed_matrices(cls, *, matrices: Sequence[np.ndarray], steps: Sequence[int],
                                sequence_id: str, current_step: int) -> "SanitizedHistoryView":
        return cls(matrices=tuple(matrices), steps=tuple(steps), sequence_id=str(sequence_id),
                   current_step=int(current_step))


__all__ = ["PartialObservationState", "PublicTopologyView", "RevealedDemandToken",
           "SanitizedHistoryView", "TruthTokenId", "readonly_array"]
