"""Proposals and the trusted deterministic checker (rlccl/uncertainty/execution.py:18-161).

``commit_proposal`` validates a whole slot before applying anything and
rejects, in this order: scenario-only proposals, an observation of another
problem stage, a stale state version, a token acted on twice, an unrevealed
token, an out-of-range edge, a source that does not hold the token, a
destination that already holds it, edge capacity, and every shared
bandwidth group.  It then applies all transfers atomically; because sources
were checked against the pre-slot state, a token received in this slot
cannot be forwarded in the same slot.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import MappingProxyType
from typing import TYPE_CHECKING, Any, Mapping

import numpy as np

from .observation import PartialObservationState, TruthTokenId
from .scenarios import ScenarioSet

if TYPE_CHECKING:
    from .problem import UncertainProblemInstance


@dataclass(frozen=True, slots=True)
class TransferAction:
    token_id: TruthTokenId
    edge_index: int

    def __post_init__(self) -> None:
        if not isinstance(self.token_id, TruthTokenId):
            raise TypeError("TransferAction requires TruthTokenId; scenario tokens are not executable")
        if isinstance(self.edge_index, (bool, np.bool_)) or not isinstance(self.edge_index, (int, np.integer)):
            raise TypeError("edge_index must be an integer")
        object.__setattr__(self, "edge_index", int(self.edge_index))


@dataclass(frozen=True, slots=True)
class Proposal:
    actions: tuple[TransferAction, ...] = ()
    scenario_set: ScenarioSet | None = None

    def __post_init__(self) -> None:
        actions = tuple(self.actions)
        if any(not isinstance(a, TransferAction) for a in actions):
            raise TypeError("Proposal actions must be TransferAction objects")
        if self.scenario_set is not None and actions:
            raise ValueError("A scenario-only proposal cannot contain executable actions")
        object.__setattr__(self, "actions", actions)

    @classmethod
    def wait(cls) -> "Proposal":
        return cls()

    @classmethod
    def from_transfers(cls, actions: tuple[TransferAction, ...]) -> "Proposal":
        return cls(actions=tuple(actions))

    @classmethod
    def scenario_only(cls, scenario_set: ScenarioSet) -> "Proposal":
        if not isinstance(scenario_set, ScenarioSet):
            raise TypeError("scenario_only requires ScenarioSet")
        return cls(scenario_set=scenario_set)

    @property
    def is_wait(self) -> bool:
        return not self.actions and self.scenario_set is None

    def to_public_payload(self) -> Mapping[str, Any]:
        return MappingProxyType({
            "actions": tuple(MappingProxyType({"token_id": a.token_id, "edge_index": a.edge_index})
                             for a in self.actions),
            "is_wait": self.is_wait,
            "scenario_set": self.scenario_set,
        })


@dataclass(frozen=True, slots=True)
class CommitResult:
    legal: bool
    applied_actions: int
    state_version: int


def validate_legacy_schedule_matrix(matrix: Any, *, expected_shape: tuple[int, int]) -> np.ndarray:
    m = np.asarray(matrix)
    if m.ndim != 2:
        raise ValueError("Legacy schedule matrix must be 2-D")
    if tuple(m.shape) != tuple(expected_shape):
        raise ValueError(f"Legacy schedule matrix shape must be {expected_shape}")
    if not np.issubdtype(m.dtype, np.number):
        raise ValueError("Legacy schedule matrix must contain numeric binary values")
    f = m.astype(np.float64, copy=False)
    if not np.all(np.isfinite(f)):
        raise ValueError("Legacy schedule matrix must contain finite values, not NaN/Inf")
    if np.any(f < 0):
        raise ValueError("Legacy schedule matrix must be nonnegative")
    if np.any((f != 0) & (f != 1)):
        raise ValueError("Legacy schedule matrix must be binary")
    out = np.array(f, dtype=np.int8, copy=True)
    out.setflags(write=False)
    return out


_EPS = 1e-12


def commit_proposal(world: "UncertainProblemInstance", observation: PartialObservationState,
                    proposal: Proposal) -> CommitResult:
    if not isinstance(observation, PartialObservationState):
        raise TypeError("commit requires PartialObservationState")
    if not isinstance(proposal, Proposal):
        raise TypeError("commit requires Proposal")
    if proposal.scenario_set is not None:
        raise ValueError("Scenario tokens are planning-only and not executable")
    if observation.sequence_id != world.sequence_id or observation.sequence_step != world.sequence_step:
        raise ValueError("Observation belongs to a different problem stage")
    if observation.state_version != world._state_version:
        raise ValueError("stale observation cannot be committed")
    if proposal.is_wait:
        return CommitResult(True, 0, world._state_version)
    topo = world.topology_info
    executable = set(observation.executable_token_ids)
    seen: set[TruthTokenId] = set()
    load = np.zeros(topo.E, dtype=np.float64)
    resolved: list[tuple[int, int]] = []
    for action in proposal.actions:
        if action.token_id in seen:
            raise ValueError("Duplicate token action conflict in one slot")
        seen.add(action.token_id)
        if action.token_id not in executable or action.token_id not in world._public_to_private:
            raise ValueError("Token is unrevealed and not executable at this stage")
        edge = int(action.edge_index)
        if edge < 0 or edge >= topo.E:
            raise ValueError("edge_index is outside valid edge range")
        token = world._public_to_private[action.token_id]
        src, dst = int(topo.edge_src[edge]), int(topo.edge_dst[edge])
        if not world._possession[token, src]:
            raise ValueError("Edge source is not a current token holder; source possession required")
        if world._possession[token, dst]:
            raise ValueError("Edge destination already holds this token")
        load[edge] += 1.0
        resolved.append((token, dst))
    if np.any(load > np.asarray(topo.capacities, dtype=float) + _EPS):
        raise ValueError("Edge capacity/bandwidth exceeded")
    for members, limit in topo.shared_constraints:
        if float(load[np.asarray(members, dtype=np.int64)].sum()) > float(limit) + _EPS:
            raise ValueError("Shared group bandwidth limit exceeded")
    for token, dst in resolved:
        world._possession[token, dst] = True
    world._state_version += 1
    return CommitResult(True, len(resolved), world._state_version)


__all__ = ["CommitResult", "Proposal", "TransferAction", "commit_proposal",
           "validate_legacy_schedule_matrix"]
