"""Proposals and the trusted, deterministic slot checker.

Interface of rlccl/uncertainty/execution.py:18-161 (``TransferAction``,
``Proposal``, ``CommitResult``, ``commit_proposal``,
``validate_legacy_schedule_matrix``) and its verdicts, in its order:

1. envelope: the observation and proposal types, no scenario tokens, the
   observation belongs to this problem stage, its state version is current
   (a wait is then legal and changes nothing);
2. per action, in proposal order: a token acted on twice, a token not
   revealed (not executable), an edge index out of range, an edge whose
   source does not hold the token, an edge whose destination already does;
3. bandwidth of the whole slot: per-edge capacity, then every shared group.

The slot is applied only after all three pass, atomically: possession is
read from the pre-slot state, so a token received in this slot cannot be
forwarded in the same slot.  Here the per-action stage resolves each action
to (token row, destination, edge) and the bandwidth stage works on the edge
column of that table (``np.bincount``) instead of accumulating loads
action by action.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import MappingProxyType
from typing import TYPE_CHECKING, Any, Mapping, Sequence

import numpy as np

from .observation import PartialObservationState, TruthTokenId
from .scenarios import ScenarioSet

if TYPE_CHECKING:
    from .problem import UncertainProblemInstance

_SLACK = 1e-12  # capacities are compared with this tolerance


class StaleObservationError(ValueError):
    """The observation's state version is no longer the world's."""


def _is_index(value: Any) -> bool:
    return isinstance(value, (int, np.integer)) and not isinstance(value, (bool, np.bool_))


@dataclass(frozen=True, slots=True)
class TransferAction:
    token_id: TruthTokenId
    edge_index: int

    def __post_init__(self) -> None:
        if not isinstance(self.token_id, TruthTokenId):
            raise TypeError("only a TruthTokenId can be transferred (scenario tokens never execute)")
        if not _is_index(self.edge_index):
            raise TypeError("edge_index is an integer")
        object.__setattr__(self, "edge_index", int(self.edge_index))


@dataclass(frozen=True, slots=True)
class Proposal:
    actions: tuple[TransferAction, ...] = ()
    scenario_set: ScenarioSet | None = None

    def __post_init__(self) -> None:
        actions = tuple(self.actions)
        if not all(isinstance(a, TransferAction) for a in actions):
            raise TypeError("every proposal action is a TransferAction")
        if actions and self.scenario_set is not None:
            raise ValueError("a scenario-only proposal carries no executable action")
        object.__setattr__(self, "actions", actions)

    @classmethod
    def wait(cls) -> "Proposal":
        return cls()

    @classmethod
    def from_transfers(cls, actions: Sequence[TransferAction]) -> "Proposal":
        return cls(actions=tuple(actions))

    @classmethod
    def scenario_only(cls, scenario_set: ScenarioSet) -> "Proposal":
        if not isinstance(scenario_set, ScenarioSet):
            raise TypeError("scenario_only takes a ScenarioSet")
        return cls(scenario_set=scenario_set)

    @property
    def is_wait(self) -> bool:
        return self.scenario_set is None and len(self.actions) == 0

    def to_public_payload(self) -> Mapping[str, Any]:
        rows = tuple(MappingProxyType({"token_id": a.token_id, "edge_index": a.edge_index}) for a in self.actions)
        return MappingProxyType({"actions": rows, "is_wait": self.is_wait, "scenario_set": self.scenario_set})


@dataclass(frozen=True, slots=True)
class CommitResult:
    legal: bool
    applied_actions: int
    state_version: int


def validate_legacy_schedule_matrix(matrix: Any, *, expected_shape: tuple[int, int]) -> np.ndarray:
    """A 0/1 schedule matrix of the legacy format as a read-only int8 copy."""
    m = np.asarray(matrix)
    if m.ndim != 2:
        raise ValueError("a legacy schedule matrix is 2-D")
    if tuple(m.shape) != tuple(expected_shape):
        raise ValueError(f"a legacy schedule matrix here has shape {expected_shape}")
    if not np.issubdtype(m.dtype, np.number):
        raise ValueError("a legacy schedule matrix holds numeric binary values")
    values = m.astype(np.float64, copy=False)
    for bad, why in ((~np.isfinite(values), "finite values (no NaN/Inf)"),
                     (values < 0, "nonnegative values"),
                     ((values != 0) & (values != 1), "binary values (0 or 1)")):
        if np.any(bad):
            raise ValueError(f"a legacy schedule matrix holds {why}")
    out = values.astype(np.int8)
    out.setflags(write=False)
    return out


def _check_envelope(world: "UncertainProblemInstance", observation: Any, proposal: Any) -> None:
    if not isinstance(observation, PartialObservationState):
        raise TypeError("commit takes a PartialObservationState")
    if not isinstance(proposal, Proposal):
        raise TypeError("commit takes a Proposal")
    if proposal.scenario_set is not None:
        raise ValueError("scenario tokens are for planning only and never execute")
    if (observation.sequence_id, observation.sequence_step) != (world.sequence_id, world.sequence_step):
        raise ValueError("the observation belongs to another problem stage")
    if observation.state_version != world._state_version:
        raise StaleObservationError("stale observation: its state version is not the world's current one")


def _resolve_actions(world: "UncertainProblemInstance", observation: PartialObservationState,
                     actions: tuple[TransferAction, ...]) -> np.ndarray:
    """[n, 3] int64 rows (token row, destination node, edge) or a ValueError
    naming the first action, in proposal order, that may not run."""
    topo = world.topology_info
    src_of, dst_of = np.asarray(topo.edge_src), np.asarray(topo.edge_dst)
    revealed = frozenset(observation.executable_token_ids)
    held = world._possession
    table = np.empty((len(actions), 3), dtype=np.int64)
    taken: set[TruthTokenId] = set()
    for i, action in enumerate(actions):
        tid, edge = action.token_id, action.edge_index
        if tid in taken:
            raise ValueError("duplicate token action conflict: one token acted on twice in a slot")
        taken.add(tid)
        row = world._public_to_private.get(tid) if tid in revealed else None
        if row is None:
            raise ValueError("the token is unrevealed and not executable at this stage")
        if not 0 <= edge < topo.E:
            raise ValueError(f"edge_index {edge} is outside 0..{topo.E - 1}")
        src, dst = int(src_of[edge]), int(dst_of[edge])
        if not held[row, src]:
            raise ValueError("the edge's source does not hold the token (source possession required)")
        if held[row, dst]:
            raise ValueError("the edge's destination already holds the token")
        table[i] = (row, dst, edge)
    return table


def _check_bandwidth(topology: Any, edges: np.ndarray) -> None:
    load = np.bincount(edges, minlength=int(topology.E)).astype(np.float64)
    if np.any(load > np.asarray(topology.capacities, dtype=np.float64) + _SLACK):
        raise ValueError("an edge's capacity (bandwidth) is exceeded")
    for members, limit in topology.shared_constraints:
        if load[np.asarray(members, dtype=np.int64)].sum() > float(limit) + _SLACK:
            raise ValueError("a shared group's bandwidth limit is exceeded")


def commit_proposal(world: "UncertainProblemInstance", observation: PartialObservationState,
                    proposal: Proposal) -> CommitResult:
    """Check a whole slot against the truth world, then apply it atomically."""
    _check_envelope(world, observation, proposal)
    if proposal.is_wait:
        return CommitResult(True, 0, world._state_version)
    table = _resolve_actions(world, observation, proposal.actions)
    _check_bandwidth(world.topology_info, table[:, 2])
    world._possession[table[:, 0], table[:, 1]] = True
    world._state_version += 1
    return CommitResult(True, int(table.shape[0]), world._state_version)


__all__ = ["CommitResult", "Proposal", "StaleObservationError", "TransferAction", "commit_proposal",
           "validate_legacy_schedule_matrix"]
