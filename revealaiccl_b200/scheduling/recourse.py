"""Binding planner ordinals to truth ids, the execution ledger and prefix repair.

Interface and verdicts of rlccl/scheduling/recourse.py:14-234: the state
records (``ExecutedActionIdentity``, ``ExecutedLedger``, ``RecourseState``,
``WaitOutcome``, ``Transition``, ``ExecutionOutcome``), the binding and
commit-recording functions and the transition reasons ("reveal",
"exhaustion", "invalidation", "continue"; "stale_observation" /
"checker_rejection" for a slot that may not run).

How this module does it:
* a plan's first batch is bound only after three groups of preconditions
  (``_PLAN_CHECKS`` on the plan against the public view, ``_check_trusted``
  on the trusted observation against the view, ``_check_first_batch`` on
  each planned hop against the current holders and distances);
* the ledger keeps a hash index beside its ordered tuple, so a replay is
  found in O(1) and a batch is appended in one step;
* whether a refused slot counts as stale is decided by the error's type
  (a stale plan revision, or a stale observation from the trusted checker),
  not by reading its message.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Any, Callable

import numpy as np

from ..uncertainty.execution import Proposal, StaleObservationError, TransferAction, commit_proposal
from ..uncertainty.observation import TruthTokenId


class StalePlanError(ValueError):
    """A plan (or its binding inputs) no longer matches the public state.

    ``stale`` marks the one case that means the plan itself is outdated (its
    revision is not the current one) as opposed to a precondition failure."""

    def __init__(self, message: str, *, stale: bool = False) -> None:
        super().__init__(message)
        self.stale = stale


class ReplayedActionError(ValueError):
    pass


@dataclass(frozen=True, slots=True)
class ExecutedActionIdentity:
    truth_token_id: Any
    edge_index: int
    plan_revision: int
    batch_ordinal: int


@dataclass(frozen=True, slots=True)
class ExecutedLedger:
    actions: tuple[ExecutedActionIdentity, ...] = ()
    _index: frozenset = field(default=frozenset(), compare=False, repr=False)

    def __post_init__(self) -> None:
        if len(self._index) != len(self.actions):
            object.__setattr__(self, "_index", frozenset(self.actions))

    @classmethod
    def empty(cls) -> "ExecutedLedger":
        return cls()

    def can_append(self, identity: ExecutedActionIdentity) -> bool:
        return identity not in self._index

    def append(self, identity: ExecutedActionIdentity) -> "ExecutedLedger":
        return self.extend((identity,))

    def extend(self, identities: tuple[ExecutedActionIdentity, ...]) -> "ExecutedLedger":
        index = set(self._index)
        for ident in identities:
            if ident in index:
                raise ReplayedActionError("an executed action (same token, edge, revision and batch) ran again")
            index.add(ident)
        return ExecutedLedger(self.actions + tuple(identities), frozenset(index))


@dataclass(frozen=True, slots=True)
class RecourseState:
    plan: Any | None
    executed_actions: tuple[ExecutedActionIdentity, ...] = ()
    discarded_actions: int = 0
    execution_start_state_version: int = 0
    reason: str = "initial"
    wait_latch: tuple[int, int] | None = None
    next_batch_index: int = 0
    current_revision: int = 0

    @classmethod
    def initial(cls, plan: Any) -> "RecourseState":
        return cls(plan=plan, execution_start_state_version=int(plan.origin_state_version),
                   current_revision=int(plan.revision))

    @classmethod
    def waiting(cls, view: Any) -> "RecourseState":
        return cls(plan=None, execution_start_state_version=int(view.state_version), reason="wait")


# (predicate on (state, view) that must hold, message, is the plan outdated)
_PLAN_CHECKS: tuple[tuple[Callable[[RecourseState, Any], bool], str, bool], ...] = (
    (lambda st, v: st.plan is not None and bool(st.plan.batches), "the plan has no batch left to execute", False),
    (lambda st, v: 0 <= int(st.plan.revision) == int(st.current_revision),
     "stale plan: its revision is not the current one", True),
    (lambda st, v: st.plan.origin_stage == v.stage, "the plan was made at another reveal stage", False),
    (lambda st, v: st.plan.origin_state_version == v.state_version,
     "the plan was made at another state version", False),
)


def _check_trusted(view: Any, trusted: Any) -> None:
    from .robust_prefix import build_scheduling_view

    if (int(trusted.stage), int(trusted.state_version)) != (int(view.stage), int(view.state_version)):
        raise StalePlanError("the trusted observation is at another stage or state version than the view")
    trusted_rows = [(int(t.source), int(t.destination), tuple(map(int, t.holders))) for t in trusted.revealed_tokens]
    public_rows = [(t.source, t.destination, t.holders) for t in view.revealed_tokens]
    if trusted_rows != public_rows:
        raise StalePlanError("the trusted and public revealed tokens differ")
    rebuilt = build_scheduling_view(trusted)
    if (rebuilt.observation_digest, rebuilt.residual_state_digest) != (view.observation_digest,
                                                                      view.residual_state_digest):
        raise StalePlanError("the trusted observation does not rebuild the view's digests")


def _check_first_batch(plan: Any, view: Any) -> None:
    from .robust_prefix import candidate_distances

    edges = np.asarray(view.topology.edges, dtype=np.int64)
    for hop in plan.batches[0]:
        token = view.revealed_tokens[hop.local_token_ordinal]
        src, dst = (int(x) for x in edges[hop.edge_index])
        if src not in token.holders or dst in token.holders:
            raise StalePlanError("a planned hop no longer starts at a holder or ends at a non-holder")
        dist = candidate_distances(view.topology, holders=token.holders, destination=token.destination,
                                   edge_index=hop.edge_index)
        if (dist.before_global, dist.after_global) != (hop.before_distance, hop.after_distance):
            raise StalePlanError("a planned hop's distances no longer hold")


def _validate_binding(state: RecourseState, view: Any, trusted: Any | None) -> None:
    for holds, message, outdated in _PLAN_CHECKS:
        if not holds(state, view):
            raise StalePlanError(message, stale=outdated)
    if trusted is not None:
        _check_trusted(view, trusted)
    _check_first_batch(state.plan, view)


def bind_action(view: Any, *, local_token_ordinal: int, edge_index: int,
                trusted_observation: Any | None = None) -> TransferAction:
    """The executable action for the public token ``local_token_ordinal``:
    its opaque truth id comes from the trusted observation at that ordinal."""
    if not isinstance(local_token_ordinal, (int, np.integer)) or isinstance(local_token_ordinal, (bool, np.bool_)):
        raise TypeError("a local token ordinal is an integer")
    ordinal = int(local_token_ordinal)
    if not 0 <= ordinal < len(view.revealed_tokens):
        raise IndexError("the local token ordinal is hidden or outside the revealed tokens")
    if trusted_observation is None:
        raise ValueError("binding a truth token identity needs the trusted observation")
    revealed = trusted_observation.revealed_tokens
    if ordinal >= len(revealed):
        raise ValueError("the trusted revealed tokens do not match the view")
    tid = revealed[ordinal].token_id
    if not isinstance(tid, TruthTokenId):
        raise TypeError("only revealed truth tokens execute")
    return TransferAction(tid, int(edge_index))


def bind_first_batch(state: RecourseState, view: Any, *, trusted_observation: Any | None = None) -> Proposal:
    _validate_binding(state, view, trusted_observation)
    if trusted_observation is None:
        raise ValueError("an executable binding needs the trusted observation")
    return Proposal.from_transfers([
        bind_action(view, local_token_ordinal=hop.local_token_ordinal, edge_index=hop.edge_index,
                    trusted_observation=trusted_observation)
        for hop in state.plan.batches[0]])


def record_committed_batch(state: RecourseState, *, proposal: Proposal, commit_result: Any,
                           fresh_observation: Any) -> RecourseState:
    """Advance the state past a batch the trusted checker applied."""
    if not commit_result.legal:
        raise ValueError("an illegal commit is never recorded")
    if int(fresh_observation.state_version) != int(commit_result.state_version):
        raise StalePlanError("the fresh observation is not at the commit's state version")
    holders = {t.token_id: t.holders for t in fresh_observation.revealed_tokens}
    edge_dst = np.asarray(fresh_observation.topology.edges, dtype=np.int64)[:, 1]
    for action in proposal.actions:
        if action.token_id not in holders:
            raise StalePlanError("a committed token is missing from the fresh revealed tokens")
        if int(edge_dst[action.edge_index]) not in holders[action.token_id]:
            raise StalePlanError("the fresh holders lack a committed destination")
    revision, ordinal = int(state.plan.revision), int(state.next_batch_index)
    ledger = ExecutedLedger(tuple(state.executed_actions)).extend(tuple(
        ExecutedActionIdentity(a.token_id, int(a.edge_index), revision, ordinal) for a in proposal.actions))
    rest = tuple(state.plan.batches[1:])
    plan = replace(state.plan, origin_state_version=int(commit_result.state_version), batches=rest,
                   structural_actions=tuple((h.local_token_ordinal, h.edge_index) for b in rest for h in b),
                   simulation_trace=tuple(state.plan.simulation_trace[1:]))
    return replace(state, plan=plan, executed_actions=ledger.actions, reason="commit",
                   next_batch_index=ordinal + 1)


def repair_prefix(state: RecourseState, view: Any, support: Any, planner: Any, *, reason: str) -> RecourseState:
    """Replan from the current view; the old plan's unexecuted hops are counted as discarded."""
    old = state.plan
    discarded = 0 if old is None else sum(map(len, old.batches))
    revision = 0 if old is None else old.revision + 1
    plan = replace(planner.plan(view, support), revision=revision)
    return replace(state, plan=plan, discarded_actions=state.discarded_actions + discarded, reason=str(reason),
                   wait_latch=None, next_batch_index=0, current_revision=revision)


@dataclass(frozen=True, slots=True)
class WaitOutcome:
    state: RecourseState
    no_common_delta: int
    fallback_delta: int


def enter_wait_latch(state: RecourseState, view: Any) -> WaitOutcome:
    """Latch a wait at (stage, state version); only a new latch counts once."""
    key = (int(view.stage), int(view.state_version))
    fresh = int(state.wait_latch != key)
    return WaitOutcome(replace(state, wait_latch=key), fresh, fresh)


@dataclass(frozen=True, slots=True)
class Transition:
    reason: str
    reveal_delta: int
    exhaustion_delta: int
    invalidation_delta: int


_TRANSITIONS = ("reveal", "exhaustion", "invalidation")


def choose_transition(*, new_stage: bool, prefix_exhausted: bool, precondition_valid: bool) -> Transition:
    """The first applicable of reveal > exhaustion > invalidation, else continue."""
    fired = (new_stage, prefix_exhausted, not precondition_valid)
    reason = next((name for name, hit in zip(_TRANSITIONS, fired) if hit), "continue")
    return Transition(reason, *(int(reason == name) for name in _TRANSITIONS))


@dataclass(frozen=True, slots=True)
class ExecutionOutcome:
    legality: bool
    stopped: bool
    illegal_reason: str | None
    fallback_delta: int
    no_common_delta: int
    commit_result: Any | None
    proposal: Proposal | None = None


def _refusal_reason(error: ValueError) -> str:
    outdated = isinstance(error, StaleObservationError) or getattr(error, "stale", False)
    return "stale_observation" if outdated else "checker_rejection"


def execute_first_batch(*, world: Any, state: RecourseState, view: Any,
                        trusted_observation: Any) -> ExecutionOutcome:
    """Bind and commit the plan's first batch; a refused slot stops execution."""
    try:
        proposal = bind_first_batch(state, view, trusted_observation=trusted_observation)
        result = commit_proposal(world, trusted_observation, proposal)
    except ValueError as error:
        return ExecutionOutcome(False, True, _refusal_reason(error), 0, 0, None, None)
    legal = bool(result.legal)
    return ExecutionOutcome(legal, not legal, None if legal else "checker_rejection", 0, 0, result, proposal)


__all__ = ["ExecutedActionIdentity", "ExecutedLedger", "ExecutionOutcome", "RecourseState",
           "ReplayedActionError", "StalePlanError", "Transition", "WaitOutcome", "bind_action",
           "bind_first_batch", "choose_transition", "enter_wait_latch", "execute_first_batch",
           "record_committed_batch", "repair_prefix"]
