"""Leakage-safe baseline policies over the public observation
(rlccl/uncertainty/baselines.py:14-215).

The shared rule (``direct_revealed_proposal``): walk revealed tokens in their
public order; skip delivered ones; among edges out of a current holder into a
non-holder that lie on a shortest path to the destination (by public
topology hop distance), try them in (target distance, edge index) order and
take the first that still fits edge capacity and every shared group.  Each
token moves at most one hop per slot.

``PartialCurrentOnlyBaseline`` is the frozen production policy of the MoE
control plane.
"""

from __future__ import annotations

from collections import deque

import numpy as np

from .execution import Proposal, TransferAction
from .observation import PartialObservationState, SanitizedHistoryView
from .scenarios import ScenarioSet


def distance_to_destination(num_nodes: int, edges: np.ndarray, destination: int) -> np.ndarray:
    """Hop distance of every node to ``destination`` (reverse BFS); unreachable = V + 1."""
    incoming: list[list[int]] = [[] for _ in range(num_nodes)]
    for s, t in np.asarray(edges, dtype=np.int64).reshape(-1, 2):
        incoming[int(t)].append(int(s))
    dist = np.full(num_nodes, num_nodes + 1, dtype=np.int64)
    dist[int(destination)] = 0
    queue = deque([int(destination)])
    while queue:
        t = queue.popleft()
        for s in sorted(incoming[t]):
            if dist[s] > dist[t] + 1:
                dist[s] = dist[t] + 1
                queue.append(s)
    return dist


def direct_revealed_proposal(observation: PartialObservationState) -> Proposal:
    topo = observation.topology
    edges = np.asarray(topo.edges, dtype=np.int64)
    caps = np.asarray(topo.capacities, dtype=np.float64)
    edge_load = np.zeros(topo.num_edges, dtype=np.float64)
    group_load = np.zeros(len(topo.shared_constraints), dtype=np.float64)
    groups_of: list[list[tuple[int, float]]] = [[] for _ in range(topo.num_edges)]
    for g, (members, limit) in enumerate(topo.shared_constraints):
        for e in members:
            groups_of[int(e)].append((g, float(limit)))
    dist_cache: dict[int, np.ndarray] = {}
    actions: list[TransferAction] = []
    for token in observation.revealed_tokens:
        if token.destination in token.holders:
            continue
        dist = dist_cache.get(token.destination)
        if dist is None:
            dist = dist_cache[token.destination] = distance_to_destination(topo.num_nodes, edges, token.destination)
        holders = set(token.holders)
        options = sorted(
            (int(dist[t]), e) for e, (s, t) in enumerate(edges.tolist())
            if s in holders and t not in holders and dist[s] == dist[t] + 1
        )
        for _, e in options:
            if edge_load[e] + 1.0 > caps[e] + 1e-12:
                continue
            if any(group_load[g] + 1.0 > lim + 1e-12 for g, lim in groups_of[e]):
                continue
            actions.append(TransferAction(token.token_id, e))
            edge_load[e] += 1.0
            for g, _ in groups_of[e]:
                group_load[g] += 1.0
            break
    return Proposal.from_transfers(tuple(actions)) if actions else Proposal.wait()


# kept under the reference's private name for call-site parity
_direct_revealed_proposal = direct_revealed_proposal


def _validate_history(observation: PartialObservationState,
                      history: SanitizedHistoryView | None) -> SanitizedHistoryView | None:
    if history is None:
        return None
    if history.sequence_id != observation.sequence_id:
        raise ValueError("History and observation must belong to the same sequence")
    if history.current_step != observation.sequence_step:
        raise ValueError("History boundary must match the current sequence step")
    if any(m.shape != observation.observed_matrix.shape for m in history.matrices):
        raise ValueError("History matrix shape must match the current topology")
    return history


def _history_scenario(observation, history, *, method: str) -> Proposal:
    checked = _validate_history(observation, history)
    if checked is None or not checked.matrices:
        return Proposal.wait()
    if method == "long_term_mean":
        matrix = np.rint(np.mean(np.stack(checked.matrices), axis=0)).astype(np.int64)
        sid = "long-term-mean"
    elif method == "previous_value":
        matrix = np.array(checked.matrices[-1], dtype=np.int64, copy=True)
        sid = "previous-value"
    else:
        raise ValueError(f"Unsupported history scenario method: {method}")
    return Proposal.scenario_only(ScenarioSet.from_matrices(
        matrices=(matrix,), weights=(1.0,), scenario_ids=(sid,),
        provenance=("same-sequence-X-before-t",)))


class _Baseline:
    method = ""

    def propose(self, observation: PartialObservationState, *,
                history: SanitizedHistoryView | None = None,
                scenarios: ScenarioSet | None = None) -> Proposal:
        raise NotImplementedError


class WaitUntilKnownBaseline(_Baseline):
    method = "wait_until_known"

    def propose(self, observation, *, history=None, scenarios=None):
        _validate_history(observation, history)
        if observation.ratio < 1.0:
            return Proposal.wait()
        return direct_revealed_proposal(observation)


class PartialCurrentOnlyBaseline(_Baseline):
    method = "partial_current_only"

    def propose(self, observation, *, history=None, scenarios=None):
        _validate_history(observation, history)
        return direct_revealed_proposal(observation)


class LongTermMeanBaseline(_Baseline):
    method = "long_term_mean"

    def propose(self, observation, *, history=None, scenarios=None):
        _validate_history(observation, history)
        if observation.revealed_tokens:
            return direct_revealed_proposal(observation)
        return _history_scenario(observation, history, method="long_term_mean")


class PreviousValueBaseline(_Baseline):
    method = "previous_value"

    def propose(self, observation, *, history=None, scenarios=None):
        _validate_history(observation, history)
        if observation.revealed_tokens:
            return direct_revealed_proposal(observation)
        return _history_scenario(observation, history, method="previous_value")


class FullInformationOracle:
    """Evaluator-only lower bound; never produces executable actions."""

    method = "full_information_oracle"
    uses_oracle = True
    upper_bound_only = True


__all__ = ["FullInformationOracle", "LongTermMeanBaseline", "PartialCurrentOnlyBaseline",
           "PreviousValueBaseline", "WaitUntilKnownBaseline", "direct_revealed_proposal",
           "distance_to_destination"]
