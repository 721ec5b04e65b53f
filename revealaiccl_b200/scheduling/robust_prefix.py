"""Reference (uncompiled) planner primitives — the oracle of the compiled scheduler.

Behaviour of rlccl/scheduling/robust_prefix.py:63-452:

* ``canonical_shortest_path``: BFS over *usable* edges (unit capacity >= 1 and
  every group containing the edge has limit >= 1), expanding each node's
  out-edges in (target node, edge index) order, so ties go to the smaller
  destination id first ("destination-first tie").  It runs a BFS per call.
* ``enumerate_candidates``: for every revealed token with 0 < d(holders, dst)
  < inf, every usable edge from a holder to a non-holder that reduces the
  global distance by exactly one; sorted by (token ordinal, edge index).
* ``pack_candidate_batch``: greedy, one hop per token, edge and group unit
  budgets.
* robust scoring (criticality, utility, robust score) and
  ``RobustPrefixPlanner`` for the research arm (H/P allowlist, lambda in
  {0, .5, 1}, K in {1, 8}).
"""

from __future__ import annotations

from dataclasses import dataclass, replace
import hashlib
import math
from typing import Any, Sequence

import numpy as np

from ..uncertainty.observation import PublicTopologyView, readonly_array

SCORE_TIE_TOLERANCE = 1e-12
LEGAL_HORIZON_PREFIX = frozenset({(2, 1), (4, 1), (4, 2), (8, 1), (8, 2), (8, 4),
                                  (16, 1), (16, 2), (16, 4), (16, 8)})


class UnreachableScenarioError(ValueError):
    pass


class InconsistentResidualError(ValueError):
    pass


class StaleSupportError(ValueError):
    pass


def canonical_digest(value: Any) -> str:
    """sha256 over a typed, length-prefixed encoding (floats by their hex form)."""
    out = bytearray()

    def enc(item: Any) -> None:
        if item is None:
            out.extend(b"N|")
        elif isinstance(item, (bool, np.bool_)):
            out.extend(b"B1|" if bool(item) else b"B0|")
        elif isinstance(item, (int, np.integer)):
            out.extend(f"I{int(item)}|".encode())
        elif isinstance(item, (float, np.floating)):
            f = float(item)
            if not math.isfinite(f):
                raise ValueError("digest values must be finite")
            out.extend(f"F{f.hex()}|".encode())
        elif isinstance(item, str):
            raw = item.encode()
            out.extend(f"S{len(raw)}:".encode() + raw + b"|")
        elif isinstance(item, np.ndarray):
            enc({"dtype": item.dtype.str, "shape": list(item.shape), "data": item.reshape(-1).tolist()})
        elif hasattr(item, "__dataclass_fields__"):
            enc({k: getattr(item, k) for k in item.__dataclass_fields__})
        elif isinstance(item, dict):
            keys = sorted(item, key=lambda k: str(k).encode())
            out.extend(f"M{len(keys)}:".encode())
            for k in keys:
                enc(str(k))
                enc(item[k])
        elif isinstance(item, (list, tuple)):
            out.extend(f"L{len(item)}:".encode())
            for v in item:
                enc(v)
        elif isinstance(item, np.generic):
            enc(item.item())
        else:
            raise TypeError(f"unsupported digest type: {type(item).__name__}")

    enc(value)
    return hashlib.sha256(bytes(out)).hexdigest()


def _topology(topology: Any) -> tuple[int, np.ndarray, np.ndarray, tuple[Any, ...]]:
    nodes = int(getattr(topology, "num_nodes", getattr(topology, "V", 0)))
    edges = np.asarray(getattr(topology, "edges"), dtype=np.int64)
    caps = np.asarray(getattr(topology, "capacities"), dtype=np.float64)
    groups = tuple(getattr(topology, "shared_constraints", ()))
    return nodes, edges, caps, groups


@dataclass(frozen=True, slots=True)
class PublicRevealedToken:
    local_ordinal: int
    source: int
    destination: int
    holders: tuple[int, ...]


@dataclass(frozen=True, slots=True)
class SchedulingObservationView:
    stage: int
    ratio: float
    state_version: int
    observed_matrix: np.ndarray
    entry_mask: np.ndarray
    source_totals: np.ndarray | None
    destination_totals: np.ndarray | None
    revealed_tokens: tuple[PublicRevealedToken, ...]
    topology: PublicTopologyView
    observation_digest: str
    residual_state_digest: str

    def __post_init__(self) -> None:
        object.__setattr__(self, "observed_matrix", readonly_array(self.observed_matrix, dtype=np.int64))
        object.__setattr__(self, "entry_mask", readonly_array(self.entry_mask, dtype=bool))
        if self.source_totals is not None:
            object.__setattr__(self, "source_totals", readonly_array(self.source_totals, dtype=np.int64))
        if self.destination_totals is not None:
            object.__setattr__(self, "destination_totals", readonly_array(self.destination_totals, dtype=np.int64))
        t = self.topology
        object.__setattr__(self, "topology", PublicTopologyView(
            t.num_nodes, t.num_edges, t.edges, t.capacities, t.shared_constraints, t.name))


def build_scheduling_view(observation: Any) -> SchedulingObservationView:
    tokens = tuple(PublicRevealedToken(i, int(t.source), int(t.destination), tuple(t.holders))
                   for i, t in enumerate(observation.revealed_tokens))
    o = observation.topology
    topo = PublicTopologyView(o.num_nodes, o.num_edges, o.edges, o.capacities,
                              o.shared_constraints, o.name)
    demand_key = (int(observation.stage), float(observation.ratio),
                  np.asarray(observation.observed_matrix), np.asarray(observation.entry_mask),
                  observation.source_totals, observation.destination_totals,
                  tuple((t.source, t.destination) for t in tokens), topo)
    residual_key = (demand_key, tuple((t.local_ordinal, t.holders) for t in tokens))
    return SchedulingObservationView(
        int(observation.stage), float(observation.ratio), int(observation.state_version),
        observation.observed_matrix, observation.entry_mask, observation.source_totals,
        observation.destination_totals, tokens, topo, canonical_digest(demand_key),
        canonical_digest(residual_key))


def atomic_units(raw: float) -> int:
    v = float(raw)
    if not math.isfinite(v) or v < 0:
        raise ValueError("capacity must be finite and nonnegative")
    return int(math.floor(v))


def edge_usable(topology: Any, edge: int) -> bool:
    _, _, caps, groups = _topology(topology)
    if atomic_units(caps[edge]) < 1:
        return False
    return all(atomic_units(limit) >= 1 for members, limit in groups if edge in members)


_usable = edge_usable


def canonical_shortest_path(topology: Any, source: int, destination: int) -> tuple[int, ...]:
    nodes, edges, _, _ = _topology(topology)
    source, destination = int(source), int(destination)
    if source == destination:
        return ()
    out: list[list[int]] = [[] for _ in range(nodes)]
    for e, (u, _v) in enumerate(edges):
        if edge_usable(topology, e):
            out[int(u)].append(e)
    for row in out:
        row.sort(key=lambda e: (int(edges[e, 1]), e))
    parent: dict[int, tuple[int, int]] = {}
    seen = {source}
    frontier = [source]
    for node in frontier:
        for e in out[node]:
            t = int(edges[e, 1])
            if t in seen:
                continue
            seen.add(t)
            parent[t] = (node, e)
            if t == destination:
                path = []
                cur = t
                while cur != source:
                    cur, pe = parent[cur]
                    path.append(pe)
                return tuple(reversed(path))
            frontier.append(t)
    raise UnreachableScenarioError(f"unreachable OD {source}->{destination}")


def _distance(topology: Any, source: int, destination: int) -> float:
    try:
        return float(len(canonical_shortest_path(topology, source, destination)))
    except UnreachableScenarioError:
        return math.inf


@dataclass(frozen=True, slots=True)
class CandidateDistances:
    source_distance: float
    edge_target_distance: float
    before_global: float
    after_global: float


def candidate_distances(topology: Any, *, holders: Sequence[int], destination: int,
                        edge_index: int) -> CandidateDistances:
    _, edges, _, _ = _topology(topology)
    s, t = map(int, edges[int(edge_index)])
    before = min(_distance(topology, h, destination) for h in holders)
    td = _distance(topology, t, destination)
    return CandidateDistances(_distance(topology, s, destination), td, before, min(before, td))


def is_strict_global_progress(topology: Any, *, holders: Sequence[int], destination: int,
                              edge_index: int) -> bool:
    d = candidate_distances(topology, holders=holders, destination=destination, edge_index=edge_index)
    return math.isfinite(d.before_global) and d.before_global > 0 and d.after_global == d.before_global - 1


@dataclass(frozen=True, slots=True)
class CandidateAction:
    local_token_ordinal: int
    edge_index: int
    before_distance: int
    after_distance: int


def enumerate_candidates(view: SchedulingObservationView) -> tuple[CandidateAction, ...]:
    if view.ratio == 0 or not view.revealed_tokens:
        return ()
    _, edges, _, _ = _topology(view.topology)
    found: list[CandidateAction] = []
    for tok in view.revealed_tokens:
        before = min(_distance(view.topology, h, tok.destination) for h in tok.holders)
        if not math.isfinite(before) or before <= 0:
            continue
        for e, (s, t) in enumerate(edges):
            if int(s) not in tok.holders or int(t) in tok.holders or not edge_usable(view.topology, e):
                continue
            after = min(before, _distance(view.topology, int(t), tok.destination))
            if after == before - 1:
                found.append(CandidateAction(tok.local_ordinal, e, int(before), int(after)))
    return tuple(sorted(found, key=lambda c: (c.local_token_ordinal, c.edge_index)))


@dataclass(frozen=True, slots=True)
class BatchLoads:
    edge_units: np.ndarray
    group_units: np.ndarray


def batch_loads(batch: Sequence[CandidateAction], topology: Any) -> BatchLoads:
    _, edges, _, groups = _topology(topology)
    edge = np.zeros(len(edges), dtype=np.int64)
    for c in batch:
        edge[c.edge_index] += 1
    group = np.asarray([sum(edge[i] for i in members) for members, _ in groups], dtype=np.int64)
    return BatchLoads(edge, group)


def can_add_candidate(batch: Sequence[CandidateAction], candidate: CandidateAction, topology: Any) -> bool:
    if any(c.local_token_ordinal == candidate.local_token_ordinal for c in batch):
        return False
    _, _, caps, groups = _topology(topology)
    loads = batch_loads((*batch, candidate), topology)
    if any(loads.edge_units[i] > atomic_units(caps[i]) for i in range(len(caps))):
        return False
    return all(loads.group_units[i] <= atomic_units(lim) for i, (_, lim) in enumerate(groups))


def pack_candidate_batch(candidates: Sequence[CandidateAction], topology: Any) -> tuple[CandidateAction, ...]:
    batch: list[CandidateAction] = []
    for c in candidates:
        if can_add_candidate(batch, c, topology):
            batch.append(c)
    return tuple(batch)


@dataclass(frozen=True, slots=True)
class ResidualProjection:
    edge_loads: np.ndarray
    group_loads: np.ndarray
    digest: str


def project_residual_scenario(scenario: Any, view: SchedulingObservationView) -> ResidualProjection:
    m = np.asarray(scenario)
    if m.shape != view.observed_matrix.shape or not np.issubdtype(m.dtype, np.number):
        raise ValueError("scenario shape/type mismatch")
    if not np.all(np.isfinite(m)) or np.any(m < 0) or np.any(m != np.floor(m)):
        raise InconsistentResidualError("negative or noninteger scenario")
    m = m.astype(np.int64)
    nodes, edges, _, groups = _topology(view.topology)
    revealed = np.zeros_like(m)
    for t in view.revealed_tokens:
        revealed[t.source, t.destination] += 1
    if np.any(m < revealed):
        raise InconsistentResidualError("insufficient scenario load for revealed tokens")
    loads = np.zeros(len(edges), dtype=np.float64)
    for s in range(nodes):
        for d in range(nodes):
            amount = int(m[s, d])
            if amount <= 0 or s == d:
                continue
            try:
                path = canonical_shortest_path(view.topology, s, d)
            except UnreachableScenarioError:
                raise UnreachableScenarioError("positive unreachable scenario demand")
            loads[list(path)] += amount
    for t in view.revealed_tokens:
        try:
            origin = canonical_shortest_path(view.topology, t.source, t.destination)
        except UnreachableScenarioError as exc:
            raise InconsistentResidualError("revealed token unreachable") from exc
        loads[list(origin)] -= 1
        if t.destination not in t.holders:
            holder = min(t.holders, key=lambda n: (_distance(view.topology, n, t.destination), n))
            loads[list(canonical_shortest_path(view.topology, holder, t.destination))] += 1
    if np.any(loads < -1e-12):
        raise InconsistentResidualError("insufficient revealed scenario load")
    loads = np.maximum(loads, 0)
    group = np.asarray([sum(loads[i] for i in members) for members, _ in groups], dtype=np.float64)
    loads.setflags(write=False)
    group.setflags(write=False)
    return ResidualProjection(loads, group, canonical_digest((loads, group)))


def criticality_for_edge(*, residual_edge_load: float, edge_units: int,
                         incident_group_loads: Sequence[float], incident_group_units: Sequence[int]) -> float:
    values = [float(residual_edge_load), *map(float, incident_group_loads)]
    if not all(math.isfinite(v) and v >= 0 for v in values):
        raise ValueError("loads must be finite nonnegative")
    out = values[0] / max(int(edge_units), 1)
    out += sum(load / max(int(u), 1) for load, u in zip(values[1:], incident_group_units))
    return float(out)


def candidate_utility(*, criticality: float, after_distance: float) -> float:
    if not math.isfinite(float(criticality)) or not math.isfinite(float(after_distance)):
        raise ValueError("Q inputs must be finite")
    return 1.0 + 0.25 * float(criticality) - 0.05 * float(after_distance)


def robust_score(q: Any, weights: Any, *, risk_lambda: float) -> float:
    v = np.asarray(q, dtype=np.float64)
    w = np.asarray(weights, dtype=np.float64)
    if v.ndim != 1 or w.shape != v.shape or not np.all(np.isfinite(v)):
        raise ValueError("Q must be finite vector")
    if not np.all(np.isfinite(w)) or np.any(w < 0) or w.sum() <= 0:
        raise ValueError("weights must be finite nonnegative with positive sum")
    p = w / w.sum()
    mean = float(p @ v)
    var = float(p @ ((v - mean) ** 2))
    return mean - float(risk_lambda) * math.sqrt(max(var, 0.0))


@dataclass(frozen=True, slots=True)
class CandidateScore:
    candidate: CandidateAction
    robust_score: float
    scenario_std: float


def score_candidates(candidates: Sequence[CandidateAction], support: Any, *,
                     risk_lambda: float) -> tuple[CandidateScore, ...]:
    projections = [project_residual_scenario(m, support.observation) for m in support.matrices]
    _, _, caps, groups = _topology(support.observation.topology)
    p = np.asarray(support.weights, dtype=float)
    p = p / p.sum()
    out = []
    for c in candidates:
        incident = [i for i, (members, _) in enumerate(groups) if c.edge_index in members]
        q = np.asarray([candidate_utility(
            criticality=criticality_for_edge(
                residual_edge_load=pr.edge_loads[c.edge_index],
                edge_units=atomic_units(caps[c.edge_index]),
                incident_group_loads=tuple(pr.group_loads[i] for i in incident),
                incident_group_units=tuple(atomic_units(groups[i][1]) for i in incident)),
            after_distance=c.after_distance) for pr in projections])
        mean = float(p @ q)
        std = float(np.sqrt(p @ ((q - mean) ** 2)))
        out.append(CandidateScore(c, robust_score(q, p, risk_lambda=risk_lambda), std))
    return tuple(out)


@dataclass(frozen=True, slots=True)
class RobustPrefixConfig:
    horizon: int
    prefix: int
    risk_lambda: float
    requested_k: int

    def __post_init__(self) -> None:
        if (int(self.horizon), int(self.prefix)) not in LEGAL_HORIZON_PREFIX:
            raise ValueError("nonallowlisted H/P")
        if float(self.risk_lambda) not in (0.0, 0.5, 1.0):
            raise ValueError("risk lambda")
        if int(self.requested_k) not in (1, 8):
            raise ValueError("requested K must be point K1 or robust K8")


@dataclass(frozen=True, slots=True)
class SimulationStep:
    projected_load_digest: str


@dataclass(frozen=True, slots=True)
class PrefixPlan:
    origin_stage: int
    origin_state_version: int
    revision: int
    support_digest: str
    config_digest: str
    batches: tuple[tuple[CandidateAction, ...], ...]
    structural_actions: tuple[tuple[int, int], ...]
    simulation_trace: tuple[SimulationStep, ...]


class RobustPrefixPlanner:
    """Plan H simulated slots with robust scores and keep the first P batches."""

    def __init__(self, config: RobustPrefixConfig) -> None:
        self.config = config

    def plan(self, observation: SchedulingObservationView, support: Any) -> PrefixPlan:
        if support.stage != observation.stage:
            raise StaleSupportError("support stage mismatch")
        if support.observation_digest != observation.observation_digest:
            raise StaleSupportError("support observation digest mismatch")
        static = canonical_digest(tuple(project_residual_scenario(m, observation).digest
                                        for m in support.matrices))
        sim = observation
        planned: list[tuple[CandidateAction, ...]] = []
        trace: list[SimulationStep] = []
        _, edges, _, _ = _topology(observation.topology)
        for _ in range(self.config.horizon):
            cands = enumerate_candidates(sim)
            if not cands:
                break
            scores = score_candidates(cands, support, risk_lambda=self.config.risk_lambda)
            ordered = [s.candidate for s in sorted(
                scores, key=lambda s: (-s.robust_score, s.candidate.local_token_ordinal, s.candidate.edge_index))]
            batch = pack_candidate_batch(ordered, sim.topology)
            if not batch:
                break
            planned.append(batch)
            trace.append(SimulationStep(static))
            holders = [set(t.holders) for t in sim.revealed_tokens]
            for a in batch:
                holders[a.local_token_ordinal].add(int(edges[a.edge_index, 1]))
            toks = tuple(replace(t, holders=tuple(sorted(holders[t.local_ordinal]))) for t in sim.revealed_tokens)
            sim = replace(sim, revealed_tokens=toks, residual_state_digest=canonical_digest(
                tuple((t.local_ordinal, t.holders) for t in toks)))
        batches = tuple(planned[: self.config.prefix])
        structural = tuple((a.local_token_ordinal, a.edge_index) for b in batches for a in b)
        return PrefixPlan(observation.stage, observation.state_version, 0, support.digest,
                          canonical_digest(self.config), batches, structural,
                          tuple(trace[: self.config.prefix]))


__all__ = [
    "SchedulingObservationView", "PublicRevealedToken", "CandidateAction", "CandidateDistances",
    "CandidateScore", "RobustPrefixConfig", "RobustPrefixPlanner", "PrefixPlan",
    "UnreachableScenarioError", "InconsistentResidualError", "StaleSupportError", "atomic_units",
    "build_scheduling_view", "canonical_digest", "canonical_shortest_path", "enumerate_candidates",
    "pack_candidate_batch", "batch_loads", "project_residual_scenario", "robust_score",
    "criticality_for_edge", "candidate_utility", "score_candidates", "candidate_distances",
    "is_strict_global_progress", "can_add_candidate", "edge_usable", "SCORE_TIE_TOLERANCE",
]
