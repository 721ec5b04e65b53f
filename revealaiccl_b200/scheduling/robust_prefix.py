"""Uncompiled planner primitives: the oracle of the compiled scheduler, and the
robust-prefix planner of the recourse study.

Semantics of rlccl/scheduling/robust_prefix.py:63-452 (kept, because the
compiled scheduler, the device control plane and the recourse runner must
reproduce them exactly):

* routes use *usable* edges only (capacity units >= 1 and every shared group
  containing the edge has limit units >= 1); a shortest route is found by BFS
  that expands each node's out-edges in (target node, edge index) order, so
  ties go to the smaller target id first ("destination-first");
* a candidate is one hop of a revealed token from a holder to a non-holder
  over a usable edge that lowers the token's distance to its destination by
  exactly one; candidates are ordered by (token ordinal, edge index);
* a batch is packed greedily from an ordered candidate list: at most one hop
  per token, within every edge's and every group's unit budget;
* the robust score of a hop is the weighted mean minus lambda times the
  weighted standard deviation, over scenarios, of
  1 + 0.25 * criticality - 0.05 * distance-after, where criticality sums the
  scenario's residual load over capacity units of the edge and of each group
  containing it.

Mechanics of this module: every topology gets one cached ``_Routes`` table,
built by a BFS from each source (V BFS runs in total, instead of one per
query): the all-pairs distance matrix and each source's BFS parent edges,
from which a canonical route is read back.  Candidate enumeration is then a
vectorised edge mask per token, batch packing keeps running edge and group
loads, and a residual projection adds whole route incidence vectors.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, replace
import hashlib
import math
from typing import Any, Sequence

import numpy as np

from ..uncertainty.observation import PublicTopologyView, readonly_array

SCORE_TIE_TOLERANCE = 1e-12
LEGAL_HORIZON_PREFIX = frozenset({(2, 1), (4, 1), (4, 2), (8, 1), (8, 2), (8, 4),
                                  (16, 1), (16, 2), (16, 4), (16, 8)})
RISK_LAMBDAS = (0.0, 0.5, 1.0)
REQUESTED_K = (1, 8)


class UnreachableScenarioError(ValueError):
    pass


class InconsistentResidualError(ValueError):
    pass


class StaleSupportError(ValueError):
    pass


# --------------------------------------------------------------------- digest
def _digest_parts(item: Any, out: bytearray) -> None:
    """Typed, length-prefixed encoding (floats by their exact hex form)."""
    stack = [item]
    while stack:
        x = stack.pop()
        if x is None:
            out += b"N|"
        elif isinstance(x, (bool, np.bool_)):
            out += b"B1|" if x else b"B0|"
        elif isinstance(x, (int, np.integer)):
            out += b"I%d|" % int(x)
        elif isinstance(x, (float, np.floating)):
            f = float(x)
            if not math.isfinite(f):
                raise ValueError("digest values must be finite")
            out += b"F" + f.hex().encode() + b"|"
        elif isinstance(x, str):
            raw = x.encode()
            out += b"S%d:" % len(raw) + raw + b"|"
        elif isinstance(x, np.ndarray):
            stack.append({"dtype": x.dtype.str, "shape": list(x.shape), "data": x.reshape(-1).tolist()})
        elif hasattr(x, "__dataclass_fields__"):
            stack.append({k: getattr(x, k) for k in x.__dataclass_fields__})
        elif isinstance(x, dict):
            keys = sorted(x, key=lambda k: str(k).encode())
            out += b"M%d:" % len(keys)
            for k in reversed(keys):  # the stack pops them back in key order
                stack.append(x[k])
                stack.append(str(k))
        elif isinstance(x, (list, tuple)):
            out += b"L%d:" % len(x)
            stack.extend(reversed(x))
        elif isinstance(x, np.generic):
            stack.append(x.item())
        else:
            raise TypeError(f"unsupported digest type: {type(x).__name__}")


def canonical_digest(value: Any) -> str:
    """sha256 of the typed encoding of ``value`` (nested containers, dataclasses, arrays)."""
    out = bytearray()
    _digest_parts(value, out)
    return hashlib.sha256(bytes(out)).hexdigest()


# ------------------------------------------------------------------- topology
def _topology(topology: Any) -> tuple[int, np.ndarray, np.ndarray, tuple[Any, ...]]:
    nodes = int(getattr(topology, "num_nodes", getattr(topology, "V", 0)))
    edges = np.asarray(topology.edges, dtype=np.int64).reshape(-1, 2)
    caps = np.asarray(topology.capacities, dtype=np.float64)
    groups = tuple(getattr(topology, "shared_constraints", ()))
    return nodes, edges, caps, groups


def atomic_units(raw: float) -> int:
    """Whole transfer units a capacity allows per slot."""
    v = float(raw)
    if not (math.isfinite(v) and v >= 0):
        raise ValueError("a capacity is finite and nonnegative")
    return int(math.floor(v))


class _Routes:
    """Usable edges, all-pairs BFS distances and canonical parent edges of one topology."""

    def __init__(self, topology: Any) -> None:
        nodes, edges, caps, groups = _topology(topology)
        self.nodes, self.edges = nodes, edges
        self.edge_units = np.asarray([atomic_units(c) for c in caps], dtype=np.int64)
        self.groups = tuple((np.asarray(list(m), dtype=np.int64), lim) for m, lim in groups)
        self.group_units = np.asarray([atomic_units(lim) if len(m) else 0 for m, lim in self.groups],
                                      dtype=np.int64)
        usable = self.edge_units >= 1
        for (members, _), units in zip(self.groups, self.group_units):
            if len(members) and units < 1:
                usable[members] = False
        self.usable = usable
        # groups containing each edge, in group order, and how many times each
        # lists the edge (a group's load counts an edge once per listing)
        self.edge_groups: list[list[int]] = [[] for _ in range(len(edges))]
        self.edge_group_mult: list[dict[int, int]] = [{} for _ in range(len(edges))]
        for g, (members, _) in enumerate(self.groups):
            for e in members.tolist():
                if g not in self.edge_group_mult[e]:
                    self.edge_groups[e].append(g)
                self.edge_group_mult[e][g] = self.edge_group_mult[e].get(g, 0) + 1
        ids = np.flatnonzero(usable)
        ids = ids[np.lexsort((ids, edges[ids, 1], edges[ids, 0]))]  # by source, then target, then edge
        starts = np.searchsorted(edges[ids, 0], np.arange(nodes + 1))
        self.dist = np.full((nodes, nodes), np.inf)
        self.parent = np.full((nodes, nodes), -1, dtype=np.int64)
        for s in range(nodes):
            self.dist[s, s] = 0.0
            queue = [s]
            for u in queue:
                for e in ids[starts[u]:starts[u + 1]].tolist():
                    t = int(edges[e, 1])
                    if self.dist[s, t] == np.inf:
                        self.dist[s, t] = self.dist[s, u] + 1.0
                        self.parent[s, t] = e
                        queue.append(t)

    def path(self, source: int, destination: int) -> tuple[int, ...]:
        if source == destination:
            return ()
        if self.dist[source, destination] == np.inf:
            raise UnreachableScenarioError(f"unreachable OD {source}->{destination}")
        hops = []
        node = destination
        while node != source:
            e = int(self.parent[source, node])
            hops.append(e)
            node = int(self.edges[e, 0])
        return tuple(reversed(hops))


_ROUTE_CACHE: "OrderedDict[tuple, _Routes]" = OrderedDict()


def _routes(topology: Any) -> _Routes:
    nodes, edges, caps, groups = _topology(topology)
    key = (nodes, edges.tobytes(), caps.tobytes(),
           tuple((tuple(int(e) for e in m), float(lim)) for m, lim in groups))
    hit = _ROUTE_CACHE.get(key)
    if hit is None:
        hit = _Routes(topology)
        _ROUTE_CACHE[key] = hit
        if len(_ROUTE_CACHE) > 64:
            _ROUTE_CACHE.popitem(last=False)
    else:
        _ROUTE_CACHE.move_to_end(key)
    return hit


def edge_usable(topology: Any, edge: int) -> bool:
    return bool(_routes(topology).usable[int(edge)])


def canonical_shortest_path(topology: Any, source: int, destination: int) -> tuple[int, ...]:
    return _routes(topology).path(int(source), int(destination))


def _distance(topology: Any, source: int, destination: int) -> float:
    return float(_routes(topology).dist[int(source), int(destination)])


# ---------------------------------------------------------------- public view
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
        for name, dtype in (("observed_matrix", np.int64), ("entry_mask", bool),
                            ("source_totals", np.int64), ("destination_totals", np.int64)):
            value = getattr(self, name)
            if value is not None:
                object.__setattr__(self, name, readonly_array(value, dtype=dtype))
        t = self.topology
        object.__setattr__(self, "topology", PublicTopologyView(
            t.num_nodes, t.num_edges, t.edges, t.capacities, t.shared_constraints, t.name))


def _residual_key(tokens: Sequence[PublicRevealedToken]) -> tuple:
    return tuple((t.local_ordinal, t.holders) for t in tokens)


def build_scheduling_view(observation: Any) -> SchedulingObservationView:
    """The planner's view of an observation, with digests of its demand part
    and of its demand plus current holders."""
    o = observation
    tokens = tuple(PublicRevealedToken(i, int(t.source), int(t.destination), tuple(t.holders))
                   for i, t in enumerate(o.revealed_tokens))
    topo = PublicTopologyView(o.topology.num_nodes, o.topology.num_edges, o.topology.edges,
                              o.topology.capacities, o.topology.shared_constraints, o.topology.name)
    demand = (int(o.stage), float(o.ratio), np.asarray(o.observed_matrix), np.asarray(o.entry_mask),
              o.source_totals, o.destination_totals, tuple((t.source, t.destination) for t in tokens), topo)
    return SchedulingObservationView(
        stage=int(o.stage), ratio=float(o.ratio), state_version=int(o.state_version),
        observed_matrix=o.observed_matrix, entry_mask=o.entry_mask, source_totals=o.source_totals,
        destination_totals=o.destination_totals, revealed_tokens=tokens, topology=topo,
        observation_digest=canonical_digest(demand),
        residual_state_digest=canonical_digest((demand, _residual_key(tokens))))


# ----------------------------------------------------------------- candidates
@dataclass(frozen=True, slots=True)
class CandidateDistances:
    source_distance: float
    edge_target_distance: float
    before_global: float
    after_global: float


def candidate_distances(topology: Any, *, holders: Sequence[int], destination: int,
                        edge_index: int) -> CandidateDistances:
    r = _routes(topology)
    src, tgt = (int(x) for x in r.edges[int(edge_index)])
    before = float(min(r.dist[int(h), int(destination)] for h in holders))
    target = float(r.dist[tgt, int(destination)])
    return CandidateDistances(float(r.dist[src, int(destination)]), target, before, min(before, target))


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
    """Every distance-lowering hop of every revealed token, by (ordinal, edge)."""
    if view.ratio == 0 or not view.revealed_tokens:
        return ()
    r = _routes(view.topology)
    src, tgt = r.edges[:, 0], r.edges[:, 1]
    out: list[CandidateAction] = []
    for token in view.revealed_tokens:
        held = np.zeros(r.nodes, dtype=bool)
        held[list(token.holders)] = True
        to_dst = r.dist[:, token.destination]
        before = float(to_dst[held].min()) if held.any() else math.inf
        if not (math.isfinite(before) and before > 0):
            continue
        # a usable hop from a holder to a non-holder whose target is one step closer
        hop = r.usable & held[src] & ~held[tgt] & (to_dst[tgt] == before - 1)
        out.extend(CandidateAction(token.local_ordinal, int(e), int(before), int(before) - 1)
                   for e in np.flatnonzero(hop).tolist())
    out.sort(key=lambda c: (c.local_token_ordinal, c.edge_index))
    return tuple(out)


@dataclass(frozen=True, slots=True)
class BatchLoads:
    edge_units: np.ndarray
    group_units: np.ndarray


def batch_loads(batch: Sequence[CandidateAction], topology: Any) -> BatchLoads:
    """Units a batch puts on every edge and on every shared group."""
    _, edges, _, groups = _topology(topology)
    per_edge = np.bincount(np.asarray([c.edge_index for c in batch], dtype=np.int64),
                           minlength=len(edges)).astype(np.int64)
    per_group = np.asarray([int(per_edge[np.asarray(list(m), dtype=np.int64)].sum()) for m, _ in groups],
                           dtype=np.int64)
    return BatchLoads(per_edge, per_group)


class _Packer:
    """Running edge and group loads of a batch under construction."""

    def __init__(self, topology: Any) -> None:
        r = _routes(topology)
        self.r = r
        self.edge_load = np.zeros(len(r.edges), dtype=np.int64)
        self.group_load = np.zeros(len(r.groups), dtype=np.int64)
        self.tokens: set[int] = set()

    def fits(self, c: CandidateAction) -> bool:
        if c.local_token_ordinal in self.tokens:
            return False
        e = c.edge_index
        if self.edge_load[e] + 1 > self.r.edge_units[e]:
            return False
        return all(self.group_load[g] + k <= self.r.group_units[g] for g, k in self.r.edge_group_mult[e].items())

    def add(self, c: CandidateAction) -> None:
        self.tokens.add(c.local_token_ordinal)
        self.edge_load[c.edge_index] += 1
        for g, k in self.r.edge_group_mult[c.edge_index].items():
            self.group_load[g] += k


def can_add_candidate(batch: Sequence[CandidateAction], candidate: CandidateAction, topology: Any) -> bool:
    packer = _Packer(topology)
    for c in batch:
        packer.add(c)
    return packer.fits(candidate)


def pack_candidate_batch(candidates: Sequence[CandidateAction], topology: Any) -> tuple[CandidateAction, ...]:
    """Greedy batch in the given candidate order."""
    packer = _Packer(topology)
    chosen = []
    for c in candidates:
        if packer.fits(c):
            packer.add(c)
            chosen.append(c)
    return tuple(chosen)


# ------------------------------------------------------- residual projections
@dataclass(frozen=True, slots=True)
class ResidualProjection:
    edge_loads: np.ndarray
    group_loads: np.ndarray
    digest: str


def project_residual_scenario(scenario: Any, view: SchedulingObservationView) -> ResidualProjection:
    """Edge and group loads a scenario still needs on canonical routes, given
    what the revealed tokens already carry (each revealed token's own route is
    replaced by the route from its closest holder, or by nothing once it has
    arrived)."""
    m = np.asarray(scenario)
    if m.shape != view.observed_matrix.shape or not np.issubdtype(m.dtype, np.number):
        raise ValueError("scenario shape/type mismatch")
    if not np.all(np.isfinite(m)) or np.any(m < 0) or np.any(m != np.floor(m)):
        raise InconsistentResidualError("a scenario holds negative or noninteger demand")
    m = m.astype(np.int64)
    r = _routes(view.topology)
    seen = np.zeros_like(m)
    for t in view.revealed_tokens:
        seen[t.source, t.destination] += 1
    if np.any(m < seen):
        raise InconsistentResidualError("the scenario has fewer units than the revealed tokens on a pair")
    loads = np.zeros(len(r.edges), dtype=np.float64)
    pairs = np.argwhere(m > 0)
    for s, d in pairs.tolist():  # row-major, so the first unreachable pair is reported
        if s == d:
            continue
        if r.dist[s, d] == np.inf:
            raise UnreachableScenarioError("a scenario has positive demand on an unreachable pair")
        loads[list(r.path(s, d))] += float(m[s, d])
    for t in view.revealed_tokens:
        if r.dist[t.source, t.destination] == np.inf:
            raise InconsistentResidualError("a revealed token's pair is unreachable")
        loads[list(r.path(t.source, t.destination))] -= 1.0
        if t.destination not in t.holders:
            best = min(t.holders, key=lambda h: (r.dist[h, t.destination], h))
            loads[list(r.path(best, t.destination))] += 1.0
    if np.any(loads < -1e-12):
        raise InconsistentResidualError("the scenario does not cover the revealed tokens' loads")
    loads = np.maximum(loads, 0.0)
    group = np.asarray([sum(loads[i] for i in members.tolist()) for members, _ in r.groups], dtype=np.float64)
    loads.setflags(write=False)
    group.setflags(write=False)
    return ResidualProjection(loads, group, canonical_digest((loads, group)))


# -------------------------------------------------------------------- scoring
def criticality_for_edge(*, residual_edge_load: float, edge_units: int,
                         incident_group_loads: Sequence[float], incident_group_units: Sequence[int]) -> float:
    """Residual load over capacity units, summed over the edge and its groups."""
    loads = [float(residual_edge_load)] + [float(v) for v in incident_group_loads]
    if not all(math.isfinite(v) and v >= 0 for v in loads):
        raise ValueError("residual loads must be finite and nonnegative")
    edge_part = loads[0] / max(int(edge_units), 1)
    group_part = sum(load / max(int(u), 1) for load, u in zip(loads[1:], incident_group_units))
    return float(edge_part + group_part)


def candidate_utility(*, criticality: float, after_distance: float) -> float:
    c, a = float(criticality), float(after_distance)
    if not (math.isfinite(c) and math.isfinite(a)):
        raise ValueError("utility inputs must be finite")
    return 1.0 + 0.25 * c - 0.05 * a


def robust_score(q: Any, weights: Any, *, risk_lambda: float) -> float:
    """Weighted mean minus lambda times weighted standard deviation of q."""
    qv = np.asarray(q, dtype=np.float64)
    w = np.asarray(weights, dtype=np.float64)
    if qv.ndim != 1 or w.shape != qv.shape or not np.all(np.isfinite(qv)):
        raise ValueError("utilities must be a finite vector")
    if not np.all(np.isfinite(w)) or np.any(w < 0) or w.sum() <= 0:
        raise ValueError("weights must be finite, nonnegative and not all zero")
    p = w / w.sum()
    mean = float(p @ qv)
    spread = float(p @ ((qv - mean) ** 2))
    return mean - float(risk_lambda) * math.sqrt(max(spread, 0.0))


@dataclass(frozen=True, slots=True)
class CandidateScore:
    candidate: CandidateAction
    robust_score: float
    scenario_std: float


def score_candidates(candidates: Sequence[CandidateAction], support: Any, *,
                     risk_lambda: float) -> tuple[CandidateScore, ...]:
    projections = [project_residual_scenario(m, support.observation) for m in support.matrices]
    r = _routes(support.observation.topology)
    p = np.asarray(support.weights, dtype=float)
    p = p / p.sum()
    scored = []
    for c in candidates:
        e = c.edge_index
        groups = r.edge_groups[e]
        q = np.asarray([candidate_utility(
            criticality=criticality_for_edge(
                residual_edge_load=pr.edge_loads[e], edge_units=int(r.edge_units[e]),
                incident_group_loads=[pr.group_loads[g] for g in groups],
                incident_group_units=[int(r.group_units[g]) for g in groups]),
            after_distance=c.after_distance) for pr in projections])
        mean = float(p @ q)
        scored.append(CandidateScore(c, robust_score(q, p, risk_lambda=risk_lambda),
                                     float(np.sqrt(p @ ((q - mean) ** 2)))))
    return tuple(scored)


# -------------------------------------------------------------------- planner
@dataclass(frozen=True, slots=True)
class RobustPrefixConfig:
    horizon: int
    prefix: int
    risk_lambda: float
    requested_k: int

    def __post_init__(self) -> None:
        if (int(self.horizon), int(self.prefix)) not in LEGAL_HORIZON_PREFIX:
            raise ValueError(f"(horizon, prefix) must be one of {sorted(LEGAL_HORIZON_PREFIX)}")
        if float(self.risk_lambda) not in RISK_LAMBDAS:
            raise ValueError(f"risk lambda must be one of {RISK_LAMBDAS}")
        if int(self.requested_k) not in REQUESTED_K:
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
    """Simulate up to ``horizon`` slots of robust-score batches on the public
    view, and keep the first ``prefix`` batches as the plan."""

    def __init__(self, config: RobustPrefixConfig) -> None:
        self.config = config

    def plan(self, observation: SchedulingObservationView, support: Any) -> PrefixPlan:
        if support.stage != observation.stage:
            raise StaleSupportError("the support was built at another reveal stage")
        if support.observation_digest != observation.observation_digest:
            raise StaleSupportError("the support was built for another observation")
        projected = canonical_digest(tuple(project_residual_scenario(m, observation).digest
                                           for m in support.matrices))
        dst_of = np.asarray(observation.topology.edges, dtype=np.int64)[:, 1]
        view, batches = observation, []
        for _ in range(self.config.horizon):
            candidates = enumerate_candidates(view)
            if not candidates:
                break
            scores = score_candidates(candidates, support, risk_lambda=self.config.risk_lambda)
            ranked = sorted(scores, key=lambda s: (-s.robust_score, s.candidate.local_token_ordinal,
                                                   s.candidate.edge_index))
            batch = pack_candidate_batch([s.candidate for s in ranked], view.topology)
            if not batch:
                break
            batches.append(batch)
            grown = {c.local_token_ordinal: {int(dst_of[c.edge_index])} for c in batch}
            tokens = tuple(replace(t, holders=tuple(sorted(set(t.holders) | grown.get(t.local_ordinal, set()))))
                           for t in view.revealed_tokens)
            view = replace(view, revealed_tokens=tokens, residual_state_digest=canonical_digest(_residual_key(tokens)))
        kept = tuple(batches[: self.config.prefix])
        return PrefixPlan(
            origin_stage=observation.stage, origin_state_version=observation.state_version, revision=0,
            support_digest=support.digest, config_digest=canonical_digest(self.config), batches=kept,
            structural_actions=tuple((c.local_token_ordinal, c.edge_index) for b in kept for c in b),
            simulation_trace=tuple(SimulationStep(projected) for _ in kept))


__all__ = [
    "SchedulingObservationView", "PublicRevealedToken", "CandidateAction", "CandidateDistances",
    "CandidateScore", "RobustPrefixConfig", "RobustPrefixPlanner", "PrefixPlan",
    "UnreachableScenarioError", "InconsistentResidualError", "StaleSupportError", "atomic_units",
    "build_scheduling_view", "canonical_digest", "canonical_shortest_path", "enumerate_candidates",
    "pack_candidate_batch", "batch_loads", "project_residual_scenario", "robust_score",
    "criticality_for_edge", "candidate_utility", "score_candidates", "candidate_distances",
    "is_strict_global_progress", "can_add_candidate", "edge_usable", "SCORE_TIE_TOLERANCE",
]
