"""Compiled, incremental, fail-closed scheduler (the fast path).

Interfaces and observable behaviour follow
rlccl/scheduling/compiled_event_driven.py:76-704:

* ``StaticPlanCompiler.compile(topology) -> CompiledPlan`` pays every graph
  search once: atomic capacity units, edge -> group mapping, usable edges,
  per-source BFS (out-edges in (target, edge) order) giving the all-pairs
  distance table and canonical paths, per-destination route templates and a
  ``StaticProof`` (fails closed).  ``compile_bfs_sources`` counts the BFS runs.
* ``IncrementalState`` holds preallocated arrays updated only by deltas;
  ``stage_ready_chunk`` makes a chunk pending (invisible to the binder and
  guard), ``consume_pending_chunk`` activates chunks strictly in ordinal
  order.  ``full_rebuild_count`` must stay 0.
* ``FastBinder.step`` = enumerate (token ordinal, then template order) ->
  greedy select (one hop per token, link and group credits) -> bind to truth
  ids.  ``runtime_bfs_calls`` stays 0: the binder never searches the graph.
* ``DynamicGuard.check/apply`` is the independent fail-closed checker; any
  exception becomes a rejection.

The array work of enumerate/select/check/apply runs in the C++ core
(``revealaiccl_b200._host``, csrc/host/scheduler_core.cpp) when it is built,
operating in place on the same NumPy arrays; the NumPy implementation below
is the reference for it and is used when the extension is absent (CPU CI).
"""

from __future__ import annotations

from dataclasses import dataclass
import hashlib
from typing import Any, Iterable, Sequence

import numpy as np

from ..uncertainty.execution import Proposal, TransferAction
from ..uncertainty.observation import TruthTokenId
from .robust_prefix import CandidateAction, atomic_units

INF = np.iinfo(np.int32).max // 4

# Reason strings of the guard, indexed by the C++ core's reason codes.
GUARD_REASONS = (None, "stale_state_version", "proposal_type", "scenario_only", "unrevealed",
                 "duplicate_in_slot", "edge_range", "source_holder", "duplicate_commit",
                 "residual_demand", "edge_capacity", "bandwidth_group")


def _native_core():
    try:
        from ..ops import _native

        if _native.has_host():
            return _native.host()
    except Exception:  # pragma: no cover - import problems fall back to NumPy
        return None
    return None


@dataclass(frozen=True, slots=True)
class RouteTemplate:
    destination: int
    edge_index: int
    source: int
    target: int
    source_distance: int
    target_distance: int
    group_indices: tuple[int, ...]


@dataclass(frozen=True, slots=True)
class StaticProof:
    topology_path_validity: bool
    endpoint_validity: bool
    resource_group_mapping: bool
    template_static_legality: bool
    canonical_path_cases: int
    template_cases: int
    digest: str

    @property
    def valid(self) -> bool:
        return (self.topology_path_validity and self.endpoint_validity
                and self.resource_group_mapping and self.template_static_legality)


@dataclass(frozen=True, slots=True)
class CompiledPlan:
    nodes: int
    edges: np.ndarray
    edge_sources: np.ndarray
    edge_targets: np.ndarray
    capacity_units: np.ndarray
    group_edges: tuple[tuple[int, ...], ...]
    group_limits: np.ndarray
    edge_to_groups: tuple[tuple[int, ...], ...]
    usable_edges: np.ndarray
    distances: np.ndarray
    canonical_paths: tuple[tuple[tuple[int, ...], ...], ...]
    templates_by_destination: tuple[tuple[RouteTemplate, ...], ...]
    proof: StaticProof
    template_order: str = "token_ordinal_then_edge_index"


_FLAT_CACHE: dict[int, tuple[CompiledPlan, dict]] = {}


def _build_flat(plan: CompiledPlan) -> dict[str, np.ndarray]:
    """Flattened (CSR) int arrays of a plan, the layout the C++ core reads."""
    t_ptr = [0]
    t_edge, t_src, t_tgt, t_td = [], [], [], []
    for group in plan.templates_by_destination:
        for t in group:
            t_edge.append(t.edge_index)
            t_src.append(t.source)
            t_tgt.append(t.target)
            t_td.append(t.target_distance)
        t_ptr.append(len(t_edge))
    g_ptr, g_members = [0], []
    for members in plan.group_edges:
        g_members.extend(members)
        g_ptr.append(len(g_members))
    eg_ptr, eg_members = [0], []
    for groups in plan.edge_to_groups:
        eg_members.extend(groups)
        eg_ptr.append(len(eg_members))

    def i32(v):
        return np.ascontiguousarray(np.asarray(v, dtype=np.int32))

    def i64(v):
        return np.ascontiguousarray(np.asarray(v, dtype=np.int64))

    return {
        "edge_src": i32(plan.edge_sources), "edge_tgt": i32(plan.edge_targets),
        "cap_units": i64(plan.capacity_units), "group_limits": i64(plan.group_limits),
        "group_ptr": i32(g_ptr), "group_members": i32(g_members),
        "edge_group_ptr": i32(eg_ptr), "edge_group_members": i32(eg_members),
        "distances": np.ascontiguousarray(plan.distances, dtype=np.int32),
        "tmpl_ptr": i32(t_ptr), "tmpl_edge": i32(t_edge), "tmpl_src": i32(t_src),
        "tmpl_tgt": i32(t_tgt), "tmpl_tdist": i32(t_td),
    }


def _plan_flat(plan: CompiledPlan) -> dict[str, np.ndarray]:
    hit = _FLAT_CACHE.get(id(plan))
    if hit is not None and hit[0] is plan:
        return hit[1]
    flat = _build_flat(plan)
    _FLAT_CACHE[id(plan)] = (plan, flat)
    return flat


class StaticPlanCompiler:
    """Compile every topology-dependent decision; the runtime never performs BFS."""

    def __init__(self) -> None:
        self.compile_bfs_sources = 0

    def compile(self, topology: Any) -> CompiledPlan:
        nodes = int(getattr(topology, "num_nodes", getattr(topology, "V", 0)))
        edges = np.array(getattr(topology, "edges"), dtype=np.int64, copy=True)
        caps = np.array(getattr(topology, "capacities"), dtype=np.float64, copy=True)
        raw_groups = tuple(getattr(topology, "shared_constraints", ()))
        if nodes <= 0 or edges.ndim != 2 or edges.shape[1] != 2:
            raise ValueError("invalid topology shape")
        if caps.shape != (len(edges),):
            raise ValueError("capacity shape mismatch")
        if np.any(edges < 0) or np.any(edges >= nodes):
            raise ValueError("edge endpoint outside topology")
        E = len(edges)
        cap_units = np.asarray([atomic_units(v) for v in caps], dtype=np.int64)
        group_edges: list[tuple[int, ...]] = []
        group_limits: list[int] = []
        edge_groups: list[list[int]] = [[] for _ in range(E)]
        for g, (members, limit) in enumerate(raw_groups):
            m = tuple(int(e) for e in members)
            if len(set(m)) != len(m):
                raise ValueError("duplicate edge in bandwidth group")
            if any(e < 0 or e >= E for e in m):
                raise ValueError("bandwidth group edge outside topology")
            group_edges.append(m)
            group_limits.append(atomic_units(limit))
            for e in m:
                edge_groups[e].append(g)
        limits = np.asarray(group_limits, dtype=np.int64)
        usable = cap_units >= 1
        for e, gs in enumerate(edge_groups):
            if any(limits[g] < 1 for g in gs):
                usable[e] = False

        out: list[list[int]] = [[] for _ in range(nodes)]
        for e, (s, _t) in enumerate(edges):
            if usable[e]:
                out[int(s)].append(e)
        for row in out:
            row.sort(key=lambda e: (int(edges[e, 1]), e))

        dist = np.full((nodes, nodes), INF, dtype=np.int32)
        paths: list[list[tuple[int, ...]]] = [[() for _ in range(nodes)] for _ in range(nodes)]
        for s in range(nodes):
            self.compile_bfs_sources += 1
            dist[s, s] = 0
            parent: dict[int, tuple[int, int]] = {}
            seen = {s}
            frontier = [s]
            for node in frontier:
                for e in out[node]:
                    t = int(edges[e, 1])
                    if t in seen:
                        continue
                    seen.add(t)
                    parent[t] = (node, e)
                    dist[s, t] = dist[s, node] + 1
                    frontier.append(t)
            for d in range(nodes):
                if d != s and dist[s, d] < INF:
                    rev = []
                    cur = d
                    while cur != s:
                        cur, e = parent[cur]
                        rev.append(e)
                    paths[s][d] = tuple(reversed(rev))

        templates: list[tuple[RouteTemplate, ...]] = []
        for d in range(nodes):
            row = []
            for e, (s, t) in enumerate(edges):
                td = int(dist[int(t), d])
                if not usable[e] or td >= INF:
                    continue
                row.append(RouteTemplate(d, e, int(s), int(t), int(dist[int(s), d]), td,
                                         tuple(edge_groups[e])))
            templates.append(tuple(row))

        canonical = tuple(tuple(r) for r in paths)
        endpoint_ok = all(0 <= t.source < nodes and 0 <= t.target < nodes for g in templates for t in g)
        mapping_ok = all(tuple(i for i, m in enumerate(group_edges) if e in m) == tuple(edge_groups[e])
                         for e in range(E))
        template_ok = all(
            bool(usable[t.edge_index]) and tuple(edge_groups[t.edge_index]) == t.group_indices
            and int(edges[t.edge_index, 0]) == t.source and int(edges[t.edge_index, 1]) == t.target
            and t.target_distance == int(dist[t.target, t.destination])
            for g in templates for t in g)
        path_ok = True
        cases = 0
        for s in range(nodes):
            for d in range(nodes):
                p = canonical[s][d]
                if s == d or dist[s, d] >= INF:
                    path_ok &= p == ()
                    continue
                cases += 1
                cur = s
                for e in p:
                    path_ok &= bool(usable[e]) and int(edges[e, 0]) == cur
                    cur = int(edges[e, 1])
                path_ok &= cur == d and len(p) == int(dist[s, d])
        material = (nodes, tuple(map(tuple, edges.tolist())), tuple(cap_units.tolist()),
                    tuple(group_edges), tuple(group_limits), canonical,
                    tuple(tuple((t.destination, t.edge_index, t.source, t.target, t.source_distance,
                                 t.target_distance, t.group_indices) for t in g) for g in templates))
        proof = StaticProof(bool(path_ok), bool(endpoint_ok), bool(mapping_ok), bool(template_ok),
                            cases, sum(len(g) for g in templates),
                            hashlib.sha256(repr(material).encode()).hexdigest())
        if not proof.valid:
            raise ValueError("static proof failed")
        for a in (edges, cap_units, limits, usable, dist):
            a.setflags(write=False)
        return CompiledPlan(nodes, edges, edges[:, 0], edges[:, 1], cap_units, tuple(group_edges),
                            limits, tuple(tuple(g) for g in edge_groups), usable, dist, canonical,
                            tuple(templates), proof)


@dataclass(frozen=True, slots=True)
class StateDigest:
    state_version: int
    ready_bitmap: int
    pending_ready_bitmap: int
    revealed_count: int
    residual_demand: tuple[tuple[int, ...], ...]
    holders: tuple[tuple[int, ...], ...]
    committed: tuple[tuple[int, ...], ...]
    link_credits: tuple[int, ...]
    group_credits: tuple[int, ...]


class IncrementalState:
    """Preallocated reveal/commit state updated only by deltas."""

    def __init__(self, plan: CompiledPlan, *, max_tokens: int, max_chunks: int = 8,
                 sequence_id: str = "", sequence_step: int = 0) -> None:
        if max_tokens <= 0 or max_chunks <= 0:
            raise ValueError("state capacities must be positive")
        self.plan = plan
        self.max_tokens = int(max_tokens)
        self.max_chunks = int(max_chunks)
        self.sequence_id = str(sequence_id)
        self.sequence_step = int(sequence_step)
        self.stage = 0
        self.ratio = 0.0
        self.state_version = 0
        self.revealed_count = 0
        self.staged_count = 0
        self.ready_bitmap = 0
        self.pending_ready_bitmap = 0
        n, E, G, T = plan.nodes, len(plan.edges), len(plan.group_edges), self.max_tokens
        self.token_ids: list[TruthTokenId | None] = [None] * T
        self.token_ordinals: dict[TruthTokenId, int] = {}
        self.sources = np.full(T, -1, dtype=np.int32)
        self.destinations = np.full(T, -1, dtype=np.int32)
        self.holders = np.zeros((T, n), dtype=bool)
        self.ready = np.zeros(T, dtype=bool)
        self.committed_bitmap = np.zeros((T, E), dtype=bool)
        self.residual_token = np.zeros(T, dtype=bool)
        self.remaining_hops = np.full(T, INF, dtype=np.int32)
        self.residual_demand = np.zeros((n, n), dtype=np.int64)
        self.chunk_starts = np.full(self.max_chunks, -1, dtype=np.int32)
        self.chunk_counts = np.zeros(self.max_chunks, dtype=np.int32)
        self.chunk_consumed = np.zeros(self.max_chunks, dtype=bool)
        self.link_credits = np.array(plan.capacity_units, dtype=np.int64, copy=True)
        self.group_credits = np.array(plan.group_limits, dtype=np.int64, copy=True)
        self._scratch_selected_tokens = np.zeros(T, dtype=bool)
        self._scratch_seen_tokens = np.zeros(T, dtype=bool)
        self._scratch_edge_load = np.zeros(E, dtype=np.int64)
        self.delta_update_count = 0
        self.full_rebuild_count = 0
        del G

    @classmethod
    def from_observation(cls, plan: CompiledPlan, observation: Any, *,
                         max_tokens: int | None = None) -> "IncrementalState":
        cap = max(int(max_tokens or len(observation.revealed_tokens) or 1), len(observation.revealed_tokens))
        st = cls(plan, max_tokens=cap, max_chunks=max(8, int(getattr(observation, "stage", 0)) + 1),
                 sequence_id=str(observation.sequence_id), sequence_step=int(observation.sequence_step))
        st.state_version = int(observation.state_version)
        st._append_ready_tokens(observation.revealed_tokens)
        st.stage = int(observation.stage)
        st.ratio = float(observation.ratio)
        if observation.revealed_tokens:
            st.ready_bitmap |= 1 << min(st.stage, st.max_chunks - 1)
        return st

    def _write_staged_token(self, ordinal: int, token: Any) -> None:
        if ordinal >= self.max_tokens:
            raise ValueError("token capacity exceeded")
        if not isinstance(token.token_id, TruthTokenId):
            raise TypeError("compiled state requires revealed truth token IDs")
        if token.token_id in self.token_ordinals:
            raise ValueError("duplicate revealed token")
        s, d = int(token.source), int(token.destination)
        n = self.plan.nodes
        if not (0 <= s < n and 0 <= d < n) or s == d:
            raise ValueError("invalid token endpoint")
        holders = tuple(int(h) for h in token.holders)
        if not holders or any(h < 0 or h >= n for h in holders):
            raise ValueError("invalid token holder")
        self.token_ids[ordinal] = token.token_id
        self.token_ordinals[token.token_id] = ordinal
        self.sources[ordinal] = s
        self.destinations[ordinal] = d
        self.holders[ordinal, :] = False
        self.holders[ordinal, list(holders)] = True

    def stage_ready_chunk(self, chunk: int, tokens: Sequence[Any]) -> None:
        i = int(chunk)
        if i < 0 or i >= self.max_chunks:
            raise ValueError("chunk outside state capacity")
        bit = 1 << i
        if self.pending_ready_bitmap & bit or self.ready_bitmap & bit:
            raise ValueError("chunk replay")
        vals = tuple(tokens)
        start = self.staged_count
        if start + len(vals) > self.max_tokens:
            raise ValueError("token capacity exceeded")
        for k, tok in enumerate(vals):
            self._write_staged_token(start + k, tok)
        self.chunk_starts[i] = start
        self.chunk_counts[i] = len(vals)
        self.staged_count += len(vals)
        self.pending_ready_bitmap |= bit

    def consume_pending_chunk(self, chunk: int) -> None:
        i = int(chunk)
        bit = 1 << i
        if not self.pending_ready_bitmap & bit:
            raise ValueError("chunk is not pending-ready")
        start, count = int(self.chunk_starts[i]), int(self.chunk_counts[i])
        if start != self.revealed_count:
            raise ValueError("out-of-order ready chunk would reorder token ordinals")
        self._activate_range(start, count)
        self.pending_ready_bitmap &= ~bit
        self.ready_bitmap |= bit
        self.chunk_consumed[i] = True
        self.delta_update_count += 1

    def _activate_range(self, start: int, count: int) -> None:
        dist = self.plan.distances
        for o in range(start, start + count):
            s, d = int(self.sources[o]), int(self.destinations[o])
            self.ready[o] = True
            residual = not bool(self.holders[o, d])
            self.residual_token[o] = residual
            if residual:
                self.residual_demand[s, d] += 1
            hs = np.flatnonzero(self.holders[o])
            self.remaining_hops[o] = int(dist[hs, d].min()) if len(hs) else INF
        self.revealed_count += count

    def _append_ready_tokens(self, tokens: Iterable[Any]) -> None:
        vals = tuple(tokens)
        start = self.staged_count
        for k, tok in enumerate(vals):
            self._write_staged_token(start + k, tok)
        self.staged_count += len(vals)
        self._activate_range(start, len(vals))
        if vals:
            self.delta_update_count += 1

    def ingest_observation_delta(self, observation: Any, *, chunk: int | None = None) -> None:
        if self.sequence_id and str(observation.sequence_id) != self.sequence_id:
            raise ValueError("observation sequence mismatch")
        if int(observation.sequence_step) != self.sequence_step:
            raise ValueError("observation step mismatch")
        if int(observation.state_version) != self.state_version:
            raise ValueError("stale observation")
        toks = tuple(observation.revealed_tokens)
        if len(toks) < self.revealed_count:
            raise ValueError("revealed prefix shrank")
        for o in range(self.revealed_count):
            if toks[o].token_id != self.token_ids[o]:
                raise ValueError("revealed token order changed")
            seen = np.zeros(self.plan.nodes, dtype=bool)
            seen[list(toks[o].holders)] = True
            if not np.array_equal(seen, self.holders[o]):
                raise ValueError("holder state divergence")
        suffix = toks[self.revealed_count:]
        if suffix:
            i = int(observation.stage if chunk is None else chunk)
            i = min(i, self.max_chunks - 1)
            self.stage_ready_chunk(i, suffix)
            self.consume_pending_chunk(i)
        self.stage = int(observation.stage)
        self.ratio = float(observation.ratio)

    def reset_slot_credits(self) -> None:
        np.copyto(self.link_credits, self.plan.capacity_units)
        np.copyto(self.group_credits, self.plan.group_limits)
        self._scratch_selected_tokens.fill(False)

    def digest(self) -> StateDigest:
        rc = self.revealed_count
        return StateDigest(
            self.state_version, self.ready_bitmap, self.pending_ready_bitmap, rc,
            tuple(tuple(int(v) for v in r) for r in self.residual_demand),
            tuple(tuple(int(v) for v in np.flatnonzero(self.holders[i])) for i in range(rc)),
            tuple(tuple(int(v) for v in np.flatnonzero(self.committed_bitmap[i])) for i in range(rc)),
            tuple(int(v) for v in self.link_credits), tuple(int(v) for v in self.group_credits))

    def native_arrays(self) -> dict[str, np.ndarray]:
        """The state arrays the C++ core reads and updates in place."""
        return {
            "sources": self.sources, "destinations": self.destinations,
            "holders": self.holders.view(np.uint8), "ready": self.ready.view(np.uint8),
            "committed": self.committed_bitmap.view(np.uint8),
            "residual": self.residual_token.view(np.uint8), "remaining_hops": self.remaining_hops,
            "residual_demand": self.residual_demand, "link_credits": self.link_credits,
            "group_credits": self.group_credits,
            "scratch_selected": self._scratch_selected_tokens.view(np.uint8),
            "scratch_seen": self._scratch_seen_tokens.view(np.uint8),
            "scratch_edge_load": self._scratch_edge_load,
        }


@dataclass(frozen=True, slots=True)
class BoundBatch:
    state_version: int
    candidates: tuple[CandidateAction, ...]
    selected: tuple[CandidateAction, ...]
    proposal: Proposal


class FastBinder:
    """Template lookup, dynamic filter, deterministic selection and binding."""

    def __init__(self, plan: CompiledPlan, *, backend: str = "auto") -> None:
        if not plan.proof.valid:
            raise ValueError("compiled plan has no valid static proof")
        self.plan = plan
        self.runtime_bfs_calls = 0
        self._core = _native_core() if backend in ("auto", "native") else None
        if backend == "native" and self._core is None:
            raise RuntimeError("native scheduler core requested but revealaiccl_b200._host is not built")

    @property
    def backend(self) -> str:
        return "native" if self._core is not None else "numpy"

    def enumerate_candidates(self, state: IncrementalState) -> tuple[CandidateAction, ...]:
        if state.ratio == 0.0 or state.revealed_count == 0:
            return ()
        if self._core is not None:
            rows = self._core.sched_enumerate(_plan_flat(self.plan), state.native_arrays(),
                                              int(state.revealed_count), int(self.plan.nodes))
            return tuple(CandidateAction(int(o), int(e), int(b), int(a)) for o, e, b, a in rows)
        out: list[CandidateAction] = []
        for o in range(state.revealed_count):
            if not state.ready[o] or not state.residual_token[o]:
                continue
            d = int(state.destinations[o])
            before = int(state.remaining_hops[o])
            if before <= 0 or before >= INF:
                continue
            for t in self.plan.templates_by_destination[d]:
                if (state.holders[o, t.source] and not state.holders[o, t.target]
                        and t.target_distance == before - 1):
                    out.append(CandidateAction(o, t.edge_index, before, before - 1))
        return tuple(out)

    def select_batch(self, state: IncrementalState,
                     candidates: Sequence[CandidateAction]) -> tuple[CandidateAction, ...]:
        if self._core is not None:
            flat = np.asarray([(c.local_token_ordinal, c.edge_index) for c in candidates],
                              dtype=np.int32).reshape(-1, 2)
            keep = self._core.sched_select(_plan_flat(self.plan), state.native_arrays(), flat,
                                           int(state.revealed_count))
            return tuple(candidates[i] for i in keep)
        state.reset_slot_credits()
        chosen: list[CandidateAction] = []
        for c in candidates:
            o, e = int(c.local_token_ordinal), int(c.edge_index)
            if o < 0 or o >= state.revealed_count or state._scratch_selected_tokens[o]:
                continue
            if state.link_credits[e] < 1:
                continue
            groups = self.plan.edge_to_groups[e]
            if any(state.group_credits[g] < 1 for g in groups):
                continue
            state._scratch_selected_tokens[o] = True
            state.link_credits[e] -= 1
            for g in groups:
                state.group_credits[g] -= 1
            chosen.append(c)
        return tuple(chosen)

    def bind(self, state: IncrementalState, selected: Sequence[CandidateAction]) -> Proposal:
        actions = []
        for c in selected:
            o = int(c.local_token_ordinal)
            if o < 0 or o >= state.revealed_count or not state.ready[o]:
                raise ValueError("candidate token is hidden or not ready")
            tid = state.token_ids[o]
            if not isinstance(tid, TruthTokenId):
                raise ValueError("candidate has no executable truth token")
            actions.append(TransferAction(tid, int(c.edge_index)))
        return Proposal.from_transfers(tuple(actions))

    def step(self, state: IncrementalState) -> BoundBatch:
        cands = self.enumerate_candidates(state)
        sel = self.select_batch(state, cands)
        return BoundBatch(state.state_version, cands, sel, self.bind(state, sel))


@dataclass(frozen=True, slots=True)
class GuardDecision:
    accepted: bool
    reason: str | None
    applied_actions: int
    state_version: int


class DynamicGuard:
    """Independent fail-closed checker equivalent to the trusted commit checker."""

    def __init__(self, plan: CompiledPlan, *, backend: str = "auto") -> None:
        self.plan = plan
        self._core = _native_core() if backend in ("auto", "native") else None
        if backend == "native" and self._core is None:
            raise RuntimeError("native scheduler core requested but revealaiccl_b200._host is not built")

    def _resolve(self, state: IncrementalState, proposal: Proposal) -> np.ndarray:
        rows = []
        for a in proposal.actions:
            o = state.token_ordinals.get(a.token_id)
            rows.append((-1 if o is None else int(o), int(a.edge_index)))
        return np.asarray(rows, dtype=np.int64).reshape(-1, 2)

    def _first_refusal(self, state: IncrementalState, proposal: Proposal, semantics: bool) -> str | None:
        """NumPy form of the guard: every action's checks are evaluated as
        columns of one table, and the verdict is the first failing check of
        the first failing action (the order the trusted checker uses), then
        the slot's edge and group budgets."""
        plan = self.plan
        E = len(plan.edges)
        n = len(proposal.actions)
        ords = np.fromiter((state.token_ordinals.get(a.token_id, -1) for a in proposal.actions), np.int64, n)
        edges = np.fromiter((int(a.edge_index) for a in proposal.actions), np.int64, n)
        o = np.clip(ords, 0, max(state.revealed_count - 1, 0))
        revealed = (ords >= 0) & (ords < state.revealed_count)
        revealed &= np.asarray(state.ready, dtype=bool)[o] if state.revealed_count else False
        # an ordinal that an earlier action of the slot already named
        _, first = np.unique(ords, return_index=True)
        earlier = np.ones(n, dtype=bool)
        earlier[first] = False
        in_range = (edges >= 0) & (edges < E)
        e = np.where(in_range, edges, 0)
        src, tgt = np.asarray(plan.edge_sources)[e], np.asarray(plan.edge_targets)[e]
        held = np.asarray(state.holders, dtype=bool)
        columns = [
            ("unrevealed", ~revealed),
            ("duplicate_in_slot", earlier),
            ("edge_range", ~in_range),
            ("source_holder", ~held[o, src]),
            ("duplicate_commit", held[o, tgt] | np.asarray(state.committed_bitmap, dtype=bool)[o, e]),
        ]
        if semantics:
            hops = np.asarray(state.remaining_hops, dtype=np.int64)[o]
            to_dst = np.asarray(plan.distances)[tgt, np.asarray(state.destinations, dtype=np.int64)[o]]
            columns.append(("residual_demand", ~np.asarray(state.residual_token, dtype=bool)[o] | (hops <= 0)
                            | (to_dst != hops - 1)))
        fails = np.stack([bad for _, bad in columns], axis=1)
        if fails.any():
            i = int(np.flatnonzero(fails.any(axis=1))[0])
            return columns[int(np.flatnonzero(fails[i])[0])][0]
        load = np.bincount(edges, minlength=E)
        if np.any(load > np.asarray(plan.capacity_units)):
            return "edge_capacity"
        for g, members in enumerate(plan.group_edges):
            if int(load[np.asarray(members, dtype=np.int64)].sum()) > int(plan.group_limits[g]):
                return "bandwidth_group"
        return None

    def check(self, state: IncrementalState, proposal: Proposal, *,
              require_scheduler_semantics: bool = False,
              expected_state_version: int | None = None) -> GuardDecision:
        try:
            if expected_state_version is not None and int(expected_state_version) != state.state_version:
                raise ValueError("stale_state_version")
            if not isinstance(proposal, Proposal):
                raise TypeError("proposal_type")
            if proposal.scenario_set is not None:
                raise ValueError("scenario_only")
            if proposal.is_wait:
                return GuardDecision(True, None, 0, state.state_version)
            if self._core is not None:
                code = self._core.sched_check(_plan_flat(self.plan), state.native_arrays(),
                                              self._resolve(state, proposal), int(state.revealed_count),
                                              bool(require_scheduler_semantics))
                if code != 0:
                    raise ValueError(GUARD_REASONS[code])
                return GuardDecision(True, None, len(proposal.actions), state.state_version + 1)
            reason = self._first_refusal(state, proposal, bool(require_scheduler_semantics))
            if reason is not None:
                raise ValueError(reason)
            return GuardDecision(True, None, len(proposal.actions), state.state_version + 1)
        except Exception as error:  # fail closed
            return GuardDecision(False, str(error), 0, state.state_version)

    def apply(self, state: IncrementalState, proposal: Proposal, *,
              require_scheduler_semantics: bool = False,
              expected_state_version: int | None = None) -> GuardDecision:
        decision = self.check(state, proposal, require_scheduler_semantics=require_scheduler_semantics,
                              expected_state_version=expected_state_version)
        if not decision.accepted or proposal.is_wait:
            return decision
        if self._core is not None:
            self._core.sched_apply(_plan_flat(self.plan), state.native_arrays(),
                                   self._resolve(state, proposal), int(self.plan.nodes))
        else:
            state.reset_slot_credits()
            dist = self.plan.distances
            for a in proposal.actions:
                o = state.token_ordinals[a.token_id]
                e = int(a.edge_index)
                t = int(self.plan.edge_targets[e])
                state.holders[o, t] = True
                state.committed_bitmap[o, e] = True
                state.link_credits[e] -= 1
                for g in self.plan.edge_to_groups[e]:
                    state.group_credits[g] -= 1
                d = int(state.destinations[o])
                if t == d and state.residual_token[o]:
                    state.residual_demand[int(state.sources[o]), d] -= 1
                    state.residual_token[o] = False
                hs = np.flatnonzero(state.holders[o])
                state.remaining_hops[o] = int(dist[hs, d].min()) if len(hs) else INF
        state.state_version = decision.state_version
        state.delta_update_count += 1
        return decision


@dataclass(frozen=True, slots=True)
class RuntimeStep:
    bound: BoundBatch
    decision: GuardDecision


class CompiledEventDrivenRuntime:
    """Single-process adapter from ready chunks to a compiled commit.

    Called only for a chunk whose ready flag was published (by the native
    event bridge or the router kernel's completion flag); it performs no
    polling, IPC, serialisation, graph search or observation rebuild."""

    def __init__(self, plan: CompiledPlan, state: IncrementalState, *, backend: str = "auto") -> None:
        if state.plan is not plan:
            raise ValueError("runtime state/plan identity mismatch")
        self.plan = plan
        self.state = state
        self.binder = FastBinder(plan, backend=backend)
        self.guard = DynamicGuard(plan, backend=backend)

    def stage_router_chunk(self, chunk: int, revealed_tokens: Sequence[Any]) -> None:
        self.state.stage_ready_chunk(chunk, revealed_tokens)

    def consume_event_ready(self, chunk: int, *, stage: int, ratio: float) -> None:
        self.state.consume_pending_chunk(chunk)
        self.state.stage = int(stage)
        self.state.ratio = float(ratio)

    def schedule_and_commit(self) -> RuntimeStep:
        bound = self.binder.step(self.state)
        decision = self.guard.apply(self.state, bound.proposal, require_scheduler_semantics=True,
                                    expected_state_version=bound.state_version)
        return RuntimeStep(bound, decision)


def structural_signature(candidates: Sequence[CandidateAction]) -> tuple[tuple[int, int, int, int], ...]:
    return tuple((int(c.local_token_ordinal), int(c.edge_index), int(c.before_distance),
                  int(c.after_distance)) for c in candidates)


__all__ = ["BoundBatch", "CompiledEventDrivenRuntime", "CompiledPlan", "DynamicGuard", "FastBinder",
           "GuardDecision", "INF", "IncrementalState", "RouteTemplate", "RuntimeStep", "StateDigest",
           "StaticPlanCompiler", "StaticProof", "structural_signature"]
