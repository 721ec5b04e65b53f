"""Finite empirical traffic ambiguity sets built from history only.

Behaviour of rlccl/uncertainty/ambiguity.py:

* descriptors of a traffic matrix: total, per-source and per-destination
  load, destination hotspot strength, off-diagonal sparsity and the offered
  load of every shared bandwidth group along the deterministic shortest path
  (BFS, neighbours in (target, edge) order);
* ``AmbiguityConstructionView``: the only input of an ordinary construction —
  the 32 strictly past matrices, the current partial observation (exact
  entries, partial-shard lower bounds, optional source / destination totals),
  the public topology, a seed and a descriptor normaliser fitted on history;
* reconciliation of a history matrix with the observation: clipping into the
  feasible box, a source-total completion (largest-remainder quotas towards the
  candidate), or an integer min-cost transport completion over unit arcs whose
  cost is one plus the change of |value - candidate| (successive shortest
  paths; equal-cost paths are compared as tuples of arc indices, so the
  completion is reproducible);
* the empirical set: reconciled support, descriptor box widened by a
  calibration radius and clipped to physical bounds, mean / variance moment
  bands, uniform witness; at ratio 1 the singleton observed matrix;
* support selection (random, worst recent cases by standardised severity,
  boundary scenarios, greedy k-centre "minimax" subset; ties to the most recent
  history offset), covering radius, truth-aware upper bound and truth distance.
"""

from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass, fields
from typing import Any, Sequence

import numpy as np

from .observation import PublicTopologyView, readonly_array

HISTORY_WINDOW = 32
MAX_ENTRY = 8


# ---------------------------------------------------------------------------
# canonical digests and validation
# ---------------------------------------------------------------------------
def _canon(v: Any) -> Any:
    if isinstance(v, np.ndarray):
        return {"dtype": v.dtype.str, "shape": list(v.shape), "bytes": np.ascontiguousarray(v).tobytes().hex()}
    if isinstance(v, dict):
        return {str(k): _canon(v[k]) for k in sorted(v)}
    if isinstance(v, (tuple, list)):
        return [_canon(x) for x in v]
    if hasattr(v, "__dataclass_fields__"):
        return {f.name: _canon(getattr(v, f.name)) for f in fields(v)}
    if isinstance(v, np.generic):
        return v.item()
    return v


def _canonical_bytes(v: Any) -> bytes:
    return json.dumps(_canon(v), sort_keys=True, separators=(",", ":"), allow_nan=False).encode("utf-8")


def _digest(v: Any) -> str:
    return hashlib.sha256(_canonical_bytes(v)).hexdigest()


def _nodes(topo: Any) -> int:
    return int(getattr(topo, "num_nodes", getattr(topo, "V", 0)))


def _groups(topo: Any) -> tuple[tuple[tuple[int, ...], float], ...]:
    return tuple((tuple(int(i) for i in idx), float(lim)) for idx, lim in topo.shared_constraints)


def _finite(v: Any, name: str, ndim: int | None = None) -> np.ndarray:
    a = np.asarray(v)
    if ndim is not None and a.ndim != ndim:
        raise ValueError(f"{name} dimensionality mismatch")
    if not np.isfinite(a).all():
        raise ValueError(f"{name} must be finite")
    return a


def _matrix(v: Any, size: int | None = None, max_entry: int = MAX_ENTRY) -> np.ndarray:
    raw = _finite(v, "traffic matrix", 2)
    if raw.shape[0] != raw.shape[1]:
        raise ValueError("traffic matrix must be square")
    if size is not None and raw.shape != (size, size):
        raise ValueError("traffic matrix shape mismatch")
    if not np.equal(raw, np.floor(raw)).all():
        raise ValueError("traffic matrix must contain integers")
    m = raw.astype(np.int64)
    if m.min() < 0 or m.max() > max_entry:
        raise ValueError(f"traffic matrix entries must be within [0,{max_entry}]")
    if np.any(np.diag(m) != 0):
        raise ValueError("traffic matrix diagonal must be zero")
    return m


def _public(topo: Any) -> PublicTopologyView:
    if isinstance(topo, PublicTopologyView):
        return PublicTopologyView(num_nodes=int(topo.num_nodes), num_edges=int(topo.num_edges),
                                  edges=np.asarray(topo.edges), capacities=np.asarray(topo.capacities),
                                  shared_constraints=topo.shared_constraints, name=topo.name)
    return PublicTopologyView.from_topology_info(topo)


# ---------------------------------------------------------------------------
# descriptors
# ---------------------------------------------------------------------------
def _bfs_path(topo: Any, src: int, dst: int) -> tuple[int, ...]:
    """Shortest-hop edge path; neighbours scanned in (target node, edge index) order."""
    edges = np.asarray(topo.edges, dtype=np.int64)
    out: dict[int, list[tuple[int, int]]] = {}
    for e, (a, b) in enumerate(edges):
        out.setdefault(int(a), []).append((int(b), e))
    parent: dict[int, tuple[int, int] | None] = {int(src): None}
    frontier = [int(src)]
    while frontier:
        nxt = []
        for u in frontier:
            if u == dst:
                path = []
                while parent[u] is not None:
                    u, e = parent[u]
                    path.append(e)
                return tuple(reversed(path))
            for v, e in sorted(out.get(u, ())):
                if v not in parent:
                    parent[v] = (u, e)
                    nxt.append(v)
        frontier = nxt
    raise ValueError(f"topology has no directed path {src}->{dst}")


def _group_coefficients(topo: Any) -> np.ndarray:
    n, groups = _nodes(topo), _groups(topo)
    coeff = np.zeros((len(groups), n, n), dtype=np.float64)
    members = [set(idx) for idx, _ in groups]
    if not members:
        return coeff
    for s in range(n):
        for d in range(n):
            if s != d:
                path = _bfs_path(topo, s, d)
                for g, m in enumerate(members):
                    coeff[g, s, d] = float(sum(e in m for e in path))
    return coeff


def group_coefficients_digest(topology: Any) -> str:
    return _digest(_group_coefficients(topology))


def descriptor_names(topology: Any) -> tuple[str, ...]:
    n = _nodes(topology)
    if n < 2:
        raise ValueError("topology must have at least two nodes")
    return ("total_traffic", *(f"source_load_{i}" for i in range(n)), *(f"destination_load_{i}" for i in range(n)),
            "hotspot_strength", "sparsity", *(f"bandwidth_group_load_{g}" for g in range(len(_groups(topology)))))


def traffic_descriptor(matrix: Any, topology: Any) -> np.ndarray:
    n = _nodes(topology)
    m = _matrix(matrix, n)
    out_l, in_l = m.sum(axis=1, dtype=np.float64), m.sum(axis=0, dtype=np.float64)
    mean_in = float(in_l.mean())
    hot = 0.0 if mean_in == 0.0 else float(in_l.max() / mean_in)
    sparsity = float(np.mean(m[~np.eye(n, dtype=bool)] == 0))
    groups = np.einsum("gij,ij->g", _group_coefficients(topology), m, optimize=True)
    return np.asarray([float(out_l.sum()), *out_l, *in_l, hot, sparsity, *groups], dtype=np.float64)


@dataclass(frozen=True, slots=True)
class DescriptorNormalizer:
    center: np.ndarray
    scale: np.ndarray

    def __post_init__(self) -> None:
        c, s = readonly_array(self.center, dtype=np.float64), readonly_array(self.scale, dtype=np.float64)
        if c.ndim != 1 or s.shape != c.shape:
            raise ValueError("normalizer center/scale shape mismatch")
        if not (np.isfinite(c).all() and np.isfinite(s).all()):
            raise ValueError("normalizer must be finite")
        if np.any(s <= 0.0):
            raise ValueError("normalizer scale must be positive")
        object.__setattr__(self, "center", c)
        object.__setattr__(self, "scale", s)

    @property
    def digest(self) -> str:
        return _digest((self.center, self.scale))


def fit_descriptor_normalizer(history_matrices: Sequence[Any], topology: Any) -> DescriptorNormalizer:
    mats = tuple(history_matrices)
    if not mats:
        raise ValueError("fit history cannot be empty")
    v = np.stack([traffic_descriptor(m, topology) for m in mats])
    scale = v.std(axis=0, ddof=0)
    scale[scale < 1e-8] = 1.0
    return DescriptorNormalizer(center=v.mean(axis=0), scale=scale)


def physical_descriptor_bounds(topology: Any, *, max_entry: int = MAX_ENTRY) -> tuple[np.ndarray, np.ndarray]:
    if int(max_entry) <= 0:
        raise ValueError("max_entry must be positive")
    n = _nodes(topology)
    coeff = _group_coefficients(topology)
    row = (n - 1) * max_entry
    high = np.asarray([n * row, *([row] * n), *([row] * n), float(n), 1.0, *(coeff.sum(axis=(1, 2)) * max_entry)],
                      dtype=np.float64)
    return readonly_array(np.zeros_like(high), dtype=np.float64), readonly_array(high, dtype=np.float64)


# ---------------------------------------------------------------------------
# construction view
# ---------------------------------------------------------------------------
def _totals(v: Any | None, size: int, label: str) -> np.ndarray | None:
    if v is None:
        return None
    raw = _finite(v, f"{label} totals", 1)
    if raw.shape != (size,) or not np.equal(raw, np.floor(raw)).all():
        raise ValueError(f"{label} totals shape/integer mismatch")
    t = raw.astype(np.int64)
    if np.any(t < 0):
        raise ValueError(f"{label} totals have negative margin")
    return readonly_array(t, dtype=np.int64)


def _bounds(observed: np.ndarray, mask: np.ndarray, mode: str, src_tot, dst_tot) -> tuple[np.ndarray, np.ndarray]:
    """Per-entry lower bound and free capacity above it: exact entries are fixed,
    partial-shard entries start at the observed count, the rest are free."""
    n = observed.shape[0]
    off = ~np.eye(n, dtype=bool)
    if np.any(np.diag(observed) != 0):
        raise ValueError("diagonal observation must be zero")
    exact = mask & off
    lower = np.where(exact | ((mode == "partial_shards") & off), observed, 0).astype(np.int64)
    cap = np.where(exact | ~off, 0, MAX_ENTRY - lower).astype(np.int64)
    if lower.min() < 0 or lower.max() > MAX_ENTRY or cap.min() < 0:
        raise ValueError("observation lower bound exceeds entry cap 8")
    for tot, axis, label in ((src_tot, 1, "source"), (dst_tot, 0, "destination")):
        if tot is not None:
            res = tot - lower.sum(axis=axis)
            if np.any(res < 0) or np.any(res > cap.sum(axis=axis)):
                raise ValueError(f"{label} residual margin is infeasible for capacity")
    if src_tot is not None and dst_tot is not None and int(src_tot.sum()) != int(dst_tot.sum()):
        raise ValueError("source/destination residual margins violate conservation")
    return lower, cap


@dataclass(frozen=True, slots=True)
class AmbiguityConstructionView:
    history_matrices: tuple[np.ndarray, ...]
    history_offsets: tuple[int, ...]
    observed_matrix: np.ndarray
    entry_mask: np.ndarray
    mode: str
    stage: int
    ratio: float
    source_totals: np.ndarray | None
    destination_totals: np.ndarray | None
    topology: PublicTopologyView
    construction_seed: int
    normalizer: DescriptorNormalizer
    history_cutoff: int

    def __post_init__(self) -> None:
        mats = tuple(self.history_matrices)
        if len(mats) != HISTORY_WINDOW:
            raise ValueError("history must contain exactly 32 matrices")
        offs = tuple(int(x) for x in self.history_offsets)
        if offs != tuple(range(-HISTORY_WINDOW, 0)):
            raise ValueError("history offsets must be strictly increasing -32..-1")
        topo = _public(self.topology)
        n = int(topo.num_nodes)
        observed = readonly_array(_matrix(self.observed_matrix, n), dtype=np.int64)
        mask = readonly_array(self.entry_mask, dtype=bool)
        if mask.shape != (n, n):
            raise ValueError("entry mask shape mismatch")
        if not np.all(np.diag(mask)):
            raise ValueError("diagonal entries must be exact")
        src, dst = _totals(self.source_totals, n, "source"), _totals(self.destination_totals, n, "destination")
        ratio = float(self.ratio)
        if not math.isfinite(ratio) or not 0.0 <= ratio <= 1.0:
            raise ValueError("ratio must be finite and in [0,1]")
        if not isinstance(self.normalizer, DescriptorNormalizer):
            raise TypeError("normalizer must be a DescriptorNormalizer")
        if self.normalizer.center.shape != (len(descriptor_names(topo)),):
            raise ValueError("normalizer descriptor dimension mismatch")
        _bounds(observed, mask, str(self.mode), src, dst)
        if int(self.history_cutoff) < HISTORY_WINDOW:
            raise ValueError("history cutoff must admit the complete 32-step window")
        for k, v in (("history_matrices", tuple(readonly_array(_matrix(m, n), dtype=np.int64) for m in mats)),
                     ("history_offsets", offs), ("observed_matrix", observed), ("entry_mask", mask),
                     ("mode", str(self.mode)), ("stage", int(self.stage)), ("ratio", ratio), ("source_totals", src),
                     ("destination_totals", dst), ("topology", topo), ("construction_seed", int(self.construction_seed)),
                     ("history_cutoff", int(self.history_cutoff)),
                     ("normalizer", DescriptorNormalizer(self.normalizer.center, self.normalizer.scale))):
            object.__setattr__(self, k, v)

    @classmethod
    def from_observation(cls, *, history_matrices: Sequence[Any], history_offsets: Sequence[int], observation: Any,
                         construction_seed: int, normalizer: DescriptorNormalizer) -> "AmbiguityConstructionView":
        opt = lambda v: None if v is None else np.asarray(v)  # noqa: E731
        return cls(history_matrices=tuple(history_matrices), history_offsets=tuple(history_offsets),
                   observed_matrix=np.asarray(observation.observed_matrix),
                   entry_mask=np.asarray(observation.entry_mask), mode=str(observation.mode),
                   stage=int(observation.stage), ratio=float(observation.ratio),
                   source_totals=opt(observation.source_totals), destination_totals=opt(observation.destination_totals),
                   topology=_public(observation.topology), construction_seed=int(construction_seed),
                   normalizer=normalizer, history_cutoff=int(observation.sequence_step))


# ---------------------------------------------------------------------------
# reconciliation
# ---------------------------------------------------------------------------
def _complete_rows(cand: np.ndarray, lower: np.ndarray, cap: np.ndarray, src_tot: np.ndarray) -> np.ndarray:
    """Fill each row up to its source total: floor of quotas proportional to the
    unmet candidate preference (or to the free capacity without any), then one
    unit each by descending quota remainder, preference, lower destination."""
    res = lower.copy()
    n = res.shape[0]
    for s in range(n):
        need = int(src_tot[s] - res[s].sum())
        while need > 0:
            free = {d: int(cap[s, d] - (res[s, d] - lower[s, d])) for d in range(n) if d != s}
            active = [d for d in free if free[d] > 0]
            if not active:
                raise ValueError("source residual margin is infeasible")
            pref = {d: max(int(cand[s, d] - res[s, d]), 0) for d in active}
            w = pref if sum(pref.values()) else {d: free[d] for d in active}
            tot_w = float(sum(w.values()))
            quota = {d: need * w[d] / tot_w for d in active}
            got = 0
            for d in active:
                a = min(free[d], int(math.floor(quota[d])), need - got)
                if a > 0:
                    res[s, d] += a
                    got += a
                if got == need:
                    break
            need -= got
            if need == 0:
                continue
            extra = 0
            for d in sorted(active, key=lambda d: (-(quota[d] - math.floor(quota[d])), -pref[d], d)):
                if need > 0 and res[s, d] - lower[s, d] < cap[s, d]:
                    res[s, d] += 1
                    need -= 1
                    extra += 1
            if got == 0 and extra == 0:
                raise ValueError("source completion made no progress")
    if not np.array_equal(res.sum(axis=1), src_tot):
        raise ValueError("source completion margin mismatch")
    return res


def _transport(cand: np.ndarray, lower: np.ndarray, cap: np.ndarray, src_tot: np.ndarray,
               dst_tot: np.ndarray) -> np.ndarray:
    """Integer min-cost completion with both margins.

    Network: super source -> row s (row residual), one unit arc per free unit
    of (s, d) with cost 1 + |v - c| - |v - 1 - c| for the unit that raises the
    entry to v (c = candidate), column d -> sink (column residual).  Arcs are
    numbered source arcs, then unit arcs row-major by unit, then sink arcs,
    each followed by its residual twin.  One unit per successive shortest path
    (Bellman-Ford rounds over the arc list; a path of equal cost replaces
    another when its tuple of arc indices is smaller).
    """
    n = lower.shape[0]
    rres = (src_tot - lower.sum(axis=1)).astype(np.int64)
    cres = (dst_tot - lower.sum(axis=0)).astype(np.int64)
    if rres.min() < 0 or cres.min() < 0:
        raise ValueError("negative residual margin is infeasible")
    if int(rres.sum()) != int(cres.sum()):
        raise ValueError("residual margins violate conservation")
    SRC, ROW, COL, SNK = 0, 1, 1 + n, 1 + 2 * n
    tail: list[int] = []
    head: list[int] = []
    capa: list[int] = []
    cost: list[int] = []

    def arc(u: int, v: int, c: int, w: int) -> int:
        i = len(tail)
        tail.extend((u, v))
        head.extend((v, u))
        capa.extend((int(c), 0))
        cost.extend((int(w), -int(w)))
        return i

    for s in range(n):
        arc(SRC, ROW + s, rres[s], 0)
    units: dict[tuple[int, int], list[int]] = {}
    for s in range(n):
        for d in range(n):
            if s == d:
                continue
            c = int(cand[s, d])
            ids = []
            for u in range(1, int(cap[s, d]) + 1):
                v = int(lower[s, d]) + u
                ids.append(arc(ROW + s, COL + d, 1, 1 + abs(v - c) - abs(v - 1 - c)))
            units[(s, d)] = ids
    for d in range(n):
        arc(COL + d, SNK, cres[d], 0)
    nodes = SNK + 1
    for _ in range(int(rres.sum())):
        dist: list[float] = [math.inf] * nodes
        path: list[tuple[int, ...] | None] = [None] * nodes
        dist[SRC], path[SRC] = 0, ()
        for _r in range(nodes - 1):
            changed = False
            for i in range(len(tail)):
                u = tail[i]
                if capa[i] <= 0 or path[u] is None:
                    continue
                v, nd = head[i], dist[u] + cost[i]
                if nd < dist[v] or (nd == dist[v] and (path[v] is None or path[u] + (i,) < path[v])):
                    dist[v], path[v] = nd, path[u] + (i,)
                    changed = True
            if not changed:
                break
        if path[SNK] is None:
            raise ValueError("integer min-cost flow has infeasible residual margins")
        for i in path[SNK]:
            capa[i] -= 1
            capa[i ^ 1] += 1  # the residual twin is the next index
    res = lower.copy()
    for (s, d), ids in units.items():
        res[s, d] += sum(capa[i] == 0 for i in ids)
    if not (np.array_equal(res.sum(axis=1), src_tot) and np.array_equal(res.sum(axis=0), dst_tot)):
        raise ValueError("min-cost-flow margin mismatch")
    return res


def _check_reconciled(m: np.ndarray, view: AmbiguityConstructionView) -> None:
    r = _matrix(m, view.observed_matrix.shape[0])
    exact = np.asarray(view.entry_mask, dtype=bool)
    obs = np.asarray(view.observed_matrix)
    if not np.array_equal(r[exact], obs[exact]):
        raise ValueError("reconciled matrix violates exact observation")
    if view.mode == "partial_shards" and np.any(r[~exact] < obs[~exact]):
        raise ValueError("reconciled matrix violates partial-shard lower bound")
    if view.source_totals is not None and not np.array_equal(r.sum(axis=1), view.source_totals):
        raise ValueError("reconciled matrix violates source totals")
    if view.destination_totals is not None and not np.array_equal(r.sum(axis=0), view.destination_totals):
        raise ValueError("reconciled matrix violates destination totals")


def reconcile_candidate(candidate: Any, view: AmbiguityConstructionView) -> np.ndarray:
    """The history matrix made consistent with the current observation."""
    if not isinstance(view, AmbiguityConstructionView):
        raise TypeError("reconciliation requires AmbiguityConstructionView")
    n = view.observed_matrix.shape[0]
    cand = _matrix(candidate, n)
    lower, cap = _bounds(np.asarray(view.observed_matrix), np.asarray(view.entry_mask), view.mode,
                         view.source_totals, view.destination_totals)
    if view.source_totals is None and view.destination_totals is not None:
        raise ValueError("destination totals without source totals are unsupported/infeasible")
    if view.source_totals is None:
        res = np.where(cap > 0, np.minimum(MAX_ENTRY, np.maximum(cand, lower)), lower).astype(np.int64)
    elif view.destination_totals is None:
        res = _complete_rows(cand, lower, cap, np.asarray(view.source_totals))
    else:
        res = _transport(cand, lower, cap, np.asarray(view.source_totals), np.asarray(view.destination_totals))
    _check_reconciled(res, view)
    return readonly_array(res, dtype=np.int64)


# ---------------------------------------------------------------------------
# the empirical set
# ---------------------------------------------------------------------------
@dataclass(frozen=True, slots=True)
class EmpiricalAmbiguitySet:
    support_matrices: tuple[np.ndarray, ...]
    history_offsets: tuple[int, ...]
    descriptor_vectors: np.ndarray
    descriptor_labels: tuple[str, ...]
    lower_bounds: np.ndarray
    upper_bounds: np.ndarray
    empirical_mean: np.ndarray
    empirical_variance: np.ndarray
    delta_mean: np.ndarray
    variance_low: np.ndarray
    variance_high: np.ndarray
    uniform_witness: np.ndarray
    normalizer: DescriptorNormalizer
    topology: PublicTopologyView
    observation_constraint_fingerprint: str
    normalizer_digest: str
    group_coefficients_digest: str
    history_cutoff: int
    construction_seed: int
    singleton_control: bool
    uses_oracle: bool = False
    upper_bound_only: bool = False

    def __post_init__(self) -> None:
        mats = tuple(readonly_array(m, dtype=np.int64) for m in self.support_matrices)
        vec = readonly_array(self.descriptor_vectors, dtype=np.float64)
        if not mats or vec.shape[0] != len(mats):
            raise ValueError("ambiguity support cannot be empty")
        object.__setattr__(self, "support_matrices", mats)
        object.__setattr__(self, "descriptor_vectors", vec)
        for k in ("lower_bounds", "upper_bounds", "empirical_mean", "empirical_variance", "delta_mean",
                  "variance_low", "variance_high", "uniform_witness"):
            object.__setattr__(self, k, readonly_array(getattr(self, k), dtype=np.float64))
        object.__setattr__(self, "topology", _public(self.topology))
        if str(self.normalizer_digest) != self.normalizer.digest:
            raise ValueError("normalizer provenance digest mismatch")
        if str(self.group_coefficients_digest) != group_coefficients_digest(self.topology):
            raise ValueError("group coefficient provenance digest mismatch")
        if int(self.history_cutoff) < HISTORY_WINDOW:
            raise ValueError("history cutoff provenance is invalid")
        object.__setattr__(self, "normalizer_digest", str(self.normalizer_digest))
        object.__setattr__(self, "group_coefficients_digest", str(self.group_coefficients_digest))
        object.__setattr__(self, "history_cutoff", int(self.history_cutoff))
        object.__setattr__(self, "construction_seed", int(self.construction_seed))

    @property
    def probability_support_size(self) -> int:
        return len(self.support_matrices)

    def validate_probability_weights(self, weights: Any) -> bool:
        """A distribution on the support whose descriptor moments stay inside the bands."""
        w = np.asarray(weights, dtype=np.float64)
        if w.shape != (self.probability_support_size,):
            raise ValueError("probability weight shape mismatch")
        if not np.isfinite(w).all():
            raise ValueError("probability weights must be finite")
        if np.any(w < 0.0):
            raise ValueError("probability weights must be nonnegative")
        if abs(float(w.sum()) - 1.0) > 1e-10:
            raise ValueError("probability weights must be normalized")
        if np.any(np.abs(w @ self.descriptor_vectors - self.empirical_mean) > self.delta_mean + 1e-10):
            raise ValueError("probability weights violate ambiguity mean moments")
        var = w @ (self.descriptor_vectors - self.empirical_mean) ** 2
        if np.any(var < self.variance_low - 1e-10) or np.any(var > self.variance_high + 1e-10):
            raise ValueError("probability weights violate ambiguity variance moments")
        return True

    def to_canonical_bytes(self) -> bytes:
        return _canonical_bytes(self)


def build_empirical_ambiguity_set(view: AmbiguityConstructionView, *,
                                  calibration_radius: float) -> EmpiricalAmbiguitySet:
    if not isinstance(view, AmbiguityConstructionView):
        raise TypeError("ordinary construction accepts only AmbiguityConstructionView")
    radius = float(calibration_radius)
    if not math.isfinite(radius) or radius < 0.0:
        raise ValueError("calibration radius must be finite and nonnegative")
    singleton = view.ratio == 1.0
    if singleton:
        m = readonly_array(view.observed_matrix, dtype=np.int64)
        _check_reconciled(m, view)
        mats, offs = (m,), (-1,)
    else:
        mats, offs = tuple(reconcile_candidate(c, view) for c in view.history_matrices), view.history_offsets
    vec = np.stack([traffic_descriptor(m, view.topology) for m in mats])
    mean = vec.mean(axis=0)
    var = ((vec - mean) ** 2).mean(axis=0)
    scale = view.normalizer.scale
    plo, phi = physical_descriptor_bounds(view.topology, max_entry=MAX_ENTRY)
    if singleton:
        lo, hi = vec[0].copy(), vec[0].copy()
    else:
        lo = np.maximum(plo, vec.min(axis=0) - radius * scale)
        hi = np.minimum(phi, vec.max(axis=0) + radius * scale)
    gdig = group_coefficients_digest(view.topology)
    fp = _digest((view.observed_matrix, view.entry_mask, view.mode, view.stage, view.ratio, view.source_totals,
                  view.destination_totals, view.normalizer.digest, gdig, view.history_offsets, view.history_cutoff))
    out = EmpiricalAmbiguitySet(
        support_matrices=mats, history_offsets=offs, descriptor_vectors=vec,
        descriptor_labels=descriptor_names(view.topology), lower_bounds=lo, upper_bounds=hi, empirical_mean=mean,
        empirical_variance=var, delta_mean=0.25 * scale, variance_low=0.5 * var,
        variance_high=1.5 * var + 0.01 * scale ** 2, uniform_witness=np.full(len(mats), 1.0 / len(mats)),
        normalizer=view.normalizer, topology=view.topology, observation_constraint_fingerprint=fp,
        normalizer_digest=view.normalizer.digest, group_coefficients_digest=gdig, history_cutoff=view.history_cutoff,
        construction_seed=view.construction_seed, singleton_control=singleton)
    out.validate_probability_weights(out.uniform_witness)
    return out


# ---------------------------------------------------------------------------
# support selection
# ---------------------------------------------------------------------------
def _pairwise(vec: np.ndarray, scale: np.ndarray) -> np.ndarray:
    z = np.asarray(vec, dtype=np.float64) / np.asarray(scale, dtype=np.float64)
    return np.sqrt(((z[:, None, :] - z[None, :, :]) ** 2).sum(axis=2))


def _selection_inputs(vectors, scale, offsets, k):
    v, s, o, k = (np.asarray(vectors, dtype=np.float64), np.asarray(scale, dtype=np.float64),
                  np.asarray(offsets, dtype=np.int64), int(k))
    if v.ndim != 2 or not np.isfinite(v).all():
        raise ValueError("selector vectors must be finite and two-dimensional")
    if s.shape != (v.shape[1],) or np.any(s <= 0.0) or not np.isfinite(s).all():
        raise ValueError("selector scale must be finite and positive")
    if o.shape != (v.shape[0],):
        raise ValueError("selector history offsets shape mismatch")
    if k <= 0 or k > v.shape[0]:
        raise ValueError("selector K exceeds finite support")
    return v, s, o, k


def _most_recent(cands, offsets) -> int:
    """Among tied candidates: the latest history offset, then the larger index."""
    return int(max(cands, key=lambda i: (int(offsets[i]), int(i))))


def _extend_farthest(dist: np.ndarray, offsets: np.ndarray, chosen: list[int], k: int) -> None:
    while len(chosen) < k:
        near = dist[:, chosen].min(axis=1)
        near[chosen] = -np.inf
        far = float(near.max())
        chosen.append(_most_recent(np.flatnonzero(np.isclose(near, far, rtol=0.0, atol=1e-12)), offsets))


def greedy_minimax_indices(vectors: Any, *, scale: Any, history_offsets: Any, k: int) -> tuple[int, ...]:
    """Greedy k-centre: start at the medoid of smallest eccentricity, then add the farthest point."""
    v, s, o, k = _selection_inputs(vectors, scale, history_offsets, k)
    dist = _pairwise(v, s)
    ecc = dist.max(axis=1)
    chosen = [_most_recent(np.flatnonzero(np.isclose(ecc, float(ecc.min()), rtol=0.0, atol=1e-12)), o)]
    _extend_farthest(dist, o, chosen, k)
    return tuple(chosen)


def boundary_indices(vectors: Any, *, lower: Any, upper: Any, scale: Any, history_offsets: Any,
                     k: int) -> tuple[int, ...]:
    """Per descriptor, the support point nearest its lower then upper bound; then farthest-point fill."""
    v, s, o, k = _selection_inputs(vectors, scale, history_offsets, k)
    lo, hi = np.asarray(lower, dtype=np.float64), np.asarray(upper, dtype=np.float64)
    if lo.shape != s.shape or hi.shape != s.shape:
        raise ValueError("boundary shape mismatch")
    chosen: list[int] = []
    for j in range(v.shape[1]):
        for target in (lo[j], hi[j]):
            if len(chosen) == k:
                return tuple(chosen)
            avail = [i for i in range(len(v)) if i not in chosen]
            dd = {i: abs(v[i, j] - target) / s[j] for i in avail}
            m = min(dd.values())
            chosen.append(_most_recent([i for i in avail if abs(dd[i] - m) <= 1e-12], o))
    if not chosen:
        chosen.extend(greedy_minimax_indices(v, scale=s, history_offsets=o, k=1))
    _extend_farthest(_pairwise(v, s), o, chosen, k)
    return tuple(chosen)


@dataclass(frozen=True, slots=True)
class SelectedSupport:
    method: str
    requested_k: int
    actual_k: int
    selected_indices: tuple[int, ...]
    history_offsets: tuple[int, ...]
    matrices: tuple[np.ndarray, ...]
    descriptor_vectors: np.ndarray
    weights: tuple[float, ...]
    uses_oracle: bool
    upper_bound_only: bool
    severity_definition: str | None = None
    approximation: str | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "matrices", tuple(readonly_array(m, dtype=np.int64) for m in self.matrices))
        object.__setattr__(self, "descriptor_vectors", readonly_array(self.descriptor_vectors, dtype=np.float64))

    def to_canonical_bytes(self) -> bytes:
        return _canonical_bytes(self)


def _severity(amb: EmpiricalAmbiguitySet) -> np.ndarray:
    """Largest standardised excess over the fit centre among the load descriptors,
    or the standardised density (negative sparsity) when that is larger."""
    v, c, s = amb.descriptor_vectors, amb.normalizer.center, amb.normalizer.scale
    sp = 2 * amb.topology.num_nodes + 2
    idx = [i for i in range(v.shape[1]) if i != sp]
    return np.maximum(((v[:, idx] - c[idx]) / s[idx]).max(axis=1), -(v[:, sp] - c[sp]) / s[sp])


def _support(amb: EmpiricalAmbiguitySet, method: str, k: int, idx: Sequence[int], *, severity: str | None = None,
             approx: str | None = None) -> SelectedSupport:
    idx = tuple(int(i) for i in idx)
    return SelectedSupport(method=method, requested_k=int(k), actual_k=len(idx), selected_indices=idx,
                           history_offsets=tuple(amb.history_offsets[i] for i in idx),
                           matrices=tuple(amb.support_matrices[i] for i in idx),
                           descriptor_vectors=amb.descriptor_vectors[list(idx)], weights=(1.0 / len(idx),) * len(idx),
                           uses_oracle=False, upper_bound_only=False, severity_definition=severity,
                           approximation=approx)


def select_support(ambiguity: EmpiricalAmbiguitySet, *, method: str, k: int,
                   replicate_seed: int | None = None) -> SelectedSupport:
    if not isinstance(ambiguity, EmpiricalAmbiguitySet):
        raise TypeError("selector requires EmpiricalAmbiguitySet")
    k, method = int(k), str(method)
    if k <= 0:
        raise ValueError("K must be positive")
    if ambiguity.singleton_control:
        return _support(ambiguity, method, k, (0,),
                        approx="deterministic_greedy_k_center" if method == "minimax_subset" else None)
    if k > len(ambiguity.support_matrices):
        raise ValueError("K exceeds finite empirical support")
    if method == "random_empirical":
        if replicate_seed is None:
            raise ValueError("random_empirical requires explicit replicate_seed")
        perm = np.random.default_rng(int(replicate_seed)).permutation(len(ambiguity.support_matrices))
        return _support(ambiguity, method, k, perm[:k])
    if method == "worst_recent_cases":
        sev = _severity(ambiguity)
        order = sorted(range(len(sev)), key=lambda i: (-float(sev[i]), -int(ambiguity.history_offsets[i])))
        return _support(ambiguity, method, k, order[:k], severity="max_upper_fit_standardized_with_density")
    if method == "boundary_scenarios":
        return _support(ambiguity, method, k, boundary_indices(
            ambiguity.descriptor_vectors, lower=ambiguity.lower_bounds, upper=ambiguity.upper_bounds,
            scale=ambiguity.normalizer.scale, history_offsets=ambiguity.history_offsets, k=k))
    if method == "minimax_subset":
        return _support(ambiguity, method, k, greedy_minimax_indices(
            ambiguity.descriptor_vectors, scale=ambiguity.normalizer.scale,
            history_offsets=ambiguity.history_offsets, k=k), approx="deterministic_greedy_k_center")
    raise ValueError(f"unknown ordinary selector: {method}")


def _rms(a: np.ndarray, b: np.ndarray, scale: np.ndarray) -> float:
    return float(np.sqrt(np.mean(((a - b) / scale) ** 2)))


def support_covering_radius(ambiguity: EmpiricalAmbiguitySet, support: SelectedSupport) -> float:
    s = ambiguity.normalizer.scale
    return float(max((min(_rms(c, x, s) for x in support.descriptor_vectors) for c in ambiguity.descriptor_vectors),
                     default=0.0))


def oracle_support_upper_bound(ambiguity: EmpiricalAmbiguitySet, *, truth: Any, k: int) -> SelectedSupport:
    """Evaluator-only: the truth plus k - 1 support points chosen farthest from the truth and each other."""
    k = int(k)
    if k <= 0:
        raise ValueError("oracle K must be positive")
    m = readonly_array(_matrix(truth, ambiguity.topology.num_nodes), dtype=np.int64)
    tv = traffic_descriptor(m, ambiguity.topology)
    want = 0 if ambiguity.singleton_control else min(max(k - 1, 0), len(ambiguity.support_matrices))
    chosen: list[int] = []
    if want:
        z = ambiguity.descriptor_vectors / ambiguity.normalizer.scale
        zt = tv / ambiguity.normalizer.scale
        while len(chosen) < want:
            avail = [i for i in range(len(z)) if i not in chosen]
            anchors = [zt] + [z[i] for i in chosen]
            near = {i: min(float(np.linalg.norm(z[i] - a)) for a in anchors) for i in avail}
            far = max(near.values())
            chosen.append(_most_recent([i for i in avail if abs(near[i] - far) <= 1e-12], ambiguity.history_offsets))
    mats = (m,) + tuple(ambiguity.support_matrices[i] for i in chosen)
    return SelectedSupport(method="oracle_support_upper_bound", requested_k=k, actual_k=len(mats),
                           selected_indices=(-1, *chosen),
                           history_offsets=(0, *[ambiguity.history_offsets[i] for i in chosen]), matrices=mats,
                           descriptor_vectors=np.vstack([tv, *[ambiguity.descriptor_vectors[i] for i in chosen]]),
                           weights=(1.0 / len(mats),) * len(mats), uses_oracle=True, upper_bound_only=True,
                           approximation="truth_plus_deterministic_greedy_k_center")


def truth_nearest_descriptor_distance(ambiguity: EmpiricalAmbiguitySet, support: SelectedSupport,
                                      truth: Any) -> float:
    v = traffic_descriptor(truth, ambiguity.topology)
    return min(_rms(v, c, ambiguity.normalizer.scale) for c in support.descriptor_vectors)


__all__ = ["AmbiguityConstructionView", "DescriptorNormalizer", "EmpiricalAmbiguitySet", "HISTORY_WINDOW",
           "MAX_ENTRY", "SelectedSupport", "boundary_indices", "build_empirical_ambiguity_set", "descriptor_names",
           "fit_descriptor_normalizer", "group_coefficients_digest", "greedy_minimax_indices",
           "oracle_support_upper_bound", "physical_descriptor_bounds", "reconcile_candidate", "select_support",
           "support_covering_radius", "traffic_descriptor", "truth_nearest_descriptor_distance"]
