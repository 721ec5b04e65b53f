"""Evaluation helpers for traffic-conditioned schedule policies.

Behaviour of rlccl/evaluation/{metrics,counterfactual,partial_demand,
sequence_evaluator}.py:

* ``cvar`` / ``summarize_rows``: empirical tail mean beyond the alpha
  quantile; completion / timeout / legality / synthesis summaries;
* counterfactual histories: one current matrix with two strictly prior
  histories, contexts built from prior matrices only, context distances,
  Levenshtein distance of action sequences, sparse schedules, edge-use L1;
* partial-demand observations: random hidden entries, random hidden shards,
  source totals only (balanced rows) and source + destination totals
  (integral transportation by shortest augmenting paths over the zero-
  diagonal bipartite graph), mapped back onto the true chunk identities so
  the action space is unchanged;
* ``evaluate_sequence_policy``: greedy slot decoding of a policy over
  sequence problems under a context ablation (baseline, mean only, full,
  shuffled donor context), with per-problem completion, legality and
  synthesis time.

The traffic audit lives in ``research.traffic_audit``.
"""

from __future__ import annotations

import time
from collections import defaultdict, deque
from collections.abc import Iterable, Mapping, Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np

from ..traffic.matrix_utils import validate_traffic_matrix
from ..traffic.moments import SlidingMomentEstimator, mean_only_context, relative_l2_error
from ..traffic.types import MomentContext


# ---------------------------------------------------------------------------
# metrics
# ---------------------------------------------------------------------------
def cvar(values, alpha: float, higher_is_worse: bool = True) -> float:
    """Mean of the values at or beyond the alpha quantile (the worse tail)."""
    a = np.asarray(values, dtype=np.float64)
    if a.size == 0:
        raise ValueError("CVaR requires at least one value")
    if not 0.0 <= alpha < 1.0:
        raise ValueError("alpha must be in [0, 1)")
    if higher_is_worse:
        return float(a[a >= np.quantile(a, alpha)].mean())
    return float(a[a <= np.quantile(a, 1.0 - alpha)].mean())


def summarize_rows(rows: Iterable[Mapping[str, Any]]) -> dict[str, float | int]:
    recs = list(rows)
    if not recs:
        raise ValueError("At least one evaluation row is required")
    steps = np.asarray([r["completion_steps"] for r in recs], dtype=np.float64)
    synth = np.asarray([r["synthesis_ms"] for r in recs], dtype=np.float64)
    out: dict[str, float | int] = {
        "num_collectives": len(recs), "completion_steps_mean": float(steps.mean()),
        "completion_steps_median": float(np.median(steps)),
        "completion_steps_p95": float(np.percentile(steps, 95)),
        "completion_steps_p99": float(np.percentile(steps, 99)),
        "completion_steps_cvar90": cvar(steps, 0.90), "completion_steps_cvar95": cvar(steps, 0.95),
        "timeout_rate": float(np.mean([bool(r["timeout"]) for r in recs])),
        "legality_rate": float(np.mean([bool(r["legal"]) for r in recs])),
        "synthesis_ms_mean": float(synth.mean()), "synthesis_ms_p95": float(np.percentile(synth, 95)),
    }
    if "fallback_level" in recs[0]:
        out["fallback_rate"] = float(np.mean([int(r["fallback_level"]) > 0 for r in recs]))
    return out


# ---------------------------------------------------------------------------
# counterfactual histories
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class CounterfactualHistoryPair:
    """One current matrix and two strictly prior history windows."""

    pair_id: str
    family: str
    seed: int
    current_matrix: np.ndarray
    history_a: tuple[np.ndarray, ...]
    history_b: tuple[np.ndarray, ...]
    mean_ref: np.ndarray
    var_ref: np.ndarray

    def __post_init__(self) -> None:
        cur = np.asarray(self.current_matrix, dtype=np.int64)
        object.__setattr__(self, "current_matrix", cur)
        for name in ("history_a", "history_b"):
            hist = tuple(np.asarray(m, dtype=np.int64) for m in getattr(self, name))
            if not hist:
                raise ValueError(f"{name} must not be empty")
            if any(m.shape != cur.shape for m in hist):
                raise ValueError(f"{name} matrix shape mismatch")
            if any(np.shares_memory(m, cur) for m in hist):
                raise ValueError(f"{name} must contain prior matrices, not current_matrix")
            object.__setattr__(self, name, hist)
        for name in ("mean_ref", "var_ref"):
            ref = np.asarray(getattr(self, name), dtype=np.float64)
            if ref.shape != cur.shape:
                raise ValueError("Reference shape mismatch")
            object.__setattr__(self, name, ref)


def context_from_prior_history(history: Sequence[np.ndarray], current_matrix: np.ndarray, mean_ref: np.ndarray,
                               var_ref: np.ndarray, *, window_size: int, min_history: int) -> MomentContext:
    """Context after feeding only the prior matrices (the last window_size of them)."""
    est = SlidingMomentEstimator(num_nodes=int(np.asarray(current_matrix).shape[0]), window_size=window_size,
                                 min_history=min_history)
    for m in list(history)[-window_size:]:
        est.update(m)
    n = est.history_length
    ctx = est.get_context(current_matrix, mean_ref, var_ref)
    if est.history_length != n:
        raise AssertionError("get_context mutated estimator history")
    return ctx


def context_distance(a: MomentContext, b: MomentContext) -> dict[str, float]:
    m = relative_l2_error(a.mean_matrix, b.mean_matrix)
    v = relative_l2_error(a.var_matrix, b.var_matrix)
    node = relative_l2_error(np.concatenate([a.send_mean, a.recv_mean]), np.concatenate([b.send_mean, b.recv_mean]))
    return {"mean_relative_l2": float(m), "variance_relative_l2": float(v), "node_load_relative_l2": float(node),
            "combined": float(m + v + node)}


def action_edit_distance(lhs: Sequence[tuple[int, ...]], rhs: Sequence[tuple[int, ...]]) -> int:
    """Levenshtein distance (unit insert / delete / substitute) between action sequences."""
    row = np.arange(len(rhs) + 1)
    for i, x in enumerate(lhs, start=1):
        prev_diag, row[0] = row[0], i
        for j, y in enumerate(rhs, start=1):
            cur = min(row[j] + 1, row[j - 1] + 1, prev_diag + (x != y))
            prev_diag, row[j] = row[j], cur
    return int(row[-1])


def sparse_schedule(schedule: Sequence[np.ndarray]) -> list[list[int]]:
    """Every scheduled transfer as [slot, chunk, edge], slot-major then row-major."""
    out: list[list[int]] = []
    for slot, y in enumerate(schedule):
        c, e = np.nonzero(np.asarray(y))
        out.extend([slot, int(ci), int(ei)] for ci, ei in zip(c, e))
    return out


def schedule_edge_use(schedule: Sequence[np.ndarray]) -> np.ndarray:
    if not schedule:
        return np.empty(0, dtype=np.int64)
    return np.sum([np.asarray(y, dtype=np.int64).sum(axis=0) for y in schedule], axis=0)


def edge_use_l1(lhs: Sequence[np.ndarray], rhs: Sequence[np.ndarray]) -> int:
    a, b = schedule_edge_use(lhs), schedule_edge_use(rhs)
    if a.shape != b.shape:
        raise ValueError("Schedule edge dimensions differ")
    return int(np.abs(a - b).sum())


def json_ready_context(ctx: MomentContext) -> dict[str, Any]:
    """Audit summary of a context (no current or future matrices)."""
    return {"history_length": int(ctx.history_length), "window_size": int(ctx.window_size),
            "mean_drift": float(ctx.mean_drift), "var_drift": float(ctx.var_drift),
            "confidence": float(ctx.confidence), "mean_matrix": np.asarray(ctx.mean_matrix).tolist(),
            "var_matrix": np.asarray(ctx.var_matrix).tolist()}


# ---------------------------------------------------------------------------
# partial-demand observations
# ---------------------------------------------------------------------------
OBSERVATION_MODES = ("random_entries", "source_totals", "source_destination_totals", "partial_shards")


@dataclass(frozen=True)
class PartialDemandObservation:
    mode: str
    hide_ratio: float | None
    observed_matrix: np.ndarray
    observation_demands: np.ndarray
    revealed_chunk_mask: np.ndarray
    metadata: dict[str, Any]

    def __post_init__(self) -> None:
        m = np.asarray(self.observed_matrix, dtype=np.int64)
        dem = np.asarray(self.observation_demands, dtype=np.float32)
        rev = np.asarray(self.revealed_chunk_mask, dtype=bool)
        validate_traffic_matrix(m)
        if dem.ndim != 2 or rev.shape != (dem.shape[0],):
            raise ValueError("Invalid observation demand/chunk-mask shape")
        if np.any(dem < 0) or not np.all(np.isfinite(dem)):
            raise ValueError("Observation demands must be finite and nonnegative")
        object.__setattr__(self, "observed_matrix", m)
        object.__setattr__(self, "observation_demands", dem)
        object.__setattr__(self, "revealed_chunk_mask", rev)


def chunk_owners(matrix: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(source, destination) of every chunk: chunks numbered row-major over the entries, one per unit."""
    m = np.asarray(matrix, dtype=np.int64)
    counts = m.ravel()
    flat = np.repeat(np.arange(counts.size), counts)
    return flat // m.shape[1], flat % m.shape[1]


def balanced_rows(source_totals: np.ndarray) -> np.ndarray:
    """Each row total spread over the off-diagonal columns, remainder to the lowest columns."""
    tot = np.asarray(source_totals, dtype=np.int64)
    n = len(tot)
    out = np.zeros((n, n), dtype=np.int64)
    for s, t in enumerate(tot):
        cols = np.array([d for d in range(n) if d != s])
        q, r = divmod(int(t), n - 1)
        out[s, cols] = q
        out[s, cols[:r]] += 1
    return out


def transport_from_margins(source_totals: np.ndarray, destination_totals: np.ndarray) -> np.ndarray:
    """Integral matrix with the given margins and a zero diagonal (max-flow, shortest augmenting paths).

    Graph: super source 0, rows 1..n, columns n+1..2n, sink 2n+1; row->column
    arcs off the diagonal with unbounded capacity.  Augmenting paths are found
    breadth first, scanning neighbours in index order, each saturating its
    bottleneck.
    """
    rows = np.asarray(source_totals, dtype=np.int64)
    cols = np.asarray(destination_totals, dtype=np.int64)
    if rows.sum() != cols.sum() or np.any(rows < 0) or np.any(cols < 0):
        raise ValueError("Invalid transportation margins")
    n, total = len(rows), int(rows.sum())
    N, sink = 2 * n + 2, 2 * n + 1
    res = np.zeros((N, N), dtype=np.int64)
    res[0, 1:n + 1] = rows
    res[1:n + 1, n + 1:2 * n + 1] = total * (1 - np.eye(n, dtype=np.int64))
    res[n + 1:2 * n + 1, sink] = cols
    flow = np.zeros((N, N), dtype=np.int64)
    sent = 0
    while True:
        parent = np.full(N, -1, dtype=np.int64)
        parent[0] = 0
        q = deque([0])
        while q and parent[sink] < 0:
            u = q.popleft()
            for v in np.flatnonzero(res[u] > 0):
                if parent[v] < 0:
                    parent[v] = u
                    q.append(int(v))
        if parent[sink] < 0:
            break
        path = [sink]
        while path[-1] != 0:
            path.append(int(parent[path[-1]]))
        path.reverse()
        amt = min(int(res[u, v]) for u, v in zip(path[:-1], path[1:]))
        for u, v in zip(path[:-1], path[1:]):
            res[u, v] -= amt
            res[v, u] += amt
            flow[u, v] += amt
            flow[v, u] -= amt
        sent += amt
    if sent != total:
        raise RuntimeError("Traffic margins are infeasible under zero diagonal")
    out = flow[1:n + 1, n + 1:2 * n + 1].astype(np.int64)
    if not (np.array_equal(out.sum(axis=1), rows) and np.array_equal(out.sum(axis=0), cols)):
        raise AssertionError("Transportation flow does not preserve margins")
    return out


def demands_for_proxy(true_matrix: np.ndarray, proxy: np.ndarray, num_chunks: int) -> np.ndarray:
    """Give each source's own chunks (in order) the proxy row's destinations (in column order)."""
    n = true_matrix.shape[0]
    src, _ = chunk_owners(true_matrix)
    dem = np.zeros((num_chunks, n), dtype=np.float32)
    for s in range(n):
        mine = np.flatnonzero(src == s)
        dests = np.repeat(np.arange(n), np.asarray(proxy[s], dtype=np.int64))
        if len(dests) != len(mine):
            raise AssertionError("Proxy row total differs from available source chunks")
        dem[mine, dests] = 1.0
    return dem


def build_partial_observation(matrix: np.ndarray, true_demands: np.ndarray, *, mode: str, hide_ratio: float | None,
                              seed: int) -> PartialDemandObservation:
    """A policy observation of one traffic matrix; the executed demand is unchanged."""
    T = np.asarray(matrix, dtype=np.int64)
    D = np.asarray(true_demands, dtype=np.int64)
    validate_traffic_matrix(T)
    src, dst = chunk_owners(T)
    nchunks = len(src)
    if nchunks != D.shape[0] or D.shape[1] != T.shape[0]:
        raise ValueError("true_demands do not match the traffic matrix chunk encoding")
    if mode not in OBSERVATION_MODES:
        raise ValueError(f"Unsupported observation mode: {mode}")
    if mode in ("random_entries", "partial_shards") and (hide_ratio is None or not 0.0 <= hide_ratio < 1.0):
        raise ValueError("random_entries/partial_shards require hide_ratio in [0,1)")
    rng = np.random.default_rng(seed)
    n = T.shape[0]
    observed = np.zeros_like(T)
    obs_dem = np.zeros(D.shape, dtype=np.float32)
    revealed = np.zeros(nchunks, dtype=bool)
    if mode in ("random_entries", "partial_shards"):
        if mode == "random_entries":
            entries = [(i, j) for i in range(n) for j in range(n) if i != j]
            hidden = set(int(x) for x in rng.choice(len(entries), size=int(round(float(hide_ratio) * len(entries))),
                                                    replace=False))
            visible_entry = np.zeros((n, n), dtype=bool)
            for k, (i, j) in enumerate(entries):
                visible_entry[i, j] = k not in hidden
            revealed = visible_entry[src, dst]
            meta = {"visible_entry_count": int(visible_entry.sum()), "total_off_diagonal_entries": len(entries),
                    "representation_note": ("Chunk identities/source ownership remain known to preserve the action "
                                            "space; hidden destination entries are zero in policy demand features.")}
        else:
            k = int(round((1.0 - float(hide_ratio)) * nchunks))
            revealed[rng.choice(nchunks, size=k, replace=False)] = True
            meta = {"visible_chunk_count": k, "total_chunk_count": nchunks}
        np.add.at(observed, (src[revealed], dst[revealed]), 1)
        obs_dem[revealed] = D[revealed]
    elif mode == "source_totals":
        observed = balanced_rows(T.sum(axis=1))
        obs_dem = demands_for_proxy(T, observed, nchunks)
        meta = {"imputation": "deterministic balanced off-diagonal allocation preserving source totals",
                "provided": "source totals only"}
        hide_ratio = None
    else:
        observed = transport_from_margins(T.sum(axis=1), T.sum(axis=0))
        obs_dem = demands_for_proxy(T, observed, nchunks)
        meta = {"imputation": ("deterministic integral max-flow using only source/destination totals and the "
                               "zero-diagonal structural constraint"),
                "provided": "source and destination totals"}
        hide_ratio = None
    validate_traffic_matrix(observed)
    return PartialDemandObservation(mode=mode, hide_ratio=hide_ratio, observed_matrix=observed,
                                    observation_demands=obs_dem, revealed_chunk_mask=revealed, metadata=meta)


# ---------------------------------------------------------------------------
# sequence policy evaluation
# ---------------------------------------------------------------------------
CONTEXT_MODES = ("baseline", "mean_only", "full", "shuffled")


def build_shuffled_context_map(problems: Sequence[tuple[str, Any]]) -> dict[str, Any]:
    """Donor context per problem: another sequence at the same step, same family when possible.

    Donors are sorted by problem id; the pick is (sum of the id's UTF-8
    bytes) mod the donor count, so the map is deterministic without a global
    random state.  A donor never comes from the problem's own sequence.
    """
    by_fs: dict[tuple[str, int], list] = defaultdict(list)
    by_s: dict[int, list] = defaultdict(list)
    for pid, p in problems:
        fam, step = str(p.metadata.get("family", "unknown")), int(p.sequence_step)
        by_fs[(fam, step)].append((pid, p))
        by_s[step].append((pid, p))
    out: dict[str, Any] = {}
    for pid, p in problems:
        fam, step = str(p.metadata.get("family", "unknown")), int(p.sequence_step)
        pool = sorted(by_fs[(fam, step)], key=lambda x: x[0])
        if len({q.sequence_id for _, q in pool}) < 2:
            pool = sorted(by_s[step], key=lambda x: x[0])
        donors = [q for _, q in pool if q.sequence_id != p.sequence_id]
        if not donors:
            raise ValueError(f"Shuffled-context evaluation requires at least two sequences at sequence step {step}")
        out[pid] = donors[sum(pid.encode("utf-8")) % len(donors)].moment_context
    return out


def _context_for(pid, problem, mode, shuffled):
    if mode == "baseline":
        return None
    if mode == "full":
        return problem.moment_context
    if mode == "mean_only":
        return mean_only_context(problem.moment_context)
    if mode == "shuffled":
        if shuffled is None or pid not in shuffled:
            raise ValueError("Missing shuffled context for problem")
        return shuffled[pid]
    raise ValueError(f"Unsupported context mode: {mode}")


def evaluate_sequence_policy(model, problems: Sequence[tuple[str, Any]], device, *, context_mode: str,
                             moment_max_entry: float = 8.0, shuffled_contexts: Mapping[str, Any] | None = None,
                             warmup: bool = True) -> list[dict[str, Any]]:
    """Greedy decoding of every problem under one context ablation; one row per problem."""
    import torch

    from ..rl.decoder import SlotDecoder
    from ..rl.scenarios import evaluate_schedule
    from ..topology.info import compute_received_chunks

    if context_mode not in CONTEXT_MODES:
        raise ValueError(f"Unsupported context mode: {context_mode}")
    if context_mode != "baseline" and getattr(model, "global_moment_feat_dim", 0) <= 0:
        raise ValueError("Moment context modes require a moment-enabled model")
    dev = torch.device(device)
    sync = (lambda: torch.cuda.synchronize(dev)) if dev.type == "cuda" else (lambda: None)
    model.eval()
    rows: list[dict[str, Any]] = []
    with torch.no_grad():
        if warmup and problems:
            pid, p = problems[0]
            SlotDecoder(p.topology_info).decode_slot(
                model, p.initial_state.copy(), p.demands.copy(), 0, p.T, train=False,
                moment_context=_context_for(pid, p, context_mode, shuffled_contexts), current_matrix=p.traffic_matrix,
                moment_max_entry=moment_max_entry)
            sync()
        for pid, p in problems:
            topo = p.topology_info
            dec = SlotDecoder(topo)
            state, dem = p.initial_state.copy(), p.demands.copy()
            ctx = _context_for(pid, p, context_mode, shuffled_contexts)
            schedule = []
            sync()
            t0 = time.perf_counter()
            done_at = p.T
            for slot in range(p.T):
                y = dec.decode_slot(model, state, dem, slot, p.T, train=False, moment_context=ctx,
                                    current_matrix=p.traffic_matrix, moment_max_entry=moment_max_entry)[0]
                schedule.append(y)
                got = compute_received_chunks(y, topo.edge_dst, topo.V)
                state = np.maximum(state, got)
                dem = dem * (1 - got)
                if not np.any(dem):
                    done_at = slot + 1
                    break
            sync()
            ms = (time.perf_counter() - t0) * 1e3
            timed_out = bool(np.any(dem))
            schedule += [np.zeros((p.C, p.E), dtype=np.int64)] * (p.T - len(schedule))
            score, err = evaluate_schedule(schedule, p)
            rows.append({"method": context_mode, "problem_id": pid, "sequence_id": p.sequence_id,
                         "sequence_step": int(p.sequence_step), "family": str(p.metadata.get("family", "unknown")),
                         "completion_steps": int(done_at), "timeout": timed_out, "legal": err == "",
                         "evaluation_error": err, "score": float(score), "synthesis_ms": float(ms)})
    return rows


__all__ = ["CONTEXT_MODES", "CounterfactualHistoryPair", "OBSERVATION_MODES", "PartialDemandObservation",
           "action_edit_distance", "balanced_rows", "build_partial_observation", "build_shuffled_context_map",
           "chunk_owners", "context_distance", "context_from_prior_history", "cvar", "demands_for_proxy",
           "edge_use_l1", "evaluate_sequence_policy", "json_ready_context", "schedule_edge_use", "sparse_schedule",
           "summarize_rows", "transport_from_margins"]
