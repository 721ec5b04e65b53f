"""History-only predictors of low-dimensional traffic summaries.

Behaviour of rlccl/models/traffic_predictor.py:

* ``RidgeMultiOutput``: standardised features (zero-variance columns keep
  scale 1), centred targets, closed-form ridge ``(Z'Z + a I) W = Z'Y``;
  state keys ``{prefix}_{x_mean,x_scale,y_mean,weights,alpha}``;
* ``deterministic_group_coefficients``: offered load per shared bandwidth
  group when every (src, dst) demand follows the greedy shortest path that
  takes the lowest-index edge reducing the hop distance;
* ``traffic_summary`` / ``summary_vector``: total, per-source and
  per-destination load, hotspot strength (max / mean destination load),
  off-diagonal sparsity, group loads;
* ``build_history_examples``: features from X_0..X_{t-1} only (window
  moments of the last ``history_window`` matrices and the last
  ``recent_steps`` summary vectors); the target is the summary of X_t;
* ``TrafficPredictorSuite``: constant, previous-value, moment-only ridge,
  recent-history ridge and an oracle row, each with a hotspot head; npz
  artifacts with the reference's key names so saved suites load in both.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Iterable, Sequence

import numpy as np


@dataclass
class RidgeMultiOutput:
    alpha: float = 1.0
    x_mean: np.ndarray | None = None
    x_scale: np.ndarray | None = None
    y_mean: np.ndarray | None = None
    weights: np.ndarray | None = None

    def _require(self) -> None:
        if self.weights is None or self.x_mean is None or self.x_scale is None or self.y_mean is None:
            raise RuntimeError("Regressor is not fitted")

    def fit(self, x: np.ndarray, y: np.ndarray) -> "RidgeMultiOutput":
        X = np.asarray(x, dtype=np.float64)
        Y = np.asarray(y, dtype=np.float64)
        if X.ndim != 2 or Y.ndim != 2 or len(X) != len(Y):
            raise ValueError("x and y must be same-length 2-D arrays")
        if len(X) == 0:
            raise ValueError("Cannot fit an empty dataset")
        self.x_mean = X.mean(axis=0)
        scale = X.std(axis=0, ddof=0)
        scale[scale < 1e-8] = 1.0
        self.x_scale = scale
        Z = (X - self.x_mean) / scale
        self.y_mean = Y.mean(axis=0)
        A = Z.T @ Z + float(self.alpha) * np.eye(Z.shape[1])
        self.weights = np.linalg.solve(A, Z.T @ (Y - self.y_mean))
        return self

    def predict(self, x: np.ndarray) -> np.ndarray:
        self._require()
        X = np.asarray(x, dtype=np.float64)
        if X.ndim != 2 or X.shape[1] != self.x_mean.shape[0]:
            raise ValueError("Feature dimension mismatch")
        return (X - self.x_mean) / self.x_scale @ self.weights + self.y_mean

    def state(self, prefix: str) -> dict[str, np.ndarray]:
        self._require()
        return {f"{prefix}_x_mean": self.x_mean, f"{prefix}_x_scale": self.x_scale,
                f"{prefix}_y_mean": self.y_mean, f"{prefix}_weights": self.weights,
                f"{prefix}_alpha": np.asarray([self.alpha], dtype=np.float64)}

    @classmethod
    def from_state(cls, values: Any, prefix: str) -> "RidgeMultiOutput":
        f = lambda k: np.asarray(values[f"{prefix}_{k}"], dtype=np.float64)  # noqa: E731
        return cls(alpha=float(f("alpha")[0]), x_mean=f("x_mean"), x_scale=f("x_scale"), y_mean=f("y_mean"),
                   weights=f("weights"))


def deterministic_group_coefficients(topology: Any) -> np.ndarray:
    """coeff[g, s, d] = number of edges of group g on the greedy shortest s->d path.

    At every node the path takes the lowest-index outgoing edge whose head is
    strictly closer to d (an offered-load proxy, not a learned schedule's
    realised load); exact and reproducible.
    """
    V, G = topology.V, len(topology.shared_constraints)
    coeff = np.zeros((G, V, V), dtype=np.float64)
    if G == 0:
        return coeff
    member = np.zeros((topology.E, G), dtype=np.float64)
    for g, (edges, _) in enumerate(topology.shared_constraints):
        for e in edges:
            member[int(e), g] += 1.0
    src = np.asarray(topology.edge_src, dtype=np.int64)
    dst = np.asarray(topology.edge_dst, dtype=np.int64)
    dist = np.asarray(topology.dist_matrix)
    order = np.argsort(src, kind="stable")  # outgoing edges of each node in index order
    starts = np.searchsorted(src[order], np.arange(V + 1))
    for d in range(V):
        # next_edge[v]: the greedy edge from v toward d
        next_edge = np.full(V, -1, dtype=np.int64)
        for v in range(V):
            if v == d:
                continue
            out = order[starts[v]:starts[v + 1]]
            closer = out[dist[dst[out], d] < dist[v, d]]
            if closer.size == 0:
                raise RuntimeError(f"No path from {v} to {d}")
            next_edge[v] = closer.min()
        for s in range(V):
            if s == d:
                continue
            v, hops = s, 0
            while v != d:
                e = next_edge[v]
                coeff[:, s, d] += member[e]
                v = int(dst[e])
                hops += 1
                if hops > V:
                    raise RuntimeError("Shortest-path proxy encountered a cycle")
    return coeff


def traffic_summary(matrix: np.ndarray, group_coefficients: np.ndarray) -> dict[str, Any]:
    T = np.asarray(matrix, dtype=np.float64)
    if T.ndim != 2 or T.shape[0] != T.shape[1]:
        raise ValueError("matrix must be square")
    out_load, in_load = T.sum(axis=1), T.sum(axis=0)
    off = ~np.eye(T.shape[0], dtype=bool)
    groups = (np.einsum("gij,ij->g", group_coefficients, T) if group_coefficients.size
              else np.empty(0, dtype=np.float64))
    return {"total": float(T.sum()), "source_load": out_load, "destination_load": in_load,
            "hotspot_destination": int(np.argmax(in_load)),
            "hotspot_strength": float(in_load.max() / max(float(in_load.mean()), 1e-8)),
            "sparsity": float(np.mean(T[off] == 0)), "bandwidth_group_load": groups}


def summary_vector(summary: dict[str, Any]) -> np.ndarray:
    """[total, source loads, destination loads, hotspot strength, sparsity, group loads]."""
    return np.concatenate([[float(summary["total"])], np.asarray(summary["source_load"], dtype=np.float64),
                           np.asarray(summary["destination_load"], dtype=np.float64),
                           [float(summary["hotspot_strength"]), float(summary["sparsity"])],
                           np.asarray(summary["bandwidth_group_load"], dtype=np.float64)]).astype(np.float64)


def _moment_features(history: np.ndarray) -> np.ndarray:
    off = ~np.eye(history.shape[1], dtype=bool)
    return np.concatenate([history.mean(axis=0)[off], history.var(axis=0, ddof=0)[off]])


def build_history_examples(sequences: Sequence[Any], *, group_coefficients: np.ndarray, history_window: int,
                           recent_steps: int, min_history: int) -> list[dict[str, Any]]:
    """One example per step t >= max(recent_steps, min_history); features read X_0..X_{t-1} only."""
    if min(history_window, recent_steps, min_history) <= 0:
        raise ValueError("History lengths must be positive")
    first = max(recent_steps, min_history)
    out: list[dict[str, Any]] = []
    for seq in sequences:
        mats = np.asarray(seq.matrices, dtype=np.float64)
        sums = [traffic_summary(m, group_coefficients) for m in mats]
        vec = np.stack([summary_vector(x) for x in sums])
        hot = np.asarray([x["hotspot_destination"] for x in sums], dtype=np.int64)
        for t in range(first, len(mats)):
            hist = mats[max(0, t - history_window):t]
            recent = vec[t - recent_steps:t]
            if hist.shape[0] == 0 or recent.shape[0] != recent_steps:  # the slices must end before t
                raise AssertionError("Invalid history-only feature slice")
            out.append({"sequence_id": seq.sequence_id, "family": seq.family, "seed": int(seq.seed), "step": t,
                        "moment_features": _moment_features(hist), "recent_features": recent.reshape(-1),
                        "previous_target": vec[t - 1].copy(), "previous_hotspot": int(hot[t - 1]),
                        "target": vec[t].copy(), "hotspot_target": int(hot[t]), "history_last_step": t - 1})
    return out


def stack_field(examples: Iterable[dict[str, Any]], name: str) -> np.ndarray:
    return np.stack([e[name] for e in examples])


_HEADS = ("moment", "recent", "moment_hotspot", "recent_hotspot")


class TrafficPredictorSuite:
    """Constant, previous-value, moment-only and recent-history predictors with hotspot heads."""

    def __init__(self, num_nodes: int, group_count: int, alpha: float = 10.0):
        self.num_nodes, self.group_count, self.alpha = int(num_nodes), int(group_count), float(alpha)
        for h in _HEADS:
            setattr(self, h, RidgeMultiOutput(self.alpha))
        self.constant_target: np.ndarray | None = None
        self.constant_hotspot: int | None = None

    @property
    def target_dim(self) -> int:
        return 1 + 2 * self.num_nodes + 2 + self.group_count

    def fit(self, examples: Sequence[dict[str, Any]]) -> "TrafficPredictorSuite":
        if not examples:
            raise ValueError("examples must not be empty")
        mom, rec, y = (stack_field(examples, k) for k in ("moment_features", "recent_features", "target"))
        lab = np.asarray([e["hotspot_target"] for e in examples], dtype=np.int64)
        if y.shape[1] != self.target_dim:
            raise ValueError("Target dimension does not match topology")
        onehot = np.eye(self.num_nodes)[lab]
        self.constant_target = y.mean(axis=0)
        self.constant_hotspot = int(np.argmax(np.bincount(lab, minlength=self.num_nodes)))
        self.moment.fit(mom, y)
        self.recent.fit(rec, y)
        self.moment_hotspot.fit(mom, onehot)
        self.recent_hotspot.fit(rec, onehot)
        return self

    def predict(self, examples: Sequence[dict[str, Any]]) -> dict[str, dict[str, np.ndarray]]:
        if self.constant_target is None or self.constant_hotspot is None:
            raise RuntimeError("Predictor suite is not fitted")
        mom, rec, prev, y = (stack_field(examples, k)
                             for k in ("moment_features", "recent_features", "previous_target", "target"))
        prev_hot = np.asarray([e["previous_hotspot"] for e in examples], dtype=np.int64)
        lab = np.asarray([e["hotspot_target"] for e in examples], dtype=np.int64)
        n = len(examples)
        return {
            "target": {"continuous": y, "hotspot": lab},
            "constant": {"continuous": np.tile(self.constant_target, (n, 1)),
                         "hotspot": np.full(n, self.constant_hotspot, dtype=np.int64)},
            "previous": {"continuous": prev, "hotspot": prev_hot},
            "moment_only": {"continuous": self.moment.predict(mom),
                            "hotspot": self.moment_hotspot.predict(mom).argmax(axis=1)},
            "recent_history": {"continuous": self.recent.predict(rec),
                               "hotspot": self.recent_hotspot.predict(rec).argmax(axis=1)},
            "oracle_current_summary": {"continuous": y.copy(), "hotspot": lab.copy()},
        }

    def save(self, path: str) -> None:
        if self.constant_target is None or self.constant_hotspot is None:
            raise RuntimeError("Predictor suite is not fitted")
        state = {"num_nodes": np.asarray([self.num_nodes], dtype=np.int64),
                 "group_count": np.asarray([self.group_count], dtype=np.int64),
                 "constant_target": self.constant_target,
                 "constant_hotspot": np.asarray([self.constant_hotspot], dtype=np.int64)}
        for h in _HEADS:
            state.update(getattr(self, h).state(h))
        np.savez_compressed(path, **state)

    @classmethod
    def load(cls, path: str) -> "TrafficPredictorSuite":
        with np.load(path) as v:
            suite = cls(int(v["num_nodes"][0]), int(v["group_count"][0]), float(v["moment_alpha"][0]))
            suite.constant_target = np.asarray(v["constant_target"], dtype=np.float64)
            suite.constant_hotspot = int(v["constant_hotspot"][0])
            for h in _HEADS:
                setattr(suite, h, RidgeMultiOutput.from_state(v, h))
        return suite


__all__ = ["RidgeMultiOutput", "TrafficPredictorSuite", "build_history_examples", "deterministic_group_coefficients",
           "stack_field", "summary_vector", "traffic_summary"]
