"""Sliding-window moments of integer traffic sequences: validation against
reference moments, a history-only sliding estimator, and controlled context
views for ablations.

Behaviour of rlccl/traffic/moment_validation.py, moment_estimator.py and
context_views.py:

* window moments are the element-wise population mean / variance over the
  window; the error of a window is the relative L2 distance
  ``||actual - ref|| / (||ref|| + eps)``, checked against the sequence's
  ``MomentBounds`` for every complete window at the configured stride;
* the estimator keeps at most ``window_size`` completed matrices of ONE
  sequence; ``get_context`` never includes (or stores) the current matrix,
  falls back to the reference moments while the history is empty, clips the
  current send/receive z-scores to ``+-z_clip`` and reports a confidence of
  ``history / min_history`` (capped at 1).
"""

from __future__ import annotations

from collections import deque
from dataclasses import replace
from typing import Any, Sequence

import numpy as np

from .matrix_utils import validate_traffic_matrix
from .types import MomentContext, TrafficSequence


def window_moments(matrices: Sequence[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    if len(matrices) == 0:
        raise ValueError("At least one traffic matrix is required")
    for m in matrices:
        validate_traffic_matrix(m)
    stack = np.stack([np.asarray(m) for m in matrices]).astype(np.float64)
    return stack.mean(axis=0), stack.var(axis=0)


def relative_l2_error(actual: np.ndarray, reference: np.ndarray, eps: float = 1e-8) -> float:
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(reference, dtype=np.float64)
    if a.shape != r.shape:
        raise ValueError(f"Moment shape mismatch: {a.shape} != {r.shape}")
    return float(np.linalg.norm(a - r) / (np.linalg.norm(r) + eps))


def validate_sequence_moment_bounds(seq: TrafficSequence) -> dict[str, Any]:
    mats = seq.matrices
    if not mats:
        raise ValueError("Traffic sequence must contain at least one matrix")
    for m in mats:
        validate_traffic_matrix(m)
    if seq.mean_ref.shape != np.asarray(mats[0]).shape or seq.var_ref.shape != np.asarray(mats[0]).shape:
        raise ValueError("Reference moments must match traffic matrix shape")
    w = int(seq.metadata.get("window_size", len(mats)))
    stride = int(seq.metadata.get("validation_stride", 1))
    allowed = float(seq.metadata.get("allowed_violation_fraction", 0.0))
    if not 1 <= w <= len(mats):
        raise ValueError("window_size must be in [1, sequence_length]")
    if stride <= 0:
        raise ValueError("validation_stride must be positive")
    if not 0.0 <= allowed <= 1.0:
        raise ValueError("allowed_violation_fraction must be in [0, 1]")
    windows = []
    for start in range(0, len(mats) - w + 1, stride):
        mean, var = window_moments(mats[start:start + w])
        me, ve = relative_l2_error(mean, seq.mean_ref), relative_l2_error(var, seq.var_ref)
        windows.append({"start": start, "end": start + w, "mean_error": me, "var_error": ve,
                        "passed": me <= seq.bounds.epsilon_mean and ve <= seq.bounds.epsilon_var})
    bad = sum(not x["passed"] for x in windows)
    frac = bad / len(windows)
    return {"passed": frac <= allowed, "num_windows": len(windows), "num_violations": bad,
            "violation_fraction": frac, "allowed_violation_fraction": allowed,
            "max_mean_error": max(x["mean_error"] for x in windows),
            "max_var_error": max(x["var_error"] for x in windows), "windows": windows}


class SlidingMomentEstimator:
    """History-only moment estimator over the completed matrices of one sequence."""

    def __init__(self, num_nodes: int, window_size: int, min_history: int, eps: float = 1e-6,
                 z_clip: float = 10.0) -> None:
        if num_nodes <= 0 or window_size <= 0:
            raise ValueError("num_nodes and window_size must be positive")
        if not 1 <= min_history <= window_size:
            raise ValueError("min_history must be in [1, window_size]")
        if eps <= 0 or z_clip <= 0:
            raise ValueError("eps and z_clip must be positive")
        self.num_nodes, self.window_size, self.min_history = int(num_nodes), int(window_size), int(min_history)
        self.eps, self.z_clip = float(eps), float(z_clip)
        self._hist: deque = deque(maxlen=self.window_size)

    @property
    def history_length(self) -> int:
        return len(self._hist)

    def _check(self, m: np.ndarray, name: str) -> np.ndarray:
        validate_traffic_matrix(m)
        a = np.asarray(m, dtype=np.int64)
        if a.shape != (self.num_nodes, self.num_nodes):
            raise ValueError(f"{name} shape must be {(self.num_nodes, self.num_nodes)}, got {a.shape}")
        return a

    def get_context(self, current_matrix: np.ndarray, mean_ref: np.ndarray, var_ref: np.ndarray) -> MomentContext:
        cur = self._check(current_matrix, "current_matrix")
        mref = np.asarray(mean_ref, dtype=np.float64)
        vref = np.asarray(var_ref, dtype=np.float64)
        shape = (self.num_nodes, self.num_nodes)
        if mref.shape != shape or vref.shape != shape:
            raise ValueError(f"Reference moment shapes must be {shape}")
        if np.any(vref < 0):
            raise ValueError("var_ref must be nonnegative")
        if self._hist:
            h = np.stack(list(self._hist)).astype(np.float64)
            mean, var = h.mean(axis=0), h.var(axis=0)
            send_std, recv_std = h.sum(axis=2).std(axis=0), h.sum(axis=1).std(axis=0)
        else:  # cold start: reference moments, independence approximation for the z scale
            mean, var = mref.copy(), vref.copy()
            send_std = np.sqrt(np.maximum(vref.sum(axis=1), 0.0))
            recv_std = np.sqrt(np.maximum(vref.sum(axis=0), 0.0))
        np.fill_diagonal(mean, 0.0)
        np.fill_diagonal(var, 0.0)
        std = np.sqrt(np.maximum(var, 0.0) + self.eps)
        np.fill_diagonal(std, 0.0)
        send_mean, recv_mean = mean.sum(axis=1), mean.sum(axis=0)
        zs = np.clip((cur.sum(axis=1, dtype=np.float64) - send_mean) / (send_std + self.eps), -self.z_clip, self.z_clip)
        zr = np.clip((cur.sum(axis=0, dtype=np.float64) - recv_mean) / (recv_std + self.eps), -self.z_clip, self.z_clip)
        n = len(self._hist)
        return MomentContext(
            history_length=n, window_size=self.window_size, mean_matrix=mean.copy(), var_matrix=var.copy(),
            std_matrix=std, send_mean=send_mean, recv_mean=recv_mean,
            send_std=np.asarray(send_std, dtype=np.float64), recv_std=np.asarray(recv_std, dtype=np.float64),
            current_send_z=zs, current_recv_z=zr,
            mean_drift=relative_l2_error(mean, mref, self.eps), var_drift=relative_l2_error(var, vref, self.eps),
            confidence=min(1.0, n / self.min_history), is_warm=n >= self.min_history)

    def update(self, completed_matrix: np.ndarray) -> None:
        self._hist.append(self._check(completed_matrix, "completed_matrix").copy())

    def state_dict(self) -> dict[str, Any]:
        return {"num_nodes": self.num_nodes, "window_size": self.window_size, "min_history": self.min_history,
                "eps": self.eps, "z_clip": self.z_clip, "history": [m.tolist() for m in self._hist]}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        for k in ("num_nodes", "window_size", "min_history"):
            if int(state[k]) != getattr(self, k):
                raise ValueError(f"Estimator {k} mismatch: {state[k]} != {getattr(self, k)}")
        hist = [self._check(np.asarray(m), "history matrix") for m in state.get("history", [])]
        if len(hist) > self.window_size:
            raise ValueError("Estimator state contains more history than window_size")
        self._hist.clear()
        self._hist.extend(m.copy() for m in hist)


def mean_only_context(ctx: MomentContext) -> MomentContext:
    """Keep the first moments; zero every variance / z feature."""
    z = np.zeros_like
    return replace(ctx, var_matrix=z(ctx.var_matrix), std_matrix=z(ctx.std_matrix), send_std=z(ctx.send_std),
                   recv_std=z(ctx.recv_std), current_send_z=z(ctx.current_send_z),
                   current_recv_z=z(ctx.current_recv_z), var_drift=0.0)


def zero_moment_context(ctx: MomentContext) -> MomentContext:
    """Zero every statistical feature, keeping shape and window metadata."""
    z = np.zeros_like
    return replace(ctx, mean_matrix=z(ctx.mean_matrix), var_matrix=z(ctx.var_matrix), std_matrix=z(ctx.std_matrix),
                   send_mean=z(ctx.send_mean), recv_mean=z(ctx.recv_mean), send_std=z(ctx.send_std),
                   recv_std=z(ctx.recv_std), current_send_z=z(ctx.current_send_z),
                   current_recv_z=z(ctx.current_recv_z), mean_drift=0.0, var_drift=0.0, confidence=0.0,
                   is_warm=False)


__all__ = ["SlidingMomentEstimator", "mean_only_context", "relative_l2_error", "validate_sequence_moment_bounds",
           "window_moments", "zero_moment_context"]
