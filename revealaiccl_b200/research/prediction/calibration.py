"""Pooled signed-residual calibration (rlccl/prediction/calibration.py).

Quantiles q10/q50/q90 are the point plus the calibration residuals'
per-component linear quantiles; each of the 64 joint scenarios of example i
is the point plus one whole residual row drawn with
``default_rng(seed + stable_index_i)``, so a scenario set depends only on
the example's stable index, not on batch order.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class CalibratedPrediction:
    q10: np.ndarray
    q50: np.ndarray
    q90: np.ndarray
    scenarios: np.ndarray


class ResidualCalibrator:
    def __init__(self, seed: int = 20260731, scenario_count: int = 64):
        if scenario_count <= 0:
            raise ValueError("scenario_count must be positive")
        self.seed, self.scenario_count = int(seed), int(scenario_count)
        self.residuals: np.ndarray | None = None
        self.residual_quantiles: np.ndarray | None = None

    def fit(self, calibration_point, signed_residuals) -> "ResidualCalibrator":
        p, r = np.asarray(calibration_point, dtype=np.float64), np.asarray(signed_residuals, dtype=np.float64)
        if p.ndim != 2 or r.ndim != 2 or p.shape != r.shape:
            raise ValueError("calibration points and signed residuals must share a 2-D shape")
        if not len(r) or not np.isfinite(r).all():
            raise ValueError("calibration residuals must be nonempty and finite")
        self.residuals = r.copy()
        self.residual_quantiles = np.quantile(r, (0.10, 0.50, 0.90), axis=0, method="linear")
        return self

    def predict(self, point, *, stable_example_indices) -> CalibratedPrediction:
        if self.residuals is None:
            raise RuntimeError("ResidualCalibrator is not fitted")
        v = np.asarray(point, dtype=np.float64)
        idx = np.asarray(stable_example_indices, dtype=np.int64)
        if v.ndim != 2 or v.shape[1] != self.residuals.shape[1]:
            raise ValueError("point prediction dimension mismatch")
        if idx.shape != (len(v),):
            raise ValueError("one stable example index is required per prediction")
        pick = np.stack([np.random.default_rng(self.seed + int(i)).integers(0, len(self.residuals),
                                                                            size=self.scenario_count) for i in idx]) \
            if len(idx) else np.zeros((0, self.scenario_count), dtype=np.int64)
        scen = v[:, None, :] + self.residuals[pick]
        q = self.residual_quantiles
        return CalibratedPrediction(v + q[0], v + q[1], v + q[2], scen)


def tail_event_recall(actual_total, predicted_q90, *, fit_threshold: float, minimum_events: int = 10) -> dict:
    """Recall of total-load tail events (actual > fit threshold) by q90 > threshold; too few events reported as such."""
    a = np.asarray(actual_total, dtype=np.float64).reshape(-1)
    u = np.asarray(predicted_q90, dtype=np.float64).reshape(-1)
    if a.shape != u.shape or not np.isfinite(a).all() or not np.isfinite(u).all():
        raise ValueError("actual and q90 arrays must be same-length and finite")
    ev = a > float(fit_threshold)
    n = int(ev.sum())
    if n < int(minimum_events):
        return {"status": "insufficient_events", "event_count": n, "recall": None}
    return {"status": "ok", "event_count": n, "recall": float(np.mean(u[ev] > float(fit_threshold)))}
