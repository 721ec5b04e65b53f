"""Sequence-level metrics, intervals, bootstrap and the H1 gate
(rlccl/prediction/statistics.py).

Gate conditions: (1) pooled total-RMSE improvement CI lower bound > 0;
(2) every base seed's mean delta > 0 and at least 4 of 5 families > 0;
(3) every primary target's CI lower bound > 0; (4) leave-one-family-out
aggregate delta >= 0, at least 3 families > 0 and at most one family with a
relative RMSE change > 10%; (5) interval calibration error <= 0.05 overall
and <= 0.10 per family, scenario calibration error <= 0.10; (6) at least 10
tail events and q90 recall >= 0.70; (7) integrity tests passed and no veto.
Too few tail events gives HOLD when every other condition passes, else FAIL.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping

import numpy as np
from scipy.stats import rankdata

PRIMARY_TARGETS = ("total_traffic", "source_load_vector", "destination_load_vector")
EXPECTED_BASE_SEEDS = {42, 142, 242}
EXPECTED_FAMILIES = {"regime_switching_long", "stochastic_volatility", "rare_shock_recovery", "hotspot_random_walk",
                     "same_moments_different_dynamics"}


def _spearman(a: np.ndarray, b: np.ndarray) -> float:
    """Pearson correlation of average ranks (ties share their mean rank); 0 for a constant side."""
    ra = rankdata(np.asarray(a, dtype=np.float64).reshape(-1), method="average")
    rb = rankdata(np.asarray(b, dtype=np.float64).reshape(-1), method="average")
    ra -= ra.mean()
    rb -= rb.mean()
    den = float(np.sqrt((ra @ ra) * (rb @ rb)))
    return float(ra @ rb / den) if den > 0.0 else 0.0


def sequence_target_metrics(actual: Mapping[str, np.ndarray], predicted: Mapping[str, np.ndarray]) -> dict:
    """MAE / RMSE / R2 / Spearman per target block, components weighted equally."""
    if set(actual) != set(predicted):
        raise ValueError("actual and predicted target blocks must match")
    out: dict[str, dict[str, float]] = {}
    for k in actual:
        t, e = np.asarray(actual[k], dtype=np.float64), np.asarray(predicted[k], dtype=np.float64)
        if t.shape != e.shape or t.size == 0:
            raise ValueError(f"shape mismatch for target {k}")
        if not (np.isfinite(t).all() and np.isfinite(e).all()):
            raise ValueError(f"target {k} contains NaN/Inf")
        t, e = t.reshape(-1), e.reshape(-1)
        err = e - t
        ss_tot = float(np.sum((t - t.mean()) ** 2))
        ss_err = float(err @ err)
        r2 = 1.0 - ss_err / ss_tot if ss_tot > 0.0 else (1.0 if ss_err == 0 else 0.0)
        out[k] = {"mae": float(np.mean(np.abs(err))), "rmse": float(np.sqrt(np.mean(err ** 2))), "r2": float(r2),
                  "spearman": _spearman(t, e)}
    return out


def hotspot_from_destination_loads(destination_loads) -> np.ndarray:
    d = np.asarray(destination_loads, dtype=np.float64)
    if d.ndim != 2 or d.shape[1] == 0:
        raise ValueError("destination_loads must be a nonempty 2-D array")
    return np.argmax(d, axis=1).astype(np.int64)


@dataclass(frozen=True)
class BootstrapResult:
    mean: float
    lower: float
    upper: float
    samples: np.ndarray


def family_stratified_paired_bootstrap(deltas, families, *, samples: int = 10_000,
                                       seed: int = 20260731) -> BootstrapResult:
    """Resample whole test sequences within each family (families in first-seen order), average, 95% CI."""
    v = np.asarray(deltas, dtype=np.float64).reshape(-1)
    lab = np.asarray(families, dtype=object).reshape(-1)
    if v.shape != lab.shape or not len(v) or not np.isfinite(v).all():
        raise ValueError("deltas/families must be same-length, nonempty, and finite")
    if samples <= 0:
        raise ValueError("samples must be positive")
    groups = [np.flatnonzero(lab == f) for f in dict.fromkeys(lab.tolist())]
    rng = np.random.default_rng(int(seed))
    draws = np.empty(int(samples))
    for i in range(int(samples)):
        draws[i] = float(np.mean(v[np.concatenate([rng.choice(g, size=len(g), replace=True) for g in groups])]))
    lo, hi = np.quantile(draws, (0.025, 0.975), method="linear")
    return BootstrapResult(float(v.mean()), float(lo), float(hi), draws)


def autocorrelation(values, *, max_lag: int = 64) -> np.ndarray:
    a = np.asarray(values, dtype=np.float64).reshape(-1)
    if not len(a) or max_lag < 0:
        raise ValueError("values must be nonempty and max_lag nonnegative")
    out = np.zeros(int(max_lag) + 1)
    out[0] = 1.0
    c = a - a.mean()
    var = float(c @ c)
    if var <= 0.0:
        return out
    for k in range(1, min(int(max_lag), len(a) - 1) + 1):
        out[k] = float(c[:-k] @ c[k:] / var)
    return out


def positive_sequence_ess(values, *, max_lag: int = 64) -> float:
    a = np.asarray(values, dtype=np.float64).reshape(-1)
    rho = autocorrelation(a, max_lag=max_lag)[1:min(len(a), max_lag + 1)]
    stop = np.flatnonzero(rho <= 0.0)
    head = rho[:stop[0]] if stop.size else rho
    return float(len(a) / (1.0 + 2.0 * float(np.sum(head))))


def quantile_interval_metrics(actual, lower, upper, *, nominal_coverage: float = 0.80) -> dict[str, float]:
    t, lo, hi = (np.asarray(x, dtype=np.float64) for x in (actual, lower, upper))
    if t.shape != lo.shape or t.shape != hi.shape or not t.size:
        raise ValueError("actual/lower/upper shapes must match and be nonempty")
    if not (np.isfinite(t).all() and np.isfinite(lo).all() and np.isfinite(hi).all()):
        raise ValueError("interval arrays contain NaN/Inf")
    if np.any(lo > hi):
        raise ValueError("interval lower bound exceeds upper bound")
    cov = float(np.mean((t >= lo) & (t <= hi)))
    return {"coverage": cov, "interval_width": float(np.mean(hi - lo)),
            "calibration_error": abs(cov - float(nominal_coverage))}


def scenario_envelope_metrics(actual, scenarios, *, nominal_coverage: float = 0.80) -> dict[str, Any]:
    t, s = np.asarray(actual, dtype=np.float64), np.asarray(scenarios, dtype=np.float64)
    if s.ndim != t.ndim + 1 or s.shape[0] != t.shape[0] or s.shape[2:] != t.shape[1:]:
        raise ValueError("scenarios must have shape [example, scenario, ...target]")
    if s.shape[1] != 64:
        raise ValueError("Gate H1 requires exactly 64 joint scenarios")
    lo = np.quantile(s, 0.10, axis=1, method="linear")
    hi = np.quantile(s, 0.90, axis=1, method="linear")
    m: dict[str, Any] = quantile_interval_metrics(t, lo, hi, nominal_coverage=nominal_coverage)
    m.update({"lower": lo, "upper": hi})
    return m


def evaluate_h1_gate(evidence: Mapping[str, Any]) -> dict[str, Any]:
    seeds, fams = evidence["seed_mean_deltas"], evidence["family_mean_deltas"]
    primary, lofo = evidence["primary_ci_lowers"], evidence["lofo"]
    prob, tail = evidence["probability"], evidence["tail"]
    pos = lambda d, thr=0.0: sum(float(x) > thr for x in d.values())  # noqa: E731
    c = {
        "condition_1": float(evidence["pooled_total_ci_lower"]) > 0.0,
        "condition_2": (set(seeds) == EXPECTED_BASE_SEEDS and all(float(x) > 0.0 for x in seeds.values())
                        and set(fams) == EXPECTED_FAMILIES and pos(fams) >= 4),
        "condition_3": set(primary) == set(PRIMARY_TARGETS) and all(float(primary[k]) > 0.0 for k in PRIMARY_TARGETS),
        "condition_4": (float(lofo["aggregate_mean_delta"]) >= 0.0 and set(lofo["family_mean_deltas"]) == EXPECTED_FAMILIES
                        and set(lofo["relative_rmse_changes"]) == EXPECTED_FAMILIES
                        and pos(lofo["family_mean_deltas"]) >= 3 and pos(lofo["relative_rmse_changes"], 0.10) <= 1),
        "condition_5": (float(prob["overall_interval_calibration_error"]) <= 0.05
                        and set(prob["family_interval_calibration_errors"]) == EXPECTED_FAMILIES
                        and all(float(x) <= 0.10 for x in prob["family_interval_calibration_errors"].values())
                        and float(prob["overall_scenario_calibration_error"]) <= 0.10),
    }
    enough = int(tail["event_count"]) >= 10
    c["condition_6"] = enough and tail.get("recall") is not None and float(tail["recall"]) >= 0.70
    c["condition_7"] = bool(evidence["integrity_tests_passed"]) and not bool(evidence["supervisor_veto"])
    c = {k: bool(v) for k, v in c.items()}
    reasons = [k for k, v in c.items() if not v]
    if not enough:
        reasons.append("insufficient_events")
        decision = "HOLD" if all(v for k, v in c.items() if k != "condition_6") else "FAIL"
    else:
        decision = "PASS" if all(c.values()) else "FAIL"
    return {"decision": decision, "conditions": c, "reasons": reasons}
