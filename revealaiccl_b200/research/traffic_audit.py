"""Descriptive audit of generated traffic-matrix sequences.

Behaviour of rlccl/evaluation/traffic_audit.py: the audit reads only the
public ``TrafficSequence`` (matrices, reference moments, bounds, metadata)
and reports, per sequence, total-load statistics and bursts, temporal
structure (autocorrelation with a positive-sequence effective sample size,
adjacent-matrix distances, hotspot dwell, duplicates and exact
periodicity), spatial concentration (shares, entropy, load variance and
skewness), rolling-window moment errors at three scales, and generation
instrumentation when the generator recorded it.  ``summarize_audits``
groups records by (family, length, seed base, dynamics variant).

Rolling moments use prefix sums (one pass per window size); distinct
matrices get integer ids once, and duplicates, periodicity and repeat ratios
compare ids.
"""

from __future__ import annotations

from collections import Counter
from typing import Any, Iterable, Sequence

import numpy as np

from ..traffic.types import TrafficSequence

DEFAULT_ACF_LAGS = (1, 2, 4, 8, 16, 32, 64)
_QUANTILES = (("p50", 0.50), ("p90", 0.90), ("p95", 0.95), ("p99", 0.99), ("p99_9", 0.999))


def _finite(x) -> float | None:
    x = float(x)
    return x if np.isfinite(x) else None


def describe(values) -> dict[str, float | None]:
    a = np.asarray(values, dtype=np.float64)
    keys = ("mean", "variance", "std", "min", "max") + tuple(k for k, _ in _QUANTILES)
    if a.size == 0:
        return {k: None for k in keys}
    out = {"mean": _finite(a.mean()), "variance": _finite(a.var(ddof=0)), "std": _finite(a.std(ddof=0)),
           "min": _finite(a.min()), "max": _finite(a.max())}
    out.update({k: _finite(np.quantile(a, q)) for k, q in _QUANTILES})
    return out


def run_lengths(mask) -> list[int]:
    """Lengths of the maximal runs of True."""
    m = np.asarray(mask, dtype=bool).astype(np.int8)
    if m.size == 0:
        return []
    edges = np.diff(np.concatenate([[0], m, [0]]))
    return (np.flatnonzero(edges == -1) - np.flatnonzero(edges == 1)).astype(int).tolist()


def autocorrelation(values, lags: Iterable[int] = DEFAULT_ACF_LAGS) -> dict[str, Any]:
    """Global-mean-normalised ACF at the requested lags and the ESS n / (1 + 2 sum of the leading positive rho)."""
    a = np.asarray(values, dtype=np.float64)
    c = a - a.mean()
    denom = float(np.dot(c, c))
    req = tuple(sorted({int(k) for k in lags if int(k) > 0}))
    if denom <= 1e-15:
        return {"defined": False, "reason": "constant series", "values": {str(k): None for k in req},
                "effective_sample_size": None}
    acf = {str(k): (_finite(np.dot(c[:-k], c[k:]) / denom) if k < len(a) else None) for k in req}
    pos, k = 0.0, 1
    while k < len(a):  # leading run of positive autocorrelations
        r = float(np.dot(c[:-k], c[k:]) / denom)
        if r <= 0.0:
            break
        pos += r
        k += 1
    ess = len(a) / (1.0 + 2.0 * pos)
    return {"defined": True, "reason": None, "values": acf, "effective_sample_size": float(np.clip(ess, 1.0, len(a)))}


def _skewness(values) -> float | None:
    a = np.asarray(values, dtype=np.float64)
    s = float(a.std(ddof=0))
    if a.size == 0 or s <= 1e-15:
        return None
    return _finite(np.mean(((a - a.mean()) / s) ** 3))


def rolling_moment_metrics(stack: np.ndarray, mean_ref: np.ndarray, var_ref: np.ndarray, window: int,
                           epsilon_mean: float, epsilon_var: float) -> dict[str, Any]:
    L = int(stack.shape[0])
    if window > L:
        return {"available": False, "reason": f"window_size={window} exceeds sequence_length={L}",
                "window_size": int(window), "num_windows": 0}
    v = stack.astype(np.float64, copy=False)
    zero = np.zeros((1,) + v.shape[1:])
    c1 = np.concatenate([zero, np.cumsum(v, axis=0)], axis=0)
    c2 = np.concatenate([zero, np.cumsum(v * v, axis=0)], axis=0)
    m = (c1[window:] - c1[:-window]) / float(window)
    var = np.maximum((c2[window:] - c2[:-window]) / float(window) - m * m, 0.0)
    axes = tuple(range(1, m.ndim))
    em = np.sqrt(np.sum((m - mean_ref) ** 2, axis=axes)) / (float(np.linalg.norm(mean_ref)) + 1e-8)
    ev = np.sqrt(np.sum((var - var_ref) ** 2, axis=axes)) / (float(np.linalg.norm(var_ref)) + 1e-8)
    bad = (em > epsilon_mean) | (ev > epsilon_var)
    return {"available": True, "reason": None, "window_size": int(window), "num_windows": int(len(em)),
            "mean_error": describe(em), "variance_error": describe(ev),
            "mean_violation_fraction": float(np.mean(em > epsilon_mean)),
            "variance_violation_fraction": float(np.mean(ev > epsilon_var)),
            "any_violation_fraction": float(np.mean(bad)),
            "max_consecutive_violation_windows": max(run_lengths(bad), default=0),
            "epsilon_mean": float(epsilon_mean), "epsilon_var": float(epsilon_var)}


def periodicity(stack: np.ndarray, max_period_lag: int) -> dict[str, Any]:
    """Exact-repeat ratio at the standard lags and at every lag whose matrix equals the first one."""
    L = int(stack.shape[0])
    # integer ids of distinct matrices (equal bytes <=> equal id)
    _, ids = np.unique(np.ascontiguousarray(stack).reshape(L, -1), axis=0, return_inverse=True)
    ids = ids.ravel()
    limit = min(int(max_period_lag), L // 2)
    lags = {k for k in DEFAULT_ACF_LAGS if k <= limit}
    lags.update(int(k) for k in np.flatnonzero(ids[1:limit + 1] == ids[0]) + 1)
    ratios: dict[str, float] = {}
    detected = best_lag = None
    best = -1.0
    for k in sorted(lags):
        r = float(np.mean(ids[:-k] == ids[k:]))
        ratios[str(k)] = r
        if r > best:
            best_lag, best = k, r
        if detected is None and r == 1.0 and np.array_equal(stack[:-k], stack[k:]):
            detected = k
    return {"detected_exact_period": detected, "strongest_checked_lag": best_lag,
            "strongest_exact_repeat_ratio": best if best_lag is not None else None,
            "exact_repeat_ratio_by_lag": ratios, "max_period_lag": limit}


def _dwell(series: np.ndarray) -> list[int]:
    """Run lengths of a categorical series."""
    if series.size == 0:
        return [1]
    cuts = np.flatnonzero(series[1:] != series[:-1]) + 1
    bounds = np.concatenate([[0], cuts, [series.size]])
    return np.diff(bounds).astype(int).tolist()


def audit_sequence(sequence: TrafficSequence, *, short_window: int = 16, medium_window: int = 128,
                   long_window: int = 512, acf_lags: Iterable[int] = DEFAULT_ACF_LAGS, max_period_lag: int = 512,
                   generation_seconds: float | None = None) -> dict[str, Any]:
    """Audit one sequence (the statistical unit)."""
    if not sequence.matrices:
        raise ValueError("Traffic sequence must contain at least one matrix")
    stack = np.stack(sequence.matrices, axis=0)
    if stack.ndim != 3 or stack.shape[1] != stack.shape[2]:
        raise ValueError("Traffic matrices must stack to [time, nodes, nodes]")
    L, n, _ = stack.shape
    off = ~np.eye(n, dtype=bool)
    md = sequence.metadata

    total = stack.sum(axis=(1, 2)).astype(np.float64)
    tstats = describe(total)
    mu, sd = float(total.mean()), float(total.std(ddof=0))
    hi2, hi3 = total > mu + 2.0 * sd, total > mu + 3.0 * sd
    bursts = np.flatnonzero(hi2)
    tstats.update({"max_to_mean_ratio": float(total.max() / mu) if mu > 0 else None,
                   "fraction_above_mean_plus_2std": float(hi2.mean()),
                   "fraction_above_mean_plus_3std": float(hi3.mean()),
                   "high_load_run_lengths": run_lengths(hi2), "high_load_run_length_stats": describe(run_lengths(hi2)),
                   "burst_intervals": np.diff(bursts).astype(int).tolist(),
                   "burst_interval_stats": describe(np.diff(bursts))})

    delta = np.diff(stack.astype(np.float64), axis=0)
    l1 = np.abs(delta).sum(axis=(1, 2))
    l2 = np.sqrt((delta * delta).sum(axis=(1, 2)))
    norm = max(float(n * (n - 1) * max(int(stack.max()), 1)), 1.0)
    recv = stack.sum(axis=1).astype(np.float64)
    send = stack.sum(axis=2).astype(np.float64)
    hot = np.argmax(recv, axis=1)
    hot_runs = _dwell(hot)
    _, first_idx = np.unique(stack.reshape(L, -1), axis=0, return_index=True)
    uniq = len(first_idx)
    near = 0.05
    nl1 = l1 / norm
    rec_name = next((k for k in ("regime_dwell_records", "volatility_dwell_records", "variant_dwell_records")
                     if md.get(k)), None)
    temporal = {
        "total_traffic_acf": autocorrelation(total, acf_lags),
        "adjacent_matrix_l1": describe(l1), "adjacent_matrix_l2": describe(l2),
        "adjacent_normalized_l1": describe(nl1),
        "hotspot_destination_dwell_lengths": hot_runs, "hotspot_destination_dwell_stats": describe(hot_runs),
        "hotspot_destination_migrations": int(np.sum(hot[1:] != hot[:-1])),
        "hotspot_destination_series": hot.astype(int).tolist(),
        "regime_dwell": ({"available": True, "source": rec_name, "lengths": [int(r["length"]) for r in md[rec_name]],
                          "statistics": describe([r["length"] for r in md[rec_name]])}
                         if rec_name is not None else
                         {"available": False, "reason": "generator output contains no latent regime labels"}),
        "exact_duplicate_ratio": float(1.0 - uniq / L), "num_unique_matrices": uniq,
        "adjacent_near_duplicate_ratio": float(np.mean(nl1 <= near)) if L > 1 else None,
        "near_duplicate_normalized_l1_threshold": near,
        "periodicity": periodicity(stack, max_period_lag),
        "labeled_hotspot_destination_series": md.get("hotspot_destination"),
        "labeled_hotspot_source_series": md.get("hotspot_source"),
        "shock_count": int(np.sum(md.get("shock_flags", []))),
    }

    denom = np.maximum(total, 1.0)
    p = stack[:, off].astype(np.float64) / denom[:, None]
    logp = np.zeros_like(p)
    logp[p > 0] = np.log(p[p > 0])
    ent = -np.sum(p * logp, axis=1)
    spatial = {
        "source_load_by_node": {str(i): describe(send[:, i]) for i in range(n)},
        "destination_load_by_node": {str(i): describe(recv[:, i]) for i in range(n)},
        "off_diagonal_sparsity": describe(np.mean(stack[:, off] == 0, axis=1)),
        "max_source_share": describe(send.max(axis=1) / denom),
        "max_destination_share": describe(recv.max(axis=1) / denom),
        "off_diagonal_entropy": describe(ent),
        "normalized_off_diagonal_entropy": describe(ent / np.log(max(n * (n - 1), 2))),
        "destination_hotspot_strength": describe(recv.max(axis=1) * n / denom),
        "source_load_variance": describe(np.var(send, axis=1, ddof=0)),
        "destination_load_variance": describe(np.var(recv, axis=1, ddof=0)),
        "source_load_skewness": _skewness(send.ravel()),
        "destination_load_skewness": _skewness(recv.ravel()),
        "bandwidth_group_concentration": {
            "available": False,
            "reason": ("TrafficSequence has source-destination demand only; mapping demand to routed topology "
                       "bandwidth groups requires a routing/schedule policy and is not identifiable here")},
    }

    windows = {str(w): rolling_moment_metrics(stack, sequence.mean_ref, sequence.var_ref, w,
                                              sequence.bounds.epsilon_mean, sequence.bounds.epsilon_var)
               for w in dict.fromkeys((short_window, medium_window, long_window))}

    attempt = int(md.get("generation_attempt", 1))
    has_inter = "pre_clip_statistics" in md
    generation = {
        "attempts": attempt, "rejections_before_acceptance": max(0, attempt - 1),
        "rejection_rate_before_acceptance": float(max(0, attempt - 1) / attempt),
        "wall_time_seconds": None if generation_seconds is None else float(generation_seconds),
        "intermediate_instrumentation_available": has_inter,
        "pre_clip": md.get("pre_clip_statistics"), "post_clip_pre_round": md.get("post_clip_statistics"),
        "post_round_pre_diagonal": None,
        "unavailable_reason": None if has_inter else (
            "generate_traffic_sequence returns only final integer matrices and does not retain pre-clip, pre-round, "
            "or rejected candidate arrays"),
        "final_integer": {
            "dtype": str(stack.dtype), "minimum": int(stack.min()), "maximum": int(stack.max()),
            "diagonal_nonzero_count": int(np.count_nonzero(np.diagonal(stack, axis1=1, axis2=2))),
            "off_diagonal_zero_fraction": float(np.mean(stack[:, off] == 0)),
            "off_diagonal_at_max_fraction": float(np.mean(stack[:, off] == int(stack.max())))},
        "smoothing_indicator": {
            "mean_adjacent_normalized_l1": float(nl1.mean()) if L > 1 else None,
            "note": "descriptive output statistic; the generator exposes no explicit smoothing stage"},
    }
    return {
        "sequence_id": sequence.sequence_id, "family": sequence.family,
        "dynamics_variant": md.get("dynamics_variant"), "seed": int(sequence.seed), "sequence_length": int(L),
        "num_nodes": int(n), "topology_name": sequence.topology_name,
        "generator_kind": md.get("generator_kind", "legacy short-horizon generator"),
        "metadata_usage": md.get("metadata_usage"), "constraint_status": md.get("constraint_status"),
        "calibration_candidates_evaluated": md.get("calibration_candidates_evaluated"),
        "spatial_distribution_validation": md.get("spatial_distribution_validation"),
        "generator_window_size": int(md.get("window_size", short_window)),
        "total_traffic": tstats, "temporal": temporal, "spatial": spatial, "multi_window_moments": windows,
        "generation": generation, "generator_multi_scale_constraints": md.get("multi_scale_constraints"),
        "generator_matrix_multi_scale_constraints": md.get("matrix_multi_scale_constraints"),
    }


def summarize_audits(records: Sequence[dict[str, Any]]) -> dict[str, Any]:
    """Aggregate audit records per (family, sequence_length, seed_base, dynamics_variant)."""
    groups: dict[tuple, list[dict[str, Any]]] = {}
    for r in records:
        groups.setdefault((r["family"], r["sequence_length"], r["seed_base"], r.get("dynamics_variant")), []).append(r)
    out = []
    for (fam, length, seed_base, variant), rows in sorted(groups.items(), key=lambda kv: tuple(map(str, kv[0]))):
        ok = [r for r in rows if r.get("status") == "success"]
        item: dict[str, Any] = {"family": fam, "sequence_length": length, "seed_base": seed_base,
                                "dynamics_variant": variant, "num_requested": len(rows), "num_succeeded": len(ok),
                                "num_failed": len(rows) - len(ok), "generation_failure_rate": (len(rows) - len(ok)) / len(rows)}
        if ok:
            wins = ok[0]["multi_window_moments"]
            item.update({
                "mean_generation_seconds": float(np.mean([r["generation"]["wall_time_seconds"] for r in ok])),
                "mean_generation_attempts": float(np.mean([r["generation"]["attempts"] for r in ok])),
                "mean_total_cv": float(np.mean([(r["total_traffic"]["std"] / r["total_traffic"]["mean"])
                                                if r["total_traffic"]["mean"] else 0.0 for r in ok])),
                "mean_exact_duplicate_ratio": float(np.mean([r["temporal"]["exact_duplicate_ratio"] for r in ok])),
                "detected_exact_periods": sorted(Counter(r["temporal"]["periodicity"]["detected_exact_period"]
                                                         for r in ok).items(), key=lambda kv: str(kv[0])),
                "window_violation_fraction": {
                    w: (float(np.mean([r["multi_window_moments"][w]["any_violation_fraction"] for r in ok
                                       if r["multi_window_moments"][w]["available"]]))
                        if any(r["multi_window_moments"][w]["available"] for r in ok) else None)
                    for w in wins},
            })
        out.append(item)
    return {"groups": out, "num_records": len(records)}


__all__ = ["DEFAULT_ACF_LAGS", "audit_sequence", "autocorrelation", "describe", "periodicity",
           "rolling_moment_metrics", "run_lengths", "summarize_audits"]
