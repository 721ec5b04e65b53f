"""Prediction-study runner (rlccl/prediction/experiment.py, artifacts.py).

Pipeline per scope (pooled, then one leave-one-family-out fold per family):
fit the suite on the fit sequences; score the two recent-history backbones
by total-traffic RMSE on the validation sequences and select one; collect
that backbone's signed residuals on the calibration sequences; on every
test sequence record, per point method and target block, MAE / RMSE / R2 /
Spearman / RMSE improvement over previous-value / hotspot accuracy, and per
target block interval and 64-scenario coverage counts plus total-traffic
tail events above the fit split's 90th percentile.  The summary (primary
CIs from the family-stratified bootstrap, seed / family means, LOFO
changes, pooled probability calibration and the data conditions of the
gate) is recomputed from the raw rows and the manifest alone, so artifact
bundles can be re-verified offline.
"""

from __future__ import annotations

import csv
import hashlib
import importlib.metadata
import json
import platform
import sys
from dataclasses import replace
from pathlib import Path
from typing import Any, Mapping, Sequence

import numpy as np

from ...topology.loader import load_topology_info
from ..traffic_predictor import deterministic_group_coefficients
from .calibration import ResidualCalibrator
from .data import (FORMAL_BASE_SEEDS, FORMAL_FAMILIES, SPLITS, HistoryExamples, SequenceSpec,
                   build_formal_sequence_specs, build_history_examples, generate_formal_sequence, sequence_digest,
                   validate_split_records)
from .models import METHOD_NAMES, HistoryPredictorSuite, select_recent_backbone
from .statistics import (PRIMARY_TARGETS, autocorrelation, family_stratified_paired_bootstrap,
                         hotspot_from_destination_loads, positive_sequence_ess, sequence_target_metrics)

CONTINUOUS_TARGETS = ("total_traffic", "source_load_vector", "destination_load_vector", "hotspot_strength", "sparsity",
                      "bandwidth_group_offered_load_vector")
POINT_METHODS = (*METHOD_NAMES, "selected_recent")
CANDIDATE_METHODS = ("recent_history_mlp", "causal_tcn")
PIPELINE_TRACE = ("fit", "validation_selection", "calibration_residuals", "test_evaluation", "lofo_refits")
SEED = 20260731
POINT_FIELDS = ("scope", "split", "held_out_family", "sequence_id", "family", "base_seed", "method", "target", "mae",
                "rmse", "r2", "spearman", "delta_rmse", "hotspot_accuracy", "acf_lag1", "ess", "raw_step_count",
                "previous_row_key")
PROBABILITY_FIELDS = ("scope", "held_out_family", "sequence_id", "family", "base_seed", "target", "coverage_numerator",
                      "coverage_denominator", "interval_width_sum", "scenario_coverage_numerator",
                      "scenario_coverage_denominator", "tail_event_count", "tail_true_positive_count")


def jsonable(v: Any) -> Any:
    if isinstance(v, dict):
        return {str(k): jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [jsonable(x) for x in v]
    if isinstance(v, np.ndarray):
        return jsonable(v.tolist())
    if isinstance(v, np.generic):
        return v.item()
    if isinstance(v, float) and not np.isfinite(v):
        raise ValueError("non-finite value in artifact")
    return v


def array_digest(a: np.ndarray) -> str:
    a = np.ascontiguousarray(np.asarray(a))
    h = hashlib.sha256()
    h.update(np.asarray(a.shape, dtype=np.int64).tobytes())
    h.update(a.dtype.str.encode("ascii"))
    h.update(a.tobytes())
    return h.hexdigest()


def target_slices(num_nodes: int, group_count: int) -> dict[str, slice]:
    widths = (1, num_nodes, num_nodes, 1, 1, group_count)
    edges = np.concatenate([[0], np.cumsum(widths)])
    return {k: slice(int(a), int(b)) for k, a, b in zip(CONTINUOUS_TARGETS, edges[:-1], edges[1:])}


# ---------------------------------------------------------------------------
# manifest
# ---------------------------------------------------------------------------
def _identities(records: Sequence[Mapping[str, Any]]) -> tuple[dict, dict]:
    ids = lambda pred: [str(r["sequence_id"]) for r in records if pred(r)]  # noqa: E731
    pooled = {f"{s}_sequence_ids": ids(lambda r, s=s: r["split"] == s) for s in SPLITS}
    lofo = {}
    for fam in dict.fromkeys(r["family"] for r in records):
        fold = {f"{s}_sequence_ids": ids(lambda r, s=s: r["split"] == s and r["family"] != fam)
                for s in ("fit", "validation", "calibration")}
        fold["test_sequence_ids"] = ids(lambda r: r["split"] == "test" and r["family"] == fam)
        lofo[str(fam)] = fold
    return pooled, lofo


def build_experiment_manifest(*, specs: Sequence[SequenceSpec], sequence_records: Sequence[Mapping[str, Any]],
                              protocol: Mapping[str, Any], source: Mapping[str, Any], command: Sequence[str],
                              environment: Mapping[str, Any], topology: Mapping[str, Any],
                              group_coefficients_digest: str) -> dict[str, Any]:
    by_id = {s.sequence_id: s for s in specs}
    if len(by_id) != len(specs):
        raise ValueError("duplicate sequence identity in specs")
    given: dict[str, Mapping[str, Any]] = {}
    for r in sequence_records:
        sid = str(r.get("sequence_id", ""))
        if not sid or sid in given:
            raise ValueError("duplicate or missing sequence identity in records")
        given[sid] = r
    if set(given) != set(by_id):
        raise ValueError("sequence record identities do not match specs")
    records = []
    for s in specs:
        if str(given[s.sequence_id].get("split")) != s.split:
            raise ValueError(f"split mismatch for {s.sequence_id}")
        records.append({"sequence_id": s.sequence_id, "family": s.family, "family_index": s.family_index,
                        "base_seed": s.base_seed, "seed_index": s.seed_index, "sequence_index": s.sequence_index,
                        "actual_seed": s.actual_seed, "split": s.split, "dynamics_variant": s.dynamics_variant,
                        "sequence_length": s.sequence_length, "generator_config": jsonable(s.generator_config),
                        "digest": str(given[s.sequence_id].get("digest", ""))})
    pooled, lofo = _identities(records)
    m = jsonable({"schema_version": 2, "protocol": dict(protocol), "source": dict(source), "command": list(command),
                  "environment": dict(environment), "topology": dict(topology),
                  "group_coefficients_digest": group_coefficients_digest,
                  "families": list(dict.fromkeys(r["family"] for r in records)),
                  "base_seeds": list(dict.fromkeys(r["base_seed"] for r in records)),
                  "methods": list(METHOD_NAMES), "point_methods": list(POINT_METHODS),
                  "continuous_targets": list(CONTINUOUS_TARGETS), "random_seed": SEED, "sequence_records": records,
                  "pooled_identity": pooled, "lofo_identities": lofo})
    validate_experiment_manifest(m)
    return m


def validate_experiment_manifest(m: Mapping[str, Any]) -> None:
    if m.get("schema_version") != 2:
        raise ValueError("manifest schema_version must be 2")
    recs = list(m["sequence_records"])
    for r in recs:
        d = str(r["digest"])
        if len(d) != 64 or set(d) - set("0123456789abcdef"):
            raise ValueError(f"invalid digest for {r['sequence_id']}")
    validate_split_records(recs)
    pooled, lofo = _identities(recs)
    if m["pooled_identity"] != pooled or m["lofo_identities"] != lofo:
        raise ValueError("manifest identities do not follow from the sequence records")
    if list(m["point_methods"]) != list(POINT_METHODS) or list(m["continuous_targets"]) != list(CONTINUOUS_TARGETS):
        raise ValueError("manifest method / target registry mismatch")


# ---------------------------------------------------------------------------
# execution
# ---------------------------------------------------------------------------
def _stack(ex: Mapping[str, HistoryExamples], ids: Sequence[str], field: str) -> np.ndarray:
    if not ids:
        raise ValueError(f"cannot stack empty sequence identity for {field}")
    return np.concatenate([np.asarray(getattr(ex[i], field)) for i in ids], axis=0)


def _predict(suite: HistoryPredictorSuite, e: HistoryExamples) -> dict[str, np.ndarray]:
    return suite.predict(e.moment_features, e.recent_history, e.previous_targets, e.ewma_targets)


def _rmse(a, b) -> float:
    return float(np.sqrt(np.mean((np.asarray(a) - np.asarray(b)) ** 2)))


def run_scope(*, scope: str, held_out_family: str, identity: Mapping[str, Sequence[str]],
              records: Mapping[str, Mapping[str, Any]], examples: Mapping[str, HistoryExamples],
              slices: Mapping[str, slice], seed: int = SEED) -> tuple[list[dict], list[dict], str]:
    fit_ids = list(identity["fit_sequence_ids"])
    r, y = _stack(examples, fit_ids, "recent_history"), _stack(examples, fit_ids, "targets")
    suite = HistoryPredictorSuite(r.shape[1], y.shape[1], seed=seed).fit(_stack(examples, fit_ids, "moment_features"),
                                                                         r, y)
    tot = slices["total_traffic"]
    points: list[dict] = []
    scores: dict[str, list[float]] = {m: [] for m in CANDIDATE_METHODS}
    for sid in identity["validation_sequence_ids"]:
        e, rec = examples[sid], records[sid]
        pred = _predict(suite, e)
        for m in CANDIDATE_METHODS:
            s = _rmse(pred[m][:, tot], e.targets[:, tot])
            scores[m].append(s)
            points.append({"scope": scope, "split": "validation", "held_out_family": held_out_family,
                           "sequence_id": sid, "family": rec["family"], "base_seed": rec["base_seed"], "method": m,
                           "target": "total_traffic", "rmse": s})
    backbone = select_recent_backbone({k: np.asarray(v) for k, v in scores.items()})

    cal_pts, cal_res = [], []
    for sid in identity["calibration_sequence_ids"]:
        e = examples[sid]
        p = _predict(suite, e)[backbone]
        cal_pts.append(p)
        cal_res.append(e.targets - p)
    cal = ResidualCalibrator(seed=seed, scenario_count=64).fit(np.concatenate(cal_pts), np.concatenate(cal_res))
    tail_thr = float(np.quantile(y[:, 0], 0.90, method="linear"))

    probs: list[dict] = []
    cursor = 0
    dst = slices["destination_load_vector"]
    for sid in identity["test_sequence_ids"]:
        e, rec = examples[sid], records[sid]
        pred = _predict(suite, e)
        n = len(e.targets)
        cp = cal.predict(pred[backbone], stable_example_indices=np.arange(cursor, cursor + n))
        cursor += n
        pred["quantile_scenario"] = cp.q50
        pred["selected_recent"] = pred[backbone]  # alias of the selected backbone, not a separate fit
        truth = {k: e.targets[:, s] for k, s in slices.items()}
        hot_true = hotspot_from_destination_loads(e.targets[:, dst])
        metrics = {m: sequence_target_metrics(truth, {k: pred[m][:, s] for k, s in slices.items()})
                   for m in POINT_METHODS}
        hot_acc = {m: float(np.mean(hotspot_from_destination_loads(pred[m][:, dst]) == hot_true))
                   for m in POINT_METHODS}
        total = truth["total_traffic"].reshape(-1)
        acf1 = float(autocorrelation(total, max_lag=1)[1])
        ess = float(positive_sequence_ess(total, max_lag=64))
        base = {"scope": scope, "held_out_family": held_out_family, "sequence_id": sid, "family": rec["family"],
                "base_seed": rec["base_seed"]}
        for m in POINT_METHODS:
            for t in CONTINUOUS_TARGETS:
                mt = metrics[m][t]
                points.append({**base, "split": "test", "method": m, "target": t, **mt,
                               "delta_rmse": metrics["previous_value"][t]["rmse"] - mt["rmse"],
                               "hotspot_accuracy": hot_acc[m], "acf_lag1": acf1, "ess": ess, "raw_step_count": n,
                               "previous_row_key": f"{scope}|{held_out_family}|{sid}|previous_value|{t}"})
        for t, s in slices.items():
            tr, lo, hi = truth[t], cp.q10[:, s], cp.q90[:, s]
            sc = cp.scenarios[:, :, s]
            slo = np.quantile(sc, 0.10, axis=1, method="linear")
            shi = np.quantile(sc, 0.90, axis=1, method="linear")
            if t == "total_traffic":
                ev = tr > tail_thr
                tp = ev & (hi > tail_thr)
            else:
                ev = tp = np.zeros(tr.shape, dtype=bool)
            probs.append({**base, "target": t, "coverage_numerator": int(np.sum((tr >= lo) & (tr <= hi))),
                          "coverage_denominator": int(tr.size), "interval_width_sum": float(np.sum(hi - lo)),
                          "scenario_coverage_numerator": int(np.sum((tr >= slo) & (tr <= shi))),
                          "scenario_coverage_denominator": int(tr.size), "tail_event_count": int(ev.sum()),
                          "tail_true_positive_count": int(tp.sum())})
    return points, probs, backbone


def probability_summary(rows: Sequence[Mapping[str, Any]]) -> dict[str, Any]:
    tot = lambda k: sum(int(r[k]) for r in rows)  # noqa: E731
    den, sden, ev, tp = (tot("coverage_denominator"), tot("scenario_coverage_denominator"), tot("tail_event_count"),
                         tot("tail_true_positive_count"))
    return {"coverage": tot("coverage_numerator") / den, "coverage_numerator": tot("coverage_numerator"),
            "coverage_denominator": den,
            "mean_interval_width": sum(float(r["interval_width_sum"]) for r in rows) / den,
            "scenario_coverage": tot("scenario_coverage_numerator") / sden,
            "scenario_coverage_numerator": tot("scenario_coverage_numerator"), "scenario_coverage_denominator": sden,
            "tail_event_count": ev, "tail_true_positive_count": tp, "tail_recall": tp / ev if ev else None,
            "tail_status": "ok" if ev >= 10 else "insufficient_events"}


def validation_selection(points: Sequence[Mapping[str, Any]], held_out_family: str = "") -> str:
    scope = "lofo" if held_out_family else "pooled"
    rows = [r for r in points if r["scope"] == scope and r["split"] == "validation"
            and r["held_out_family"] == held_out_family]
    return select_recent_backbone({m: np.asarray([float(r["rmse"]) for r in rows if r["method"] == m])
                                   for m in CANDIDATE_METHODS})


def recompute_summary(points: Sequence[Mapping[str, Any]], probs: Sequence[Mapping[str, Any]],
                      manifest: Mapping[str, Any], *, require_formal: bool) -> dict[str, Any]:
    validate_experiment_manifest(manifest)
    recs = list(manifest["sequence_records"])
    fams, seeds = list(manifest["families"]), [int(s) for s in manifest["base_seeds"]]
    if require_formal:
        counts = {s: sum(r["split"] == s for r in recs) for s in SPLITS}
        if (len(recs) != 75 or fams != list(FORMAL_FAMILIES) or seeds != list(FORMAL_BASE_SEEDS)
                or counts != {"fit": 30, "validation": 15, "calibration": 15, "test": 15}):
            raise ValueError("formal summary requires exact 75-sequence identity coverage")
    sel = [r for r in points if r["scope"] == "pooled" and r["split"] == "test" and r["method"] == "selected_recent"]
    ci = {}
    for t in PRIMARY_TARGETS:
        rows = [r for r in sel if r["target"] == t]
        b = family_stratified_paired_bootstrap(np.asarray([float(r["delta_rmse"]) for r in rows]),
                                               np.asarray([r["family"] for r in rows], dtype=object),
                                               samples=10_000, seed=SEED)
        ci[t] = {"mean": b.mean, "lower": b.lower, "upper": b.upper}
    tot = [r for r in sel if r["target"] == "total_traffic"]
    mean_of = lambda rows, key="delta_rmse": float(np.mean([float(r[key]) for r in rows]))  # noqa: E731
    seed_means = {str(s): mean_of([r for r in tot if int(r["base_seed"]) == s]) for s in seeds}
    fam_means = {f: mean_of([r for r in tot if r["family"] == f]) for f in fams}
    lofo_means, lofo_rel = {}, {}
    for f in fams:
        fold = [r for r in points if r["scope"] == "lofo" and r["held_out_family"] == f and r["split"] == "test"
                and r["target"] == "total_traffic"]
        s_rows = [r for r in fold if r["method"] == "selected_recent"]
        p_rows = [r for r in fold if r["method"] == "previous_value"]
        lofo_means[f] = mean_of(s_rows)
        lofo_rel[f] = mean_of(s_rows, "rmse") / mean_of(p_rows, "rmse") - 1.0
    pp_rows = [r for r in probs if r["scope"] == "pooled" and r["target"] == "total_traffic"]
    pooled = probability_summary(pp_rows)
    fam_cal = {f: abs(float(probability_summary([r for r in pp_rows if r["family"] == f])["coverage"]) - 0.80)
               for f in fams}
    exact_f, exact_s = set(fams) == set(FORMAL_FAMILIES), set(seeds) == set(FORMAL_BASE_SEEDS)
    lofo_agg = float(np.mean(list(lofo_means.values())))
    cond = {
        "condition_1": ci["total_traffic"]["lower"] > 0.0,
        "condition_2": exact_s and all(v > 0.0 for v in seed_means.values()) and exact_f
        and sum(v > 0.0 for v in fam_means.values()) >= 4,
        "condition_3": all(ci[t]["lower"] > 0.0 for t in PRIMARY_TARGETS),
        "condition_4": exact_f and lofo_agg >= 0.0 and sum(v > 0.0 for v in lofo_means.values()) >= 3
        and sum(v > 0.10 for v in lofo_rel.values()) <= 1,
        "condition_5": exact_f and abs(float(pooled["coverage"]) - 0.80) <= 0.05
        and all(v <= 0.10 for v in fam_cal.values()) and abs(float(pooled["scenario_coverage"]) - 0.80) <= 0.10,
        "condition_6": int(pooled["tail_event_count"]) >= 10 and pooled["tail_recall"] is not None
        and float(pooled["tail_recall"]) >= 0.70,
    }
    return jsonable({
        "schema_version": 2, "gate_status": "PENDING_SUPERVISOR", "pipeline_trace": list(PIPELINE_TRACE),
        "selected_backbone": validation_selection(points),
        "lofo_selected_backbones": {f: validation_selection(points, f) for f in fams},
        "calibration_sequence_ids": list(manifest["pooled_identity"]["calibration_sequence_ids"]),
        "identity_counts": {"families": len(fams), "base_seeds": len(seeds),
                            "pooled_test_sequences": len(manifest["pooled_identity"]["test_sequence_ids"]),
                            "lofo_test_sequences": sum(len(v["test_sequence_ids"])
                                                       for v in manifest["lofo_identities"].values()),
                            "point_methods": len(POINT_METHODS), "continuous_targets": len(CONTINUOUS_TARGETS)},
        "primary_delta_ci": ci, "seed_mean_deltas": seed_means, "family_mean_deltas": fam_means,
        "lofo": {"aggregate_mean_delta": lofo_agg, "family_mean_deltas": lofo_means,
                 "relative_rmse_changes": lofo_rel},
        "probability": {"pooled": pooled, "family_interval_calibration_errors": fam_cal},
        "conditions": {k: bool(v) for k, v in cond.items()},
    })


def execute(*, manifest: Mapping[str, Any], sequences: Mapping[str, Any], group_coefficients: np.ndarray,
            output_dir: str | Path | None, require_formal: bool) -> dict[str, Any]:
    recs = {r["sequence_id"]: r for r in manifest["sequence_records"]}
    if set(sequences) != set(recs):
        raise ValueError("generated sequence identities do not match manifest")
    ex = {sid: build_history_examples(s, group_coefficients=group_coefficients) for sid, s in sequences.items()}
    n = int(np.asarray(next(iter(sequences.values())).matrices[0]).shape[0])
    sl = target_slices(n, int(group_coefficients.shape[0]))
    points, probs, _ = run_scope(scope="pooled", held_out_family="", identity=manifest["pooled_identity"],
                                 records=recs, examples=ex, slices=sl)
    for fam, ident in manifest["lofo_identities"].items():
        p, q, _ = run_scope(scope="lofo", held_out_family=fam, identity=ident, records=recs, examples=ex, slices=sl)
        points += p
        probs += q
    out = {"manifest": jsonable(manifest), "point_rows": jsonable(points), "probability_rows": jsonable(probs),
           "summary": recompute_summary(points, probs, manifest, require_formal=require_formal)}
    if output_dir is not None:
        write_artifacts(output_dir, **out)
    return out


def write_artifacts(output_dir: str | Path, *, manifest, point_rows, probability_rows, summary) -> None:
    """manifest.json, the two raw CSV tables and summary.json (which must equal its recomputation)."""
    again = recompute_summary(point_rows, probability_rows, manifest,
                              require_formal=len(manifest["sequence_records"]) == 75)
    if jsonable(summary) != again:
        raise ValueError("summary does not equal raw+manifest recomputation")
    d = Path(output_dir)
    d.mkdir(parents=True, exist_ok=True)

    def dump(name, value):
        with (d / name).open("w", encoding="utf-8", newline="\n") as fh:
            json.dump(jsonable(value), fh, indent=2, sort_keys=True, ensure_ascii=False, allow_nan=False)
            fh.write("\n")

    def table(name, rows, fields):
        with (d / name).open("w", encoding="utf-8", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=list(fields), extrasaction="raise", lineterminator="\n")
            w.writeheader()
            w.writerows(rows)

    dump("manifest.json", manifest)
    table("raw_sequence_metrics.csv", point_rows, POINT_FIELDS)
    table("raw_probability_metrics.csv", probability_rows, PROBABILITY_FIELDS)
    dump("summary.json", again)


def _environment() -> dict[str, str]:
    return {"python": platform.python_version(), "numpy": np.__version__,
            "sklearn": importlib.metadata.version("scikit-learn"), "platform": platform.platform()}


def toy_specs(length: int = 48) -> list[SequenceSpec]:
    """The first two families at the first base seed, shortened to `length` steps."""
    out = []
    for s in build_formal_sequence_specs():
        if s.family in FORMAL_FAMILIES[:2] and s.base_seed == FORMAL_BASE_SEEDS[0]:
            cfg = dict(s.generator_config, sequence_length=length)
            out.append(replace(s, sequence_length=length, generator_config=cfg))
    return out


def run_toy_experiment(*, output_dir: str | Path | None = None, length: int = 48) -> dict[str, Any]:
    """The full four-split + LOFO pipeline on ten short generated sequences (seconds)."""
    specs = toy_specs(length)
    seqs = {s.sequence_id: generate_formal_sequence(s) for s in specs}
    recs = [{"sequence_id": s.sequence_id, "split": s.split, "digest": sequence_digest(seqs[s.sequence_id].matrices)}
            for s in specs]
    g = np.ones((1, 4, 4))
    np.fill_diagonal(g[0], 0.0)
    m = build_experiment_manifest(specs=specs, sequence_records=recs, protocol={"kind": "toy"},
                                  source={"kind": "toy"}, command=["run_toy_experiment"], environment=_environment(),
                                  topology={"name": "ToyComplete4"}, group_coefficients_digest=array_digest(g))
    return execute(manifest=m, sequences=seqs, group_coefficients=g, output_dir=output_dir, require_formal=False)


def run_formal_experiment(output_dir: str | Path = "outputs/h1_predictability") -> dict[str, Any]:
    """The frozen 75-sequence design on Rear4GPU's group coefficients."""
    specs = build_formal_sequence_specs()
    topo = load_topology_info("Rear4GPU")
    g = deterministic_group_coefficients(topo)
    seqs = {s.sequence_id: generate_formal_sequence(s) for s in specs}
    recs = [{"sequence_id": s.sequence_id, "split": s.split, "digest": sequence_digest(seqs[s.sequence_id].matrices)}
            for s in specs]
    m = build_experiment_manifest(specs=specs, sequence_records=recs, protocol={"kind": "formal"},
                                  source={"kind": "revealaiccl_b200.research.prediction"}, command=list(sys.argv),
                                  environment=_environment(), topology={"name": "Rear4GPU"},
                                  group_coefficients_digest=array_digest(g))
    return execute(manifest=m, sequences=seqs, group_coefficients=g, output_dir=output_dir, require_formal=True)


def read_artifacts(output_dir: str | Path) -> dict[str, Any]:
    """Read a bundle back and re-verify its summary from the raw tables."""
    d = Path(output_dir)
    manifest = json.loads((d / "manifest.json").read_text())
    summary = json.loads((d / "summary.json").read_text())

    def rows(name, ints, floats):
        out = []
        with (d / name).open(newline="") as fh:
            for r in csv.DictReader(fh):
                for k in list(r):
                    if r[k] == "":
                        del r[k]
                    elif k in ints:
                        r[k] = int(r[k])
                    elif k in floats:
                        r[k] = float(r[k])
                out.append(r)
        return out

    pts = rows("raw_sequence_metrics.csv", {"base_seed", "raw_step_count"},
               {"mae", "rmse", "r2", "spearman", "delta_rmse", "hotspot_accuracy", "acf_lag1", "ess"})
    for r in pts:
        r.setdefault("held_out_family", "")
    prs = rows("raw_probability_metrics.csv", {"base_seed", "coverage_numerator", "coverage_denominator",
                                               "scenario_coverage_numerator", "scenario_coverage_denominator",
                                               "tail_event_count", "tail_true_positive_count"},
               {"interval_width_sum"})
    for r in prs:
        r.setdefault("held_out_family", "")
    again = recompute_summary(pts, prs, manifest, require_formal=len(manifest["sequence_records"]) == 75)
    if again != summary:
        raise ValueError("artifact summary does not match its raw tables")
    return {"manifest": manifest, "point_rows": pts, "probability_rows": prs, "summary": summary}


def main(argv: Sequence[str] | None = None) -> None:
    import argparse
    ap = argparse.ArgumentParser(description="history-only traffic prediction study")
    ap.add_argument("--toy", action="store_true", help="ten short sequences instead of the 75-sequence design")
    ap.add_argument("--output-dir", default="outputs/h1_predictability")
    a = ap.parse_args(argv)
    res = run_toy_experiment(output_dir=a.output_dir) if a.toy else run_formal_experiment(a.output_dir)
    print(json.dumps(res["summary"]["conditions"], sort_keys=True))


if __name__ == "__main__":
    main()
