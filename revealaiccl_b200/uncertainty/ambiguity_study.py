"""Phase-3B empirical-ambiguity study: design, case evaluation, statistics, gate.

The study asks whether a small support selected from an empirical ambiguity
set (``ambiguity.py``) represents the unknown traffic matrix of a partially
revealed step well, and whether the chosen selector beats random sampling of
the same set.  It follows the frozen protocol of
rlccl/uncertainty/ambiguity_experiment.py (constants :51-94, sequence design
:212-248, registry :308-352, observation model :1562-1655, calibration
:370-440, validation selection :487-529, case metrics :566-686, bootstrap
:819-861, gate :880-982); the pipeline here is this package's own:

* ``build_sequence_specs`` — 5 long-horizon families x 3 base seeds x 5 splits
  (fit, fit, validation, calibration, test), Rear4GPU, 1024 steps;
* ``observe`` — one matrix revealed by mode and ratio with a seeded entry
  order (the order of random draws is part of the protocol, so equal seeds
  give equal observations);
* calibration: per sequence the 0.9 quantile ("higher") of the exceedance
  score of the history box, then the 0.9 quantile over sequences, gives the
  radius that widens every ambiguity box;
* validation: the ordinary selector with the smallest mean nearest-RMS
  distance at K = 8 over unknown ratios (ties in a fixed order);
* test: every case (checkpoint x mode x ratio x K x method; random sampling
  averaged over 8 replicates) scored with ``case_metrics``; per sequence the
  selected method's mean distance minus random's is the paired delta, with a
  family-stratified bootstrap CI (10,000 resamples, seed 20260731);
* leave-one-family-out folds, a six-condition gate, CSV/JSON artifacts that
  ``recompute_summary`` rebuilds from the raw rows and compares.

``run_study(scale=...)``: ``"formal"`` is the full protocol; ``"quick"`` keeps
every structure but fewer checkpoints, sequences per family and K values, for
a run in minutes; ``"toy"`` is a one-sequence smoke run.

    python -m revealaiccl_b200.uncertainty.ambiguity_study --scale quick --out out/phase3b
"""

from __future__ import annotations

import argparse
import csv
import hashlib
import json
import math
import time
from collections import defaultdict
from dataclasses import asdict, dataclass, fields
from pathlib import Path
from typing import Any, Mapping, Sequence

import numpy as np

from ..traffic.long_horizon import LONG_HORIZON_FAMILIES, SAME_MOMENT_VARIANTS, LongHorizonTrafficConfig
from .ambiguity import (
    HISTORY_WINDOW,
    AmbiguityConstructionView,
    build_empirical_ambiguity_set,
    descriptor_names,
    fit_descriptor_normalizer,
    oracle_support_upper_bound,
    physical_descriptor_bounds,
    select_support,
    support_covering_radius,
    traffic_descriptor,
)
from .observation import PartialObservationState, PublicTopologyView

# ---------------------------------------------------------------------------
# protocol constants (preregistered; changing one changes the study)
# ---------------------------------------------------------------------------
FAMILIES = tuple(LONG_HORIZON_FAMILIES)
BASE_SEEDS = (342, 442, 542)
SPLITS = ("fit", "fit", "validation", "calibration", "test")
SEQUENCE_LENGTH = 1024
MAX_ENTRY = 8
CHECKPOINTS = tuple(range(32, 993, 64))
REVEAL_MODES = ("random_entries", "source_totals_first", "source_destination_totals_first", "partial_shards",
                "time_based_arrival")
REVEAL_RATIOS = (0.0, 0.25, 0.5, 0.75, 1.0)
UNKNOWN_RATIOS = REVEAL_RATIOS[:-1]
REQUESTED_K = (1, 4, 8, 16)
ORDINARY_METHODS = ("random_empirical", "worst_recent_cases", "boundary_scenarios", "minimax_subset")
ALL_METHODS = ORDINARY_METHODS + ("oracle_support_upper_bound",)
TIE_ORDER = ("minimax_subset", "boundary_scenarios", "worst_recent_cases", "random_empirical")
RANDOM_REPLICATES = 8
SELECTION_K = 8
BOOTSTRAP_REPLICATES = 10_000
BOOTSTRAP_SEED = 20260731
CALIBRATION_QUANTILE = 0.9


def observation_seed(record_index: int, checkpoint: int, mode_index: int) -> int:
    return 31_000_000 + int(record_index) * 100_000 + int(checkpoint) * 10 + int(mode_index)


def replicate_seed(case_index: int, replicate: int) -> int:
    if not 0 <= int(replicate) < RANDOM_REPLICATES:
        raise ValueError("replicate index outside [0, 8)")
    return 41_000_000 + int(case_index) * 100 + int(replicate)


# ---------------------------------------------------------------------------
# design
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class SequenceSpec:
    sequence_id: str
    family: str
    base_seed: int
    seed_index: int
    sequence_index: int
    seed: int
    split: str
    variant: str | None
    record_index: int

    def generator_config(self, length: int = SEQUENCE_LENGTH) -> LongHorizonTrafficConfig:
        return LongHorizonTrafficConfig(num_nodes=4, sequence_length=length, family=self.family, seed=self.seed,
                                        mean_level=2.0, std_level=1.5, max_entry=MAX_ENTRY,
                                        calibration_candidates=1, topology_name="Rear4GPU",
                                        dynamics_variant=self.variant)


def build_sequence_specs() -> tuple[SequenceSpec, ...]:
    """All 75 sequence specifications (no traffic is generated here)."""
    out = []
    for fi, fam in enumerate(FAMILIES):
        for si, base in enumerate(BASE_SEEDS):
            for qi, split in enumerate(SPLITS):
                seed = base + fi * 1_000_000 + qi * 10_000
                variant = SAME_MOMENT_VARIANTS[(si + qi) % 4] if fam == "same_moments_different_dynamics" else None
                out.append(SequenceSpec(f"{fam}-base{base}-sequence{qi}-seed{seed}", fam, base, si, qi, seed, split,
                                        variant, len(out)))
    return tuple(out)


@dataclass(frozen=True)
class StudyScale:
    """How much of the protocol a run evaluates."""
    name: str
    checkpoints: tuple[int, ...]
    bases: tuple[int, ...]                 # base seeds kept (sequences per family and split)
    families: tuple[str, ...]
    requested_k: tuple[int, ...]
    bootstrap_replicates: int
    sequence_length: int

    @classmethod
    def named(cls, name: str) -> "StudyScale":
        if name == "formal":
            return cls(name, CHECKPOINTS, BASE_SEEDS, FAMILIES, REQUESTED_K, BOOTSTRAP_REPLICATES, SEQUENCE_LENGTH)
        if name == "quick":
            return cls(name, CHECKPOINTS[::5], BASE_SEEDS, FAMILIES, (4, 8), 2000, SEQUENCE_LENGTH)
        if name == "toy":
            return cls(name, (32, 96), BASE_SEEDS[:1], FAMILIES[:1], (8,), 200, 160)
        raise ValueError(f"unknown study scale {name!r}")


def case_identities(specs: Sequence[SequenceSpec], scale: StudyScale) -> list[tuple[str, int, int, int, int, int]]:
    """(split, record, checkpoint, mode, stage, K) of every evaluated case, sorted;
    fit sequences never enter evaluation.  Case indices are positions here."""
    out = [(s.split, s.record_index, cp, mi, st, k) for s in specs if s.split != "fit"
           for cp in scale.checkpoints for mi in range(len(REVEAL_MODES))
           for st in range(len(REVEAL_RATIOS)) for k in scale.requested_k]
    out.sort()
    if len(set(out)) != len(out):
        raise ValueError("duplicate case identity")
    return out


# ---------------------------------------------------------------------------
# observation model
# ---------------------------------------------------------------------------
def observe(matrix: Any, *, mode: str, ratio: float, seed: int, topology: PublicTopologyView,
            sequence_id: str = "", step: int = 0, family: str = "") -> tuple[PartialObservationState, float]:
    """Reveal one matrix: a seeded order of the off-diagonal entries (and an
    arrival time each, drawn for every mode), then by mode: the first
    floor(ratio n) entries, the entries that arrived by `ratio`, or (partial
    shards) a seeded prefix of the unit tokens, an entry exact once all its
    units are seen.  Totals modes add the source (and destination) totals.
    Returns the observation and the fraction of off-diagonal entries exact."""
    x = np.asarray(matrix, dtype=np.int64)
    n = x.shape[0]
    off = [(i, j) for i in range(n) for j in range(n) if i != j]
    rng = np.random.default_rng(int(seed))
    order = np.asarray(off, dtype=np.int64)[rng.permutation(len(off))]
    arrival = rng.uniform(np.nextafter(0.0, 1.0), 1.0, size=len(off))
    mask = np.eye(n, dtype=bool)
    seen = np.zeros_like(x)
    full = ratio == 1.0
    if mode == "partial_shards":
        units = np.repeat(np.asarray(off, dtype=np.int64), [int(x[i, j]) for i, j in off], axis=0)
        if len(units):
            units = units[rng.permutation(len(units))]
        take = len(units) if full else int(math.floor(ratio * len(units)))
        if take:
            np.add.at(seen, (units[:take, 0], units[:take, 1]), 1)
        if full:
            mask[:] = True
            seen = x.copy()
        else:
            for i, j in off:
                if x[i, j] > 0 and seen[i, j] == x[i, j]:
                    mask[i, j] = True
    else:
        if mode == "time_based_arrival":
            chosen = order if full else order[arrival <= ratio]
        else:
            chosen = order[: len(order) if full else int(math.floor(ratio * len(order)))]
        if len(chosen):
            mask[chosen[:, 0], chosen[:, 1]] = True
        seen[mask] = x[mask]
    src = x.sum(axis=1) if mode in ("source_totals_first", "source_destination_totals_first") else None
    dst = x.sum(axis=0) if mode == "source_destination_totals_first" else None
    frac = float(np.count_nonzero(mask & ~np.eye(n, dtype=bool)) / len(off))
    obs = PartialObservationState(sequence_id=sequence_id, sequence_step=int(step), family=family, mode=mode,
                                  stage=REVEAL_RATIOS.index(float(ratio)), ratio=float(ratio), entry_mask=mask,
                                  observed_matrix=seen, unknown_mask=~mask, revealed_tokens=(), source_totals=src,
                                  destination_totals=dst, topology=topology, state_version=0)
    return obs, frac


def construction_view(matrices: Sequence[np.ndarray], spec: SequenceSpec, *, checkpoint: int, mode_index: int,
                      ratio: float, topology: PublicTopologyView, normalizer: Any) -> tuple[AmbiguityConstructionView, float]:
    seed = observation_seed(spec.record_index, checkpoint, mode_index)
    obs, frac = observe(matrices[checkpoint], mode=REVEAL_MODES[mode_index], ratio=ratio, seed=seed,
                        topology=topology, sequence_id=spec.sequence_id, step=checkpoint, family=spec.family)
    view = AmbiguityConstructionView.from_observation(
        history_matrices=tuple(matrices[checkpoint - HISTORY_WINDOW: checkpoint]),
        history_offsets=tuple(range(-HISTORY_WINDOW, 0)), observation=obs, construction_seed=seed,
        normalizer=normalizer)
    return view, frac


# ---------------------------------------------------------------------------
# scores and metrics
# ---------------------------------------------------------------------------
def exceedance_score(lower: Any, upper: Any, descriptor: Any, scale: Any) -> float:
    """Largest scaled distance of the descriptor outside [lower, upper] (0 inside)."""
    lo, hi, v, s = (np.asarray(a, dtype=np.float64) for a in (lower, upper, descriptor, scale))
    if not (lo.shape == hi.shape == v.shape == s.shape) or lo.ndim != 1:
        raise ValueError("descriptor / bound shape mismatch")
    if not all(np.isfinite(a).all() for a in (lo, hi, v, s)) or np.any(s <= 0) or np.any(lo > hi):
        raise ValueError("calibration inputs must be finite with positive scale and ordered bounds")
    return float(np.max(np.maximum(np.maximum(lo - v, v - hi) / s, 0.0)))


def calibration_radius(rows: Sequence[Mapping[str, Any]], *, exclude_family: str | None = None) -> float:
    per_seq: dict[str, list[float]] = defaultdict(list)
    for r in rows:
        if exclude_family is None or r["family"] != exclude_family:
            per_seq[str(r["sequence_id"])].append(float(r["score"]))
    if not per_seq:
        raise ValueError("no calibration rows")
    q = [float(np.quantile(np.asarray(v), CALIBRATION_QUANTILE, method="higher")) for _, v in sorted(per_seq.items())]
    return float(np.quantile(np.asarray(q), CALIBRATION_QUANTILE, method="higher"))


@dataclass(frozen=True)
class CaseMetrics:
    nearest_rms_distance: float
    nearest_matrix_l1_distance: int
    covering_radius: float
    mean_pairwise_diversity: float
    duplicate_fraction: float
    actual_k: int
    requested_k: int
    component_coverage: float
    joint_coverage: int
    physical_normalized_mean_width: float
    zero_physical_range_components: int
    total_tail_events: int
    total_tail_hits: int
    group_tail_events: int
    group_tail_hits: int
    hotspot_event: int
    hotspot_hit: int


@dataclass(frozen=True)
class TailThresholds:
    total_index: int
    total: float
    group_indices: tuple[int, ...]
    groups: np.ndarray


def tail_thresholds(fit_descriptors: np.ndarray, topology: PublicTopologyView) -> TailThresholds:
    """Upper-tail thresholds from the fit split: the 0.9 quantile of the total
    load and of every bandwidth-group load descriptor."""
    names = descriptor_names(topology)
    ti = names.index("total_traffic")
    gi = tuple(i for i, nm in enumerate(names) if nm.startswith("bandwidth_group_load_"))
    d = np.asarray(fit_descriptors, dtype=np.float64)
    return TailThresholds(ti, float(np.quantile(d[:, ti], 0.9)), gi,
                          np.asarray([np.quantile(d[:, i], 0.9) for i in gi], dtype=np.float64))


def _rms(a: np.ndarray, b: np.ndarray, s: np.ndarray) -> float:
    return float(np.sqrt(np.mean(((a - b) / s) ** 2)))


def _hotspot(matrix: np.ndarray) -> int:
    m = np.asarray(matrix, dtype=np.int64).copy()
    np.fill_diagonal(m, 0)
    return int(np.argmax(m.sum(axis=0)))


def case_metrics(ambiguity: Any, support: Any, truth: Any, *, physical: tuple[np.ndarray, np.ndarray],
                 tails: TailThresholds, truth_in_observation: bool = True) -> CaseMetrics:
    """How well `support` represents the truth, and what the ambiguity box covers."""
    topo = ambiguity.topology
    scale = ambiguity.normalizer.scale
    t = np.asarray(truth, dtype=np.int64)
    tv = traffic_descriptor(t, topo)
    sv = np.asarray(support.descriptor_vectors, dtype=np.float64)
    mats = [np.asarray(m, dtype=np.int64) for m in support.matrices]
    offd = ~np.eye(t.shape[0], dtype=bool)
    near = min(_rms(tv, v, scale) for v in sv)
    l1 = min(int(np.abs(t[offd] - m[offd]).sum()) for m in mats)
    pair = [_rms(sv[a], sv[b], scale) for a in range(len(sv)) for b in range(a + 1, len(sv))]
    unique = len({hashlib.sha256(np.ascontiguousarray(m).tobytes()).hexdigest() for m in mats})
    lo, hi = ambiguity.lower_bounds, ambiguity.upper_bounds
    inside = (tv >= lo - 1.000001e-10) & (tv <= hi + 1.000001e-10)
    plo, phi = physical
    rng = phi - plo
    pos = rng > 0
    tev = int(tv[tails.total_index] > tails.total)
    thit = int(tev and sv[:, tails.total_index].max() > tails.total)
    gev = ghit = 0
    for idx, thr in zip(tails.group_indices, tails.groups):
        ev = int(tv[idx] > thr)
        gev += ev
        ghit += int(ev and sv[:, idx].max() > thr)
    return CaseMetrics(
        nearest_rms_distance=float(near), nearest_matrix_l1_distance=l1,
        covering_radius=support_covering_radius(ambiguity, support) if not support.uses_oracle else 0.0,
        mean_pairwise_diversity=float(np.mean(pair)) if pair else 0.0,
        duplicate_fraction=1.0 - unique / len(mats), actual_k=len(mats), requested_k=int(support.requested_k),
        component_coverage=float(inside.mean()), joint_coverage=int(bool(inside.all()) and truth_in_observation),
        physical_normalized_mean_width=float(np.mean((hi[pos] - lo[pos]) / rng[pos])) if pos.any() else 0.0,
        zero_physical_range_components=int((~pos).sum()), total_tail_events=tev, total_tail_hits=thit,
        group_tail_events=gev, group_tail_hits=ghit, hotspot_event=1,
        hotspot_hit=int(_hotspot(t) in {_hotspot(m) for m in mats}))


def _mean_metrics(values: Sequence[CaseMetrics]) -> dict[str, float]:
    return {f.name: float(np.mean([getattr(v, f.name) for v in values])) for f in fields(CaseMetrics)}


# ---------------------------------------------------------------------------
# selection, statistics, gate
# ---------------------------------------------------------------------------
def select_method(rows: Sequence[Mapping[str, Any]]) -> tuple[str, dict[str, float]]:
    """The ordinary selector with the smallest mean (over sequences of the mean
    over cases) nearest-RMS distance at K = 8 and unknown ratios."""
    if any(r["method"] == "oracle_support_upper_bound" or r.get("uses_oracle") for r in rows):
        raise ValueError("oracle rows cannot take part in the selection")
    per: dict[tuple[str, str], list[float]] = defaultdict(list)
    for r in rows:
        if r["method"] in ORDINARY_METHODS and int(r["requested_k"]) == SELECTION_K and float(r["reveal_ratio"]) < 1.0:
            per[(str(r["sequence_id"]), str(r["method"]))].append(float(r["nearest_rms_distance"]))
    seqs = sorted({s for s, _ in per})
    if not seqs:
        raise ValueError("no validation rows at K = 8")
    means = {}
    for m in ORDINARY_METHODS:
        if any((s, m) not in per for s in seqs):
            raise ValueError(f"validation rows incomplete for {m}")
        means[m] = float(np.mean([np.mean(per[(s, m)]) for s in seqs]))
    best = min(means.values())
    return next(m for m in TIE_ORDER if abs(means[m] - best) <= 1e-12), means


def paired_deltas(seq_rows: Sequence[Mapping[str, Any]], method: str, k: int = SELECTION_K) -> list[dict[str, Any]]:
    """Per sequence: random's mean nearest distance minus the method's (positive:
    the method represents the truth better than random sampling)."""
    by = {(r["sequence_id"], r["method"]): r for r in seq_rows if int(r["requested_k"]) == k}
    out = []
    for (sid, m), r in sorted(by.items()):
        if m != method:
            continue
        rnd = by.get((sid, "random_empirical"))
        if rnd is None:
            raise ValueError(f"no random rows for {sid}")
        out.append({"sequence_id": sid, "family": r["family"], "base_seed": r["base_seed"],
                    "paired_delta": float(rnd["nearest_rms_distance"]) - float(r["nearest_rms_distance"])})
    return out


def family_bootstrap(deltas: Sequence[Mapping[str, Any]], *, replicates: int = BOOTSTRAP_REPLICATES,
                     seed: int = BOOTSTRAP_SEED) -> dict[str, Any]:
    """Mean paired delta and its 95% percentile CI, resampling sequences within
    each family (families kept fixed)."""
    fam: dict[str, list[float]] = defaultdict(list)
    for r in sorted(deltas, key=lambda r: (r["family"], int(r["base_seed"]), r["sequence_id"])):
        fam[str(r["family"])].append(float(r["paired_delta"]))
    if not fam:
        raise ValueError("no paired deltas")
    groups = [np.asarray(fam[f]) for f in sorted(fam)]
    rng = np.random.default_rng(int(seed))
    draws = np.empty(int(replicates))
    for b in range(int(replicates)):
        draws[b] = np.mean(np.concatenate([g[rng.integers(0, len(g), size=len(g))] for g in groups]))
    allv = np.concatenate(groups)
    return {"sequence_count": int(allv.size), "family_count": len(groups), "replicates": int(replicates),
            "seed": int(seed), "mean_delta": float(allv.mean()), "ci_lower": float(np.quantile(draws, 0.025)),
            "ci_upper": float(np.quantile(draws, 0.975))}


@dataclass(frozen=True)
class GateDecision:
    data_status: str                      # PASS / FAIL / HOLD
    failed_conditions: tuple[int, ...]
    insufficient_conditions: tuple[int, ...]


def _rate(hits: float, events: float) -> float:
    if events <= 0 or hits < 0 or hits > events:
        raise ValueError("invalid event / hit counts")
    return hits / events


def evaluate_gate(ev: Mapping[str, Any]) -> GateDecision:
    """The six conditions: (1) joint coverage >= 0.85 overall and >= 0.80 in
    every family; (2) paired-delta CI above 0, every base seed positive, at
    least 4 of 5 families positive; (3) LOFO aggregate >= 0, at least 3
    families positive, at most one family degraded by more than 10 %; (4)
    total / group / hotspot tail recall >= 0.70 with at least 10 events each
    (else HOLD); (5) mean normalised width <= 0.75, no invalid ordinary case,
    singleton coverage 1 at ratio 1, finite timings; (6) integrity checks."""
    failed, insufficient = [], []
    if not (ev["selected_joint_coverage"] >= 0.85 and ev["selected_joint_coverage_by_family"]
            and all(v >= 0.80 for v in ev["selected_joint_coverage_by_family"].values())):
        failed.append(1)
    fam = list(ev["paired_delta_by_family"].values())
    if not (ev["paired_delta_ci95"][0] > 0 and ev["paired_delta_by_base_seed"]
            and all(v > 0 for v in ev["paired_delta_by_base_seed"].values())
            and sum(v > 0 for v in fam) >= min(4, len(fam))):
        failed.append(2)
    lofo = list(ev["lofo_delta_by_family"].values())
    degr = list(ev["lofo_relative_degradation_by_family"].values())
    if not (ev["lofo_aggregate_delta"] >= 0 and sum(v > 0 for v in lofo) >= min(3, len(lofo))
            and sum(v > 0.10 for v in degr) <= 1):
        failed.append(3)
    if ev["total_tail_events"] < 10 or ev["group_tail_events"] < 10:
        insufficient.append(4)
    elif not (_rate(ev["total_tail_hits"], ev["total_tail_events"]) >= 0.70
              and _rate(ev["group_tail_hits"], ev["group_tail_events"]) >= 0.70
              and _rate(ev["hotspot_hits"], ev["hotspot_events"]) >= 0.70):
        failed.append(4)
    if not (ev["selected_mean_physical_normalized_width"] <= 0.75
            and all(v == 0.0 for v in ev["ordinary_invalid_or_empty_rate"].values())
            and ev["ratio1_singleton_coverage"] == 1.0 and ev["all_timings_finite"]):
        failed.append(5)
    if not (ev["integrity_checks_complete"] and ev["integrity_checks_passed"]):
        failed.append(6)
    status = "FAIL" if failed else ("HOLD" if insufficient else "PASS")
    return GateDecision(status, tuple(failed), tuple(insufficient))


# ---------------------------------------------------------------------------
# the pipeline
# ---------------------------------------------------------------------------
class _Study:
    def __init__(self, scale: StudyScale, topology: Any) -> None:
        from ..traffic.long_horizon import generate_long_horizon_sequence

        self.scale = scale
        self.topo = topology if isinstance(topology, PublicTopologyView) \
            else PublicTopologyView.from_topology_info(topology)
        self.specs = tuple(s for s in build_sequence_specs()
                           if s.family in scale.families and s.base_seed in scale.bases)
        self.mats: dict[str, list[np.ndarray]] = {}
        self.digests: dict[str, str] = {}
        for s in self.specs:
            seq = generate_long_horizon_sequence(s.generator_config(scale.sequence_length))
            self.mats[s.sequence_id] = [np.asarray(m, dtype=np.int64) for m in seq.matrices]
            self.digests[s.sequence_id] = hashlib.sha256(np.ascontiguousarray(
                np.stack(self.mats[s.sequence_id])).tobytes()).hexdigest()
        if len(set(self.digests.values())) != len(self.digests):
            raise ValueError("two sequences of the design are identical")
        fit = [m for s in self.specs if s.split == "fit" for m in self.mats[s.sequence_id]]
        self.normalizer = fit_descriptor_normalizer(fit, self.topo)
        self.physical = physical_descriptor_bounds(self.topo, max_entry=MAX_ENTRY)
        self.tails = tail_thresholds(np.stack([traffic_descriptor(m, self.topo) for m in fit]), self.topo)
        self.case_index = {ident: i for i, ident in enumerate(case_identities(self.specs, scale))}

    def _split(self, name: str, family: str | None = None, exclude: str | None = None) -> list[SequenceSpec]:
        return [s for s in self.specs if s.split == name and (family is None or s.family == family)
                and (exclude is None or s.family != exclude)]

    def calibration_rows(self) -> list[dict[str, Any]]:
        rows = []
        for s in self._split("calibration"):
            for cp in self.scale.checkpoints:
                truth = traffic_descriptor(self.mats[s.sequence_id][cp], self.topo)
                for mi, mode in enumerate(REVEAL_MODES):
                    for ratio in UNKNOWN_RATIOS:
                        view, _ = construction_view(self.mats[s.sequence_id], s, checkpoint=cp, mode_index=mi,
                                                    ratio=ratio, topology=self.topo, normalizer=self.normalizer)
                        raw = build_empirical_ambiguity_set(view, calibration_radius=0.0)
                        rows.append({"sequence_id": s.sequence_id, "family": s.family, "checkpoint": cp,
                                     "reveal_mode": mode, "reveal_ratio": ratio,
                                     "score": exceedance_score(raw.lower_bounds, raw.upper_bounds, truth,
                                                               self.normalizer.scale)})
        return rows

    def case_rows(self, specs: Sequence[SequenceSpec], radius: float, methods: Sequence[str],
                  ratios: Sequence[float] = REVEAL_RATIOS) -> list[dict[str, Any]]:
        rows = []
        for s in specs:
            mats = self.mats[s.sequence_id]
            for cp in self.scale.checkpoints:
                truth = mats[cp]
                for mi, mode in enumerate(REVEAL_MODES):
                    for st, ratio in enumerate(REVEAL_RATIOS):
                        if ratio not in ratios:
                            continue
                        view, frac = construction_view(mats, s, checkpoint=cp, mode_index=mi, ratio=ratio,
                                                       topology=self.topo, normalizer=self.normalizer)
                        t0 = time.perf_counter()
                        amb = build_empirical_ambiguity_set(view, calibration_radius=radius)
                        t_build = time.perf_counter() - t0
                        for k in self.scale.requested_k:
                            ci = self.case_index[(s.split, s.record_index, cp, mi, st, k)]
                            for m in methods:
                                t1 = time.perf_counter()
                                if m == "random_empirical" and ratio < 1.0:
                                    met = _mean_metrics([case_metrics(
                                        amb, select_support(amb, method=m, k=k, replicate_seed=replicate_seed(ci, r)),
                                        truth, physical=self.physical, tails=self.tails)
                                        for r in range(RANDOM_REPLICATES)])
                                else:
                                    sup = (oracle_support_upper_bound(amb, truth=truth, k=k)
                                           if m == "oracle_support_upper_bound" else
                                           select_support(amb, method=m, k=k,
                                                          **({"replicate_seed": replicate_seed(ci, 0)}
                                                             if m == "random_empirical" else {})))
                                    met = asdict(case_metrics(amb, sup, truth, physical=self.physical,
                                                              tails=self.tails))
                                rows.append({"case_index": ci, "sequence_id": s.sequence_id, "split": s.split,
                                             "family": s.family, "base_seed": s.base_seed, "checkpoint": cp,
                                             "reveal_mode": mode, "reveal_ratio": ratio, "entry_fraction": frac,
                                             "requested_k": k, "method": m, **met,
                                             "uses_oracle": m == "oracle_support_upper_bound", "invalid_or_empty": 0,
                                             "construction_seconds": t_build,
                                             "selector_seconds": time.perf_counter() - t1,
                                             "sequence_digest": self.digests[s.sequence_id]})
        return rows


def sequence_rows(case_rows: Sequence[Mapping[str, Any]]) -> list[dict[str, Any]]:
    """Per (sequence, method, K) over unknown ratios: mean nearest distance and
    the tail / hotspot event and hit sums."""
    g: dict[tuple[str, str, int], list[Mapping[str, Any]]] = defaultdict(list)
    for r in case_rows:
        if float(r["reveal_ratio"]) < 1.0:
            g[(str(r["sequence_id"]), str(r["method"]), int(r["requested_k"]))].append(r)
    out = []
    for (sid, m, k), rs in sorted(g.items()):
        sums = {key: float(sum(float(r[key]) for r in rs)) for key in
                ("total_tail_events", "total_tail_hits", "group_tail_events", "group_tail_hits", "hotspot_event",
                 "hotspot_hit", "joint_coverage")}
        out.append({"sequence_id": sid, "method": m, "requested_k": k, "family": rs[0]["family"],
                    "base_seed": rs[0]["base_seed"], "cases": len(rs),
                    "nearest_rms_distance": float(np.mean([float(r["nearest_rms_distance"]) for r in rs])),
                    "joint_coverage": sums["joint_coverage"] / len(rs),
                    "physical_normalized_mean_width": float(np.mean([float(r["physical_normalized_mean_width"])
                                                                     for r in rs])),
                    **{k2: v for k2, v in sums.items() if k2 != "joint_coverage"}})
    return out


def _evidence(test_cases, test_seq, selected, boot, lofo) -> dict[str, Any]:
    sel = [r for r in test_cases if r["method"] == selected and int(r["requested_k"]) == SELECTION_K
           and float(r["reveal_ratio"]) < 1.0]
    fams = sorted({r["family"] for r in sel})
    deltas = paired_deltas(test_seq, selected)
    by_fam = {f: float(np.mean([d["paired_delta"] for d in deltas if d["family"] == f])) for f in fams}
    by_seed = {str(b): float(np.mean([d["paired_delta"] for d in deltas if int(d["base_seed"]) == b]))
               for b in sorted({int(d["base_seed"]) for d in deltas})}
    ratio1 = [r for r in test_cases if float(r["reveal_ratio"]) == 1.0 and r["method"] in ORDINARY_METHODS]
    ordinary = [r for r in test_cases if r["method"] in ORDINARY_METHODS]
    return {
        "selected_joint_coverage": float(np.mean([r["joint_coverage"] for r in sel])),
        "selected_joint_coverage_by_family": {f: float(np.mean([r["joint_coverage"] for r in sel
                                                                if r["family"] == f])) for f in fams},
        "paired_delta_ci95": [boot["ci_lower"], boot["ci_upper"]],
        "paired_delta_by_base_seed": by_seed, "paired_delta_by_family": by_fam,
        "lofo_aggregate_delta": lofo["aggregate_delta"], "lofo_delta_by_family": lofo["delta_by_family"],
        "lofo_relative_degradation_by_family": lofo["relative_degradation_by_family"],
        "total_tail_events": int(sum(r["total_tail_events"] for r in sel)),
        "total_tail_hits": float(sum(r["total_tail_hits"] for r in sel)),
        "group_tail_events": int(sum(r["group_tail_events"] for r in sel)),
        "group_tail_hits": float(sum(r["group_tail_hits"] for r in sel)),
        "hotspot_events": int(sum(r["hotspot_event"] for r in sel)),
        "hotspot_hits": float(sum(r["hotspot_hit"] for r in sel)),
        "selected_mean_physical_normalized_width": float(np.mean([r["physical_normalized_mean_width"] for r in sel])),
        "ordinary_invalid_or_empty_rate": {m: float(np.mean([r["invalid_or_empty"] for r in ordinary
                                                             if r["method"] == m])) for m in ORDINARY_METHODS},
        "ratio1_singleton_coverage": float(np.mean([r["joint_coverage"] for r in ratio1])) if ratio1 else 0.0,
        "all_timings_finite": all(math.isfinite(r["construction_seconds"]) and math.isfinite(r["selector_seconds"])
                                  for r in test_cases),
        "integrity_checks_complete": True,
        "integrity_checks_passed": len({r["sequence_digest"] for r in test_cases}) == len(
            {r["sequence_id"] for r in test_cases}),
    }


def recompute_summary(raw: Mapping[str, Sequence[Mapping[str, Any]]], *, bootstrap_replicates: int) -> dict[str, Any]:
    """Everything of the summary, rebuilt from the raw tables alone."""
    radius = calibration_radius(raw["calibration"])
    selected, means = select_method(raw["validation"])
    test_seq = sequence_rows(raw["test"])
    boot = family_bootstrap(paired_deltas(test_seq, selected), replicates=bootstrap_replicates)
    lofo = lofo_summary(raw["lofo"])
    ev = _evidence(raw["test"], test_seq, selected, boot, lofo)
    gate = evaluate_gate(ev)
    return {"calibration_radius": radius, "selected_method": selected, "selected_k": SELECTION_K,
            "validation_means": means, "bootstrap": boot, "lofo": lofo, "evidence": ev,
            "data_status": gate.data_status, "failed_conditions": list(gate.failed_conditions),
            "insufficient_conditions": list(gate.insufficient_conditions)}


def lofo_summary(rows: Sequence[Mapping[str, Any]]) -> dict[str, Any]:
    """Per held-out family: the fold's selected method's paired delta on that
    family's test sequences, and its relative degradation against the pooled
    selection's delta on the same sequences."""
    by: dict[str, list[Mapping[str, Any]]] = defaultdict(list)
    for r in rows:
        by[str(r["held_out_family"])].append(r)
    delta = {f: float(np.mean([float(r["fold_delta"]) for r in rs])) for f, rs in sorted(by.items())}
    pooled = {f: float(np.mean([float(r["pooled_delta"]) for r in rs])) for f, rs in sorted(by.items())}
    degr = {f: (0.0 if abs(pooled[f]) < 1e-12 else max(0.0, (pooled[f] - delta[f]) / abs(pooled[f])))
            for f in delta}
    return {"aggregate_delta": float(np.mean(list(delta.values()))) if delta else 0.0,
            "delta_by_family": delta, "relative_degradation_by_family": degr,
            "fold_methods": {f: rs[0]["fold_method"] for f, rs in sorted(by.items())}}


def run_study(scale: str = "quick", *, out_dir: str | Path | None = None, topology: Any = None) -> dict[str, Any]:
    """Run the study at `scale` and (with out_dir) write its artifacts; returns the summary."""
    from ..topology.loader import load_rear4_topology

    sc = StudyScale.named(scale)
    topo = topology if topology is not None else load_rear4_topology()[0]
    st = _Study(sc, topo)
    calib = st.calibration_rows()
    radius = calibration_radius(calib)
    valid = st.case_rows(st._split("validation"), radius, ORDINARY_METHODS, UNKNOWN_RATIOS)
    selected, _ = select_method(valid)
    test = st.case_rows(st._split("test"), radius, ALL_METHODS)
    test_seq = sequence_rows(test)
    pooled = {d["sequence_id"]: d["paired_delta"] for d in paired_deltas(test_seq, selected)}
    lofo_rows = []
    for fam in sorted({s.family for s in st.specs}):
        fold_radius = calibration_radius(calib, exclude_family=fam) if len(sc.families) > 1 else radius
        fold_valid = [r for r in valid if r["family"] != fam] or valid
        fold_method, _ = select_method(fold_valid)
        fold_test = st.case_rows(st._split("test", family=fam), fold_radius,
                                 sorted({fold_method, "random_empirical"}), UNKNOWN_RATIOS)
        for d in paired_deltas(sequence_rows(fold_test), fold_method):
            lofo_rows.append({"held_out_family": fam, "sequence_id": d["sequence_id"], "fold_method": fold_method,
                              "fold_radius": fold_radius, "fold_delta": d["paired_delta"],
                              "pooled_delta": pooled[d["sequence_id"]]})
    raw = {"calibration": calib, "validation": valid, "test": test, "lofo": lofo_rows}
    summary = recompute_summary(raw, bootstrap_replicates=sc.bootstrap_replicates)
    summary.update(scale=sc.name, sequences=len(st.specs), test_cases=len(test))
    if out_dir is not None:
        write_artifacts(out_dir, raw, test_seq, summary)
    return summary


def _json_default(v: Any) -> Any:
    if isinstance(v, (np.integer,)):
        return int(v)
    if isinstance(v, (np.floating,)):
        return float(v)
    if isinstance(v, np.ndarray):
        return v.tolist()
    raise TypeError(type(v))


def write_artifacts(out_dir: str | Path, raw: Mapping[str, Sequence[Mapping[str, Any]]],
                    seq_rows: Sequence[Mapping[str, Any]], summary: Mapping[str, Any]) -> dict[str, str]:
    """Raw tables as CSV, the summary as JSON, and a manifest of sha256 digests."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    digests = {}
    tables = dict(raw)
    tables["test_sequences"] = seq_rows
    for name, rows in tables.items():
        path = out / f"raw_{name}.csv"
        with path.open("w", newline="") as fh:
            if rows:
                w = csv.DictWriter(fh, fieldnames=list(rows[0].keys()))
                w.writeheader()
                w.writerows(rows)
        digests[path.name] = hashlib.sha256(path.read_bytes()).hexdigest()
    (out / "summary.json").write_text(json.dumps(summary, indent=2, sort_keys=True, default=_json_default))
    digests["summary.json"] = hashlib.sha256((out / "summary.json").read_bytes()).hexdigest()
    (out / "manifest.json").write_text(json.dumps({"artifacts": digests}, indent=2, sort_keys=True))
    return digests


def read_raw_tables(out_dir: str | Path) -> dict[str, list[dict[str, Any]]]:
    """The raw tables of an artifact directory with numeric fields restored."""
    def conv(v: str) -> Any:
        if v in ("True", "False"):
            return v == "True"
        try:
            return int(v)
        except ValueError:
            try:
                return float(v)
            except ValueError:
                return v

    res = {}
    for name in ("calibration", "validation", "test", "lofo"):
        with (Path(out_dir) / f"raw_{name}.csv").open() as fh:
            res[name] = [{k: conv(v) for k, v in r.items()} for r in csv.DictReader(fh)]
    return res


def main(argv: Sequence[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--scale", default="quick", choices=("toy", "quick", "formal"))
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    s = run_study(args.scale, out_dir=args.out)
    print(json.dumps({k: s[k] for k in ("scale", "sequences", "test_cases", "calibration_radius", "selected_method",
                                         "data_status", "failed_conditions", "insufficient_conditions")},
                     default=_json_default))


if __name__ == "__main__":
    main()
