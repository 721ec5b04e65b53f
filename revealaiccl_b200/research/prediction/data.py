"""Preregistered sequences and leakage-safe examples (rlccl/prediction/data.py).

75 sequences = 5 long-horizon families x 3 base seeds (42, 142, 242) x 5
split slots (fit, fit, validation, calibration, test); seed =
base + 1e6 * family index + 1e4 * slot; same-moment variants rotate with
(seed index + slot).  An example at step t >= recent_steps reads the
summaries of steps t-8..t-1 and the window moments of matrices
max(0, t-16)..t-1; the target is the summary of step t.
"""

from __future__ import annotations

import hashlib
from dataclasses import asdict, dataclass
from typing import Any, Iterable, Mapping, Sequence

import numpy as np

from ...traffic.long_horizon import (LONG_HORIZON_FAMILIES, SAME_MOMENT_VARIANTS, LongHorizonTrafficConfig,
                                     generate_long_horizon_sequence)
from ..traffic_predictor import summary_vector, traffic_summary

FORMAL_FAMILIES = tuple(LONG_HORIZON_FAMILIES)
FORMAL_BASE_SEEDS = (42, 142, 242)
FORMAL_SEQUENCE_LENGTH = 1024
FORMAL_SPLITS = ("fit", "fit", "validation", "calibration", "test")
RECENT_STEPS = 8
MOMENT_WINDOW = 16
SPLITS = ("fit", "validation", "calibration", "test")


@dataclass(frozen=True)
class SequenceSpec:
    sequence_id: str
    family: str
    family_index: int
    base_seed: int
    seed_index: int
    sequence_index: int
    actual_seed: int
    split: str
    dynamics_variant: str | None
    sequence_length: int
    generator_config: dict[str, Any]


@dataclass(frozen=True)
class HistoryExamples:
    sequence_ids: np.ndarray
    families: np.ndarray
    seeds: np.ndarray
    steps: np.ndarray
    history_last_steps: np.ndarray
    recent_history: np.ndarray      # [N, recent_steps, target_dim]
    moment_features: np.ndarray     # [N, 2 n (n - 1)]
    previous_targets: np.ndarray
    ewma_targets: np.ndarray
    targets: np.ndarray
    hotspot_targets: np.ndarray
    previous_hotspots: np.ndarray


@dataclass
class Standardizers:
    input_mean: np.ndarray
    input_scale: np.ndarray
    target_mean: np.ndarray
    target_scale: np.ndarray

    def transform_inputs(self, v):
        return (np.asarray(v, dtype=np.float64) - self.input_mean) / self.input_scale

    def transform_targets(self, v):
        return (np.asarray(v, dtype=np.float64) - self.target_mean) / self.target_scale

    def inverse_targets(self, v):
        return np.asarray(v, dtype=np.float64) * self.target_scale + self.target_mean

    def state_dict(self) -> dict[str, np.ndarray]:
        return {k: getattr(self, k).copy() for k in ("input_mean", "input_scale", "target_mean", "target_scale")}


def generator_config(family: str, seed: int, variant: str | None, length: int = FORMAL_SEQUENCE_LENGTH) -> dict:
    return asdict(LongHorizonTrafficConfig(num_nodes=4, sequence_length=length, family=family, seed=seed,
                                           mean_level=2.0, std_level=1.5, max_entry=8, calibration_candidates=1,
                                           topology_name="Rear4GPU", dynamics_variant=variant))


def build_formal_sequence_specs() -> list[SequenceSpec]:
    """The frozen 75-sequence design (no traffic generated)."""
    out = []
    for fi, fam in enumerate(FORMAL_FAMILIES):
        for si, base in enumerate(FORMAL_BASE_SEEDS):
            for qi, split in enumerate(FORMAL_SPLITS):
                seed = base + fi * 1_000_000 + qi * 10_000
                var = SAME_MOMENT_VARIANTS[(si + qi) % 4] if fam == "same_moments_different_dynamics" else None
                out.append(SequenceSpec(f"{fam}-base{base}-sequence{qi}-seed{seed}", fam, fi, base, si, qi, seed, split,
                                        var, FORMAL_SEQUENCE_LENGTH, generator_config(fam, seed, var)))
    return out


def generate_formal_sequence(spec: SequenceSpec):
    seq = generate_long_horizon_sequence(LongHorizonTrafficConfig(**dict(spec.generator_config)))
    seq.sequence_id = spec.sequence_id
    seq.metadata.update({"formal_base_seed": spec.base_seed, "formal_sequence_index": spec.sequence_index,
                         "formal_split": spec.split})
    return seq


def sequence_digest(matrices: Iterable[np.ndarray]) -> str:
    """SHA-256 over (shape, dtype, bytes) of every matrix, then the count."""
    h = hashlib.sha256()
    n = 0
    for m in matrices:
        a = np.ascontiguousarray(np.asarray(m))
        h.update(np.asarray(a.shape, dtype=np.int64).tobytes())
        h.update(a.dtype.str.encode("ascii"))
        h.update(a.tobytes())
        n += 1
    h.update(np.asarray([n], dtype=np.int64).tobytes())
    return h.hexdigest()


def validate_split_records(records: Iterable[Mapping[str, Any]]) -> None:
    """No sequence id and no sequence digest may appear twice (across or within splits)."""
    ids: dict[str, str] = {}
    digests: dict[str, str] = {}
    for r in records:
        sid, dig, split = str(r["sequence_id"]), str(r["digest"]), str(r["split"])
        if split not in SPLITS:
            raise ValueError(f"Unknown split: {split}")
        if sid in ids:
            raise ValueError(f"sequence id overlap/duplicate: {sid} in {ids[sid]} and {split}")
        if dig in digests:
            raise ValueError(f"digest overlap/duplicate: {dig} in {digests[dig]} and {split}")
        ids[sid], digests[dig] = split, split


def ewma_rows(v: np.ndarray, alpha: float = 0.30) -> np.ndarray:
    """Post-update EWMA states: s_0 = v_0, s_t = alpha v_t + (1 - alpha) s_{t-1}."""
    v = np.asarray(v, dtype=np.float64)
    out = np.empty_like(v)
    s = v[0].copy()
    for i in range(len(v)):
        if i:
            s = alpha * v[i] + (1.0 - alpha) * s
        out[i] = s
    return out


def _window_moment_features(mats: np.ndarray, steps: np.ndarray, window: int) -> np.ndarray:
    """[mean, var] of the off-diagonal entries over matrices max(0, t - window)..t-1, per step t (prefix sums)."""
    n = mats.shape[1]
    off = ~np.eye(n, dtype=bool)
    flat = mats[:, off]
    c1 = np.concatenate([np.zeros((1, flat.shape[1])), np.cumsum(flat, axis=0)])
    c2 = np.concatenate([np.zeros((1, flat.shape[1])), np.cumsum(flat * flat, axis=0)])
    lo = np.maximum(0, steps - window)
    cnt = (steps - lo)[:, None].astype(np.float64)
    mean = (c1[steps] - c1[lo]) / cnt
    var = np.maximum((c2[steps] - c2[lo]) / cnt - mean * mean, 0.0)
    return np.concatenate([mean, var], axis=1)


def build_history_examples(sequence, *, group_coefficients: np.ndarray, recent_steps: int = RECENT_STEPS,
                           moment_window: int = MOMENT_WINDOW) -> HistoryExamples:
    """Examples at t >= recent_steps; features read matrices 0..t-1 only."""
    if recent_steps <= 0 or moment_window <= 0:
        raise ValueError("history windows must be positive")
    mats = np.asarray(sequence.matrices, dtype=np.float64)
    if mats.ndim != 3 or mats.shape[1] != mats.shape[2]:
        raise ValueError("sequence matrices must have shape [time, node, node]")
    g = np.asarray(group_coefficients, dtype=np.float64)
    if g.ndim != 3 or g.shape[1:] != mats.shape[1:]:
        raise ValueError("group_coefficients must have shape [group, node, node]")
    if len(mats) <= recent_steps:
        raise ValueError("sequence is too short for the recent-history window")
    sums = [traffic_summary(m, g) for m in mats]
    vec = np.stack([summary_vector(s) for s in sums]).astype(np.float64)
    hot = np.asarray([s["hotspot_destination"] for s in sums], dtype=np.int64)
    ew = ewma_rows(vec)
    steps = np.arange(recent_steps, len(mats), dtype=np.int64)
    recent = np.lib.stride_tricks.sliding_window_view(vec, recent_steps, axis=0)[:len(steps)].transpose(0, 2, 1)
    n = len(steps)
    return HistoryExamples(
        sequence_ids=np.full(n, str(sequence.sequence_id), dtype=object),
        families=np.full(n, str(sequence.family), dtype=object), seeds=np.full(n, int(sequence.seed), dtype=np.int64),
        steps=steps, history_last_steps=steps - 1, recent_history=np.ascontiguousarray(recent),
        moment_features=_window_moment_features(mats, steps, moment_window),
        previous_targets=vec[steps - 1].copy(), ewma_targets=ew[steps - 1].copy(), targets=vec[steps].copy(),
        hotspot_targets=hot[steps].copy(), previous_hotspots=hot[steps - 1].copy())


def fit_standardizers(inputs: np.ndarray, targets: np.ndarray) -> Standardizers:
    """Scaling statistics of the fit split (inputs pooled over every axis but the last)."""
    x, y = np.asarray(inputs, dtype=np.float64), np.asarray(targets, dtype=np.float64)
    if x.ndim < 2 or y.ndim != 2 or len(x) != len(y) or not len(x):
        raise ValueError("inputs and targets must be nonempty same-length arrays")
    red = tuple(range(x.ndim - 1))
    guard = lambda s: np.where(s < 1e-8, 1.0, s)  # noqa: E731
    return Standardizers(x.mean(axis=red), guard(x.std(axis=red, ddof=0)), y.mean(axis=0), guard(y.std(axis=0, ddof=0)))


def build_lofo_fold(specs: Sequence[SequenceSpec], held_out_family: str) -> dict[str, list[SequenceSpec]]:
    """Leave-one-family-out: the held-out family only in test, absent from every other split."""
    if held_out_family not in FORMAL_FAMILIES:
        raise ValueError(f"Unknown held-out family: {held_out_family}")
    out: dict[str, list[SequenceSpec]] = {s: [] for s in SPLITS}
    for sp in specs:
        if sp.split == "test":
            if sp.family == held_out_family:
                out["test"].append(sp)
        elif sp.family != held_out_family:
            out[sp.split].append(sp)
    return out
