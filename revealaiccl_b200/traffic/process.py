"""Moment-bounded, non-Gaussian All-to-All-V traffic processes.

Generator of rlccl/traffic/process_generator.py, same recipe so that equal
configurations give equal sequences:

1. a family profile over one period of ``window_size`` steps, standardised
   to mean 0 / std 1 (smooth_ar: two sines; alternating_burst: +-1 with a
   slower +-0.15 ripple; moving_hotspot: a Gaussian pulse of width W/8 on the
   circular distance; sparse_switching: a small sine plus a +1.5 block on the
   first W/4 steps; bimodal: -1 / +1 halves; heavy_tail_clipped: one spike of
   max(4, sqrt(W)) plus a unit bump at W/2 for W >= 8);
2. per distinct (mean, var) target, an integer period: the affine map
   ``rint(clip(mean + offset + std * factor * profile, 0, max_entry))`` over
   offsets linspace(-0.75, 0.75, 13) x factors linspace(0.5, 1.5, 21) that
   minimises the squared relative errors of the period's mean and variance;
3. each off-diagonal pair gets that period rolled by a family-specific phase
   (hotspot: by destination, switching / burst / heavy tail: by an affine
   function of (src, dst)) shifted by ``seed % window_size``, or a random phase
   from the seeded generator for the other families;
4. the period is tiled to ``sequence_length``; the candidate is accepted when
   every complete window meets the moment bounds, else regenerated (up to
   ``max_generation_attempts``).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import ClassVar

import numpy as np

from .moments import validate_sequence_moment_bounds
from .types import MomentBounds, TrafficSequence

FAMILIES = ("smooth_ar", "alternating_burst", "moving_hotspot", "sparse_switching", "bimodal",
            "heavy_tail_clipped")


@dataclass
class TrafficProcessConfig:
    num_nodes: int
    sequence_length: int
    window_size: int
    mean_level: float
    std_level: float
    max_entry: int
    epsilon_mean: float
    epsilon_var: float
    family: str
    seed: int
    max_generation_attempts: int = 100
    mean_ref: np.ndarray | None = None
    var_ref: np.ndarray | None = None
    topology_name: str = "unknown"
    validation_stride: int = 1
    allowed_violation_fraction: float = 0.0

    FAMILIES: ClassVar[tuple[str, ...]] = FAMILIES

    def __post_init__(self) -> None:
        if self.num_nodes < 2:
            raise ValueError("num_nodes must be at least 2")
        if self.window_size <= 1 or self.sequence_length < self.window_size:
            raise ValueError("sequence_length must be >= window_size > 1")
        if self.mean_level < 0 or self.std_level < 0:
            raise ValueError("mean_level and std_level must be nonnegative")
        if self.max_entry <= 0:
            raise ValueError("max_entry must be positive")
        if self.family not in FAMILIES:
            raise ValueError(f"Unknown traffic family {self.family!r}; expected one of {FAMILIES}")
        if self.max_generation_attempts <= 0 or self.validation_stride <= 0:
            raise ValueError("max_generation_attempts and validation_stride must be positive")
        if not 0.0 <= self.allowed_violation_fraction <= 1.0:
            raise ValueError("allowed_violation_fraction must be in [0, 1]")


def family_profile(family: str, w: int) -> np.ndarray:
    t = np.arange(w, dtype=np.float64)
    if family == "smooth_ar":
        x = np.sin(2 * np.pi * t / w) + 0.30 * np.sin(4 * np.pi * t / w + 0.4)
    elif family == "alternating_burst":
        ti = t.astype(int)
        x = np.where(ti % 2 == 0, -1.0, 1.0) + 0.15 * np.where(ti % 4 < 2, -1.0, 1.0)
    elif family == "moving_hotspot":
        d = np.minimum(t, w - t)
        x = np.exp(-0.5 * (d / max(w / 8.0, 1.0)) ** 2)
    elif family == "sparse_switching":
        x = 0.20 * np.sin(2 * np.pi * t / w)
        x[:max(1, w // 4)] += 1.5
    elif family == "bimodal":
        x = np.where(t >= w // 2, 1.0, -1.0)
    elif family == "heavy_tail_clipped":
        x = np.zeros(w)
        x[0] = max(4.0, np.sqrt(w))
        if w >= 8:
            x[w // 2] = 1.0
    else:
        raise ValueError(f"Unsupported family: {family}")
    x = x - x.mean()
    s = x.std()
    if s < 1e-12:
        raise ValueError("Family profile must have nonzero variance")
    return x / s


def calibrate_integer_period(profile: np.ndarray, mean: float, var: float, max_entry: int) -> np.ndarray:
    std = float(np.sqrt(max(var, 0.0)))
    factors = np.linspace(0.50, 1.50, 21) if std > 0 else np.array([0.0])
    ms, vs = max(abs(mean), 1.0), max(abs(var), 1.0)
    best, best_score = None, np.inf
    for off in np.linspace(-0.75, 0.75, 13):
        for fac in factors:
            v = np.rint(np.clip(mean + off + std * fac * profile, 0, max_entry)).astype(np.int64)
            score = ((v.mean() - mean) / ms) ** 2 + ((v.var() - var) / vs) ** 2
            if score < best_score:
                best, best_score = v, score
    return best


def _pair_phase(family: str, src: int, dst: int, n: int, w: int, rng: np.random.Generator, base: int) -> int:
    if family == "moving_hotspot":
        return (dst * w // n + base) % w
    if family == "sparse_switching":
        return (src * n + dst + base) % w
    if family == "alternating_burst":
        return (src + dst + base) % w
    if family == "heavy_tail_clipped":
        return (3 * src + 5 * dst + base) % w
    return int(rng.integers(0, w))


def _references(cfg: TrafficProcessConfig) -> tuple[np.ndarray, np.ndarray]:
    n = cfg.num_nodes
    mref = (np.full((n, n), cfg.mean_level, dtype=np.float64) if cfg.mean_ref is None
            else np.asarray(cfg.mean_ref, dtype=np.float64).copy())
    vref = (np.full((n, n), cfg.std_level ** 2, dtype=np.float64) if cfg.var_ref is None
            else np.asarray(cfg.var_ref, dtype=np.float64).copy())
    if cfg.mean_ref is None:
        np.fill_diagonal(mref, 0.0)
    if cfg.var_ref is None:
        np.fill_diagonal(vref, 0.0)
    if mref.shape != (n, n) or vref.shape != (n, n):
        raise ValueError(f"mean_ref and var_ref must both have shape {(n, n)}")
    if not (np.all(np.isfinite(mref)) and np.all(np.isfinite(vref))):
        raise ValueError("Reference moments must be finite")
    if np.any(mref < 0) or np.any(vref < 0):
        raise ValueError("Reference mean and variance must be nonnegative")
    if np.any(np.diag(mref) != 0) or np.any(np.diag(vref) != 0):
        raise ValueError("Reference moment diagonals must be zero")
    return mref, vref


def _candidate(cfg: TrafficProcessConfig, mref, vref, rng) -> list[np.ndarray]:
    w, n = cfg.window_size, cfg.num_nodes
    prof = family_profile(cfg.family, w)
    period = np.zeros((w, n, n), dtype=np.int64)
    base = int(cfg.seed % w)
    cache: dict[tuple[float, float], np.ndarray] = {}
    for s in range(n):
        for d in range(n):
            if s == d:
                continue
            key = (float(mref[s, d]), float(vref[s, d]))
            if key not in cache:
                cache[key] = calibrate_integer_period(prof, key[0], key[1], cfg.max_entry)
            period[:, s, d] = np.roll(cache[key], _pair_phase(cfg.family, s, d, n, w, rng, base))
    reps = -(-cfg.sequence_length // w)
    seq = np.tile(period, (reps, 1, 1))[:cfg.sequence_length]
    return [m.copy() for m in seq]


def _config_meta(cfg: TrafficProcessConfig) -> dict:
    d = asdict(cfg)
    for k in ("mean_ref", "var_ref"):
        if d[k] is not None:
            d[k] = np.asarray(d[k]).tolist()
    return d


def generate_traffic_sequence(cfg: TrafficProcessConfig) -> TrafficSequence:
    mref, vref = _references(cfg)
    bounds = MomentBounds(cfg.epsilon_mean, cfg.epsilon_var)
    rng = np.random.default_rng(cfg.seed)
    diag = None
    for attempt in range(1, cfg.max_generation_attempts + 1):
        seq = TrafficSequence(
            sequence_id=f"{cfg.family}-seed{cfg.seed}", topology_name=cfg.topology_name, family=cfg.family,
            seed=cfg.seed, matrices=_candidate(cfg, mref, vref, rng), mean_ref=mref, var_ref=vref, bounds=bounds,
            metadata={"schema_version": 1, "window_size": cfg.window_size, "validation_stride": cfg.validation_stride,
                      "allowed_violation_fraction": cfg.allowed_violation_fraction, "generation_attempt": attempt,
                      "generator_config": _config_meta(cfg)})
        diag = validate_sequence_moment_bounds(seq)
        if diag["passed"]:
            seq.metadata["validation"] = {k: v for k, v in diag.items() if k != "windows"}
            return seq
    raise RuntimeError(
        f"Unable to generate a moment-bounded integer traffic sequence after {cfg.max_generation_attempts} "
        f"attempts for family={cfg.family!r}; max_mean_error={diag['max_mean_error']:.6f}, "
        f"max_var_error={diag['max_var_error']:.6f}, bounds=({cfg.epsilon_mean}, {cfg.epsilon_var})")


__all__ = ["FAMILIES", "TrafficProcessConfig", "calibrate_integer_period", "family_profile",
           "generate_traffic_sequence"]
