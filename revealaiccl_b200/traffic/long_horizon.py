"""Long-horizon stochastic traffic processes.

Behaviour of rlccl/traffic/long_horizon_generator.py (same configuration
fields, same random-draw order, so equal configurations give equal
sequences and metadata):

* a scalar total-load process ``S_t`` per family (long regimes with AR(1)
  noise, stochastic volatility, rare shocks with geometric recovery, a calm
  AR(1) for the hotspot walk, and four "same moments, different dynamics"
  latents scaled to one configured total std);
* a normalised spatial process ``P_t`` over the off-diagonal pairs
  (log-normal AR(1) noise times a per-step mode: balanced, single source /
  destination hotspot, dual hotspot, sparse support, cross-group
  concentration, random-walk hotspot);
* integerisation of ``S_t * P_t`` by a largest-deficit allocator with a
  per-entry cap (``max_entry``) and a 1e-9 jitter for tie order;
* rolling short / medium / long window checks of the realised totals and of
  the matrices against configured (never realised) reference moments, and up
  to ``calibration_candidates`` independently seeded candidates, keeping the
  least-violating one.

The random streams: ``SeedSequence([seed, candidate]).spawn(3)`` gives the
total, spatial and allocation generators.  AR(1) innovations are drawn as one
standard-normal block and scaled (numpy's scalar ``normal`` is
``loc + scale * standard_normal``, so the stream is the same one value at a
time or as a block).  The allocator keeps a heap of deficits instead of a
full argmax per unit; the deficit of an entry is recomputed with the same
floating-point expression after each increment and ties break on the lower
flat index, so the allocation is identical.
"""

from __future__ import annotations

import heapq
from dataclasses import asdict, dataclass
from typing import Any, ClassVar

import numpy as np

from .matrix_utils import validate_traffic_matrix
from .types import MomentBounds, TrafficSequence

LONG_HORIZON_FAMILIES = ("regime_switching_long", "stochastic_volatility", "rare_shock_recovery",
                         "hotspot_random_walk", "same_moments_different_dynamics")
SAME_MOMENT_VARIANTS = ("smooth", "random_switching", "long_regime", "shock_recovery")
SPATIAL_MODES = ("balanced", "single_source_hotspot", "single_destination_hotspot", "dual_hotspot",
                 "sparse_support", "cross_group_concentration", "hotspot_random_walk")


@dataclass(frozen=True)
class LongHorizonTrafficConfig:
    num_nodes: int = 4
    sequence_length: int = 1024
    family: str = "regime_switching_long"
    seed: int = 42
    mean_level: float = 2.0
    std_level: float = 1.5
    max_entry: int = 8
    base_level: float | None = None
    ar_coefficient: float = 0.80
    short_noise_scale: float = 0.06
    regime_levels: tuple[float, float, float] = (0.75, 1.00, 1.25)
    regime_dwell_range: tuple[int, int] = (32, 512)
    shock_probability: float = 0.003
    shock_magnitude: float = 1.50
    shock_duration_range: tuple[int, int] = (4, 16)
    recovery_rate: float = 0.94
    minimum_total: float = 4.0
    maximum_total: float | None = None
    short_window: int = 16
    medium_window: int = 128
    long_window: int = 512
    medium_epsilon_mean: float = 0.60
    medium_epsilon_var: float = 6.00
    medium_allowed_violation_fraction: float = 0.20
    medium_matrix_epsilon_mean: float = 1.10
    medium_matrix_epsilon_var: float = 3.50
    long_epsilon_mean: float = 0.30
    long_epsilon_var: float = 3.00
    long_allowed_violation_fraction: float = 0.05
    long_matrix_epsilon_mean: float = 0.70
    long_matrix_epsilon_var: float = 2.50
    spatial_mode: str | None = None
    hotspot_dwell_range: tuple[int, int] = (8, 96)
    hotspot_strength_range: tuple[float, float] = (2.5, 5.0)
    source_groups: tuple[int, ...] | None = None
    dynamics_variant: str | None = None
    calibration_candidates: int = 3
    topology_name: str = "Rear4GPU"

    FAMILIES: ClassVar[tuple[str, ...]] = LONG_HORIZON_FAMILIES
    SPATIAL_MODES: ClassVar[tuple[str, ...]] = SPATIAL_MODES
    SAME_MOMENT_VARIANTS: ClassVar[tuple[str, ...]] = SAME_MOMENT_VARIANTS

    def __post_init__(self) -> None:
        if self.num_nodes < 2:
            raise ValueError("num_nodes must be at least two")
        if self.short_window <= 1 or self.sequence_length < self.short_window:
            raise ValueError("sequence_length must be >= short_window > 1")
        if self.family not in LONG_HORIZON_FAMILIES:
            raise ValueError(f"Unsupported long-horizon family: {self.family}")
        if self.mean_level <= 0 or self.std_level < 0 or self.max_entry <= 0:
            raise ValueError("mean_level/max_entry must be positive and std_level nonnegative")
        if not -0.999 < self.ar_coefficient < 0.999:
            raise ValueError("ar_coefficient must be in (-0.999, 0.999)")
        if not 0.0 <= self.shock_probability <= 1.0:
            raise ValueError("shock_probability must be in [0, 1]")
        if not 0.0 < self.recovery_rate < 1.0:
            raise ValueError("recovery_rate must be in (0, 1)")
        if self.spatial_mode is not None and self.spatial_mode not in SPATIAL_MODES:
            raise ValueError(f"Unsupported spatial_mode: {self.spatial_mode}")
        if self.dynamics_variant is not None and self.dynamics_variant not in SAME_MOMENT_VARIANTS:
            raise ValueError(f"Unsupported dynamics_variant: {self.dynamics_variant}")
        for name in ("regime_dwell_range", "shock_duration_range", "hotspot_dwell_range"):
            lo_hi = getattr(self, name)
            if len(lo_hi) != 2 or lo_hi[0] <= 0 or lo_hi[1] < lo_hi[0]:
                raise ValueError(f"{name} must be a positive ordered pair")
        for name in ("medium_allowed_violation_fraction", "long_allowed_violation_fraction"):
            if not 0.0 <= getattr(self, name) <= 1.0:
                raise ValueError(f"{name} must be in [0, 1]")
        if self.calibration_candidates <= 0:
            raise ValueError("calibration_candidates must be positive")
        if self.source_groups is not None and len(self.source_groups) != self.num_nodes:
            raise ValueError("source_groups must contain one group id per node")

    @property
    def pairs(self) -> int:
        return self.num_nodes * (self.num_nodes - 1)

    @property
    def base_total(self) -> float:
        return float(self.base_level if self.base_level is not None else self.mean_level * self.pairs)

    @property
    def max_total(self) -> float:
        cap = float(self.max_entry * self.pairs)
        return cap if self.maximum_total is None else min(cap, float(self.maximum_total))


# ---------------------------------------------------------------------------
# scalar building blocks
# ---------------------------------------------------------------------------
def ar1(length: int, phi: float, sigma, rng: np.random.Generator) -> np.ndarray:
    """Stationary-scaled AR(1): x_0 = 0, x_t = phi x_{t-1} + N(0, sigma_t sqrt(1 - phi^2))."""
    scale = np.broadcast_to(np.asarray(sigma, dtype=np.float64), (length,)) * np.sqrt(max(1.0 - phi * phi, 1e-6))
    z = rng.standard_normal(max(length - 1, 0))
    eps = scale[1:] * z
    out = np.zeros(length, dtype=np.float64)
    prev = 0.0
    for i in range(1, length):
        prev = phi * prev + eps[i - 1]
        out[i] = prev
    return out


def dwell_states(length: int, labels: tuple, dwell: tuple[int, int],
                 rng: np.random.Generator) -> tuple[np.ndarray, list[dict[str, Any]]]:
    """Piecewise-constant label path: uniform dwell in [lo, hi], then a jump to a different label."""
    path = np.empty(length, dtype=object)
    runs: list[dict[str, Any]] = []
    pos, cur = 0, int(rng.integers(0, len(labels)))
    while pos < length:
        end = min(length, pos + int(rng.integers(dwell[0], dwell[1] + 1)))
        path[pos:end] = labels[cur]
        runs.append({"state": labels[cur], "start": pos, "end": end, "length": end - pos})
        cur = int(rng.choice([i for i in range(len(labels)) if i != cur]))
        pos = end
    return path, runs


def _geometric_tail(series: np.ndarray, start: int, amplitude: float, rate: float, floor: float) -> int:
    """Add amplitude * rate^j at start + j - 1 (j >= 1) while the residual exceeds floor; returns the end."""
    residual, cur = amplitude, start
    while cur < len(series) and residual > floor:
        residual *= rate
        series[cur] += residual
        cur += 1
    return cur


def same_moment_latent(length: int, variant: str, cfg: LongHorizonTrafficConfig,
                       rng: np.random.Generator) -> tuple[np.ndarray, dict[str, Any]]:
    """Zero-mean, unit-std latent with the variant's dynamics."""
    meta: dict[str, Any] = {"dynamics_variant": variant}
    if variant == "smooth":
        x = ar1(length, 0.975, 1.0, rng)
    elif variant in ("random_switching", "long_regime"):
        labels, dwell, phi, sig = (((-1.0, 1.0), (4, 32), 0.4, 0.20) if variant == "random_switching"
                                   else ((-1.0, 0.0, 1.0), (64, 256), 0.85, 0.15))
        path, runs = dwell_states(length, labels, dwell, rng)
        x = path.astype(np.float64) + ar1(length, phi, sig, rng)
        meta["variant_dwell_records"] = runs
    elif variant == "shock_recovery":
        x = ar1(length, 0.75, 0.18, rng)
        flags = np.zeros(length, dtype=np.int8)
        starts = sorted({int(v) for v in rng.integers(32, max(33, length - 32), size=max(1, length // 512))})
        for st in starts:
            amp = float(rng.uniform(3.0, 5.0))
            dur = int(rng.integers(4, 13))
            stop = min(length, st + dur)
            x[st:stop] += amp
            flags[st:stop] = 1
            _geometric_tail(x, st + dur, amp, cfg.recovery_rate, 0.05)
        meta["variant_shock_flags"] = flags.astype(int).tolist()
    else:
        raise ValueError(f"Unknown same-moment variant: {variant}")
    x = x - x.mean()
    s = float(x.std(ddof=0))
    if s <= 1e-12:
        raise RuntimeError("same-moment latent process became constant")
    return x / s, meta


def _add_shock(comp: np.ndarray, flags: np.ndarray, start: int, dur: int, amp: float, rate: float,
               floor: float) -> dict[str, Any]:
    end = min(len(comp), start + dur)
    comp[start:end] += amp
    flags[start:end] = 1
    rec_end = _geometric_tail(comp, end, amp, rate, floor)
    return {"start": start, "end": end, "duration": end - start, "amplitude": amp, "recovery_end": rec_end}


def total_load(cfg: LongHorizonTrafficConfig, rng: np.random.Generator) -> tuple[np.ndarray, dict[str, Any]]:
    """S_t for the family, mean-shifted to the base total and clipped to [minimum_total, max_total]."""
    L, base = cfg.sequence_length, cfg.base_total
    meta: dict[str, Any] = {}
    regime = np.full(L, "normal", dtype=object)
    flags = np.zeros(L, dtype=np.int8)
    shock = np.zeros(L, dtype=np.float64)
    vol = np.full(L, "calm", dtype=object)
    fam = cfg.family
    if fam == "regime_switching_long":
        regime, runs = dwell_states(L, ("low", "normal", "high"), cfg.regime_dwell_range, rng)
        level = dict(zip(("low", "normal", "high"), cfg.regime_levels))
        total = (np.asarray([base * level[s] for s in regime], dtype=np.float64)
                 + ar1(L, cfg.ar_coefficient, base * cfg.short_noise_scale, rng))
        meta["regime_dwell_records"] = runs
    elif fam == "stochastic_volatility":
        vol, runs = dwell_states(L, ("calm", "volatile"), (32, 256), rng)
        total = base + ar1(L, cfg.ar_coefficient, np.where(vol == "calm", base * 0.025, base * 0.18), rng)
        regime = vol.copy()
        meta["volatility_dwell_records"] = runs
    elif fam == "rare_shock_recovery":
        total = base + ar1(L, cfg.ar_coefficient, base * cfg.short_noise_scale, rng)
        lo, hi = cfg.shock_duration_range
        records: list[dict[str, Any]] = []
        cur = 1
        while cur < L:
            if rng.random() < cfg.shock_probability:
                dur = int(rng.integers(lo, hi + 1))
                amp = base * cfg.shock_magnitude * float(rng.uniform(0.8, 1.2))
                rec = _add_shock(shock, flags, cur, dur, amp, cfg.recovery_rate, base * 0.02)
                records.append(rec)
                cur = rec["recovery_end"]
            else:
                cur += 1
        if not records:  # guarantee one event per sequence
            cur = int(rng.integers(max(1, L // 4), max(2, 3 * L // 4)))
            records.append(_add_shock(shock, flags, cur, min(hi, max(1, L - cur)), base * cfg.shock_magnitude,
                                      cfg.recovery_rate, base * 0.02))
        total += shock
        regime = np.where(flags > 0, "shock", np.where(shock > 0, "recovery", "normal"))
        meta["shock_records"] = records
    elif fam == "hotspot_random_walk":
        total = base + ar1(L, cfg.ar_coefficient, base * 0.04, rng)
    else:  # same_moments_different_dynamics
        variant = cfg.dynamics_variant or SAME_MOMENT_VARIANTS[cfg.seed % len(SAME_MOMENT_VARIANTS)]
        latent, vmeta = same_moment_latent(L, variant, cfg, rng)
        total = base + cfg.std_level * np.sqrt(cfg.pairs) * latent
        meta.update(vmeta)
        regime = np.full(L, variant, dtype=object)
        if "variant_shock_flags" in vmeta:
            flags = np.asarray(vmeta["variant_shock_flags"], dtype=np.int8)
    # one global shift keeps the dynamics (no rejection of short unusual windows)
    total = np.clip(total + (base - float(total.mean())), cfg.minimum_total, cfg.max_total)
    meta.update({"latent_regime": regime.tolist(), "shock_flags": flags.astype(int).tolist(),
                 "shock_component": shock.tolist(), "volatility_state": vol.tolist(), "target_total_mean": base})
    return total, meta


# ---------------------------------------------------------------------------
# spatial process
# ---------------------------------------------------------------------------
def hotspot_walk(cfg: LongHorizonTrafficConfig, rng: np.random.Generator):
    """Per-step hotspot (source, destination, strength): source steps -1/0/+1, destination +-1 per dwell."""
    L, n = cfg.sequence_length, cfg.num_nodes
    src = np.empty(L, dtype=np.int64)
    dst = np.empty(L, dtype=np.int64)
    strength = np.empty(L, dtype=np.float64)
    runs: list[dict[str, Any]] = []
    s, d = int(rng.integers(0, n)), int(rng.integers(0, n))
    pos = 0
    while pos < L:
        end = min(L, pos + int(rng.integers(cfg.hotspot_dwell_range[0], cfg.hotspot_dwell_range[1] + 1)))
        g = float(rng.uniform(*cfg.hotspot_strength_range))
        src[pos:end], dst[pos:end], strength[pos:end] = s, d, g
        runs.append({"start": pos, "end": end, "length": end - pos, "source": s, "destination": d, "strength": g})
        s = (s + int(rng.choice((-1, 0, 1)))) % n
        d = (d + int(rng.choice((-1, 1)))) % n
        pos = end
    return src, dst, strength, runs


_FAMILY_MODE = {
    "regime_switching_long": lambda m, t: {"low": "balanced", "normal": "single_source_hotspot",
                                           "high": "dual_hotspot"}[str(m["latent_regime"][t])],
    "stochastic_volatility": lambda m, t: "sparse_support" if m["volatility_state"][t] == "volatile" else "balanced",
    "rare_shock_recovery": lambda m, t: "dual_hotspot" if m["shock_component"][t] > 0 else "balanced",
    "hotspot_random_walk": lambda m, t: "hotspot_random_walk",
    "same_moments_different_dynamics": lambda m, t: "balanced",
}


def spatial_distribution(cfg: LongHorizonTrafficConfig, total_meta: dict[str, Any],
                         rng: np.random.Generator) -> tuple[np.ndarray, dict[str, Any]]:
    """P_t: [L, n, n] probabilities with a structurally zero diagonal."""
    L, n = cfg.sequence_length, cfg.num_nodes
    off = ~np.eye(n, dtype=bool)
    src, dst, strength, runs = hotspot_walk(cfg, rng)
    groups = np.asarray(cfg.source_groups if cfg.source_groups is not None
                        else tuple(i // max(1, n // 2) for i in range(n)), dtype=np.int64)
    cross = (groups[:, None] != groups[None, :]) & off
    pair_index = np.argwhere(off)
    probs = np.zeros((L, n, n), dtype=np.float64)
    noise = np.zeros((n, n), dtype=np.float64)
    support = off.copy()
    refresh_at = 0
    mode_of = _FAMILY_MODE[cfg.family]
    lookup = {"latent_regime": total_meta["latent_regime"], "volatility_state": total_meta["volatility_state"],
              "shock_component": total_meta["shock_component"]}
    modes: list[str] = []
    for t in range(L):
        mode = cfg.spatial_mode if cfg.spatial_mode is not None else mode_of(lookup, t)
        modes.append(mode)
        noise = 0.92 * noise + rng.normal(0.0, 0.05 if mode == "balanced" else 0.10, size=(n, n))
        w = np.exp(np.clip(noise, -1.5, 1.5))
        w[~off] = 0.0
        g, s, d = strength[t], int(src[t]), int(dst[t])
        if mode == "single_source_hotspot":
            w[s, :] *= g
        elif mode == "single_destination_hotspot":
            w[:, d] *= g
        elif mode == "dual_hotspot":
            w[s, :] *= g
            w[:, d] *= g
        elif mode == "sparse_support":
            if t >= refresh_at:
                pick = rng.choice(len(pair_index), size=max(n, len(pair_index) // 3), replace=False)
                support = np.zeros((n, n), dtype=bool)
                support[tuple(pair_index[pick].T)] = True
                refresh_at = t + int(rng.integers(8, 65))
            w[~support] *= 0.02
        elif mode == "cross_group_concentration":
            w[cross] *= g
        elif mode == "hotspot_random_walk":
            w[:, d] *= g
            w[s, :] *= np.sqrt(g)
        elif mode != "balanced":
            raise ValueError(mode)
        w[~off] = 0.0
        probs[t] = w / w.sum()
    return probs, {"spatial_mode": modes, "hotspot_source": src.astype(int).tolist(),
                   "hotspot_destination": dst.astype(int).tolist(), "hotspot_strength": strength.tolist(),
                   "hotspot_dwell_records": runs, "source_groups": groups.astype(int).tolist()}


def allocate_integer(total: float, probs: np.ndarray, max_entry: int,
                     rng: np.random.Generator) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Largest-deficit integerisation of total * probs with entries capped at max_entry.

    Each unit goes to the available entry with the largest
    ``target * p - count + jitter`` (lower flat index on ties); entries at
    the cap and the diagonal are unavailable.  Returns (matrix, raw, clipped).
    """
    n = probs.shape[0]
    off = ~np.eye(n, dtype=bool)
    target = int(np.clip(np.rint(total), 0, max_entry * int(off.sum())))
    raw = float(total) * probs
    clipped = np.clip(raw, 0.0, max_entry)
    p = probs.ravel()
    jitter = rng.uniform(0.0, 1e-9, size=p.size)
    share = target * p
    counts = np.zeros(p.size, dtype=np.int64)
    heap = [(-(share[i] - 0 + jitter[i]), i) for i in np.flatnonzero(off.ravel())]
    heapq.heapify(heap)
    for _ in range(target):
        if not heap:
            break
        _, i = heapq.heappop(heap)
        counts[i] += 1
        if counts[i] < max_entry:
            heapq.heappush(heap, (-(share[i] - counts[i] + jitter[i]), i))
    out = counts.reshape(n, n)
    np.fill_diagonal(out, 0)
    return out, raw, clipped


# ---------------------------------------------------------------------------
# rolling multi-scale checks
# ---------------------------------------------------------------------------
def rolling_moments(values: np.ndarray, window: int) -> tuple[np.ndarray, np.ndarray]:
    """Population mean / variance of every length-`window` run along axis 0 (prefix sums)."""
    v = np.asarray(values, dtype=np.float64)
    zero = np.zeros((1,) + v.shape[1:])
    c1 = np.concatenate([zero, np.cumsum(v, axis=0)], axis=0)
    c2 = np.concatenate([zero, np.cumsum(v * v, axis=0)], axis=0)
    m = (c1[window:] - c1[:-window]) / float(window)
    var = np.maximum((c2[window:] - c2[:-window]) / float(window) - m * m, 0.0)
    return m, var


def _window_check(err_m: np.ndarray, err_v: np.ndarray, window: int, eps_m, eps_v, allowed) -> dict[str, Any]:
    out: dict[str, Any] = {"available": True, "window_size": window, "num_windows": int(len(err_m)),
                           "mean_error_mean": float(err_m.mean()), "mean_error_max": float(err_m.max()),
                           "variance_error_mean": float(err_v.mean()), "variance_error_max": float(err_v.max()),
                           "epsilon_mean": eps_m, "epsilon_variance": eps_v, "allowed_violation_fraction": allowed}
    if eps_m is None or eps_v is None or allowed is None:
        out.update({"hard_or_soft_bound_applied": False, "violation_fraction": None, "passed": True})
        return out
    frac = float(((err_m > eps_m) | (err_v > eps_v)).mean())
    out.update({"hard_or_soft_bound_applied": True, "violation_fraction": frac,
                "violation_magnitude": {"mean_excess_max": float(np.maximum(err_m - eps_m, 0.0).max()),
                                        "variance_excess_max": float(np.maximum(err_v - eps_v, 0.0).max())},
                "passed": frac <= allowed})
    return out


def scalar_window_check(values: np.ndarray, window: int, ref_mean: float, ref_var: float,
                        eps_m=None, eps_v=None, allowed=None) -> dict[str, Any]:
    """Relative errors |m - ref| / max(|ref|, 1) of every window of a scalar series."""
    if window > len(values):
        return {"available": False, "window_size": window, "num_windows": 0}
    m, v = rolling_moments(values, window)
    return _window_check(np.abs(m - ref_mean) / max(abs(ref_mean), 1.0),
                         np.abs(v - ref_var) / max(abs(ref_var), 1.0), window, eps_m, eps_v, allowed)


def matrix_window_check(stack: np.ndarray, window: int, mean_ref: np.ndarray, var_ref: np.ndarray,
                        eps_m=None, eps_v=None, allowed=None) -> dict[str, Any]:
    """Relative L2 errors ||m - ref|| / (||ref|| + 1e-8) of every window of a matrix series."""
    if window > len(stack):
        return {"available": False, "window_size": window, "num_windows": 0}
    m, v = rolling_moments(stack, window)
    axes = tuple(range(1, m.ndim))
    em = np.sqrt(np.sum((m - mean_ref) ** 2, axis=axes)) / (float(np.linalg.norm(mean_ref)) + 1e-8)
    ev = np.sqrt(np.sum((v - var_ref) ** 2, axis=axes)) / (float(np.linalg.norm(var_ref)) + 1e-8)
    return _window_check(em, ev, window, eps_m, eps_v, allowed)


def _summary(x: np.ndarray) -> dict[str, float]:
    a = np.asarray(x, dtype=np.float64)
    return {"mean": float(a.mean()), "variance": float(a.var(ddof=0)), "p99": float(np.quantile(a, 0.99)),
            "maximum": float(a.max())}


# ---------------------------------------------------------------------------
# candidates
# ---------------------------------------------------------------------------
def build_candidate(cfg: LongHorizonTrafficConfig, index: int) -> TrafficSequence:
    total_rng, spatial_rng, alloc_rng = (np.random.default_rng(s)
                                         for s in np.random.SeedSequence([cfg.seed, index]).spawn(3))
    totals, tmeta = total_load(cfg, total_rng)
    probs, smeta = spatial_distribution(cfg, tmeta, spatial_rng)
    mats, raws, clips = [], [], []
    for s_t, p_t in zip(totals, probs):
        m, raw, clipped = allocate_integer(s_t, p_t, cfg.max_entry, alloc_rng)
        validate_traffic_matrix(m)
        mats.append(m)
        raws.append(raw)
        clips.append(clipped)
    stack = np.stack(mats)
    realised = stack.sum(axis=(1, 2)).astype(np.float64)
    n = cfg.num_nodes
    off = ~np.eye(n, dtype=bool)
    mean_ref = np.where(off, cfg.mean_level, 0.0)
    var_ref = np.where(off, cfg.std_level ** 2, 0.0)
    ref_total_mean = cfg.base_total
    # configured (never realised) total variance; rare shocks raise it by design
    ref_total_var = float((cfg.std_level * np.sqrt(cfg.pairs)) ** 2)
    if cfg.family == "rare_shock_recovery":
        ref_total_var = max(ref_total_var, (0.30 * ref_total_mean) ** 2)
    levels = (("short", cfg.short_window, None, None, None, None, None),
              ("medium", cfg.medium_window, cfg.medium_epsilon_mean, cfg.medium_epsilon_var,
               cfg.medium_matrix_epsilon_mean, cfg.medium_matrix_epsilon_var, cfg.medium_allowed_violation_fraction),
              ("long", cfg.long_window, cfg.long_epsilon_mean, cfg.long_epsilon_var,
               cfg.long_matrix_epsilon_mean, cfg.long_matrix_epsilon_var, cfg.long_allowed_violation_fraction))
    scalar = {name: scalar_window_check(realised, w, ref_total_mean, ref_total_var, em, ev, frac)
              for name, w, em, ev, _, _, frac in levels}
    matrix = {name: matrix_window_check(stack, w, mean_ref, var_ref, mm, mv, frac)
              for name, w, _, _, mm, mv, frac in levels}
    meta: dict[str, Any] = {
        "schema_version": 1, "generator_kind": "long-horizon generator", "generator_name": "long_horizon_v1",
        "family": cfg.family, "seed": cfg.seed, "sequence_length": cfg.sequence_length,
        "window_size": cfg.short_window, "generator_config": asdict(cfg),
        "metadata_usage": "audit/evaluation only; latent state is not a policy input",
        "total_traffic": realised.astype(int).tolist(), "total_traffic_pre_integer": totals.tolist(),
        "pre_clip_statistics": _summary(np.stack(raws)[:, off]),
        "post_clip_statistics": _summary(np.stack(clips)[:, off]),
        "post_integer_statistics": _summary(stack[:, off]),
        "diagonal_zeroing": {"pre_nonzero_count": 0, "post_nonzero_count": 0,
                             "note": "P_t diagonal is structurally zero before integerization"},
        "spatial_distribution_validation": {
            "minimum_probability": float(probs.min()), "maximum_probability": float(probs.max()),
            "maximum_sum_error": float(np.max(np.abs(probs.sum(axis=(1, 2)) - 1.0))),
            "diagonal_nonzero_count": int(np.count_nonzero(np.diagonal(probs, axis1=1, axis2=2)))},
        "multi_scale_constraints": scalar, "matrix_multi_scale_constraints": matrix,
        "reference_total_mean": ref_total_mean, "reference_total_variance": ref_total_var,
        "generation_attempt": index + 1, **tmeta, **smeta,
    }
    variant = meta.get("dynamics_variant")
    return TrafficSequence(sequence_id=f"{cfg.family}{'-' + variant if variant else ''}-seed{cfg.seed}",
                           topology_name=cfg.topology_name, family=cfg.family, seed=cfg.seed, matrices=mats,
                           mean_ref=mean_ref, var_ref=var_ref,
                           bounds=MomentBounds(cfg.long_epsilon_mean, cfg.long_epsilon_var), metadata=meta)


def constraint_penalty(seq: TrafficSequence) -> float:
    """Sum over medium/long scalar and matrix checks of (violation fraction - allowed)+."""
    pen = 0.0
    for key in ("multi_scale_constraints", "matrix_multi_scale_constraints"):
        for level in ("medium", "long"):
            c = seq.metadata[key][level]
            if c["available"]:
                pen += max(float(c["violation_fraction"]) - float(c["allowed_violation_fraction"]), 0.0)
    return pen


def generate_long_horizon_sequence(cfg: LongHorizonTrafficConfig) -> TrafficSequence:
    """Best of up to ``calibration_candidates`` candidates; stops at the first that violates nothing."""
    best, best_pen = None, float("inf")
    for i in range(cfg.calibration_candidates):
        cand = build_candidate(cfg, i)
        pen = constraint_penalty(cand)
        if pen < best_pen:
            best, best_pen = cand, pen
        if pen <= 0.0:
            break
    best.metadata["calibration_candidates_evaluated"] = int(best.metadata["generation_attempt"])
    best.metadata["constraint_penalty"] = float(best_pen)
    best.metadata["constraint_status"] = "passed" if best_pen <= 0.0 else "best_effort"
    return best


def generate_same_moment_group(cfg: LongHorizonTrafficConfig) -> dict[str, TrafficSequence]:
    """The four same-moment dynamics variants of one configuration."""
    if cfg.family != "same_moments_different_dynamics":
        raise ValueError("generate_same_moment_group requires same_moments_different_dynamics")
    base = asdict(cfg)
    return {v: generate_long_horizon_sequence(LongHorizonTrafficConfig(**{**base, "dynamics_variant": v}))
            for v in SAME_MOMENT_VARIANTS}


__all__ = ["LONG_HORIZON_FAMILIES", "LongHorizonTrafficConfig", "SAME_MOMENT_VARIANTS", "SPATIAL_MODES",
           "allocate_integer", "build_candidate", "constraint_penalty", "generate_long_horizon_sequence",
           "generate_same_moment_group", "matrix_window_check", "rolling_moments", "scalar_window_check"]
