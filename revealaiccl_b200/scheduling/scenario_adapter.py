"""Observation-bound scenario supports (rlccl/scheduling/scenario_adapter.py:47-156).

An ordinary planner may only receive supports built without oracle
information; the truth-assisted (oracle) support is evaluator-only and marked
``uses_oracle``/``upper_bound_only``.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Mapping, Sequence

import numpy as np

from ..uncertainty.observation import readonly_array
from .robust_prefix import canonical_digest


@dataclass(frozen=True, slots=True)
class ScenarioSupport:
    method: str
    requested_k: int
    actual_k: int
    matrices: tuple[np.ndarray, ...]
    weights: tuple[float, ...]
    provenance: Mapping[str, Any]
    stage: int
    observation_digest: str
    observation: Any
    digest: str
    uses_oracle: bool = False
    upper_bound_only: bool = False

    def __post_init__(self) -> None:
        mats = tuple(readonly_array(m, dtype=np.int64) for m in self.matrices)
        w = tuple(float(v) for v in self.weights)
        if not mats or len(mats) != self.actual_k or len(w) != self.actual_k:
            raise ValueError("actual_k must match nonempty matrices and weights")
        shape = mats[0].shape
        if len(shape) != 2 or shape[0] != shape[1] or any(m.shape != shape for m in mats):
            raise ValueError("scenario matrices must be same-size square matrices")
        if any(np.any(m < 0) or np.any(np.diag(m) != 0) for m in mats):
            raise ValueError("scenario matrices must be nonnegative with zero diagonal")
        if any(not np.isfinite(v) or v <= 0 for v in w):
            raise ValueError("scenario weights must be finite and positive")
        total = sum(w)
        object.__setattr__(self, "matrices", mats)
        object.__setattr__(self, "weights", tuple(v / total for v in w))
        object.__setattr__(self, "provenance", MappingProxyType(dict(self.provenance)))


def scenario_support_from_matrices(*, matrices: Sequence[np.ndarray], weights: Sequence[float],
                                   method: str, requested_k: int, uses_oracle: bool,
                                   upper_bound_only: bool, provenance: Mapping[str, Any],
                                   observation: Any) -> ScenarioSupport:
    if uses_oracle or upper_bound_only:
        raise ValueError("oracle/upper-bound support is forbidden for an ordinary planner")
    mats = tuple(np.asarray(m) for m in matrices)
    w = tuple(float(v) for v in weights)
    if int(requested_k) <= 0:
        raise ValueError("requested_k must be positive")
    if len(mats) != len(w) or not mats:
        raise ValueError("matrices and weights must have equal positive length")
    payload = (str(method), int(requested_k), mats, w, dict(provenance), int(observation.stage),
               str(observation.observation_digest))
    return ScenarioSupport(str(method), int(requested_k), len(mats), mats, w, dict(provenance),
                           int(observation.stage), str(observation.observation_digest), observation,
                           canonical_digest(payload))


def scenario_support_from_selected(selected: Any, *, observation: Any) -> ScenarioSupport:
    prov = {"selected_indices": tuple(getattr(selected, "selected_indices", ())),
            "history_offsets": tuple(getattr(selected, "history_offsets", ())),
            "severity_definition": getattr(selected, "severity_definition", None),
            "approximation": getattr(selected, "approximation", None)}
    return scenario_support_from_matrices(
        matrices=selected.matrices, weights=selected.weights, method=selected.method,
        requested_k=selected.requested_k, uses_oracle=selected.uses_oracle,
        upper_bound_only=selected.upper_bound_only, provenance=prov, observation=observation)


def oracle_support_from_matrices(*, matrices: Sequence[np.ndarray], weights: Sequence[float],
                                 requested_k: int, provenance: Mapping[str, Any],
                                 observation: Any) -> ScenarioSupport:
    """Evaluator-only truth-assisted support (duplicates merged, weights summed)."""
    mats = tuple(np.asarray(m) for m in matrices)
    w = tuple(float(v) for v in weights)
    if not mats or len(mats) != len(w):
        raise ValueError("oracle matrices and weights must have equal positive length")
    if int(requested_k) != 8 or len(mats) > 8:
        raise ValueError("oracle support requires requested K8 and actual K in 1..8")
    uniq: list[np.ndarray] = []
    uw: list[float] = []
    pos: dict[tuple, int] = {}
    for m, v in zip(mats, w):
        c = np.ascontiguousarray(m, dtype=np.int64)
        key = (c.dtype.str, c.shape, c.tobytes())
        if key in pos:
            uw[pos[key]] += v
        else:
            pos[key] = len(uniq)
            uniq.append(c)
            uw.append(v)
    payload = ("oracle_scenario_robust_reference", requested_k, tuple(uniq), tuple(uw),
               dict(provenance), observation.stage, observation.observation_digest)
    return ScenarioSupport("oracle_scenario_robust_reference", 8, len(uniq), tuple(uniq), tuple(uw),
                           dict(provenance), int(observation.stage), str(observation.observation_digest),
                           observation, canonical_digest(payload), True, True)


__all__ = ["ScenarioSupport", "oracle_support_from_matrices", "scenario_support_from_matrices",
           "scenario_support_from_selected"]
