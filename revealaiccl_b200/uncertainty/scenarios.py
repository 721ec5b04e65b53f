"""Planning scenarios: demand matrices a planner may reason about but never execute.

A scenario's tokens carry ids in their own ``scenario:`` namespace, so the
trusted checker (``execution.commit_proposal``), which accepts only
``TruthTokenId``, can never be handed one.  Interface and verdicts follow
rlccl/uncertainty/scenarios.py:15-119 (field names, the id namespace, the
per-scenario token order source-major then destination then local index);
the construction here is vectorised: the token list of a matrix is the
row-major expansion of its entries, produced with one ``np.repeat``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np

from ..traffic.matrix_utils import validate_traffic_matrix
from .observation import readonly_array

SCENARIO_NAMESPACE = "scenario:"


@dataclass(frozen=True, slots=True)
class ScenarioTokenId:
    value: str

    def __post_init__(self) -> None:
        if not (isinstance(self.value, str) and self.value.startswith(SCENARIO_NAMESPACE)):
            raise ValueError(f"a scenario token id lives in the {SCENARIO_NAMESPACE!r} namespace")

    def __str__(self) -> str:
        return self.value


@dataclass(frozen=True, slots=True)
class ScenarioDemandToken:
    token_id: ScenarioTokenId
    source: int
    destination: int

    def __post_init__(self) -> None:
        if not isinstance(self.token_id, ScenarioTokenId):
            raise TypeError("a scenario demand token needs a ScenarioTokenId")
        if min(self.source, self.destination) < 0 or self.source == self.destination:
            raise ValueError("scenario demand endpoints must be two distinct nonnegative nodes")


def _expand_tokens(scenario_id: str, matrix: np.ndarray) -> tuple[ScenarioDemandToken, ...]:
    """One token per unit of demand, in row-major entry order."""
    n = matrix.shape[1]
    cells = np.repeat(np.arange(matrix.size, dtype=np.int64), matrix.reshape(-1))
    return tuple(ScenarioDemandToken(ScenarioTokenId(f"{SCENARIO_NAMESPACE}{scenario_id}:{local}"),
                                     int(cell // n), int(cell % n))
                 for local, cell in enumerate(cells.tolist()))


@dataclass(frozen=True, slots=True)
class ScenarioSet:
    matrices: tuple[np.ndarray, ...]
    weights: tuple[float, ...]
    scenario_ids: tuple[str, ...]
    provenance: tuple[str, ...]
    scenario_tokens: tuple[tuple[ScenarioDemandToken, ...], ...]

    def __post_init__(self) -> None:
        given = [np.asarray(m) for m in self.matrices]
        for m in given:
            validate_traffic_matrix(m)
        matrices = tuple(readonly_array(m, dtype=np.int64) for m in given)
        ids = tuple(map(str, self.scenario_ids))
        provenance = tuple(map(str, self.provenance))
        raw_weights = np.asarray(list(self.weights), dtype=np.float64)
        groups = tuple(tuple(g) for g in self.scenario_tokens)
        count = len(matrices)
        lengths = {len(raw_weights), len(ids), len(provenance)}
        if count == 0 or lengths != {count}:
            raise ValueError("scenario matrices, weights, ids and provenance must be non-empty and of equal length")
        if len(frozenset(ids)) != count:
            raise ValueError("scenario ids repeat")
        if not np.all(np.isfinite(raw_weights)) or np.any(raw_weights < 0):
            raise ValueError("scenario weights must be finite and nonnegative")
        total = float(raw_weights.sum())
        if total <= 0:
            raise ValueError("scenario weights sum to zero")
        if len(groups) != count:
            raise ValueError("one scenario token group is needed per matrix")
        frozen = {"matrices": matrices, "weights": tuple(float(w) / total for w in raw_weights.tolist()),
                  "scenario_ids": ids, "provenance": provenance, "scenario_tokens": groups}
        for name, value in frozen.items():
            object.__setattr__(self, name, value)

    @classmethod
    def from_matrices(cls, *, matrices: Sequence[np.ndarray], weights: Sequence[float],
                      scenario_ids: Sequence[str], provenance: Sequence[str]) -> "ScenarioSet":
        given = [np.asarray(m) for m in matrices]
        for m in given:  # validate before any cast, so a fractional entry is refused, not truncated
            validate_traffic_matrix(m)
        owned = [np.array(m, dtype=np.int64, copy=True) for m in given]
        ids = [str(v) for v in scenario_ids]
        groups = tuple(_expand_tokens(sid, m) for sid, m in zip(ids, owned))
        return cls(matrices=tuple(owned), weights=tuple(weights), scenario_ids=tuple(ids),
                   provenance=tuple(provenance), scenario_tokens=groups)


__all__ = ["ScenarioDemandToken", "ScenarioSet", "ScenarioTokenId"]
