"""Planning-only scenarios whose tokens live in a non-executable namespace
(rlccl/uncertainty/scenarios.py:15-119).  A ``ScenarioTokenId`` must start
with ``scenario:``; the trusted checker never accepts one."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np

from ..traffic.matrix_utils import validate_traffic_matrix
from .observation import readonly_array


@dataclass(frozen=True, slots=True)
class ScenarioTokenId:
    value: str

    def __post_init__(self) -> None:
        if not isinstance(self.value, str) or not self.value.startswith("scenario:"):
            raise ValueError("Scenario token IDs must use the scenario: namespace")

    def __str__(self) -> str:
        return self.value


@dataclass(frozen=True, slots=True)
class ScenarioDemandToken:
    token_id: ScenarioTokenId
    source: int
    destination: int

    def __post_init__(self) -> None:
        if not isinstance(self.token_id, ScenarioTokenId):
            raise TypeError("ScenarioDemandToken requires ScenarioTokenId")
        if self.source < 0 or self.destination < 0 or self.source == self.destination:
            raise ValueError("Invalid scenario demand endpoints")


@dataclass(frozen=True, slots=True)
class ScenarioSet:
    matrices: tuple[np.ndarray, ...]
    weights: tuple[float, ...]
    scenario_ids: tuple[str, ...]
    provenance: tuple[str, ...]
    scenario_tokens: tuple[tuple[ScenarioDemandToken, ...], ...]

    def __post_init__(self) -> None:
        raw = tuple(np.asarray(m) for m in self.matrices)
        for m in raw:
            validate_traffic_matrix(m)
        mats = tuple(readonly_array(m, dtype=np.int64) for m in raw)
        weights = tuple(float(w) for w in self.weights)
        ids = tuple(str(v) for v in self.scenario_ids)
        prov = tuple(str(v) for v in self.provenance)
        n = len(mats)
        if not n or not (len(weights) == len(ids) == len(prov) == n):
            raise ValueError("Scenario fields must be non-empty and aligned")
        if len(set(ids)) != n:
            raise ValueError("scenario_ids must be unique")
        if any(not np.isfinite(w) or w < 0 for w in weights):
            raise ValueError("Scenario weights must be finite and nonnegative")
        total = float(sum(weights))
        if total <= 0:
            raise ValueError("Scenario weights must have positive total")
        tokens = tuple(tuple(g) for g in self.scenario_tokens)
        if len(tokens) != n:
            raise ValueError("Scenario token groups must align with matrices")
        object.__setattr__(self, "matrices", mats)
        object.__setattr__(self, "weights", tuple(w / total for w in weights))
        object.__setattr__(self, "scenario_ids", ids)
        object.__setattr__(self, "provenance", prov)
        object.__setattr__(self, "scenario_tokens", tokens)

    @classmethod
    def from_matrices(cls, *, matrices: Sequence[np.ndarray], weights: Sequence[float],
                      scenario_ids: Sequence[str], provenance: Sequence[str]) -> "ScenarioSet":
        copied = tuple(np.array(m, dtype=np.int64, copy=True) for m in matrices)
        ids = tuple(str(v) for v in scenario_ids)
        groups = []
        for sid, m in zip(ids, copied):
            validate_traffic_matrix(m)
            toks = []
            local = 0
            for s in range(m.shape[0]):
                for d in range(m.shape[1]):
                    for _ in range(int(m[s, d])):
                        toks.append(ScenarioDemandToken(ScenarioTokenId(f"scenario:{sid}:{local}"), s, d))
                        local += 1
            groups.append(tuple(toks))
        return cls(copied, tuple(weights), ids, tuple(provenance), tuple(groups))


__all__ = ["ScenarioDemandToken", "ScenarioSet", "ScenarioTokenId"]
