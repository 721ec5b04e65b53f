"""Serializable types of moment-bounded traffic sequences (rlccl/traffic/types.py).

``MomentBounds`` (relative-L2 tolerances on mean / variance),
``MomentContext`` (history-only sliding moments seen by a policy at one
step) and ``TrafficSequence`` (a seeded sequence of traffic matrices with its
reference moments); all round-trip through JSON dicts.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any

import numpy as np


def _arr(v: Any, dtype=np.float64) -> np.ndarray:
    return np.asarray(v, dtype=dtype)


def _jsonable(v: Any) -> Any:
    if isinstance(v, np.ndarray):
        return v.tolist()
    if isinstance(v, np.generic):
        return v.item()
    if isinstance(v, dict):
        return {str(k): _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    return v


@dataclass(frozen=True)
class MomentBounds:
    epsilon_mean: float
    epsilon_var: float
    norm: str = "relative_l2"

    def __post_init__(self) -> None:
        if self.epsilon_mean < 0 or self.epsilon_var < 0:
            raise ValueError("Moment tolerances must be nonnegative")
        if self.norm != "relative_l2":
            raise ValueError(f"Unsupported moment norm: {self.norm}")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "MomentBounds":
        return cls(**d)


_MC_ARRAYS = ("mean_matrix", "var_matrix", "std_matrix", "send_mean", "recv_mean", "send_std", "recv_std",
              "current_send_z", "current_recv_z")


@dataclass
class MomentContext:
    history_length: int
    window_size: int
    mean_matrix: np.ndarray
    var_matrix: np.ndarray
    std_matrix: np.ndarray
    send_mean: np.ndarray
    recv_mean: np.ndarray
    send_std: np.ndarray
    recv_std: np.ndarray
    current_send_z: np.ndarray
    current_recv_z: np.ndarray
    mean_drift: float
    var_drift: float
    confidence: float
    is_warm: bool

    def __post_init__(self) -> None:
        for name in _MC_ARRAYS:
            setattr(self, name, _arr(getattr(self, name)))
        self.confidence = float(np.clip(self.confidence, 0.0, 1.0))

    def to_dict(self) -> dict:
        return _jsonable(asdict(self))

    @classmethod
    def from_dict(cls, d: dict) -> "MomentContext":
        v = dict(d)
        for name in _MC_ARRAYS:
            v[name] = _arr(v[name])
        return cls(**v)


@dataclass
class TrafficSequence:
    sequence_id: str
    topology_name: str
    family: str
    seed: int
    matrices: list
    mean_ref: np.ndarray
    var_ref: np.ndarray
    bounds: MomentBounds
    metadata: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.matrices = [_arr(m, np.int64) for m in self.matrices]
        self.mean_ref = _arr(self.mean_ref)
        self.var_ref = _arr(self.var_ref)
        if isinstance(self.bounds, dict):
            self.bounds = MomentBounds.from_dict(self.bounds)

    def to_dict(self) -> dict:
        return {"sequence_id": self.sequence_id, "topology_name": self.topology_name, "family": self.family,
                "seed": int(self.seed), "matrices": [m.tolist() for m in self.matrices],
                "mean_ref": self.mean_ref.tolist(), "var_ref": self.var_ref.tolist(),
                "bounds": self.bounds.to_dict(), "metadata": _jsonable(self.metadata)}

    @classmethod
    def from_dict(cls, d: dict) -> "TrafficSequence":
        return cls(d["sequence_id"], d["topology_name"], d["family"], int(d["seed"]),
                   [_arr(m, np.int64) for m in d["matrices"]], _arr(d["mean_ref"]), _arr(d["var_ref"]),
                   MomentBounds.from_dict(d["bounds"]), dict(d.get("metadata", {})))


__all__ = ["MomentBounds", "MomentContext", "TrafficSequence"]
