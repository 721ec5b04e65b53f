"""All-to-All-V traffic matrices <-> chunk scenarios (rlccl/traffic/matrix_utils.py:8-95).

A traffic matrix ``X[src, dst] = k`` means ``src`` must deliver ``k`` atomic
chunks to ``dst``; it must be square, finite, nonnegative, integer-valued and
zero on the diagonal.
"""

from __future__ import annotations

from typing import Any

import numpy as np


def validate_traffic_matrix(matrix: np.ndarray) -> None:
    a = np.asarray(matrix)
    if a.ndim != 2 or a.shape[0] != a.shape[1]:
        raise ValueError(f"Traffic matrix must be square, got shape {a.shape}")
    if not np.issubdtype(a.dtype, np.number):
        raise ValueError("Traffic matrix must be numeric")
    if not np.all(np.isfinite(a)):
        raise ValueError("Traffic matrix must contain only finite values")
    if np.any(a < 0):
        raise ValueError("Traffic matrix entries must be nonnegative")
    if not np.all(a == np.floor(a)):
        raise ValueError("Traffic matrix entries must be integer-valued")
    if np.any(np.diag(a) != 0):
        raise ValueError("Traffic matrix diagonal must be zero")


def traffic_matrix_to_scenario(matrix: np.ndarray, **metadata: Any) -> dict[str, Any]:
    """One chunk per unit of demand, ordered by (src, dst): initial_state marks
    the source, demands mark the destination.  A zero matrix gives C = 0."""
    validate_traffic_matrix(matrix)
    traffic = np.asarray(matrix, dtype=np.int64)
    n = traffic.shape[0]
    src, dst = np.nonzero(traffic)
    counts = traffic[src, dst]
    chunk_src = np.repeat(src, counts)
    chunk_dst = np.repeat(dst, counts)
    c = int(counts.sum())
    initial_state = np.zeros((c, n), dtype=np.int64)
    demands = np.zeros((c, n), dtype=np.int64)
    initial_state[np.arange(c), chunk_src] = 1
    demands[np.arange(c), chunk_dst] = 1
    scenario = dict(metadata)
    scenario.update({
        "type": "all_to_all_v", "V": n, "traffic_matrix": traffic.tolist(), "C": c,
        "initial_state": initial_state.tolist(), "demands": demands.tolist(),
    })
    return scenario


def scenario_to_traffic_matrix(scenario: dict[str, Any]) -> np.ndarray:
    """Return the stored matrix, or rebuild it when every chunk has exactly one
    source and one (different) destination."""
    if scenario.get("traffic_matrix") is not None:
        m = np.asarray(scenario["traffic_matrix"])
        validate_traffic_matrix(m)
        return m.astype(np.int64, copy=True)
    init = np.asarray(scenario.get("initial_state"))
    dem = np.asarray(scenario.get("demands"))
    if init.size == 0 and dem.size == 0 and int(scenario.get("C", -1)) == 0:
        n = int(scenario.get("V", 0))
        if n <= 0:
            raise ValueError("Empty scenarios need positive V metadata")
        return np.zeros((n, n), dtype=np.int64)
    if init.ndim != 2 or dem.ndim != 2 or init.shape != dem.shape:
        raise ValueError("Scenario needs same-shaped 2-D initial_state and demands")
    n = init.shape[1]
    out = np.zeros((n, n), dtype=np.int64)
    for c in range(init.shape[0]):
        s = np.flatnonzero(init[c])
        d = np.flatnonzero(dem[c])
        if len(s) != 1 or len(d) != 1:
            raise ValueError("Cannot reconstruct All-to-All-V traffic: each chunk must have "
                             "exactly one source and one destination")
        if s[0] == d[0]:
            raise ValueError("All-to-All-V chunks cannot demand their source node")
        out[s[0], d[0]] += 1
    validate_traffic_matrix(out)
    return out
