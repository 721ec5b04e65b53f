"""Topology and collective-problem records.

``TopologyInfo`` and ``ProblemInstance`` keep the field names of the
reference (rlccl/envs/problem.py:33-263) because the RL checkpoint layout,
scenario caches and scheduler interfaces are keyed on them:

* ``TopologyInfo(V, E, edges, capacities, shared_constraints)`` with derived
  ``edge_src``, ``edge_dst``, ``dist_matrix`` (hop counts, unreachable =
  V + 1) and ``group_map`` (edge -> [(group, limit)]).
* ``ProblemInstance(V, C, E, T, capacities, topology, demands, initial_state,
  shared_constraints, ...)`` with ``to_dict``/``from_dict`` JSON round-trip.

Shortest hop distances are computed by a BFS from every source (all links
have unit hop cost), not by the reference's dense Floyd-Warshall.
"""

from __future__ import annotations

from collections import deque
from dataclasses import asdict, is_dataclass
import os
from typing import Any, Sequence

import numpy as np


def _json_compatible(value: Any) -> Any:
    if isinstance(value, np.ndarray):
        return value.tolist()
    if isinstance(value, np.generic):
        return value.item()
    if is_dataclass(value) and not isinstance(value, type):
        return _json_compatible(asdict(value))
    if isinstance(value, dict):
        return {str(k): _json_compatible(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_json_compatible(v) for v in value]
    return value


def hop_distances(num_nodes: int, edges: np.ndarray) -> np.ndarray:
    """All-pairs hop distances as float32; unreachable pairs get ``V + 1``."""
    unreachable = float(num_nodes + 1)
    dist = np.full((num_nodes, num_nodes), unreachable, dtype=np.float32)
    adjacency: list[list[int]] = [[] for _ in range(num_nodes)]
    for u, v in np.asarray(edges, dtype=np.int64).reshape(-1, 2):
        adjacency[int(u)].append(int(v))
    for source in range(num_nodes):
        dist[source, source] = 0.0
        queue = deque([source])
        while queue:
            node = queue.popleft()
            for nxt in adjacency[node]:
                if dist[source, nxt] == unreachable:
                    dist[source, nxt] = dist[source, node] + 1.0
                    queue.append(nxt)
    return dist


class TopologyInfo:
    """Static link graph: nodes, directed edges, capacities, shared groups."""

    def __init__(self, V, E, edges, capacities, shared_constraints, cache_dir=None, name=None):
        self.V = int(V)
        self.E = int(E)
        self.edges = np.asarray(edges, dtype=np.int64).reshape(-1, 2)
        self.capacities = np.asarray(capacities, dtype=np.float64)
        self.shared_constraints = [
            (list(int(e) for e in idx), float(limit)) for idx, limit in shared_constraints
        ]
        self.cache_dir = cache_dir
        self.name = name
        if self.edges.shape[0] != self.E or self.capacities.shape != (self.E,):
            raise ValueError("edge/capacity count does not match E")
        self.edge_src = self.edges[:, 0]
        self.edge_dst = self.edges[:, 1]
        self.dist_matrix = self._shortest_paths()
        self.group_map: dict[int, list[tuple[int, float]]] = {}
        for g_idx, (edge_indices, limit) in enumerate(self.shared_constraints):
            for e in edge_indices:
                self.group_map.setdefault(int(e), []).append((g_idx, float(limit)))

    @property
    def num_nodes(self) -> int:
        return self.V

    def _shortest_paths(self) -> np.ndarray:
        if self.cache_dir is not None:
            cache_file = os.path.join(self.cache_dir, "shortest_paths.npy")
            if os.path.exists(cache_file):
                try:
                    dist = np.load(cache_file)
                    if dist.shape == (self.V, self.V):
                        return dist
                except Exception:
                    pass
        dist = hop_distances(self.V, self.edges)
        if self.cache_dir is not None:
            try:
                os.makedirs(self.cache_dir, exist_ok=True)
                np.save(os.path.join(self.cache_dir, "shortest_paths.npy"), dist)
            except OSError:
                pass
        return dist

    def to_dict(self) -> dict:
        return {
            "V": self.V,
            "E": self.E,
            "edges": self.edges.tolist(),
            "capacities": self.capacities.tolist(),
            "shared_constraints": _json_compatible(self.shared_constraints),
            "cache_dir": self.cache_dir,
            "name": self.name,
        }

    @classmethod
    def from_dict(cls, data: dict) -> "TopologyInfo":
        return cls(
            V=data["V"], E=data["E"], edges=np.array(data["edges"]),
            capacities=np.array(data["capacities"]),
            shared_constraints=data.get("shared_constraints", []),
            cache_dir=data.get("cache_dir"), name=data.get("name"),
        )


class ProblemInstance:
    """A collective-schedule problem: chunk demands over a topology for T slots."""

    def __init__(self, num_nodes, num_chunks, num_edges, time_limit, capacities, topology,
                 demands, initial_state, shared_constraints=None, topology_info=None,
                 traffic_matrix=None, scenario_type=None, sequence_id=None, sequence_step=None,
                 moment_context=None, metadata=None):
        self.V = int(num_nodes)
        self.C = int(num_chunks)
        self.E = int(num_edges)
        self.T = int(time_limit)
        self.capacities = np.asarray(capacities)
        self.k = np.min(self.capacities) if len(self.capacities) > 0 else 0
        self.topology = topology
        self.demands = np.asarray(demands)
        self.initial_state = np.asarray(initial_state)
        self.shared_constraints = shared_constraints if shared_constraints is not None else []
        self.traffic_matrix = None if traffic_matrix is None else np.asarray(traffic_matrix).copy()
        self.scenario_type = scenario_type
        self.sequence_id = sequence_id
        self.sequence_step = sequence_step
        self.moment_context = moment_context
        self.metadata = dict(metadata) if metadata is not None else {}
        self.topology_info = topology_info if topology_info is not None else TopologyInfo(
            self.V, self.E, np.array(topology), np.array(capacities), self.shared_constraints
        )

    def to_dict(self) -> dict:
        return {
            "V": self.V, "C": self.C, "E": self.E, "T": self.T,
            "capacities": _json_compatible(self.capacities),
            "topology": _json_compatible(self.topology),
            "demands": _json_compatible(self.demands),
            "initial_state": _json_compatible(self.initial_state),
            "shared_constraints": _json_compatible(self.shared_constraints),
            "topology_info": self.topology_info.to_dict(),
            "traffic_matrix": _json_compatible(self.traffic_matrix),
            "scenario_type": self.scenario_type,
            "sequence_id": self.sequence_id,
            "sequence_step": self.sequence_step,
            "moment_context": _json_compatible(self.moment_context),
            "metadata": _json_compatible(self.metadata),
        }

    @classmethod
    def from_dict(cls, data: dict) -> "ProblemInstance":
        topo = data.get("topology_info")
        moment = data.get("moment_context")
        if moment is not None:
            from ..traffic.types import MomentContext

            moment = MomentContext.from_dict(moment)
        return cls(
            num_nodes=data["V"], num_chunks=data["C"], num_edges=data["E"], time_limit=data["T"],
            capacities=np.array(data["capacities"]),
            topology=[tuple(e) for e in data["topology"]],
            demands=np.array(data["demands"]), initial_state=np.array(data["initial_state"]),
            shared_constraints=data.get("shared_constraints", []),
            topology_info=TopologyInfo.from_dict(topo) if topo else None,
            traffic_matrix=data.get("traffic_matrix"), scenario_type=data.get("scenario_type"),
            sequence_id=data.get("sequence_id"), sequence_step=data.get("sequence_step"),
            moment_context=moment, metadata=data.get("metadata"),
        )


def compute_received_chunks(Y_t: np.ndarray, edge_dst: np.ndarray, V: int) -> np.ndarray:
    """N_t[c, v] = 1 iff some edge e with Y_t[c, e] = 1 ends at v (rlccl/envs/problem.py:266-296)."""
    Y = np.asarray(Y_t)
    out = np.zeros((Y.shape[0], int(V)), dtype=np.int32)
    chunks, edges = np.nonzero(Y)
    if chunks.size:
        out[chunks, np.asarray(edge_dst)[edges]] = 1
    return out


def normalize_capacities(capacities: np.ndarray, shared: Sequence) -> tuple[np.ndarray, list]:
    """Divide every capacity and group limit by the minimum link capacity
    (rlccl/envs/evaluator.py:359-388)."""
    caps = np.asarray(capacities, dtype=np.float64)
    minimum = float(np.min(caps)) if caps.size else 0.0
    if minimum > 0:
        return caps / minimum, [(list(idx), float(limit) / minimum) for idx, limit in shared]
    return caps, [(list(idx), float(limit)) for idx, limit in shared]
