"""Evaluator-owned truth world (rlccl/uncertainty/problem.py:16-143).

``UncertainProblemInstance`` expands a private truth traffic matrix into
atomic tokens ``(source, destination, local_index)`` ordered by (source,
destination, local index), tracks token possession per node, and issues an
opaque ``TruthTokenId`` — ``"truth:" + sha256(seq|step|reveal_seed|src|dst|local)``
— only when a token is revealed.  It is a capability: ordinary planners only
ever see ``PartialObservationState``.
"""

from __future__ import annotations

from copy import deepcopy
from hashlib import sha256
from typing import Any, Mapping

import numpy as np

from ..topology.info import TopologyInfo
from ..traffic.matrix_utils import validate_traffic_matrix
from .observation import PublicTopologyView, TruthTokenId


class UncertainProblemInstance:
    def __init__(self, *, truth_matrix: np.ndarray, topology_info: TopologyInfo, time_limit: int,
                 sequence_id: str, sequence_step: int, family: str,
                 generator_metadata: Mapping[str, Any]) -> None:
        validate_traffic_matrix(np.asarray(truth_matrix))
        truth = np.array(truth_matrix, dtype=np.int64, copy=True)
        n = int(topology_info.V)
        if truth.shape != (n, n):
            raise ValueError("Traffic matrix and topology node count mismatch")
        if int(time_limit) <= 0:
            raise ValueError("time_limit must be positive")
        self.topology_info = TopologyInfo(
            n, int(topology_info.E), np.array(topology_info.edges, dtype=np.int64, copy=True),
            np.array(topology_info.capacities, dtype=np.float64, copy=True),
            [(list(int(e) for e in idx), float(lim)) for idx, lim in topology_info.shared_constraints],
            name=getattr(topology_info, "name", None),
        )
        self.public_topology = PublicTopologyView.from_topology_info(self.topology_info)
        self.time_limit = int(time_limit)
        self.sequence_id = str(sequence_id)
        self.sequence_step = int(sequence_step)
        self.family = str(family)
        self._truth = truth
        self._generator_metadata = deepcopy(dict(generator_metadata))
        atomic: list[tuple[int, int, int]] = []
        pairs: dict[tuple[int, int], list[int]] = {}
        for s in range(n):
            for d in range(n):
                if s == d:
                    continue
                idx = []
                for local in range(int(truth[s, d])):
                    idx.append(len(atomic))
                    atomic.append((s, d, local))
                pairs[(s, d)] = idx
        self._atomic = tuple(atomic)
        self._pair_indices = pairs
        self._possession = np.zeros((len(atomic), n), dtype=bool)
        if atomic:
            self._possession[np.arange(len(atomic)), [a[0] for a in atomic]] = True
        self._public_to_private: dict[TruthTokenId, int] = {}
        self._private_to_public: dict[int, TruthTokenId] = {}
        self._state_version = 0

    @classmethod
    def from_traffic_matrix(cls, **kwargs: Any) -> "UncertainProblemInstance":
        return cls(**kwargs)

    @property
    def _token_count(self) -> int:
        return len(self._atomic)

    @property
    def _node_count(self) -> int:
        return self._truth.shape[0]

    def _indices_for_pair(self, source: int, destination: int) -> tuple[int, ...]:
        return tuple(self._pair_indices[(int(source), int(destination))])

    def _issue_token_id(self, token_index: int, *, reveal_seed: int) -> TruthTokenId:
        known = self._private_to_public.get(int(token_index))
        if known is not None:
            return known
        s, d, local = self._atomic[int(token_index)]
        material = f"{self.sequence_id}|{self.sequence_step}|{reveal_seed}|{s}|{d}|{local}".encode()
        tid = TruthTokenId("truth:" + sha256(material).hexdigest())
        self._private_to_public[int(token_index)] = tid
        self._public_to_private[tid] = int(token_index)
        return tid

    def _token_record(self, token_index: int) -> tuple[int, int, tuple[int, ...]]:
        s, d, _ = self._atomic[int(token_index)]
        holders = tuple(int(v) for v in np.flatnonzero(self._possession[int(token_index)]))
        return s, d, holders

    def commit(self, observation: Any, proposal: Any) -> Any:
        from .execution import commit_proposal

        return commit_proposal(self, observation, proposal)

    def is_complete(self) -> bool:
        return all(self._possession[i, d] for i, (_, d, _) in enumerate(self._atomic))

    def residual_count(self) -> int:
        return sum(0 if self._possession[i, d] else 1 for i, (_, d, _) in enumerate(self._atomic))


__all__ = ["UncertainProblemInstance"]
