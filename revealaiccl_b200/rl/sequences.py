"""Temporally ordered All-to-All-V problem sequences with history-only moment context.

Behaviour of rlccl/envs/sequence_env.py (``TrafficSequenceRunner``) and
rlccl/training/sequence_sampler.py (``build_sequence_problems``): the
problem of step t carries the context of matrices 0..t-1 only — the
estimator takes X_t after the step's problem has been handed out — and
sequence seeds are ``seed + 10000 * family_index + sequence_index``.
"""

from __future__ import annotations

from collections.abc import Iterator
from dataclasses import dataclass
from typing import Any

import numpy as np

from ..topology.info import ProblemInstance
from ..traffic.matrix_utils import traffic_matrix_to_scenario
from ..traffic.moments import SlidingMomentEstimator
from ..traffic.process import TrafficProcessConfig, generate_traffic_sequence
from ..traffic.types import MomentContext, TrafficSequence


class TrafficSequenceRunner:
    """Yields (problem, context, record) per step; context never includes the step's own matrix."""

    def __init__(self, sequence: TrafficSequence, topology_info, *, time_limit: int = 20,
                 min_history: int | None = None, estimator_eps: float = 1e-6) -> None:
        if topology_info.V != sequence.mean_ref.shape[0]:
            raise ValueError("Traffic sequence and topology node counts do not match")
        if time_limit <= 0:
            raise ValueError("time_limit must be positive")
        self.sequence, self.topology_info, self.time_limit = sequence, topology_info, int(time_limit)
        self.window_size = int(sequence.metadata.get("window_size", len(sequence.matrices)))
        self.min_history = int(min_history if min_history is not None else self.window_size)
        self.estimator_eps = float(estimator_eps)

    def _problem(self, step: int, matrix: np.ndarray, ctx: MomentContext) -> ProblemInstance:
        seq, topo = self.sequence, self.topology_info
        sc = traffic_matrix_to_scenario(matrix, sequence_id=seq.sequence_id, sequence_step=step, family=seq.family)
        C = sc["C"]
        return ProblemInstance(
            num_nodes=topo.V, num_chunks=C, num_edges=topo.E, time_limit=self.time_limit,
            capacities=topo.capacities, topology=topo.edges,
            demands=np.asarray(sc["demands"], dtype=np.int64).reshape(C, topo.V),
            initial_state=np.asarray(sc["initial_state"], dtype=np.int64).reshape(C, topo.V),
            shared_constraints=topo.shared_constraints, topology_info=topo, traffic_matrix=matrix,
            scenario_type="all_to_all_v", sequence_id=seq.sequence_id, sequence_step=step, moment_context=ctx,
            metadata={"family": seq.family, **seq.metadata})

    def __iter__(self) -> Iterator[tuple[ProblemInstance, MomentContext, dict[str, Any]]]:
        seq = self.sequence
        est = SlidingMomentEstimator(num_nodes=self.topology_info.V, window_size=self.window_size,
                                     min_history=self.min_history, eps=self.estimator_eps)
        for step, m in enumerate(seq.matrices):
            ctx = est.get_context(m, seq.mean_ref, seq.var_ref)
            yield (self._problem(step, m, ctx), ctx,
                   {"sequence_id": seq.sequence_id, "sequence_step": step, "family": seq.family, "seed": seq.seed})
            est.update(m)  # only after the step's problem is out


@dataclass(frozen=True)
class SequenceDatasetConfig:
    families: tuple[str, ...]
    num_sequences_per_family: int
    sequence_length: int
    window_size: int
    min_history: int
    mean_level: float
    std_level: float
    max_entry: int
    epsilon_mean: float
    epsilon_var: float
    seed: int
    time_limit: int = 20


def build_sequence_problems(topology_info, cfg: SequenceDatasetConfig):
    """(problems [(id, problem)], sequences, records) with contexts computed in temporal order."""
    if cfg.num_sequences_per_family <= 0:
        raise ValueError("num_sequences_per_family must be positive")
    problems, sequences, records = [], [], []
    for fi, fam in enumerate(cfg.families):
        for si in range(cfg.num_sequences_per_family):
            seed = cfg.seed + fi * 10000 + si
            seq = generate_traffic_sequence(TrafficProcessConfig(
                num_nodes=topology_info.V, sequence_length=cfg.sequence_length, window_size=cfg.window_size,
                mean_level=cfg.mean_level, std_level=cfg.std_level, max_entry=cfg.max_entry,
                epsilon_mean=cfg.epsilon_mean, epsilon_var=cfg.epsilon_var, family=fam, seed=seed,
                topology_name=topology_info.name or "unknown"))
            ids = []
            for prob, _, rec in TrafficSequenceRunner(seq, topology_info, time_limit=cfg.time_limit,
                                                      min_history=cfg.min_history):
                pid = f"{seq.sequence_id}-step{rec['sequence_step']}"
                problems.append((pid, prob))
                ids.append(pid)
            sequences.append(seq)
            records.append({"sequence_id": seq.sequence_id, "family": fam, "seed": seed, "problem_ids": ids})
    return problems, sequences, records


__all__ = ["SequenceDatasetConfig", "TrafficSequenceRunner", "build_sequence_problems"]
