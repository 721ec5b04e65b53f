"""Paired evaluation of reveal-aware policies (rlccl/uncertainty/evaluation.py:32-591).

``EvaluationManifest`` pins the evaluation identity with three canonical
digests (truth bytes; versioned topology payload; versioned reveal/config
payload).  ``PairedEvaluationRunner`` gives every method a fresh world and a
fresh reveal process from the same manifest, runs slots until the truth is
delivered or ``time_limit`` is hit, commits every executable proposal through
the trusted checker, and emits one ``RecourseMetrics`` raw row per method.
The full-information oracle row is the provable four-term completion lower
bound (longest shortest path, total work / total unit capacity, per-source
egress and per-destination ingress), shared groups relaxed.
"""

from __future__ import annotations

from copy import deepcopy
from dataclasses import asdict, dataclass
from hashlib import sha256
import json
import math
from time import perf_counter
from typing import Any, Mapping, Sequence

import numpy as np

from ..topology.info import TopologyInfo
from ..traffic.matrix_utils import validate_traffic_matrix
from .baselines import (FullInformationOracle, LongTermMeanBaseline, PartialCurrentOnlyBaseline,
                        PreviousValueBaseline, WaitUntilKnownBaseline)
from .execution import Proposal
from .observation import PartialObservationState, SanitizedHistoryView
from .problem import UncertainProblemInstance
from .reveal import DemandRevealProcess


@dataclass(frozen=True, slots=True)
class RecourseMetrics:
    """One raw evaluation row (rlccl/uncertainty/metrics.py:10-50).

    ``completion`` counts elapsed execution slots (time_limit + 1 when
    unfinished); ``reveal_wait`` is the first slot with an executable action;
    ``recourse_count`` counts changes of the public proposal after slot 0;
    ``wasted_plan`` is the L1 distance of the first scenario-only plan to the
    final truth."""

    completion: int
    oracle_regret: float
    reveal_wait: int
    recourse_count: int
    replanned_actions: int
    wasted_plan: int
    synthesis_time_ms: float
    replan_time_ms: float
    legality: bool
    timeout: bool
    sequence_id: str
    family: str
    seed: int
    topology: str
    reveal_stage: int
    reveal_mode: str
    method: str
    manifest_id: str
    truth_digest: str
    topology_digest: str
    config_digest: str
    checker_version: str

    def to_raw_row(self) -> dict[str, Any]:
        return asdict(self)


def canonical_json_digest(payload: Mapping[str, Any]) -> str:
    return sha256(json.dumps(payload, ensure_ascii=False, sort_keys=True,
                             separators=(",", ":")).encode()).hexdigest()


def truth_digest(matrix: np.ndarray) -> str:
    return sha256(np.ascontiguousarray(matrix).tobytes()).hexdigest()


def topology_digest(topology: TopologyInfo) -> str:
    return canonical_json_digest({
        "version": "uncertainty-topology-v1",
        "V": int(topology.V), "E": int(topology.E),
        "edges": [[int(s), int(d)] for s, d in np.asarray(topology.edges)],
        "capacities_float_hex": [float(v).hex() for v in np.asarray(topology.capacities, dtype=np.float64)],
        "shared_groups": [{"edge_indices": [int(e) for e in idx], "limit_float_hex": float(lim).hex()}
                          for idx, lim in topology.shared_constraints],
    })


def config_digest(*, reveal_mode: str, ratios: Sequence[float], reveal_seed: int, timeout: int,
                  time_limit: int, checker_version: str) -> str:
    return canonical_json_digest({
        "version": "uncertainty-config-v1",
        "reveal_mode": str(reveal_mode),
        "normalized_ratios_float_hex": [float(v).hex() for v in ratios],
        "reveal_seed": int(reveal_seed), "timeout": int(timeout),
        "time_limit": int(time_limit), "checker_version": str(checker_version),
    })


@dataclass(frozen=True, slots=True)
class EvaluationManifest:
    manifest_id: str
    sequence_id: str
    family: str
    history_provenance: str
    truth_digest: str
    topology_digest: str
    config_digest: str
    reveal_mode: str
    ratios: tuple[float, ...]
    reveal_seed: int
    timeout: int
    time_limit: int
    checker_version: str

    def __post_init__(self) -> None:
        object.__setattr__(self, "ratios", tuple(float(v) for v in self.ratios))
        if self.timeout <= 0:
            raise ValueError("timeout limit must be positive")
        if self.time_limit <= 0:
            raise ValueError("time_limit must be positive")

    @classmethod
    def create(cls, *, manifest_id: str, sequence_id: str, family: str, history_provenance: str,
               truth_matrix: np.ndarray, topology_info: TopologyInfo, reveal_mode: str,
               ratios: Sequence[float], reveal_seed: int, timeout: int, time_limit: int,
               checker_version: str) -> "EvaluationManifest":
        raw = np.asarray(truth_matrix)
        validate_traffic_matrix(raw)
        r = tuple(float(v) for v in ratios)
        return cls(str(manifest_id), str(sequence_id), str(family), str(history_provenance),
                   truth_digest(np.array(raw, dtype=np.int64)), topology_digest(topology_info),
                   config_digest(reveal_mode=reveal_mode, ratios=r, reveal_seed=reveal_seed,
                                 timeout=timeout, time_limit=time_limit, checker_version=checker_version),
                   str(reveal_mode), r, int(reveal_seed), int(timeout), int(time_limit),
                   str(checker_version))


@dataclass(slots=True)
class Episode:
    world: UncertainProblemInstance
    reveal_process: DemandRevealProcess
    manifest: EvaluationManifest
    _slot: int = 0

    def next_observation(self) -> PartialObservationState:
        obs = self.reveal_process.observation_for_slot(self._slot)
        self._slot += 1
        return obs

    def next_full_observation(self) -> PartialObservationState:
        obs = self.reveal_process.full_observation()
        self._slot += 1
        return obs


def _ceil_div(a: int, b: int) -> int:
    return (int(a) + int(b) - 1) // int(b)


def oracle_completion_lower_bound(truth: np.ndarray, topology: TopologyInfo, time_limit: int) -> int:
    pairs = np.argwhere(np.asarray(truth) > 0)
    if len(pairs) == 0:
        return 0
    n = int(topology.V)
    edges = np.asarray(topology.edges, dtype=np.int64)
    units = np.asarray([max(0, math.floor(float(v))) for v in topology.capacities], dtype=np.int64)
    total = int(units.sum())
    if total <= 0:
        return int(time_limit) + 1
    dist = np.full((n, n), n + 1, dtype=np.int64)
    np.fill_diagonal(dist, 0)
    out_cap = np.zeros(n, dtype=np.int64)
    in_cap = np.zeros(n, dtype=np.int64)
    for e, (s, d) in enumerate(edges):
        c = int(units[e])
        if c <= 0:
            continue
        dist[int(s), int(d)] = 1
        out_cap[int(s)] += c
        in_cap[int(d)] += c
    for k in range(n):
        dist = np.minimum(dist, dist[:, [k]] + dist[[k], :])
    lb_path = 0
    work = 0
    for s, d in pairs:
        hops = int(dist[s, d])
        if hops > n or out_cap[s] <= 0 or in_cap[d] <= 0:
            return int(time_limit) + 1
        lb_path = max(lb_path, hops)
        work += int(truth[s, d]) * hops
    lb_work = _ceil_div(work, total)
    lb_src = max(_ceil_div(int(truth[s].sum()), int(out_cap[s])) for s in range(n) if int(truth[s].sum()) > 0)
    lb_dst = max(_ceil_div(int(truth[:, d].sum()), int(in_cap[d])) for d in range(n) if int(truth[:, d].sum()) > 0)
    lb = max(lb_path, lb_work, lb_src, lb_dst)
    return int(time_limit) + 1 if lb > int(time_limit) else int(lb)


def proposal_signature(proposal: Proposal) -> tuple[Any, ...]:
    if proposal.scenario_set is not None:
        sc = proposal.scenario_set
        return ("scenario", tuple((str(m.dtype), tuple(m.shape), m.tobytes()) for m in sc.matrices),
                sc.weights, sc.scenario_ids, sc.provenance)
    if proposal.actions:
        return ("actions", tuple((str(a.token_id), a.edge_index) for a in proposal.actions))
    return ("wait",)


_METHODS = ("full_information_oracle", "wait_until_known", "partial_current_only",
            "long_term_mean", "previous_value")


class PairedEvaluationRunner:
    def __init__(self, *, manifest: EvaluationManifest, truth_matrix: np.ndarray,
                 history_matrices: Sequence[np.ndarray], topology_info: TopologyInfo,
                 generator_metadata: Mapping[str, Any]) -> None:
        if not isinstance(manifest, EvaluationManifest):
            raise TypeError("manifest must be EvaluationManifest")
        raw = np.asarray(truth_matrix)
        validate_traffic_matrix(raw)
        if raw.shape != (int(topology_info.V), int(topology_info.V)):
            raise ValueError("Truth matrix shape must match topology")
        truth = np.array(raw, dtype=np.int64, copy=True)
        if truth_digest(truth) != manifest.truth_digest:
            raise ValueError("Manifest truth digest does not match input truth")
        if topology_digest(topology_info) != manifest.topology_digest:
            raise ValueError("Manifest topology digest does not match input topology")
        if config_digest(reveal_mode=manifest.reveal_mode, ratios=manifest.ratios,
                         reveal_seed=manifest.reveal_seed, timeout=manifest.timeout,
                         time_limit=manifest.time_limit,
                         checker_version=manifest.checker_version) != manifest.config_digest:
            raise ValueError("Manifest config digest does not match evaluation config")
        hist = []
        for m in history_matrices:
            a = np.asarray(m)
            validate_traffic_matrix(a)
            if a.shape != truth.shape:
                raise ValueError("Each history matrix shape must match truth/topology")
            hist.append(np.array(a, dtype=np.int64, copy=True))
        self.manifest = manifest
        self._truth = truth
        self._history = tuple(hist)
        self._topology = TopologyInfo(
            int(topology_info.V), int(topology_info.E),
            np.array(topology_info.edges, dtype=np.int64, copy=True),
            np.array(topology_info.capacities, dtype=np.float64, copy=True),
            [(list(int(e) for e in idx), float(lim)) for idx, lim in topology_info.shared_constraints],
            name=getattr(topology_info, "name", None))
        self._metadata = deepcopy(dict(generator_metadata))

    def build_episode(self, method: str) -> Episode:
        if method not in _METHODS:
            raise ValueError(f"Unknown evaluation method: {method}")
        world = UncertainProblemInstance.from_traffic_matrix(
            truth_matrix=self._truth, topology_info=self._topology,
            time_limit=self.manifest.time_limit, sequence_id=self.manifest.sequence_id,
            sequence_step=len(self._history), family=self.manifest.family,
            generator_metadata=deepcopy(self._metadata))
        reveal = DemandRevealProcess(problem=world, mode=self.manifest.reveal_mode,
                                     ratios=self.manifest.ratios, seed=self.manifest.reveal_seed)
        return Episode(world, reveal, self.manifest)

    def _history_view(self) -> SanitizedHistoryView:
        return SanitizedHistoryView.from_completed_matrices(
            matrices=self._history, steps=tuple(range(len(self._history))),
            sequence_id=self.manifest.sequence_id, current_step=len(self._history))

    def _row(self, *, method, world, completion, oracle_completion, reveal_stage, reveal_wait,
             recourse_count, replanned_actions, wasted_plan, synthesis_time_ms, replan_time_ms,
             legality, legal_attempts, commit_attempts, timeout, uses_oracle, upper_bound_only,
             legality_error=None) -> dict[str, Any]:
        m = self.manifest
        metrics = RecourseMetrics(
            int(completion), float(completion - oracle_completion), int(reveal_wait),
            int(recourse_count), int(replanned_actions), int(wasted_plan), float(synthesis_time_ms),
            float(replan_time_ms), bool(legality), bool(timeout), m.sequence_id, m.family,
            m.reveal_seed, str(getattr(world.topology_info, "name", None) or "unnamed"),
            int(reveal_stage), m.reveal_mode, method, m.manifest_id, m.truth_digest,
            m.topology_digest, m.config_digest, m.checker_version)
        row = metrics.to_raw_row()
        row.update({
            "legal": metrics.legality,
            "legality_rate": 1.0 if commit_attempts == 0 else legal_attempts / commit_attempts,
            "uses_oracle": bool(uses_oracle), "upper_bound_only": bool(upper_bound_only),
            "reveal_seed": m.reveal_seed, "history_provenance": m.history_provenance,
            "ratios": m.ratios, "time_limit": m.time_limit, "timeout_limit": m.timeout,
        })
        if legality_error is not None:
            row["legality_error"] = legality_error
        return row

    def run_oracle(self, oracle: FullInformationOracle) -> dict[str, Any]:
        if not isinstance(oracle, FullInformationOracle):
            raise TypeError("run_oracle requires FullInformationOracle")
        episode = self.build_episode(oracle.method)
        t0 = perf_counter()
        completion = oracle_completion_lower_bound(self._truth, self._topology, self.manifest.time_limit)
        synth = (perf_counter() - t0) * 1000.0
        row = self._row(method=oracle.method, world=episode.world, completion=completion,
                        oracle_completion=completion, reveal_stage=len(self.manifest.ratios) - 1,
                        reveal_wait=0, recourse_count=0, replanned_actions=0, wasted_plan=0,
                        synthesis_time_ms=synth, replan_time_ms=0.0, legality=True,
                        legal_attempts=0, commit_attempts=0,
                        timeout=completion == self.manifest.time_limit + 1,
                        uses_oracle=True, upper_bound_only=True)
        row.update({"reference_kind": "provable_full_information_lower_bound", "executable": False,
                    "legality_basis": "vacuous_no_executable_actions"})
        return row

    def run_method(self, baseline: Any, *, oracle_completion: int | None = None) -> dict[str, Any]:
        if oracle_completion is None:
            oracle_completion = int(self.run_oracle(FullInformationOracle())["completion"])
        episode = self.build_episode(baseline.method)
        history = self._history_view()
        limit = self.manifest.time_limit
        completion = 0 if episode.world.is_complete() else limit + 1
        first_action = None
        prev_sig = None
        recourse = replanned = 0
        wasted = None
        synth = replan = 0.0
        legal_attempts = commit_attempts = 0
        legality, error, final_stage = True, None, 0
        for slot in range(limit):
            if episode.world.is_complete():
                break
            obs = episode.next_observation()
            final_stage = obs.stage
            t0 = perf_counter()
            proposal = baseline.propose(obs, history=history, scenarios=None)
            dt = (perf_counter() - t0) * 1000.0
            if slot == 0:
                synth = dt
            else:
                replan += dt
                replanned += len(proposal.actions)
            sig = proposal_signature(proposal)
            if prev_sig is not None and sig != prev_sig:
                recourse += 1
            prev_sig = sig
            if proposal.scenario_set is not None:
                if wasted is None:
                    wasted = int(np.abs(np.asarray(proposal.scenario_set.matrices[0]) - self._truth).sum())
            elif proposal.actions:
                if first_action is None:
                    first_action = slot
                commit_attempts += 1
                try:
                    result = episode.world.commit(obs, proposal)
                except (TypeError, ValueError) as caught:
                    legality, error = False, str(caught)
                    break
                legal_attempts += int(result.legal)
            if episode.world.is_complete():
                completion = slot + 1
                break
        return self._row(method=baseline.method, world=episode.world, completion=completion,
                         oracle_completion=oracle_completion, reveal_stage=final_stage,
                         reveal_wait=limit if first_action is None else first_action,
                         recourse_count=recourse, replanned_actions=replanned,
                         wasted_plan=0 if wasted is None else wasted, synthesis_time_ms=synth,
                         replan_time_ms=replan, legality=legality, legal_attempts=legal_attempts,
                         commit_attempts=commit_attempts, timeout=not episode.world.is_complete(),
                         uses_oracle=False, upper_bound_only=False, legality_error=error)

    _run_ordinary = run_method

    def run_default_baselines(self) -> list[dict[str, Any]]:
        oracle = self.run_oracle(FullInformationOracle())
        oc = int(oracle["completion"])
        return [oracle] + [self.run_method(b, oracle_completion=oc) for b in (
            WaitUntilKnownBaseline(), PartialCurrentOnlyBaseline(), LongTermMeanBaseline(),
            PreviousValueBaseline())]


__all__ = ["EvaluationManifest", "Episode", "PairedEvaluationRunner", "RecourseMetrics",
           "canonical_json_digest", "config_digest", "oracle_completion_lower_bound",
           "proposal_signature", "topology_digest", "truth_digest"]
