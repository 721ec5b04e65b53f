"""Collective scenario generation, the schema-v2 scenario cache and the
schedule evaluator of the schedule-search stack (rlccl/envs/evaluator.py:83-619).

Scenario families (mixture 50% All-to-All-V, 30% AllGather, 20% AllToAll):
* All-to-All-V: X[i, j] uniform in {0..4}, zero diagonal (never all-zero);
* AllGather: every node owns k in {1, 2, 3} chunks every other node needs;
* AllToAll: one chunk per ordered (src, dst) pair, src == dst chunks need nothing.
The cache is keyed by a sha256 of the canonical generator config and is
regenerated when the schema version, generator name or hash differ.

``evaluate_schedule``: per slot checks edge capacity, shared groups and
source possession; score = -completion_step + 0.001 * sum_t satisfied_t/(t+1);
any violation scores -(T + 2).
"""

from __future__ import annotations

import hashlib
import json
import os
from typing import Any

import numpy as np

from ..topology.info import ProblemInstance, compute_received_chunks
from ..traffic.matrix_utils import traffic_matrix_to_scenario

SCENARIO_SCHEMA_VERSION = 2
LEGACY_GENERATOR_NAME = "legacy_mixed_v2"


def generate_all_to_all_v_scenario(V: int, rng) -> dict:
    m = rng.integers(0, 5, size=(V, V))
    np.fill_diagonal(m, 0)
    if not np.any(m):
        if V < 2:
            raise ValueError("All-to-All-V requires at least two nodes")
        m[0, 1] = 1
    return traffic_matrix_to_scenario(m)


def generate_allgather_scenario(V: int, chunks_per_node: int, rng=None) -> dict:
    k = int(chunks_per_node)
    C = V * k
    init = np.zeros((C, V), dtype=int)
    dem = np.zeros((C, V), dtype=int)
    for node in range(V):
        for j in range(k):
            c = node * k + j
            init[c, node] = 1
            dem[c, :] = 1
            dem[c, node] = 0
    return {"type": "allgather", "chunks_per_node": k, "C": C, "initial_state": init.tolist(),
            "demands": dem.tolist()}


def generate_alltoall_scenario(V: int, chunks_per_dest: int, rng=None) -> dict:
    k = int(chunks_per_dest)
    C = V * V * k
    init = np.zeros((C, V), dtype=int)
    dem = np.zeros((C, V), dtype=int)
    for s in range(V):
        for d in range(V):
            for j in range(k):
                c = s * V * k + d * k + j
                init[c, s] = 1
                if s != d:
                    dem[c, d] = 1
    return {"type": "alltoall", "chunks_per_dest": k, "C": C, "initial_state": init.tolist(), "demands": dem.tolist()}


def generate_scenarios(V: int, num_scenarios: int, seed: int) -> list[dict]:
    rng = np.random.default_rng(seed)
    n_a2av = int(num_scenarios * 0.5)
    n_ag = int(num_scenarios * 0.3)
    n_a2a = num_scenarios - n_a2av - n_ag
    out = []
    for _ in range(n_a2av):
        out.append(generate_all_to_all_v_scenario(V, rng))
    for _ in range(n_ag):
        out.append(generate_allgather_scenario(V, rng.integers(1, 4), rng))
    for _ in range(n_a2a):
        out.append(generate_alltoall_scenario(V, 1, rng))
    rng.shuffle(out)
    for i, s in enumerate(out):
        s["id"] = i
    return out


def legacy_generator_config(V: int, num_scenarios: int, seed: int) -> dict:
    return {"V": int(V), "num_scenarios": int(num_scenarios), "seed": int(seed),
            "mixture": {"all_to_all_v": 0.5, "allgather": 0.3, "alltoall": 0.2}, "all_to_all_v_range": [0, 4]}


def config_hash(config: dict) -> str:
    return hashlib.sha256(json.dumps(config, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def load_or_generate_scenarios(path: str, V: int, num_scenarios: int, seed: int,
                               generator_name: str = LEGACY_GENERATOR_NAME, generator_config: dict | None = None):
    cfg = generator_config or legacy_generator_config(V, num_scenarios, seed)
    h = config_hash(cfg)
    if os.path.exists(path):
        with open(path, "r", encoding="utf-8") as f:
            data = json.load(f)
        if (isinstance(data, dict) and data.get("schema_version") == SCENARIO_SCHEMA_VERSION
                and data.get("generator_name") == generator_name and data.get("generator_config_hash") == h
                and isinstance(data.get("scenarios"), list)):
            return data["scenarios"]
    scenarios = generate_scenarios(V, num_scenarios, seed)
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    with open(path, "w", encoding="utf-8") as f:
        json.dump({"schema_version": SCENARIO_SCHEMA_VERSION, "generator_name": generator_name,
                   "generator_config": cfg, "generator_config_hash": h, "V": V, "num_scenarios": num_scenarios,
                   "seed": seed, "scenarios": scenarios}, f, indent=2)
    return scenarios


def build_problem_from_scenario(V, E, edges, capacities, shared_constraints, scenario: dict, T: int = 20,
                                topology_info=None) -> ProblemInstance:
    C = scenario["C"]
    init = np.asarray(scenario["initial_state"], dtype=int).reshape(C, V)
    dem = np.asarray(scenario["demands"], dtype=int).reshape(C, V)
    meta = {k: v for k, v in scenario.items() if k not in ("initial_state", "demands", "traffic_matrix")}
    return ProblemInstance(V, C, E, T, capacities, edges, dem, init, shared_constraints, topology_info=topology_info,
                           traffic_matrix=scenario.get("traffic_matrix"), scenario_type=scenario.get("type"),
                           sequence_id=scenario.get("sequence_id"), sequence_step=scenario.get("sequence_step"),
                           metadata=meta)


def evaluate_schedule(schedule, problem) -> tuple[float, str]:
    error_score = -(problem.T + 2)
    if len(schedule) > problem.T:
        return error_score, "Schedule length exceeds time limit"
    state = problem.initial_state.copy()
    demands = problem.demands.copy()
    weighted = 0.0
    completion = len(schedule)
    topo = getattr(problem, "topology_info", None)
    edge_dst = (np.asarray(topo.edge_dst, dtype=np.int64) if topo is not None and hasattr(topo, "edge_dst")
                else np.asarray(problem.topology, dtype=np.int64)[:, 1])
    caps = np.asarray(problem.capacities, dtype=float)
    for t, Y in enumerate(schedule):
        Y = np.asarray(Y)
        if Y.shape != (problem.C, problem.E):
            return error_score, f"Invalid shape for Y_{t}: {Y.shape}, expected ({problem.C}, {problem.E})"
        loads = Y.sum(axis=0)
        if np.any(loads > caps + 1e-6):
            i = int(np.flatnonzero(loads > caps + 1e-6)[0])
            return error_score, f"Bandwidth constraint violated at step {t} on edge {i} ({loads[i]} > {caps[i]})"
        for members, limit in problem.shared_constraints:
            gl = float(np.sum(loads[list(members)]))
            if gl > float(limit) + 1e-6:
                return error_score, f"Shared bandwidth constraint violated at step {t} (load {gl} > {limit})"
        for e in range(problem.E):
            u = int(np.asarray(problem.topology[e])[0])
            for c in np.flatnonzero(Y[:, e] == 1):
                if state[c, u] == 0:
                    return error_score, f"Feasibility violated at step {t}: Node {u} sends chunk {c} but doesn't have it"
        N = compute_received_chunks(Y, edge_dst, problem.V)
        weighted += float(np.sum(N * demands)) / (t + 1)
        state = np.maximum(state, N)
        demands = demands * (1 - N)
        if np.sum(demands) == 0:
            completion = t + 1
            break
    return -completion + 0.001 * weighted, ""


def generate_train_test_split(topologies: dict[str, Any], *, num_train: int = 80, num_test: int = 20,
                              seed: int = 42, cache_dir: str | None = None, T: int = 20):
    """Per topology: train scenarios from ``seed`` and test scenarios from ``seed + 10000``."""
    train, test = [], []
    for name, topo in topologies.items():
        V = int(topo.V)
        paths = {k: (os.path.join(cache_dir, f"{name}_scenarios_{LEGACY_GENERATOR_NAME}_{k}.json") if cache_dir else None)
                 for k in ("train", "test")}
        for split, n, s in (("train", num_train, seed), ("test", num_test, seed + 10000)):
            if n <= 0:
                continue
            scs = (load_or_generate_scenarios(paths[split], V, n, s) if paths[split] else generate_scenarios(V, n, s))
            target = train if split == "train" else test
            for sc in scs:
                target.append((f"{name}:{sc['id']}", build_problem_from_scenario(
                    V, topo.E, topo.edges, topo.capacities, topo.shared_constraints, sc, T=T, topology_info=topo)))
    return train, test


__all__ = ["LEGACY_GENERATOR_NAME", "SCENARIO_SCHEMA_VERSION", "build_problem_from_scenario", "config_hash",
           "evaluate_schedule", "generate_all_to_all_v_scenario", "generate_allgather_scenario",
           "generate_alltoall_scenario", "generate_scenarios", "generate_train_test_split",
           "legacy_generator_config", "load_or_generate_scenarios"]
