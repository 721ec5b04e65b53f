"""Solve one collective on one topology with a trained schedule policy.

    python -m revealaiccl_b200.rl.single_problem --model_path runs/Rear4GPU_best.pth \\
        --topology Rear4GPU --collective allgather --chunk_factor 2 [--time_limit 30] \\
        [--root_node 0] [--output_dir ./test_results] [--export_xml] [--xml_instances 1] \\
        [--xml_fusion] [--device cpu] [--hidden_dim 128]

Capability of the reference's scripts/test_single_problem.py:28-565: build
an AllGather, AllToAll, AllReduce (modelled as every chunk reaching every
node) or Broadcast problem with ``chunk_factor`` chunks per source over every
node of the topology, decode it slot by slot with the policy (greedy), score
it with the schedule evaluator, and write a readable strategy file, an
optional MSCCL XML program (AllGather and AllToAll, through
``xml_export.schedule_to_msccl_xml`` with the topology's switch and NIC
vertices traced through, and checked by simulation) and a summary.

Problem layouts (chunk ids):
* AllGather / AllReduce: chunk ``s * cf + j`` starts at node s and is
  demanded by every other node;
* AllToAll: chunk ``(s * V + d) * cf + j`` starts at s and is demanded by d
  (s == d chunks have no demand);
* Broadcast: all ``cf`` chunks start at the root, every other node demands them.
"""

from __future__ import annotations

import argparse
from datetime import datetime
import json
import os
from typing import Callable

import numpy as np
import torch

from ..models.policy import SlotLevelPolicy
from ..topology.info import ProblemInstance
from ..topology.loader import ensure_bundled, load_topology_info, node_roles
from .decoder import SlotDecoder, rollout
from .scenarios import evaluate_schedule
from .xml_export import schedule_to_msccl_xml


def _problem(topo, initial: np.ndarray, demands: np.ndarray, T: int, kind: str) -> ProblemInstance:
    return ProblemInstance(num_nodes=topo.V, num_chunks=initial.shape[0], num_edges=topo.E, time_limit=T,
                           capacities=topo.capacities, topology=topo.edges, demands=demands,
                           initial_state=initial, shared_constraints=topo.shared_constraints,
                           topology_info=topo, scenario_type=kind)


def allgather_problem(topo, chunk_factor: int, T: int = 30) -> ProblemInstance:
    V, cf = topo.V, int(chunk_factor)
    owner = np.repeat(np.arange(V), cf)
    initial = np.zeros((V * cf, V), dtype=np.int64)
    initial[np.arange(V * cf), owner] = 1
    return _problem(topo, initial, 1 - initial, T, "allgather")


def allreduce_problem(topo, chunk_factor: int, T: int = 30) -> ProblemInstance:
    """Every node's chunks must end on every node (the reduce is not modelled)."""
    p = allgather_problem(topo, chunk_factor, T)
    p.scenario_type = "allreduce"
    return p


def alltoall_problem(topo, chunk_factor: int, T: int = 30) -> ProblemInstance:
    V, cf = topo.V, int(chunk_factor)
    ids = np.arange(V * V * cf)
    src = ids // (V * cf)
    dst = (ids // cf) % V
    initial = np.zeros((ids.size, V), dtype=np.int64)
    initial[ids, src] = 1
    demands = np.zeros_like(initial)
    off = src != dst
    demands[ids[off], dst[off]] = 1
    return _problem(topo, initial, demands, T, "alltoall")


def broadcast_problem(topo, chunk_factor: int, root_node: int = 0, T: int = 30) -> ProblemInstance:
    V, cf = topo.V, int(chunk_factor)
    if not 0 <= root_node < V:
        raise ValueError(f"root node {root_node} outside 0..{V - 1}")
    initial = np.zeros((cf, V), dtype=np.int64)
    initial[:, root_node] = 1
    return _problem(topo, initial, 1 - initial, T, "broadcast")


BUILDERS: dict[str, Callable[..., ProblemInstance]] = {
    "allgather": allgather_problem, "alltoall": alltoall_problem,
    "allreduce": allreduce_problem, "broadcast": broadcast_problem,
}


def solve(problem: ProblemInstance, model, *, log=print) -> tuple[list[np.ndarray], int]:
    model.eval()
    with torch.no_grad():
        schedule, done = rollout(SlotDecoder(problem.topology_info), model, problem, train=False)
    for t, Y in enumerate(schedule[:done]):
        n = int(np.asarray(Y).sum())
        if n:
            log(f"  slot {t}: {n} transfers")
    return schedule, done


def readable_strategy(schedule, problem: ProblemInstance, topo_name: str, chunk_factor: int) -> str:
    edges = np.asarray(problem.topology, dtype=np.int64).reshape(-1, 2)
    used = [t for t, Y in enumerate(schedule) if np.asarray(Y).sum() > 0]
    out = ["=" * 80, f"Collective schedule - {problem.scenario_type}", "=" * 80,
           f"topology: {topo_name}", f"nodes: {problem.V}", f"edges: {problem.E}", f"chunks: {problem.C}",
           f"chunk factor: {chunk_factor}", f"time limit: {problem.T}", f"slots used: {len(used)}", "", "edges:"]
    out += [f"  edge {e}: node {u} -> node {v} (capacity {int(problem.capacities[e])})"
            for e, (u, v) in enumerate(edges.tolist())]
    out += ["", "-" * 80, "transfers per slot (grouped by sending node)", "-" * 80]
    load = np.zeros(problem.E, dtype=np.int64)
    for t in used:
        c_idx, e_idx = np.nonzero(np.asarray(schedule[t]))
        load += np.bincount(e_idx, minlength=problem.E)
        out.append(f"\nslot {t}:")
        for u in sorted(set(edges[e_idx, 0].tolist())):
            out.append(f"  node {u} sends:")
            out += [f"    chunk {c} -> node {edges[e, 1]} (edge {e})"
                    for c, e in zip(c_idx.tolist(), e_idx.tolist()) if edges[e, 0] == u]
    total = int(sum(np.asarray(Y).sum() for Y in schedule))
    out += ["", "=" * 80, "statistics", "=" * 80, f"transfers: {total}", "", "transfers per slot:"]
    out += [f"  slot {t}: {int(np.asarray(schedule[t]).sum())}" for t in used]
    busiest = [e for e in np.argsort(-load, kind="stable").tolist() if load[e] > 0][:20]
    out += ["", f"busiest edges (top {len(busiest)}):"]
    out += [f"  edge {e} (node {edges[e, 0]} -> node {edges[e, 1]}): {int(load[e])} uses" for e in busiest]
    return "\n".join(out) + "\n"


def export_xml(schedule, problem: ProblemInstance, topo_name: str, path: str, *, instances: int = 1,
               fusion: bool = False) -> str:
    kind = problem.scenario_type
    if kind not in ("allgather", "alltoall"):
        raise ValueError(f"XML export covers AllGather and AllToAll, not {kind}")
    roles = node_roles(topo_name)
    is_switch = np.asarray([r != "gpu" for r in roles]) if roles else np.zeros(problem.V, dtype=bool)
    edges = np.asarray(problem.topology, dtype=np.int64).reshape(-1, 2)
    post = None
    if kind == "alltoall":
        post = np.asarray(problem.demands).copy()
        silent = post.sum(axis=1) == 0  # s == d chunks stay where they start
        post[silent] = np.asarray(problem.initial_state)[silent]
    xml = schedule_to_msccl_xml(schedule, edge_src=edges[:, 0], edge_dst=edges[:, 1],
                                pre_condition=problem.initial_state, post_condition=post, is_switch=is_switch,
                                collective=kind, name=f"raiccl_{kind}", instances=instances,
                                instr_fusion=fusion, check=True)
    with open(path, "w", encoding="utf-8") as f:
        f.write(xml)
    return xml


def run(args) -> dict:
    os.makedirs(args.output_dir, exist_ok=True)
    device = torch.device(args.device if (not args.device.startswith("cuda") or torch.cuda.is_available()) else "cpu")
    ck = torch.load(args.model_path, map_location=device, weights_only=False)
    state = ck["model_state_dict"] if isinstance(ck, dict) and "model_state_dict" in ck else ck
    model = SlotLevelPolicy(5, 2, 5, 2, args.hidden_dim).to(device)
    model.load_state_dict(state)
    ensure_bundled()
    topo = load_topology_info(args.topology)
    build = BUILDERS[args.collective]
    problem = (build(topo, args.chunk_factor, args.root_node, args.time_limit) if args.collective == "broadcast"
               else build(topo, args.chunk_factor, args.time_limit))
    print(f"{args.collective} on {args.topology}: {problem.C} chunks, {int(problem.demands.sum())} demands")
    schedule, done = solve(problem, model)
    score, error = evaluate_schedule(schedule, problem)
    transfers = int(sum(np.asarray(Y).sum() for Y in schedule))
    result = {"collective": args.collective, "topology": args.topology, "chunk_factor": args.chunk_factor,
              "time_limit": args.time_limit, "score": float(score), "error": error or None,
              "completion_steps": None if error else -int(score // 1), "transfers": transfers}
    tag = f"{args.topology}_{args.collective}_cf{args.chunk_factor}"
    strategy = os.path.join(args.output_dir, f"strategy_{tag}.txt")
    with open(strategy, "w", encoding="utf-8") as f:
        f.write(readable_strategy(schedule, problem, args.topology, args.chunk_factor))
    result["strategy_file"] = strategy
    if args.export_xml:
        xml_path = os.path.join(args.output_dir, f"{tag}_inst{args.xml_instances}.xml")
        try:
            export_xml(schedule, problem, args.topology, xml_path, instances=args.xml_instances,
                       fusion=args.xml_fusion)
            result["xml_file"] = xml_path
        except ValueError as exc:
            result["xml_error"] = str(exc)
    result["finished"] = datetime.now().isoformat(timespec="seconds")
    with open(os.path.join(args.output_dir, "test_summary.json"), "w", encoding="utf-8") as f:
        json.dump(result, f, indent=2)
    print(json.dumps(result))
    return result


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="revealaiccl_b200.rl.single_problem", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model_path", required=True)
    ap.add_argument("--topology", required=True)
    ap.add_argument("--collective", required=True, choices=sorted(BUILDERS))
    ap.add_argument("--chunk_factor", type=int, required=True)
    ap.add_argument("--time_limit", type=int, default=30)
    ap.add_argument("--root_node", type=int, default=0)
    ap.add_argument("--output_dir", default="./test_results")
    ap.add_argument("--export_xml", action="store_true")
    ap.add_argument("--xml_instances", type=int, default=1)
    ap.add_argument("--xml_fusion", action="store_true")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--hidden_dim", type=int, default=128)
    run(ap.parse_args(argv))


__all__ = ["BUILDERS", "allgather_problem", "allreduce_problem", "alltoall_problem", "broadcast_problem",
           "export_xml", "readable_strategy", "run", "solve"]

if __name__ == "__main__":
    main()
