"""Old-vs-compiled scheduler equivalence runner (scripts/run_r2_c0_equivalence.py).

E1 (static): every compiled plan's four static proofs hold and its canonical
shortest path (destination-first ties) equals the uncompiled planner's for
every (source, destination), reachability included.
E2 (single step): for random truths and reveal stages, one compiled binder
step (candidates, selection, bound proposal) equals the uncompiled path
built from the same observation.
E3 (trajectory): slot by slot until completion, binder output equals the
uncompiled path and the dynamic guard's verdict, applied count and state
version equal the trusted commit checker's, with no state rebuild and no
runtime BFS.

Corpus: five 4-node fixtures (complete graph with capacity 2, the same with
two shared groups, a diamond with ties, a bidirectional line, zero and
fractional capacities) plus the bundled Rear4GPU topology; each on the NumPy
core and, when built, the native C++ core.  The report carries per-step
latency distributions of both paths and a gate: zero mismatches.

    python -m revealaiccl_b200.bench.equivalence --out equivalence.json
"""

from __future__ import annotations

import argparse
import json
import time
from typing import Any

import numpy as np

from ..ops import _native
from ..scheduling import compiled as C
from ..scheduling import robust_prefix as R
from ..scheduling.recourse import bind_action
from ..topology import TopologyInfo, load_rear4_topology
from ..uncertainty import DemandRevealProcess, Proposal, UncertainProblemInstance, commit_proposal

RATIOS = (0.0, 0.25, 0.5, 0.75, 1.0)


def corpus() -> list[TopologyInfo]:
    full = [(a, b) for a in range(4) for b in range(4) if a != b]
    diamond = [(0, 1), (0, 2), (1, 3), (2, 3), (1, 0), (2, 0), (3, 1), (3, 2)]
    line = [(0, 1), (1, 0), (1, 2), (2, 1), (2, 3), (3, 2)]

    def mk(name, edges, caps, groups):
        return TopologyInfo(4, len(edges), np.asarray(edges, dtype=np.int64), np.asarray(caps, dtype=np.float64),
                            groups, name=name)

    return [mk("complete-cap2", full, [2.0] * 12, []),
            mk("complete-shared", full, [2.0] * 12, [([0, 1, 3, 4], 2.0), ([1, 2, 5], 1.0)]),
            mk("diamond-ties", diamond, [1.0] * 8, [([0, 1], 1.0)]),
            mk("line-bidirectional", line, [1.0, 1.5, 2.0, 2.0, 1.0, 1.0], [([2, 3], 1.0)]),
            mk("zero-and-fractional", full, [0.0, 0.5] + [1.0] * 10, []),
            load_rear4_topology()[0]]


def _dist(v: list[float]) -> dict[str, Any]:
    if not v:
        return {"count": 0}
    a = np.asarray(v)
    return {"count": len(v), "p50": float(np.percentile(a, 50)), "p95": float(np.percentile(a, 95)),
            "p99": float(np.percentile(a, 99)), "min": float(a.min()), "max": float(a.max())}


def _old_step(obs):
    view = R.build_scheduling_view(obs)
    cands = R.enumerate_candidates(view)
    sel = R.pack_candidate_batch(cands, view.topology)
    prop = Proposal.from_transfers(tuple(bind_action(view, local_token_ordinal=c.local_token_ordinal,
                                                     edge_index=c.edge_index, trusted_observation=obs) for c in sel))
    return cands, sel, prop


class _Tally:
    def __init__(self) -> None:
        self.tests = self.mismatches = 0
        self.details: list[dict] = []

    def check(self, case: str, field: str, old, new) -> None:
        self.tests += 1
        if old != new:
            self.mismatches += 1
            if len(self.details) < 50:
                self.details.append({"case": case, "field": field, "old": repr(old), "new": repr(new)})

    def report(self) -> dict:
        return {"tests": self.tests, "mismatches": self.mismatches, "details": self.details}


def run_e1(topos) -> dict:
    t = _Tally()
    for topo in topos:
        plan = C.StaticPlanCompiler().compile(topo)
        pr = plan.proof
        for f in ("topology_path_validity", "endpoint_validity", "resource_group_mapping", "template_static_legality"):
            t.check(topo.name, f, True, bool(getattr(pr, f)))
        for s in range(plan.nodes):
            for d in range(plan.nodes):
                try:
                    ref, reach = R.canonical_shortest_path(topo, s, d), True
                except R.UnreachableScenarioError:
                    ref, reach = (), False
                got_reach = s == d or int(plan.distances[s, d]) < np.iinfo(np.int32).max // 4
                t.check(f"{topo.name}:{s}->{d}", "path", (reach, ref), (got_reach, plan.canonical_paths[s][d]))
    return t.report()


def _world(topo, truth, sid, seed):
    w = UncertainProblemInstance.from_traffic_matrix(truth_matrix=truth, topology_info=topo, time_limit=160,
                                                     sequence_id=sid, sequence_step=8, family="equivalence",
                                                     generator_metadata={"seed": seed})
    return w, DemandRevealProcess(problem=w, mode="partial_shards", ratios=RATIOS, seed=seed)


def run_e2_e3(topos, backend: str, cases: int, seed: int) -> tuple[dict, dict, dict]:
    e2, e3 = _Tally(), _Tally()
    lat = {"old_ms": [], "compiled_ms": [], "guard_ms": []}
    rng = np.random.default_rng(seed)
    for topo in topos:
        plan = C.StaticPlanCompiler().compile(topo)
        for case in range(cases):
            truth = rng.integers(0, 4, size=(plan.nodes, plan.nodes))
            np.fill_diagonal(truth, 0)
            name = f"{topo.name}#{case}"
            world, reveal = _world(topo, truth, name, int(rng.integers(1 << 30)))
            # E2: a single step at every reveal stage from a fresh state
            for stage in range(len(RATIOS)):
                obs = reveal.observation_for_stage(stage)
                st = C.IncrementalState.from_observation(plan, obs)
                cands, sel, prop = _old_step(obs)
                b = C.FastBinder(plan, backend=backend).step(st)
                e2.check(f"{name}@{stage}", "candidates", C.structural_signature(cands),
                         C.structural_signature(b.candidates))
                e2.check(f"{name}@{stage}", "selected", C.structural_signature(sel), C.structural_signature(b.selected))
                e2.check(f"{name}@{stage}", "proposal", prop, b.proposal)
            # E3: the whole trajectory
            world, reveal = _world(topo, truth, name, int(rng.integers(1 << 30)))
            st = C.IncrementalState(plan, max_tokens=max(1, int(truth.sum())), max_chunks=256, sequence_id=name,
                                    sequence_step=8)
            binder, guard = C.FastBinder(plan, backend=backend), C.DynamicGuard(plan, backend=backend)
            for slot in range(world.time_limit):
                obs = reveal.observation_for_slot(slot)
                st.ingest_observation_delta(obs, chunk=slot)
                t0 = time.perf_counter()
                cands, sel, prop = _old_step(obs)
                t1 = time.perf_counter()
                b = binder.step(st)
                t2 = time.perf_counter()
                dec = guard.apply(st, b.proposal, require_scheduler_semantics=True,
                                  expected_state_version=b.state_version)
                t3 = time.perf_counter()
                lat["old_ms"].append((t1 - t0) * 1e3)
                lat["compiled_ms"].append((t2 - t1) * 1e3)
                lat["guard_ms"].append((t3 - t2) * 1e3)
                e3.check(f"{name}/{slot}", "candidates", C.structural_signature(cands),
                         C.structural_signature(b.candidates))
                e3.check(f"{name}/{slot}", "proposal", prop, b.proposal)
                try:
                    res = commit_proposal(world, obs, prop)
                    ref = (True, res.applied_actions, res.state_version)
                except Exception as exc:  # the trusted checker rejected: the guard must too
                    ref = (False, type(exc).__name__, None)
                got = ((dec.accepted, dec.applied_actions, dec.state_version) if dec.accepted
                       else (False, ref[1] if not ref[0] else dec.reason, None))
                e3.check(f"{name}/{slot}", "guard", ref, got)
                if world.is_complete():
                    break
            e3.check(name, "rebuilds", 0, st.full_rebuild_count)
            e3.check(name, "runtime_bfs", 0, binder.runtime_bfs_calls)
    return e2.report(), e3.report(), {k: _dist(v) for k, v in lat.items()}


def run(cases: int = 8, seed: int = 20260810) -> dict[str, Any]:
    topos = corpus()
    out: dict[str, Any] = {"topologies": [t.name for t in topos], "e1": run_e1(topos), "backends": {}}
    for be in ["numpy"] + (["native"] if _native.has_host() else []):
        e2, e3, lat = run_e2_e3(topos, be, cases, seed)
        out["backends"][be] = {"e2": e2, "e3": e3, "latency": lat}
    out["pass"] = out["e1"]["mismatches"] == 0 and all(
        b["e2"]["mismatches"] == 0 and b["e3"]["mismatches"] == 0 for b in out["backends"].values())
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="compiled scheduler equivalence (E1/E2/E3)")
    ap.add_argument("--cases", type=int, default=8, help="random truths per topology")
    ap.add_argument("--seed", type=int, default=20260810)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    rep = run(a.cases, a.seed)
    if a.out:
        with open(a.out, "w") as fh:
            json.dump(rep, fh, indent=2)
    print(json.dumps({"pass": rep["pass"], "e1": rep["e1"]["mismatches"],
                      **{f"{k}_e2": v["e2"]["mismatches"] for k, v in rep["backends"].items()},
                      **{f"{k}_e3": v["e3"]["mismatches"] for k, v in rep["backends"].items()},
                      **{f"{k}_compiled_p50_ms": v["latency"]["compiled_ms"].get("p50")
                         for k, v in rep["backends"].items()}}))
    if not rep["pass"]:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
