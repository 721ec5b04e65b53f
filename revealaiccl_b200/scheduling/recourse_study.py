"""Recourse study: revealed-only scheduling with robust-prefix plans and repair.

Capability of the reference's Phase-4 experiment
(rlccl/scheduling/phase4_experiment.py): one episode per (sequence,
checkpoint, reveal mode, method) over a truth matrix taken from a
long-horizon traffic sequence, planned only from what is revealed plus the
sequence's strictly earlier matrices, executed slot by slot through the
trusted checker, with an event ledger that recomputes the episode's
metrics, and paired statistics of each method against a comparator.

Methods (names are the study's vocabulary, roles as in the reference):

==================================== ============== ===========================
method                               role           plan source
==================================== ============== ===========================
full_information_lower_bound         lower bound    oracle completion bound
full_information_executable_reference executable ref the full observation
wait_until_known                     ordinary       waits for the last stage
partial_current_only                 ordinary       greedy on revealed tokens
long_term_mean_point_plan            ordinary point mean of the last 32 steps
previous_value_point_plan            ordinary point the previous step
h1_best_point_plan                   ordinary point per-entry linear trend
scenario_robust_prefix               H2 candidate   the last 8 steps, K8
oracle_scenario_robust_reference     oracle ceiling the truth (evaluator only)
==================================== ============== ===========================

Episode loop (own design over this package's modules): the reveal stage
advances every ``slots_per_stage`` slots; a planning method keeps a
``RecourseState``: a robust-prefix plan over its support (reconciled with
what is revealed) is built when there is none, when the stage advanced (the
old suffix is discarded) or when it is exhausted; the first batch is bound
to truth ids, committed by the trusted checker and recorded.  A slot with
nothing to do latches a wait once per (stage, state version).  The episode
ends complete, illegal (a refused commit) or at the slot limit.

``validate_event_ledger`` checks the ledger fail-closed (order, slots,
counts, state versions) and ``recompute_episode`` rebuilds completion,
executed actions and legality from it alone; the runner requires both to
agree with the episode it returns.

    python -m revealaiccl_b200.scheduling.recourse_study --toy --out runs/recourse
"""

from __future__ import annotations

import argparse
import csv
from dataclasses import dataclass, field
import json
from pathlib import Path
import time
from typing import Any, Mapping, Sequence

import numpy as np

from ..topology.info import TopologyInfo
from ..uncertainty.evaluation import oracle_completion_lower_bound
from ..uncertainty.execution import commit_proposal
from ..uncertainty.problem import UncertainProblemInstance
from ..uncertainty.reveal import DemandRevealProcess
from .recourse import RecourseState, bind_first_batch, record_committed_batch, bind_action
from .robust_prefix import (RobustPrefixConfig, RobustPrefixPlanner, build_scheduling_view, canonical_digest,
                            enumerate_candidates, pack_candidate_batch)
from .scenario_adapter import oracle_support_from_matrices, scenario_support_from_matrices

METHODS = ("full_information_lower_bound", "full_information_executable_reference", "wait_until_known",
           "partial_current_only", "long_term_mean_point_plan", "previous_value_point_plan",
           "h1_best_point_plan", "scenario_robust_prefix", "oracle_scenario_robust_reference")
ROLES = {
    "full_information_lower_bound": ("lower_bound", True, False),
    "full_information_executable_reference": ("executable_reference", True, True),
    "wait_until_known": ("ordinary", False, True),
    "partial_current_only": ("ordinary", False, True),
    "long_term_mean_point_plan": ("ordinary_point", False, True),
    "previous_value_point_plan": ("ordinary_point", False, True),
    "h1_best_point_plan": ("ordinary_point", False, True),
    "scenario_robust_prefix": ("h2_candidate", False, True),
    "oracle_scenario_robust_reference": ("oracle_ceiling", True, True),
}  # method -> (role, uses the truth, executable)
PLANNED = METHODS[4:]
POINT = METHODS[4:7]
EVENT_KINDS = ("episode_start", "wait_latch_entered", "suffix_discarded", "plan_built", "proposal_bound",
               "checker_rejected", "action_committed", "batch_committed", "episode_end")


@dataclass(frozen=True)
class EpisodeSpec:
    truth: np.ndarray
    topology: TopologyInfo
    history: tuple[np.ndarray, ...]
    reveal_mode: str = "partial_shards"
    ratios: tuple[float, ...] = (0.0, 0.25, 0.5, 0.75, 1.0)
    reveal_seed: int = 0
    sequence_id: str = "seq"
    step: int = 0
    family: str = "toy"
    base_seed: int = 0


@dataclass
class EpisodeResult:
    method: str
    role: str
    completion_slots: int
    first_action_slot: int
    executed_actions: int
    discarded_actions: int
    legality: bool
    end_reason: str
    online_ns: int
    events: list[dict[str, Any]] = field(default_factory=list)


# ------------------------------------------------------------------ supports
def _reconcile(candidate: np.ndarray, observation) -> np.ndarray:
    """A point candidate made consistent with what is revealed: integer,
    nonnegative, zero diagonal, equal to the observed entries where they are
    known and never below the revealed tokens of a pair."""
    m = np.rint(np.clip(np.asarray(candidate, dtype=np.float64), 0, None)).astype(np.int64)
    known = np.asarray(observation.entry_mask, dtype=bool)
    m[known] = np.asarray(observation.observed_matrix, dtype=np.int64)[known]
    seen = np.zeros_like(m)
    for t in observation.revealed_tokens:
        seen[t.source, t.destination] += 1
    m = np.maximum(m, seen)
    np.fill_diagonal(m, 0)
    return m


def _trend(history: Sequence[np.ndarray], window: int = 8) -> np.ndarray:
    """Per-entry least-squares line over the last ``window`` steps, one step ahead."""
    h = np.asarray(history[-window:], dtype=np.float64)
    x = np.arange(len(h), dtype=np.float64)
    xc = x - x.mean()
    slope = np.tensordot(xc, h - h.mean(axis=0), axes=(0, 0)) / max(float(xc @ xc), 1e-12)
    return h.mean(axis=0) + slope * (len(h) - x.mean())


def _support(method: str, spec: EpisodeSpec, trusted, view, final_stage: bool):
    hist = spec.history
    if final_stage:
        mats = (np.asarray(trusted.observed_matrix, dtype=np.int64),)
    elif method == "long_term_mean_point_plan":
        mats = (_reconcile(np.mean(np.stack(hist[-32:]), axis=0), trusted),)
    elif method == "previous_value_point_plan":
        mats = (_reconcile(hist[-1], trusted),)
    elif method == "h1_best_point_plan":
        mats = (_reconcile(_trend(hist), trusted),)
    elif method == "scenario_robust_prefix":
        mats = tuple(_reconcile(m, trusted) for m in hist[-8:])
    else:  # oracle ceiling: the truth itself
        mats = (np.asarray(spec.truth, dtype=np.int64),)
    if method == "oracle_scenario_robust_reference":
        return oracle_support_from_matrices(matrices=mats, weights=(1.0,) * len(mats), requested_k=8,
                                            provenance={"truth": True}, observation=view)
    return scenario_support_from_matrices(matrices=mats, weights=(1.0 / len(mats),) * len(mats),
                                          method="point" if method in POINT else "history_scenarios",
                                          requested_k=1 if method in POINT else 8, uses_oracle=False,
                                          upper_bound_only=False, provenance={"method": method},
                                          observation=view)


# ------------------------------------------------------------------- episode
def run_episode(spec: EpisodeSpec, method: str, *, planner_config: tuple[int, int, float] = (8, 4, 0.5),
                slots: int = 80, slots_per_stage: int = 4) -> EpisodeResult:
    if method not in ROLES:
        raise ValueError(f"unknown method {method!r}")
    role, _, executable = ROLES[method]
    world = UncertainProblemInstance(truth_matrix=spec.truth, topology_info=spec.topology, time_limit=slots,
                                     sequence_id=spec.sequence_id, sequence_step=spec.step, family=spec.family,
                                     generator_metadata={})
    reveal = DemandRevealProcess(problem=world, mode=spec.reveal_mode, ratios=spec.ratios, seed=spec.reveal_seed)
    last_stage = len(spec.ratios) - 1
    events: list[dict[str, Any]] = []

    def emit(kind: str, slot: int, reason: str = "", **extra: Any) -> None:
        events.append({"index": len(events), "kind": kind, "slot": int(slot), "reason": reason,
                       "method": method, **extra})

    emit("episode_start", -1)
    res = EpisodeResult(method, role, slots + 1, slots, 0, 0, True, "", 0)
    if not executable:
        res.completion_slots = oracle_completion_lower_bound(np.asarray(spec.truth), spec.topology, slots)
        res.first_action_slot = 0
        res.end_reason = "lower_bound_complete" if res.completion_slots <= slots else "lower_bound_timeout"
        emit("episode_end", min(res.completion_slots, slots), res.end_reason)
        res.events = events
        return res
    h, p, lam = planner_config
    planner = RobustPrefixPlanner(RobustPrefixConfig(h, p, 0.0 if method in POINT else lam,
                                                     1 if method in POINT else 8))
    state: RecourseState | None = None
    active_stage = -1
    latch = None
    t0 = time.perf_counter_ns()
    slot = 0
    for slot in range(slots):
        if world.is_complete():
            res.completion_slots = slot
            break
        stage = last_stage if method == "full_information_executable_reference" else min(slot // slots_per_stage,
                                                                                         last_stage)
        trusted = reveal.observation_for_stage(stage)
        view = build_scheduling_view(trusted)
        if method == "wait_until_known" and stage < last_stage:
            if latch != (stage, trusted.state_version):
                latch = (stage, trusted.state_version)
                emit("wait_latch_entered", slot, "no_common_action", stage=stage)
            continue
        if method in PLANNED:
            exhausted = state is None or state.plan is None or not state.plan.batches
            if exhausted or active_stage != stage:
                discarded = 0
                if state is not None and state.plan is not None and active_stage != stage and state.plan.batches:
                    discarded = sum(len(b) for b in state.plan.batches)
                    emit("suffix_discarded", slot, "reveal", stage=stage, action_count=discarded)
                support = _support(method, spec, trusted, view, stage == last_stage)
                plan = planner.plan(view, support)
                revision = 0 if state is None else state.current_revision + 1
                from dataclasses import replace

                plan = replace(plan, revision=revision)
                reason = "initial" if state is None else ("reveal" if active_stage != stage else "exhaustion")
                state = RecourseState(plan=plan, executed_actions=() if state is None else state.executed_actions,
                                      discarded_actions=(0 if state is None else state.discarded_actions) + discarded,
                                      execution_start_state_version=trusted.state_version, reason=reason,
                                      current_revision=revision)
                res.discarded_actions = state.discarded_actions
                active_stage = stage
                emit("plan_built", slot, reason, stage=stage, plan_revision=revision,
                     batch_count=len(plan.batches), action_count=sum(len(b) for b in plan.batches),
                     support_digest=support.digest)
            batch = state.plan.batches[0] if state.plan.batches else ()
        else:
            batch = pack_candidate_batch(enumerate_candidates(view), view.topology)
        if not batch:
            if latch != (stage, trusted.state_version):
                latch = (stage, trusted.state_version)
                emit("wait_latch_entered", slot, "no_common_action", stage=stage)
            continue
        if method in PLANNED:
            proposal = bind_first_batch(state, view, trusted_observation=trusted)
        else:
            from ..uncertainty.execution import Proposal

            proposal = Proposal.from_transfers([bind_action(view, local_token_ordinal=c.local_token_ordinal,
                                                            edge_index=c.edge_index, trusted_observation=trusted)
                                                for c in batch])
        before = trusted.state_version
        emit("proposal_bound", slot, stage=stage, action_count=len(proposal.actions), state_version_before=before)
        try:
            result = commit_proposal(world, trusted, proposal)
        except (TypeError, ValueError) as exc:
            res.legality = False
            emit("checker_rejected", slot, type(exc).__name__, stage=stage, action_count=len(proposal.actions))
            break
        if proposal.actions and res.first_action_slot == slots:
            res.first_action_slot = slot
        res.executed_actions += len(proposal.actions)
        for c, a in zip(batch, proposal.actions):
            emit("action_committed", slot, stage=stage, local_token_ordinal=c.local_token_ordinal,
                 edge_index=a.edge_index, binding=canonical_digest(str(a.token_id))[:16])
        if method in PLANNED:
            state = record_committed_batch(state, proposal=proposal, commit_result=result,
                                           fresh_observation=reveal.observation_for_stage(stage))
        emit("batch_committed", slot, stage=stage, action_count=len(proposal.actions), state_version_before=before,
             state_version_after=result.state_version)
    else:
        slot = slots
        if world.is_complete():
            res.completion_slots = slots
    res.online_ns = time.perf_counter_ns() - t0
    if not res.legality:
        res.completion_slots, res.end_reason = slots + 1, "illegal"
    elif res.completion_slots <= slots:
        res.end_reason = "complete"
    else:
        res.end_reason = "discrete_timeout"
    emit("episode_end", min(res.completion_slots, slots), res.end_reason)
    res.events = events
    return res


# -------------------------------------------------------------------- ledger
class LedgerError(ValueError):
    pass


def validate_event_ledger(events: Sequence[Mapping[str, Any]]) -> None:
    """Fail-closed structure checks of one episode's events."""
    if not events or events[0]["kind"] != "episode_start" or events[-1]["kind"] != "episode_end":
        raise LedgerError("a ledger starts with episode_start and ends with episode_end")
    if any(e["kind"] not in EVENT_KINDS for e in events):
        raise LedgerError("unknown event kind")
    if [e["index"] for e in events] != list(range(len(events))):
        raise LedgerError("event indices are not consecutive")
    last_slot = -1
    pending = None
    version = None
    for e in events[1:-1]:
        if e["slot"] < last_slot:
            raise LedgerError(f"event {e['index']}: slot goes backwards")
        last_slot = e["slot"]
        if e["kind"] == "proposal_bound":
            if pending is not None:
                raise LedgerError(f"event {e['index']}: a proposal before the previous one was settled")
            pending = {"slot": e["slot"], "n": e["action_count"], "seen": 0}
            if version is not None and e["state_version_before"] != version:
                raise LedgerError(f"event {e['index']}: stale state version")
        elif e["kind"] == "action_committed":
            if pending is None or pending["slot"] != e["slot"]:
                raise LedgerError(f"event {e['index']}: an action outside its proposal")
            pending["seen"] += 1
        elif e["kind"] == "batch_committed":
            if pending is None or pending["seen"] != pending["n"] or e["action_count"] != pending["n"]:
                raise LedgerError(f"event {e['index']}: batch count does not match its actions")
            if e["state_version_after"] != e["state_version_before"] + 1:
                raise LedgerError(f"event {e['index']}: a commit must advance the state version by one")
            version = e["state_version_after"]
            pending = None
        elif e["kind"] == "checker_rejected":
            if pending is None:
                raise LedgerError(f"event {e['index']}: a rejection without a proposal")
            pending = None
    if pending is not None:
        raise LedgerError("the last proposal was never settled")


def recompute_episode(events: Sequence[Mapping[str, Any]], *, slots: int = 80) -> dict[str, Any]:
    """Completion, executed actions and legality rebuilt from the ledger alone."""
    validate_event_ledger(events)
    end = events[-1]
    legal = not any(e["kind"] == "checker_rejected" for e in events)
    executed = sum(1 for e in events if e["kind"] == "action_committed")
    if end["reason"] in ("complete", "lower_bound_complete"):
        completion = end["slot"]
    else:
        completion = slots + 1
    return {"completion_slots": completion, "executed_actions": executed, "legality": legal}


# ----------------------------------------------------------------- the study
def toy_specs(*, families: Sequence[str] = ("regime_switching_long", "stochastic_volatility",
                                            "rare_shock_recovery"),
              base_seeds: Sequence[int] = (642, 742), checkpoints: Sequence[int] = (40, 72),
              reveal_modes: Sequence[str] = ("partial_shards", "source_totals_first"),
              topology: str = "Rear4GPU") -> list[EpisodeSpec]:
    """Episodes over long-horizon traffic sequences on a bundled topology."""
    from ..topology.loader import ensure_bundled, load_topology_info
    from ..traffic.long_horizon import LongHorizonTrafficConfig, generate_long_horizon_sequence

    ensure_bundled()
    topo = load_topology_info(topology)
    specs = []
    for fam in families:
        for seed in base_seeds:
            seq = generate_long_horizon_sequence(LongHorizonTrafficConfig(
                num_nodes=int(topo.V), sequence_length=max(checkpoints) + 1, family=fam, seed=seed))
            for ci, cp in enumerate(checkpoints):
                for mi, mode in enumerate(reveal_modes):
                    specs.append(EpisodeSpec(
                        truth=np.asarray(seq.matrices[cp], dtype=np.int64), topology=topo,
                        history=tuple(np.asarray(m, dtype=np.int64) for m in seq.matrices[max(0, cp - 32):cp]),
                        reveal_mode=mode, reveal_seed=seed * 1000 + ci * 10 + mi,
                        sequence_id=f"{fam}:{seed}", step=cp, family=fam, base_seed=seed))
    return specs


def run_study(specs: Sequence[EpisodeSpec], *, methods: Sequence[str] = METHODS, comparator: str = "partial_current_only",
              candidate: str = "scenario_robust_prefix", slots: int = 80,
              planner_config: tuple[int, int, float] = (8, 4, 0.5)) -> dict[str, Any]:
    """Every method on every episode; the ledger of each must validate and
    rebuild the episode; paired completion deltas of the candidate against
    the comparator with a bootstrap CI of the median and a gate."""
    from ..bench.paired import bootstrap_median

    rows = []
    for i, spec in enumerate(specs):
        for m in methods:
            r = run_episode(spec, m, planner_config=planner_config, slots=slots)
            again = recompute_episode(r.events, slots=slots)
            if (again["completion_slots"], again["executed_actions"], again["legality"]) != \
                    (r.completion_slots, r.executed_actions, r.legality):
                raise LedgerError(f"episode {i} {m}: the ledger does not rebuild the episode")
            rows.append({"episode": i, "family": spec.family, "base_seed": spec.base_seed, "step": spec.step,
                         "reveal_mode": spec.reveal_mode, "method": m, "role": r.role,
                         "completion_slots": r.completion_slots, "first_action_slot": r.first_action_slot,
                         "executed_actions": r.executed_actions, "discarded_actions": r.discarded_actions,
                         "legality": r.legality, "end_reason": r.end_reason, "online_us": r.online_ns / 1e3,
                         "events": len(r.events)})
    by = {(r["episode"], r["method"]): r for r in rows}
    deltas = [by[(i, comparator)]["completion_slots"] - by[(i, candidate)]["completion_slots"]
              for i in range(len(specs))]
    ci = bootstrap_median([float(d) for d in deltas]) if deltas else {"ci95_lower": 0.0, "ci95_upper": 0.0}
    per_seed = {}
    for i, spec in enumerate(specs):
        per_seed.setdefault(spec.base_seed, []).append(deltas[i])
    seeds_positive = sum(1 for v in per_seed.values() if float(np.median(v)) > 0)
    summary = {
        "episodes": len(specs), "methods": list(methods),
        "completion_mean": {m: float(np.mean([by[(i, m)]["completion_slots"] for i in range(len(specs))]))
                            for m in methods},
        "all_legal": all(r["legality"] for r in rows),
        "paired": {"candidate": candidate, "comparator": comparator,
                   "median_delta_slots": float(np.median(deltas)) if deltas else 0.0,
                   "ci95": [ci["ci95_lower"], ci["ci95_upper"]],
                   "seeds_positive": seeds_positive, "seeds": len(per_seed)},
    }
    summary["paired"]["gate_pass"] = bool(summary["paired"]["ci95"][0] > 0 and seeds_positive * 3 >= 2 * len(per_seed))
    return {"rows": rows, "summary": summary}


def write_study(result: Mapping[str, Any], out: Path) -> Path:
    out.mkdir(parents=True, exist_ok=True)
    rows = result["rows"]
    with open(out / "episodes.csv", "w", newline="", encoding="utf-8") as f:
        w = csv.DictWriter(f, fieldnames=list(rows[0]))
        w.writeheader()
        w.writerows(rows)
    (out / "summary.json").write_text(json.dumps(result["summary"], indent=1), encoding="utf-8")
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--toy", action="store_true", help="a small grid (3 families x 2 seeds x 2 checkpoints x 2 modes)")
    ap.add_argument("--out", default="recourse_study")
    ap.add_argument("--horizon", type=int, default=8)
    ap.add_argument("--prefix", type=int, default=4)
    ap.add_argument("--risk-lambda", type=float, default=0.5)
    args = ap.parse_args(argv)
    specs = toy_specs() if args.toy else toy_specs(families=("regime_switching_long", "stochastic_volatility",
                                                            "rare_shock_recovery", "hotspot_random_walk",
                                                            "same_moments_different_dynamics"),
                                                  base_seeds=(642, 742, 842), checkpoints=(40, 72, 104, 136),
                                                  reveal_modes=("random_entries", "source_totals_first",
                                                                "source_destination_totals_first",
                                                                "partial_shards", "time_based_arrival"))
    res = run_study(specs, planner_config=(args.horizon, args.prefix, args.risk_lambda))
    write_study(res, Path(args.out))
    print(json.dumps(res["summary"]))


__all__ = ["EpisodeResult", "EpisodeSpec", "LedgerError", "METHODS", "ROLES", "recompute_episode", "run_episode",
           "run_study", "toy_specs", "validate_event_ledger", "write_study"]

if __name__ == "__main__":
    main()
