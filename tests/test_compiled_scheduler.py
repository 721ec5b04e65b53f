"""Compiled scheduler (StaticPlanCompiler / IncrementalState / FastBinder /
DynamicGuard) against the uncompiled reference planner and the trusted checker.

Covers the reference's contracts (tests/test_r2_compiled_scheduler.py): exact
canonical BFS with destination-first ties, exact candidate and tie order,
pending chunks invisible, guard == checker accept/apply, duplicate commit,
capacity and group limits, unrevealed rejection, delta ingest without
rebuild, no runtime BFS, in-order activation, fail-closed proof — plus a
randomized static / single-step / trajectory equivalence harness run on both
the NumPy core and the C++ core.
"""

from __future__ import annotations

import numpy as np
import pytest

from revealaiccl_b200.ops import _native
from revealaiccl_b200.scheduling import compiled as C
from revealaiccl_b200.scheduling import robust_prefix as R
from revealaiccl_b200.scheduling.recourse import bind_action
from revealaiccl_b200.topology import TopologyInfo, load_rear4_topology
from revealaiccl_b200.uncertainty import (DemandRevealProcess, Proposal, TransferAction,
                                          UncertainProblemInstance, commit_proposal)

BACKENDS = ["numpy"] + (["native"] if _native.has_host() else [])


def topo(edges, caps=None, groups=(), nodes=4):
    return TopologyInfo(nodes, len(edges), np.asarray(edges, dtype=np.int64),
                        np.asarray(caps or (1.0,) * len(edges), dtype=np.float64), list(groups),
                        name="unit")


def episode(t, truth, ratio=1.0, seed=20260810):
    world = UncertainProblemInstance.from_traffic_matrix(
        truth_matrix=truth, topology_info=t, time_limit=80, sequence_id="unit", sequence_step=8,
        family="unit", generator_metadata={})
    ratios = (0.0, ratio, 1.0) if ratio < 1.0 else (0.0, 1.0)
    reveal = DemandRevealProcess(problem=world, mode="partial_shards", ratios=ratios, seed=seed)
    return world, reveal, reveal.observation_for_stage(1)


def old_path(observation):
    view = R.build_scheduling_view(observation)
    cands = R.enumerate_candidates(view)
    sel = R.pack_candidate_batch(cands, view.topology)
    proposal = Proposal.from_transfers(tuple(
        bind_action(view, local_token_ordinal=c.local_token_ordinal, edge_index=c.edge_index,
                    trusted_observation=observation) for c in sel))
    return view, cands, sel, proposal


@pytest.mark.parametrize("backend", BACKENDS)
def test_compiler_matches_canonical_bfs_destination_first(backend):
    edges = ((3, 2), (2, 0), (0, 3), (1, 2), (2, 3), (3, 0), (1, 3), (2, 1), (3, 1), (0, 1), (1, 2))
    t = topo(edges)
    plan = C.StaticPlanCompiler().compile(t)
    assert plan.proof.valid
    for s in range(4):
        for d in range(4):
            expect = () if s == d else R.canonical_shortest_path(t, s, d)
            assert plan.canonical_paths[s][d] == expect
    # 0 -> 2: both 0->1->2 and 0->3->2 are two hops; BFS expands 0's out-edges
    # in target order so node 1 (edge 9) is discovered first.
    assert plan.canonical_paths[0][2][0] == 9


@pytest.mark.parametrize("backend", BACKENDS)
def test_candidate_and_tie_order_exact(backend):
    t = topo(((0, 1), (0, 2), (1, 3), (2, 3), (1, 0), (2, 0), (3, 0)))
    truth = np.zeros((4, 4), dtype=np.int64)
    truth[0, 3] = 2
    _, _, obs = episode(t, truth)
    _, cands, sel, _ = old_path(obs)
    plan = C.StaticPlanCompiler().compile(t)
    state = C.IncrementalState.from_observation(plan, obs, max_tokens=64)
    bound = C.FastBinder(plan, backend=backend).step(state)
    assert C.structural_signature(bound.candidates) == C.structural_signature(cands)
    assert C.structural_signature(bound.selected) == C.structural_signature(sel)
    assert tuple(c.edge_index for c in bound.selected) == (0, 1)


@pytest.mark.parametrize("backend", BACKENDS)
def test_pending_chunk_is_invisible(backend):
    t = topo(((0, 1), (1, 2), (2, 3), (0, 2), (1, 3)))
    truth = np.zeros((4, 4), dtype=np.int64)
    truth[0, 3] = 2
    _, reveal, obs = episode(t, truth, ratio=0.5)
    plan = C.StaticPlanCompiler().compile(t)
    state = C.IncrementalState.from_observation(plan, obs, max_tokens=64)
    binder = C.FastBinder(plan, backend=backend)
    before = C.structural_signature(binder.step(state).selected)
    hidden = reveal.full_observation().revealed_tokens[len(obs.revealed_tokens):]
    state.stage_ready_chunk(7, hidden)
    assert C.structural_signature(binder.step(state).selected) == before
    assert state.pending_ready_bitmap != 0 and state.revealed_count == len(obs.revealed_tokens)


@pytest.mark.parametrize("backend", BACKENDS)
def test_guard_accept_and_apply_match_trusted_checker(backend):
    t, _ = load_rear4_topology()
    truth = np.array([[0, 2, 1, 0], [1, 0, 0, 2], [0, 3, 0, 1], [1, 1, 1, 0]])
    world, _, obs = episode(t, truth)
    plan = C.StaticPlanCompiler().compile(t)
    state = C.IncrementalState.from_observation(plan, obs, max_tokens=64)
    bound = C.FastBinder(plan, backend=backend).step(state)
    decision = C.DynamicGuard(plan, backend=backend).apply(
        state, bound.proposal, require_scheduler_semantics=True,
        expected_state_version=bound.state_version)
    result = commit_proposal(world, obs, bound.proposal)
    assert decision.accepted and result.legal
    assert decision.applied_actions == result.applied_actions
    assert decision.state_version == result.state_version
    for o in range(state.revealed_count):
        private = world._public_to_private[state.token_ids[o]]
        assert tuple(np.flatnonzero(world._possession[private])) == tuple(np.flatnonzero(state.holders[o]))


@pytest.mark.parametrize("backend", BACKENDS)
def test_guard_rejections_fail_closed(backend):
    t = topo(((0, 1), (1, 2), (0, 2)), caps=(1.0, 1.0, 1.0), groups=(((0, 2), 1.0),), nodes=3)
    truth = np.zeros((3, 3), dtype=np.int64)
    truth[0, 2] = 2
    truth[0, 1] = 1
    _, _, obs = episode(t, truth)
    plan = C.StaticPlanCompiler().compile(t)
    guard = C.DynamicGuard(plan, backend=backend)
    state = C.IncrementalState.from_observation(plan, obs, max_tokens=8)
    ids = [tok.token_id for tok in obs.revealed_tokens]
    by_dst = {}
    for tok in obs.revealed_tokens:
        by_dst.setdefault(tok.destination, []).append(tok.token_id)
    two = by_dst[2]
    # same edge twice exceeds capacity
    d = guard.check(state, Proposal.from_transfers((TransferAction(two[0], 2), TransferAction(two[1], 2))))
    assert not d.accepted and d.reason == "edge_capacity"
    # edges 0 and 2 share a group of limit 1
    d = guard.check(state, Proposal.from_transfers((TransferAction(two[0], 2), TransferAction(by_dst[1][0], 0))))
    assert not d.accepted and d.reason == "bandwidth_group"
    # duplicate token in one slot
    d = guard.check(state, Proposal.from_transfers((TransferAction(two[0], 2), TransferAction(two[0], 0))))
    assert not d.accepted and d.reason == "duplicate_in_slot"
    # source must hold the token
    d = guard.check(state, Proposal.from_transfers((TransferAction(two[0], 1),)))
    assert not d.accepted and d.reason == "source_holder"
    # stale version
    d = guard.check(state, Proposal.wait(), expected_state_version=state.state_version + 1)
    assert not d.accepted and d.reason == "stale_state_version"
    # unknown token id
    from revealaiccl_b200.uncertainty import TruthTokenId
    d = guard.check(state, Proposal.from_transfers((TransferAction(TruthTokenId("truth:nope"), 0),)))
    assert not d.accepted and d.reason == "unrevealed"
    # apply then duplicate commit on the same edge
    ok = guard.apply(state, Proposal.from_transfers((TransferAction(two[0], 2),)))
    assert ok.accepted
    d = guard.check(state, Proposal.from_transfers((TransferAction(two[0], 2),)))
    assert not d.accepted and d.reason == "duplicate_commit"
    assert len(ids) == 3


@pytest.mark.parametrize("backend", BACKENDS)
def test_delta_ingest_no_rebuild_and_no_runtime_bfs(backend, monkeypatch):
    t, _ = load_rear4_topology()
    truth = np.array([[0, 2, 1, 0], [1, 0, 0, 2], [0, 3, 0, 1], [1, 1, 1, 0]])
    world = UncertainProblemInstance.from_traffic_matrix(
        truth_matrix=truth, topology_info=t, time_limit=80, sequence_id="unit", sequence_step=8,
        family="unit", generator_metadata={})
    reveal = DemandRevealProcess(problem=world, mode="partial_shards", ratios=(0.0, 0.25, 0.5, 1.0), seed=5)
    plan = C.StaticPlanCompiler().compile(t)
    state = C.IncrementalState(plan, max_tokens=64, sequence_id="unit", sequence_step=8)

    def boom(*a, **k):
        raise AssertionError("runtime BFS is forbidden")

    monkeypatch.setattr(R, "canonical_shortest_path", boom)
    binder = C.FastBinder(plan, backend=backend)
    for stage in range(1, 4):
        obs = reveal.observation_for_stage(stage)
        state.ingest_observation_delta(obs, chunk=stage)
        binder.step(state)
    assert state.full_rebuild_count == 0
    assert binder.runtime_bfs_calls == 0
    assert state.delta_update_count == 3


def test_out_of_order_consume_rejected():
    t, _ = load_rear4_topology()
    truth = np.array([[0, 2, 0, 0], [0, 0, 0, 0], [0, 0, 0, 1], [0, 0, 0, 0]])
    _, _, obs = episode(t, truth)
    plan = C.StaticPlanCompiler().compile(t)
    state = C.IncrementalState(plan, max_tokens=8)
    toks = obs.revealed_tokens
    state.stage_ready_chunk(0, toks[:1])
    state.stage_ready_chunk(1, toks[1:])
    with pytest.raises(ValueError, match="out-of-order"):
        state.consume_pending_chunk(1)
    state.consume_pending_chunk(0)
    state.consume_pending_chunk(1)
    assert state.revealed_count == len(toks)


def test_bad_group_mapping_fails_closed():
    t = topo(((0, 1), (1, 0)), groups=(((0, 0), 1.0),), nodes=2)
    with pytest.raises(ValueError):
        C.StaticPlanCompiler().compile(t)


def _random_topology(rng, nodes):
    edges = [(u, v) for u in range(nodes) for v in range(nodes) if u != v and rng.random() < 0.55]
    for u in range(nodes):  # ring keeps it strongly connected
        edges.append((u, (u + 1) % nodes))
    caps = [float(rng.choice([0.5, 1.0, 1.0, 2.0, 2.7])) for _ in edges]
    groups = []
    for _ in range(int(rng.integers(0, 3))):
        members = sorted(set(int(x) for x in rng.choice(len(edges), size=min(3, len(edges)), replace=False)))
        groups.append((members, float(rng.choice([1.0, 2.0, 3.5]))))
    return TopologyInfo(nodes, len(edges), np.asarray(edges, dtype=np.int64), np.asarray(caps), groups, name="rand")


@pytest.mark.parametrize("backend", BACKENDS)
@pytest.mark.parametrize("seed", range(12))
def test_randomized_trajectory_equivalence(backend, seed):
    """Static, single-step and trajectory equivalence: at every slot the compiled
    candidates, selection and proposal equal the reference path, and the guard's
    verdict / applied count / version equal the trusted checker's."""
    rng = np.random.default_rng(1000 + seed)
    nodes = int(rng.integers(3, 7))
    t = _random_topology(rng, nodes)
    truth = rng.integers(0, 3, size=(nodes, nodes))
    np.fill_diagonal(truth, 0)
    world = UncertainProblemInstance.from_traffic_matrix(
        truth_matrix=truth, topology_info=t, time_limit=40, sequence_id=f"rand{seed}",
        sequence_step=1, family="rand", generator_metadata={})
    reveal = DemandRevealProcess(problem=world, mode="partial_shards",
                                 ratios=(0.0, 0.25, 0.5, 0.75, 1.0), seed=seed)
    plan = C.StaticPlanCompiler().compile(t)
    for s in range(nodes):
        for d in range(nodes):
            if s != d:
                try:
                    ref = R.canonical_shortest_path(t, s, d)
                except R.UnreachableScenarioError:
                    ref = ()
                assert plan.canonical_paths[s][d] == ref
    state = C.IncrementalState(plan, max_tokens=max(1, int(truth.sum())), max_chunks=64,
                               sequence_id=f"rand{seed}", sequence_step=1)
    binder = C.FastBinder(plan, backend=backend)
    guard = C.DynamicGuard(plan, backend=backend)
    for slot in range(30):
        obs = reveal.observation_for_slot(slot)
        state.ingest_observation_delta(obs, chunk=slot)
        _, cands, sel, proposal = old_path(obs)
        bound = binder.step(state)
        assert C.structural_signature(bound.candidates) == C.structural_signature(cands)
        assert C.structural_signature(bound.selected) == C.structural_signature(sel)
        assert bound.proposal == proposal
        decision = guard.apply(state, bound.proposal, require_scheduler_semantics=True,
                               expected_state_version=bound.state_version)
        result = commit_proposal(world, obs, proposal)
        assert decision.accepted and result.legal
        assert decision.applied_actions == result.applied_actions
        assert decision.state_version == result.state_version
        if world.is_complete():
            break
    assert state.full_rebuild_count == 0 and binder.runtime_bfs_calls == 0


def test_equivalence_runner_reports_zero_mismatches():
    """The E1/E2/E3 runner over the six-topology corpus (one random truth each)."""
    from revealaiccl_b200.bench import equivalence as eq

    rep = eq.run(cases=1, seed=7)
    assert rep["pass"] and rep["e1"]["tests"] > 6 * 16
    for be in rep["backends"].values():
        assert be["e2"]["tests"] > 0 and be["e3"]["tests"] > 0 and be["latency"]["compiled_ms"]["count"] > 0
