"""Differential tests of the uncertainty oracle and the planner primitives
against the reference package, when its tree is installed under baseline/_ref.

The same randomized topologies, truth matrices, reveal schedules and
proposals go through both packages; every verdict must agree: revealed token
ids and holders, the trusted checker's accept / refuse decision (by error
class) and its effect on possession, scenario token expansion, candidate
enumeration, canonical routes, batch packing, residual projections, robust
scores, robust-prefix plans and the recourse binding / recording flow.
Digests are not compared (the two packages encode them differently).
"""

from __future__ import annotations

import importlib
from pathlib import Path
import sys
from types import SimpleNamespace

import numpy as np
import pytest

from revealaiccl_b200.scheduling import recourse as my_rec
from revealaiccl_b200.scheduling import robust_prefix as my_rp
from revealaiccl_b200.topology.info import TopologyInfo as MyTopo
from revealaiccl_b200.uncertainty import execution as my_ex
from revealaiccl_b200.uncertainty import observation as my_obs
from revealaiccl_b200.uncertainty import reveal as my_rv
from revealaiccl_b200.uncertainty import scenarios as my_sc
from revealaiccl_b200.uncertainty.problem import UncertainProblemInstance as MyWorld

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
MODES = ("random_entries", "source_totals_first", "source_destination_totals_first", "partial_shards",
         "time_based_arrival")


def _ref(name):
    if not (REF_ROOT / "rlccl").exists():
        pytest.skip("reference tree not installed under baseline/_ref")
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    return importlib.import_module(name)


def _random_topology(rng, nodes):
    edges = [(s, d) for s in range(nodes) for d in range(nodes) if s != d and rng.random() < 0.55]
    # keep a ring so that most pairs are reachable, plus a few duplicates
    edges += [(i, (i + 1) % nodes) for i in range(nodes)]
    edges += [edges[int(rng.integers(len(edges)))] for _ in range(int(rng.integers(0, 3)))]
    caps = rng.choice([0.0, 0.5, 1.0, 1.0, 1.7, 2.0, 3.0], size=len(edges))
    groups = []
    for _ in range(int(rng.integers(0, 4))):
        members = sorted(set(rng.choice(len(edges), size=int(rng.integers(1, 4)), replace=True).tolist()))
        groups.append((members, float(rng.choice([0.5, 1.0, 2.0, 3.0]))))
    return np.asarray(edges, dtype=np.int64), caps.astype(np.float64), groups


def _pair(rng, nodes, max_units=3):
    edges, caps, groups = _random_topology(rng, nodes)
    ref_topo = _ref("rlccl.envs.problem").TopologyInfo(nodes, len(edges), edges.copy(), caps.copy(),
                                                        [(list(m), lim) for m, lim in groups], name="rand")
    mine = MyTopo(nodes, len(edges), edges, caps, groups, name="rand")
    truth = rng.integers(0, max_units + 1, size=(nodes, nodes))
    np.fill_diagonal(truth, 0)
    return mine, ref_topo, truth


def _worlds(mine_topo, ref_topo, truth, seq="diff", step=3):
    ref_world = _ref("rlccl.uncertainty.problem").UncertainProblemInstance(
        truth_matrix=truth, topology_info=ref_topo, time_limit=50, sequence_id=seq, sequence_step=step,
        family="diff", generator_metadata={})
    my_world = MyWorld(truth_matrix=truth, topology_info=mine_topo, time_limit=50, sequence_id=seq,
                       sequence_step=step, family="diff", generator_metadata={})
    return my_world, ref_world


def _tokens(obs):
    return [(str(t.token_id), t.source, t.destination, tuple(t.holders)) for t in obs.revealed_tokens]


def _verdict(fn):
    """("ok", result) or ("raise", error class name); both packages name their errors alike."""
    try:
        out = fn()
    except (ValueError, TypeError, IndexError) as e:
        return ("raise", type(e).__name__)
    return ("ok", out)


def _kind(fn):
    """'ok' or the builtin error family (ValueError / TypeError / IndexError) raised."""
    try:
        fn()
    except ValueError:
        return "ValueError"
    except TypeError:
        return "TypeError"
    except IndexError:
        return "IndexError"
    return "ok"


@pytest.mark.parametrize("seed", range(12))
def test_reveal_and_trusted_checker_agree(seed):
    ref_rv = _ref("rlccl.uncertainty.reveal")
    ref_ex = _ref("rlccl.uncertainty.execution")
    rng = np.random.default_rng(7000 + seed)
    nodes = int(rng.integers(3, 6))
    mine_topo, ref_topo, truth = _pair(rng, nodes)
    mode = MODES[seed % len(MODES)]
    ratios = (0.0, 0.4, 0.7, 1.0)
    my_world, ref_world = _worlds(mine_topo, ref_topo, truth)
    mine = my_rv.DemandRevealProcess(problem=my_world, mode=mode, ratios=ratios, seed=seed)
    theirs = ref_rv.DemandRevealProcess(problem=ref_world, mode=mode, ratios=ratios, seed=seed)
    for stage in range(len(ratios)):
        for _slot in range(3):
            mo, ro = mine.observation_for_stage(stage), theirs.observation_for_stage(stage)
            assert _tokens(mo) == _tokens(ro)
            for key in ("entry_mask", "observed_matrix", "unknown_mask"):
                assert np.array_equal(getattr(mo, key), getattr(ro, key))
            mp, rp = mo.to_policy_payload(), ro.to_policy_payload()
            assert list(mp) == list(rp) and list(mp["topology"]) == list(rp["topology"])
            # a random slot: mostly plausible hops, some bad ones
            acts = []
            for t in mo.revealed_tokens:
                if rng.random() < 0.3:
                    cand = [e for e in range(mine_topo.E)
                            if mine_topo.edges[e, 0] in t.holders and mine_topo.edges[e, 1] not in t.holders]
                    e = int(rng.choice(cand)) if cand and rng.random() < 0.9 else int(rng.integers(-1, mine_topo.E + 1))
                    acts.append((str(t.token_id), e))
            if acts and rng.random() < 0.15:
                acts.append(acts[0])  # duplicate token
            my_p = my_ex.Proposal.from_transfers([my_ex.TransferAction(my_obs.TruthTokenId(a), e) for a, e in acts])
            ref_obs_mod = _ref("rlccl.uncertainty.observation")
            ref_p = ref_ex.Proposal.from_transfers(
                tuple(ref_ex.TransferAction(ref_obs_mod.TruthTokenId(a), e) for a, e in acts))
            mv = _kind(lambda: my_ex.commit_proposal(my_world, mo, my_p))
            rv = _kind(lambda: ref_ex.commit_proposal(ref_world, ro, ref_p))
            assert mv == rv, (acts, mv, rv)
            assert my_world._state_version == ref_world._state_version
            assert np.array_equal(my_world._possession, ref_world._possession)
            # the old observation is now stale when the slot applied
            if mv == "ok" and acts:
                assert _kind(lambda: my_ex.commit_proposal(my_world, mo, my_ex.Proposal.wait())) == "ValueError"
                assert _kind(lambda: ref_ex.commit_proposal(ref_world, ro, ref_ex.Proposal.wait())) == "ValueError"


def test_scenario_tokens_and_legacy_matrix_agree():
    ref_sc = _ref("rlccl.uncertainty.scenarios")
    ref_ex = _ref("rlccl.uncertainty.execution")
    rng = np.random.default_rng(11)
    mats = [rng.integers(0, 3, size=(4, 4)) for _ in range(3)]
    for m in mats:
        np.fill_diagonal(m, 0)
    kw = dict(matrices=mats, weights=[1.0, 2.0, 0.5], scenario_ids=["a", "b", "c"], provenance=["x", "y", "z"])
    mine, theirs = my_sc.ScenarioSet.from_matrices(**kw), ref_sc.ScenarioSet.from_matrices(**kw)
    assert mine.weights == theirs.weights
    for mg, rg in zip(mine.scenario_tokens, theirs.scenario_tokens):
        assert [(str(t.token_id), t.source, t.destination) for t in mg] == \
               [(str(t.token_id), t.source, t.destination) for t in rg]
    bad_weights = dict(kw, weights=[0.0, 0.0, 0.0])
    assert _kind(lambda: my_sc.ScenarioSet.from_matrices(**bad_weights)) == \
           _kind(lambda: ref_sc.ScenarioSet.from_matrices(**bad_weights)) == "ValueError"
    frac = dict(kw, matrices=[m + 0.5 * np.eye(4) * 0 + (0.5 if i == 0 else 0) for i, m in enumerate(mats)])
    assert _kind(lambda: my_sc.ScenarioSet.from_matrices(**frac)) == _kind(lambda: ref_sc.ScenarioSet.from_matrices(**frac))
    for candidate in ([[0, 1], [1, 0]], [[0, 2], [1, 0]], [[0, -1], [1, 0]], [[0, np.nan], [1, 0]], [[0, 1]],
                      [[0.0, 1.0], [1.0, 0.0]]):
        m_kind = _kind(lambda: my_ex.validate_legacy_schedule_matrix(candidate, expected_shape=(2, 2)))
        r_kind = _kind(lambda: ref_ex.validate_legacy_schedule_matrix(candidate, expected_shape=(2, 2)))
        assert m_kind == r_kind, candidate


def _views(rng, mine_topo, ref_topo, nodes, count):
    ref_rp = _ref("rlccl.scheduling.robust_prefix")
    ref_obs = _ref("rlccl.uncertainty.observation")
    toks = []
    for i in range(count):
        s, d = (int(x) for x in rng.choice(nodes, size=2, replace=False))
        holders = sorted({s} | set(rng.choice(nodes, size=int(rng.integers(0, 2))).tolist()))
        toks.append((i, s, d, tuple(holders)))
    obs = rng.integers(0, 3, size=(nodes, nodes))
    np.fill_diagonal(obs, 0)

    def view(mod, obs_mod, topo):
        pt = obs_mod.PublicTopologyView.from_topology_info(topo)
        return mod.SchedulingObservationView(
            1, 0.5, 0, obs, np.ones((nodes, nodes), dtype=bool), None, None,
            tuple(mod.PublicRevealedToken(*t) for t in toks), pt, "d", "r")

    return view(my_rp, my_obs, mine_topo), view(ref_rp, ref_obs, ref_topo), toks


def _cands(cs):
    return [(c.local_token_ordinal, c.edge_index, c.before_distance, c.after_distance) for c in cs]


@pytest.mark.parametrize("seed", range(16))
def test_planner_primitives_agree(seed):
    ref_rp = _ref("rlccl.scheduling.robust_prefix")
    rng = np.random.default_rng(9100 + seed)
    nodes = int(rng.integers(3, 7))
    mine_topo, ref_topo, _ = _pair(rng, nodes)
    for s in range(nodes):
        for d in range(nodes):
            mv = _verdict(lambda: my_rp.canonical_shortest_path(mine_topo, s, d))
            rv = _verdict(lambda: ref_rp.canonical_shortest_path(ref_topo, s, d))
            assert mv == rv, (s, d)
    my_view, ref_view, toks = _views(rng, mine_topo, ref_topo, nodes, int(rng.integers(1, 9)))
    mc, rc = my_rp.enumerate_candidates(my_view), ref_rp.enumerate_candidates(ref_view)
    assert _cands(mc) == _cands(rc)
    for t in toks:
        for e in range(len(mine_topo.edges)):
            m = my_rp.candidate_distances(mine_topo, holders=t[3], destination=t[2], edge_index=e)
            r = ref_rp.candidate_distances(ref_topo, holders=t[3], destination=t[2], edge_index=e)
            assert (m.source_distance, m.edge_target_distance, m.before_global, m.after_global) == \
                   (r.source_distance, r.edge_target_distance, r.before_global, r.after_global)
    order = list(range(len(mc)))
    rng.shuffle(order)
    mb = my_rp.pack_candidate_batch([mc[i] for i in order], my_view.topology)
    rb = ref_rp.pack_candidate_batch([rc[i] for i in order], ref_view.topology)
    assert _cands(mb) == _cands(rb)
    ml, rl = my_rp.batch_loads(mb, mine_topo), ref_rp.batch_loads(rb, ref_topo)
    assert np.array_equal(ml.edge_units, rl.edge_units) and np.array_equal(ml.group_units, rl.group_units)
    # residual projections and robust scores over random scenarios
    scen = []
    for _ in range(3):
        m = rng.integers(0, 3, size=(nodes, nodes))
        np.fill_diagonal(m, 0)
        for _, s, d, _ in toks:
            m[s, d] += 1
        scen.append(m)
    for m in scen + [np.zeros((nodes, nodes), dtype=np.int64)]:
        mv = _verdict(lambda: my_rp.project_residual_scenario(m, my_view))
        rv = _verdict(lambda: ref_rp.project_residual_scenario(m, ref_view))
        assert mv[0] == rv[0], (mv, rv)
        if mv[0] == "ok":
            assert np.array_equal(mv[1].edge_loads, rv[1].edge_loads)
            assert np.array_equal(mv[1].group_loads, rv[1].group_loads)
        else:
            assert mv == rv
    if all(_verdict(lambda: ref_rp.project_residual_scenario(m, ref_view))[0] == "ok" for m in scen):
        weights = [1.0, 2.0, 3.0]
        ms = SimpleNamespace(observation=my_view, matrices=scen, weights=weights, stage=1,
                             observation_digest="d", digest="sd")
        rs = SimpleNamespace(observation=ref_view, matrices=scen, weights=weights, stage=1,
                             observation_digest="d", digest="sd")
        for lam in (0.0, 0.5, 1.0):
            a = my_rp.score_candidates(mc, ms, risk_lambda=lam)
            b = ref_rp.score_candidates(rc, rs, risk_lambda=lam)
            assert [(x.robust_score, x.scenario_std) for x in a] == [(x.robust_score, x.scenario_std) for x in b]
        for h, p in ((4, 2), (8, 4), (2, 1)):
            cfg_m = my_rp.RobustPrefixConfig(h, p, 0.5, 8)
            cfg_r = ref_rp.RobustPrefixConfig(h, p, 0.5, 8)
            pm = my_rp.RobustPrefixPlanner(cfg_m).plan(my_view, ms)
            pr = ref_rp.RobustPrefixPlanner(cfg_r).plan(ref_view, rs)
            assert pm.structural_actions == pr.structural_actions
            assert [_cands(b) for b in pm.batches] == [_cands(b) for b in pr.batches]
            assert len(pm.simulation_trace) == len(pr.simulation_trace)


@pytest.mark.parametrize("seed", range(6))
def test_recourse_flow_agrees(seed):
    """Plan, bind, commit and record the first batch in both packages; then a
    stale replay and a stale revision are refused with the same reasons."""
    ref_rp = _ref("rlccl.scheduling.robust_prefix")
    ref_rec = _ref("rlccl.scheduling.recourse")
    ref_rv = _ref("rlccl.uncertainty.reveal")
    rng = np.random.default_rng(4400 + seed)
    nodes = 4
    mine_topo, ref_topo, truth = _pair(rng, nodes, max_units=2)
    my_world, ref_world = _worlds(mine_topo, ref_topo, truth)
    mine = my_rv.DemandRevealProcess(problem=my_world, mode="partial_shards", ratios=(0.0, 1.0), seed=seed)
    theirs = ref_rv.DemandRevealProcess(problem=ref_world, mode="partial_shards", ratios=(0.0, 1.0), seed=seed)
    mo, ro = mine.observation_for_stage(1), theirs.observation_for_stage(1)
    mv, rv = my_rp.build_scheduling_view(mo), ref_rp.build_scheduling_view(ro)
    scen = [np.asarray(truth)]
    ms = SimpleNamespace(observation=mv, matrices=scen, weights=[1.0], stage=mv.stage,
                         observation_digest=mv.observation_digest, digest="s")
    rs = SimpleNamespace(observation=rv, matrices=scen, weights=[1.0], stage=rv.stage,
                         observation_digest=rv.observation_digest, digest="s")
    try:
        rplan = ref_rp.RobustPrefixPlanner(ref_rp.RobustPrefixConfig(4, 2, 0.0, 1)).plan(rv, rs)
    except ValueError:
        with pytest.raises(ValueError):
            my_rp.RobustPrefixPlanner(my_rp.RobustPrefixConfig(4, 2, 0.0, 1)).plan(mv, ms)
        return
    mplan = my_rp.RobustPrefixPlanner(my_rp.RobustPrefixConfig(4, 2, 0.0, 1)).plan(mv, ms)
    assert mplan.structural_actions == rplan.structural_actions
    mst, rst = my_rec.RecourseState.initial(mplan), ref_rec.RecourseState.initial(rplan)
    if not mplan.batches:
        a = my_rec.execute_first_batch(world=my_world, state=mst, view=mv, trusted_observation=mo)
        b = ref_rec.execute_first_batch(world=ref_world, state=rst, view=rv, trusted_observation=ro)
        assert (a.legality, a.illegal_reason) == (b.legality, b.illegal_reason)
        return
    a = my_rec.execute_first_batch(world=my_world, state=mst, view=mv, trusted_observation=mo)
    b = ref_rec.execute_first_batch(world=ref_world, state=rst, view=rv, trusted_observation=ro)
    assert (a.legality, a.stopped, a.illegal_reason) == (b.legality, b.stopped, b.illegal_reason)
    if not a.legality:
        return
    assert a.commit_result.applied_actions == b.commit_result.applied_actions
    fresh_m, fresh_r = mine.observation_for_stage(1), theirs.observation_for_stage(1)
    mst2 = my_rec.record_committed_batch(mst, proposal=a.proposal, commit_result=a.commit_result,
                                         fresh_observation=fresh_m)
    rst2 = ref_rec.record_committed_batch(rst, proposal=b.proposal, commit_result=b.commit_result,
                                          fresh_observation=fresh_r)
    assert mst2.plan.structural_actions == rst2.plan.structural_actions
    assert mst2.next_batch_index == rst2.next_batch_index == 1
    assert len(mst2.executed_actions) == len(rst2.executed_actions)
    # replaying the executed batch against the old view: both refuse, same reason
    a2 = my_rec.execute_first_batch(world=my_world, state=mst, view=mv, trusted_observation=mo)
    b2 = ref_rec.execute_first_batch(world=ref_world, state=rst, view=rv, trusted_observation=ro)
    assert (a2.legality, a2.illegal_reason) == (b2.legality, b2.illegal_reason)
    # a stale revision
    from dataclasses import replace
    a3 = my_rec.execute_first_batch(world=my_world, state=replace(mst2, current_revision=5),
                                    view=my_rp.build_scheduling_view(fresh_m), trusted_observation=fresh_m)
    b3 = ref_rec.execute_first_batch(world=ref_world, state=replace(rst2, current_revision=5),
                                     view=ref_rp.build_scheduling_view(fresh_r), trusted_observation=fresh_r)
    assert (a3.legality, a3.illegal_reason) == (b3.legality, b3.illegal_reason)
    # ledger replay protection
    ident = my_rec.ExecutedActionIdentity("t", 1, 0, 0)
    led = my_rec.ExecutedLedger.empty().append(ident)
    assert not led.can_append(ident)
    with pytest.raises(my_rec.ReplayedActionError):
        led.append(ident)
    for new_stage, exhausted, valid in ((True, False, True), (False, True, True), (False, False, False),
                                        (False, False, True)):
        assert my_rec.choose_transition(new_stage=new_stage, prefix_exhausted=exhausted,
                                        precondition_valid=valid) == \
            my_rec.Transition(*tuple(ref_rec.choose_transition(new_stage=new_stage, prefix_exhausted=exhausted,
                                                               precondition_valid=valid).__getattribute__(f)
                                     for f in ("reason", "reveal_delta", "exhaustion_delta", "invalidation_delta")))
