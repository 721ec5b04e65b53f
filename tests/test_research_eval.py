"""Evaluation helpers (CVaR, counterfactual histories, partial-demand
observations, sequence-policy ablations), the traffic audit and the
history-only sequence runner; differential against the reference modules
when its tree is installed under baseline/_ref."""

import importlib
import json
from pathlib import Path
import sys

import numpy as np
import pytest
import torch

from revealaiccl_b200.models.policy import SlotLevelPolicy
from revealaiccl_b200.research import evaluation as ev
from revealaiccl_b200.research import traffic_audit as ta
from revealaiccl_b200.rl.sequences import SequenceDatasetConfig, TrafficSequenceRunner, build_sequence_problems
from revealaiccl_b200.topology import ensure_bundled, load_topology_info
from revealaiccl_b200.traffic import long_horizon as lh
from revealaiccl_b200.traffic.matrix_utils import traffic_matrix_to_scenario

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _ref(name):
    if not (REF_ROOT / "rlccl").exists():
        return None
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    try:
        return importlib.import_module(name)
    except Exception:
        return None


def _json(x):
    return json.loads(json.dumps(x, default=lambda o: o.tolist() if hasattr(o, "tolist") else str(o)))


@pytest.fixture(scope="module")
def topo():
    ensure_bundled()
    return load_topology_info("Rear4GPU")


def test_cvar_and_summary():
    v = np.arange(100, dtype=float)
    assert ev.cvar(v, 0.9) == pytest.approx(v[v >= np.quantile(v, 0.9)].mean())
    assert ev.cvar(v, 0.9, higher_is_worse=False) == pytest.approx(v[v <= np.quantile(v, 0.1)].mean())
    rows = [{"completion_steps": s, "synthesis_ms": 1.0, "timeout": s > 8, "legal": True, "fallback_level": s % 2}
            for s in range(10)]
    s = ev.summarize_rows(rows)
    assert s["num_collectives"] == 10 and s["timeout_rate"] == 0.1 and s["fallback_rate"] == 0.5
    with pytest.raises(ValueError):
        ev.cvar([], 0.5)


def test_edit_distance_and_schedules():
    assert ev.action_edit_distance([(1,), (2,), (3,)], [(1,), (3,)]) == 1
    assert ev.action_edit_distance([], [(1,), (2,)]) == 2
    assert ev.action_edit_distance([(0, 1)], [(1, 0)]) == 1
    y = [np.array([[0, 1], [1, 0]]), np.array([[1, 1], [0, 0]])]
    assert ev.sparse_schedule(y) == [[0, 0, 1], [0, 1, 0], [1, 0, 0], [1, 0, 1]]
    assert ev.schedule_edge_use(y).tolist() == [2, 2]
    assert ev.edge_use_l1(y, y[:1]) == 2


def test_counterfactual_contexts_use_prior_history_only():
    rng = np.random.default_rng(0)
    mats = [rng.integers(0, 5, size=(4, 4)) * (1 - np.eye(4, dtype=np.int64)) for _ in range(10)]
    ref = np.ones((4, 4)) - np.eye(4)
    pair = ev.CounterfactualHistoryPair("p", "f", 0, mats[9], tuple(mats[:4]), tuple(mats[4:9]), ref, ref)
    a = ev.context_from_prior_history(pair.history_a, pair.current_matrix, ref, ref, window_size=8, min_history=2)
    b = ev.context_from_prior_history(pair.history_b, pair.current_matrix, ref, ref, window_size=3, min_history=2)
    assert a.history_length == 4 and b.history_length == 3
    d = ev.context_distance(a, b)
    assert d["combined"] == pytest.approx(d["mean_relative_l2"] + d["variance_relative_l2"] + d["node_load_relative_l2"])
    assert set(ev.json_ready_context(a)) >= {"mean_matrix", "var_matrix", "confidence"}
    with pytest.raises(ValueError):
        ev.CounterfactualHistoryPair("p", "f", 0, mats[9], (mats[9],), (mats[0],), ref, ref)


@pytest.mark.parametrize("mode", ev.OBSERVATION_MODES)
def test_partial_observation_preserves_chunk_identities(mode):
    T = np.array([[0, 2, 1], [0, 0, 3], [2, 1, 0]])
    sc = traffic_matrix_to_scenario(T)
    D = np.asarray(sc["demands"]).reshape(sc["C"], 3)
    o = ev.build_partial_observation(T, D, mode=mode, hide_ratio=0.5 if mode in ("random_entries", "partial_shards")
                                     else None, seed=3)
    src, _ = ev.chunk_owners(T)
    assert o.observation_demands.shape == D.shape
    if mode in ("source_totals", "source_destination_totals"):
        assert np.array_equal(o.observed_matrix.sum(axis=1), T.sum(axis=1)) and not o.revealed_chunk_mask.any()
        if mode == "source_destination_totals":
            assert np.array_equal(o.observed_matrix.sum(axis=0), T.sum(axis=0))
        # each source's chunks carry exactly the proxy row
        for s in range(3):
            assert np.array_equal(o.observation_demands[src == s].sum(axis=0), o.observed_matrix[s])
    else:
        assert np.array_equal(o.observation_demands[o.revealed_chunk_mask], D[o.revealed_chunk_mask])
        assert not o.observation_demands[~o.revealed_chunk_mask].any()
        assert o.observed_matrix.sum() == o.revealed_chunk_mask.sum()


def test_transport_from_margins_infeasible():
    with pytest.raises(RuntimeError):
        ev.transport_from_margins(np.array([3, 0]), np.array([3, 0]))  # all mass would need the diagonal


def test_audit_reports_structure():
    seq = lh.generate_long_horizon_sequence(lh.LongHorizonTrafficConfig(family="rare_shock_recovery", seed=2,
                                                                        sequence_length=600))
    a = ta.audit_sequence(seq, generation_seconds=0.2)
    assert a["temporal"]["shock_count"] > 0 and a["multi_window_moments"]["512"]["num_windows"] == 89
    assert a["temporal"]["total_traffic_acf"]["defined"]
    assert 1.0 <= a["temporal"]["total_traffic_acf"]["effective_sample_size"] <= 600
    assert ta.run_lengths([1, 1, 0, 1, 0, 0, 1, 1, 1]) == [2, 1, 3]
    per = np.tile(np.arange(4).reshape(4, 1, 1), (5, 2, 2))  # period 4
    assert ta.periodicity(per, 10)["detected_exact_period"] == 4
    r = dict(a, status="success", seed_base=0)
    s = ta.summarize_audits([r, dict(r, status="failed")])
    assert s["groups"][0]["num_failed"] == 1 and s["num_records"] == 2


def test_runner_context_excludes_current_step(topo):
    seq = lh.generate_long_horizon_sequence(lh.LongHorizonTrafficConfig(seed=1, sequence_length=40))
    out = list(TrafficSequenceRunner(seq, topo, time_limit=12, min_history=4))
    assert len(out) == 40
    p5, ctx5, rec5 = out[5]
    expect = np.stack(seq.matrices[:5]).astype(float).mean(0)
    np.fill_diagonal(expect, 0)
    assert ctx5.history_length == 5 and np.allclose(ctx5.mean_matrix, expect)
    assert p5.sequence_step == 5 and p5.moment_context is ctx5 and np.array_equal(p5.traffic_matrix, seq.matrices[5])
    assert out[0][1].history_length == 0


def test_sequence_policy_ablations(topo):
    cfg = SequenceDatasetConfig(families=("smooth_ar", "bimodal"), num_sequences_per_family=2, sequence_length=10,
                                window_size=4, min_history=2, mean_level=1.0, std_level=0.6, max_entry=3,
                                epsilon_mean=0.6, epsilon_var=1.5, seed=5, time_limit=12)
    problems, seqs, recs = build_sequence_problems(topo, cfg)
    assert len(problems) == 40 and recs[1]["seed"] == 6 and recs[2]["seed"] == 10005
    probs = [p for p in problems if p[1].C > 0 and p[1].sequence_step in (5, 6)]
    assert len({p.sequence_id for _, p in probs}) >= 2
    torch.manual_seed(0)
    from revealaiccl_b200.rl.decoder import GLOBAL_MOMENT_FEAT_DIM, MOMENT_NODE_FEAT_DIM
    model = SlotLevelPolicy(5 + MOMENT_NODE_FEAT_DIM, 2, 9, 2, 32, global_moment_feat_dim=GLOBAL_MOMENT_FEAT_DIM)
    shuffled = ev.build_shuffled_context_map(probs)
    for pid, p in probs:
        assert shuffled[pid] is not p.moment_context
    for mode in ev.CONTEXT_MODES:
        rows = ev.evaluate_sequence_policy(model, probs, "cpu", context_mode=mode, shuffled_contexts=shuffled,
                                           warmup=mode == "baseline")
        assert len(rows) == len(probs) and all(r["legal"] for r in rows)
        assert all(1 <= r["completion_steps"] <= 12 for r in rows)
    with pytest.raises(ValueError):
        ev.evaluate_sequence_policy(SlotLevelPolicy(5, 2, 5, 2, 32), probs, "cpu", context_mode="full")


def test_matches_reference_modules():
    ra = _ref("rlccl.evaluation.traffic_audit")
    rp = _ref("rlccl.evaluation.partial_demand")
    if ra is None or rp is None:
        pytest.skip("reference tree not installed under baseline/_ref")
    for fam in lh.LONG_HORIZON_FAMILIES:
        seq = lh.generate_long_horizon_sequence(lh.LongHorizonTrafficConfig(family=fam, seed=4, sequence_length=520))
        assert _json(ta.audit_sequence(seq, generation_seconds=1.0)) == _json(ra.audit_sequence(seq, generation_seconds=1.0))
    rng = np.random.default_rng(1)
    for trial in range(12):
        n = int(rng.integers(2, 6))
        T = rng.integers(0, 4, size=(n, n))
        np.fill_diagonal(T, 0)
        if T.sum() == 0:
            continue
        sc = traffic_matrix_to_scenario(T)
        D = np.asarray(sc["demands"]).reshape(sc["C"], n)
        for mode in ev.OBSERVATION_MODES:
            hr = 0.3 if mode in ("random_entries", "partial_shards") else None
            x = ev.build_partial_observation(T, D, mode=mode, hide_ratio=hr, seed=trial)
            y = rp.build_partial_observation(T, D, mode=mode, hide_ratio=hr, seed=trial)
            assert np.array_equal(x.observed_matrix, y.observed_matrix)
            assert np.array_equal(x.observation_demands, y.observation_demands)
            assert np.array_equal(x.revealed_chunk_mask, y.revealed_chunk_mask) and x.metadata == y.metadata
