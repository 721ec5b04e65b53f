"""History-only prediction study: preregistered design, leakage-safe
examples, causal TCN gradients, residual calibration, statistics, the H1
gate and a toy end-to-end run with artifact read-back; differential against
the reference modules when its tree is installed under baseline/_ref."""

import importlib
from pathlib import Path
import sys

import numpy as np
import pytest

from revealaiccl_b200.research.prediction import calibration as cal
from revealaiccl_b200.research.prediction import data as pdata
from revealaiccl_b200.research.prediction import experiment as exp
from revealaiccl_b200.research.prediction import models as pm
from revealaiccl_b200.research.prediction import statistics as st

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


def test_formal_design():
    specs = pdata.build_formal_sequence_specs()
    assert len(specs) == 75 and len({s.sequence_id for s in specs}) == 75
    assert {s.split for s in specs} == set(pdata.SPLITS)
    assert sum(s.split == "fit" for s in specs) == 30
    s = specs[5 * 3 + 2]  # family 1, base 42, slot 2
    assert s.actual_seed == 42 + 1_000_000 + 20_000 and s.split == "validation"
    fold = pdata.build_lofo_fold(specs, "rare_shock_recovery")
    assert all(x.family == "rare_shock_recovery" for x in fold["test"])
    assert not any(x.family == "rare_shock_recovery" for k in ("fit", "validation", "calibration") for x in fold[k])
    with pytest.raises(ValueError):
        pdata.validate_split_records([{"sequence_id": "a", "digest": "x", "split": "fit"},
                                      {"sequence_id": "b", "digest": "x", "split": "test"}])


def test_examples_read_only_the_past():
    spec = exp.toy_specs(40)[0]
    seq = pdata.generate_formal_sequence(spec)
    g = np.ones((1, 4, 4))
    np.fill_diagonal(g[0], 0)
    ex = pdata.build_history_examples(seq, group_coefficients=g)
    assert np.array_equal(ex.steps, np.arange(8, 40)) and np.array_equal(ex.history_last_steps, ex.steps - 1)
    m = np.asarray(seq.matrices, dtype=float)
    t = 20
    i = t - 8
    off = ~np.eye(4, dtype=bool)
    hist = m[t - 16:t]
    assert np.allclose(ex.moment_features[i], np.concatenate([hist.mean(0)[off], hist.var(0)[off]]))
    seq.matrices[t] = seq.matrices[t] + 1 - np.eye(4, dtype=np.int64)  # perturb X_t only
    ex2 = pdata.build_history_examples(seq, group_coefficients=g)
    assert np.array_equal(ex2.recent_history[i], ex.recent_history[i])
    assert np.array_equal(ex2.moment_features[i], ex.moment_features[i])
    assert not np.array_equal(ex2.targets[i], ex.targets[i])


def test_tcn_gradients_match_finite_differences():
    rng = np.random.default_rng(0)
    tcn = pm.NumpyCausalTCN(3, 2, kernel_size=3, hidden_channels=4, l2=1e-3, seed=1)
    x, y = rng.normal(size=(5, 6, 3)), rng.normal(size=(5, 2))
    _, g = tcn.loss_and_gradients(x, y)
    for name in tcn._PARAMETERS:
        p = getattr(tcn, name)
        num = np.zeros_like(p)
        for idx in np.ndindex(p.shape):
            old = p[idx]
            p[idx] = old + 1e-6
            lp = tcn.loss(x, y)
            p[idx] = old - 1e-6
            lm = tcn.loss(x, y)
            p[idx] = old
            num[idx] = (lp - lm) / 2e-6
        assert np.allclose(g[name], num, rtol=1e-5, atol=1e-7), name
    # causality: the output at the last step does not depend on padding beyond the start
    h = tcn.temporal_hidden(x)
    x2 = x.copy()
    x2[:, -1] += 1.0
    assert np.allclose(tcn.temporal_hidden(x2)[:, :-1], h[:, :-1])


def test_tcn_fit_reduces_loss_and_round_trips(tmp_path):
    rng = np.random.default_rng(2)
    x = rng.normal(size=(64, 8, 3))
    y = np.stack([x[:, -1, 0] + 0.5 * x[:, -2, 1], x[:, :, 2].mean(1)], axis=1)
    tcn = pm.NumpyCausalTCN(3, 2, epochs=30, batch_size=16, seed=3)
    hist = tcn.fit(x, y)
    assert hist[-1] < hist[0] * 0.5
    tcn.save(tmp_path / "tcn.npz")
    again = pm.NumpyCausalTCN.load(tmp_path / "tcn.npz")
    assert np.allclose(again.predict(x), tcn.predict(x))


def test_calibrator_and_tail_recall():
    rng = np.random.default_rng(4)
    pts, res = rng.normal(size=(200, 3)), rng.normal(size=(200, 3))
    c = cal.ResidualCalibrator(seed=5).fit(pts, res)
    p = c.predict(pts[:10], stable_example_indices=np.arange(10))
    assert p.scenarios.shape == (10, 64, 3) and np.all(p.q10 <= p.q90)
    again = c.predict(pts[5:10], stable_example_indices=np.arange(5, 10))  # depends only on the stable index
    assert np.array_equal(again.scenarios, p.scenarios[5:])
    r = cal.tail_event_recall(np.arange(20.0), np.arange(20.0) + 1, fit_threshold=4.5)
    assert r["status"] == "ok" and r["event_count"] == 15 and r["recall"] == 1.0
    assert cal.tail_event_recall(np.arange(5.0), np.arange(5.0), fit_threshold=3)["status"] == "insufficient_events"


def test_statistics():
    m = st.sequence_target_metrics({"a": np.array([[1.0], [2.0], [3.0]])}, {"a": np.array([[1.0], [2.0], [4.0]])})
    assert m["a"]["rmse"] == pytest.approx(np.sqrt(1 / 3)) and m["a"]["spearman"] == pytest.approx(1.0)
    b = st.family_stratified_paired_bootstrap(np.array([1.0, 2.0, 3.0, 4.0]), np.array(["x", "x", "y", "y"]),
                                              samples=500, seed=1)
    assert b.lower <= b.mean <= b.upper
    x = np.sin(np.arange(200) / 5.0)
    assert 1.0 <= st.positive_sequence_ess(x) < 200
    ev = {"pooled_total_ci_lower": 0.1, "seed_mean_deltas": {42: 1, 142: 1, 242: 1},
          "family_mean_deltas": {f: 1 for f in st.EXPECTED_FAMILIES}, "primary_ci_lowers": {t: 1 for t in st.PRIMARY_TARGETS},
          "lofo": {"aggregate_mean_delta": 1, "family_mean_deltas": {f: 1 for f in st.EXPECTED_FAMILIES},
                   "relative_rmse_changes": {f: 0 for f in st.EXPECTED_FAMILIES}},
          "probability": {"overall_interval_calibration_error": 0.01,
                          "family_interval_calibration_errors": {f: 0.01 for f in st.EXPECTED_FAMILIES},
                          "overall_scenario_calibration_error": 0.01},
          "tail": {"event_count": 12, "recall": 0.8}, "integrity_tests_passed": True, "supervisor_veto": False}
    assert st.evaluate_h1_gate(ev)["decision"] == "PASS"
    assert st.evaluate_h1_gate(dict(ev, tail={"event_count": 3, "recall": None}))["decision"] == "HOLD"
    assert st.evaluate_h1_gate(dict(ev, pooled_total_ci_lower=-1))["decision"] == "FAIL"


def test_toy_experiment_end_to_end(tmp_path):
    res = exp.run_toy_experiment(output_dir=tmp_path, length=40)
    s = res["summary"]
    assert s["selected_backbone"] in exp.CANDIDATE_METHODS
    assert set(s["lofo_selected_backbones"]) == set(pdata.FORMAL_FAMILIES[:2])
    assert s["identity_counts"]["pooled_test_sequences"] == 2
    assert len(res["point_rows"]) > 0 and len(res["probability_rows"]) == 2 * 2 * len(exp.CONTINUOUS_TARGETS)
    back = exp.read_artifacts(tmp_path)
    assert back["summary"] == s


def test_matches_reference_modules():
    rs = _ref("rlccl.prediction.statistics")
    rm = _ref("rlccl.prediction.models")
    rc = _ref("rlccl.prediction.calibration")
    rd = _ref("rlccl.prediction.data")
    if None in (rs, rm, rc, rd):
        pytest.skip("reference tree not installed under baseline/_ref")
    mine_specs, their_specs = pdata.build_formal_sequence_specs(), rd.build_formal_sequence_specs()
    assert [s.sequence_id for s in mine_specs] == [s.sequence_id for s in their_specs]
    assert [s.generator_config for s in mine_specs] == [s.generator_config for s in their_specs]
    rng = np.random.default_rng(7)
    a, b = rng.normal(size=(40, 3)), rng.normal(size=(40, 3))
    b[:5] = a[:5]
    m1, m2 = st.sequence_target_metrics({"k": a}, {"k": b})["k"], rs.sequence_target_metrics({"k": a}, {"k": b})["k"]
    assert m1 == pytest.approx(m2)
    x = rng.normal(size=(32, 6, 3))
    y = rng.normal(size=(32, 2))
    mine = pm.NumpyCausalTCN(3, 2, epochs=3, batch_size=8, seed=9)
    theirs = rm.NumpyCausalTCN(3, 2, epochs=3, batch_size=8, seed=9)
    assert np.allclose(mine.fit(x, y), theirs.fit(x, y), rtol=1e-10)
    assert np.allclose(mine.predict(x), theirs.predict(x), rtol=1e-9)
    c1 = cal.ResidualCalibrator(seed=3).fit(a, b)
    c2 = rc.ResidualCalibrator(seed=3).fit(a, b)
    p1 = c1.predict(a[:4], stable_example_indices=np.arange(4))
    p2 = c2.predict(a[:4], stable_example_indices=np.arange(4))
    assert np.array_equal(p1.scenarios, p2.scenarios) and np.array_equal(p1.q90, p2.q90)
    d = rng.normal(size=30)
    fam = np.array(["x"] * 10 + ["y"] * 20, dtype=object)
    r1 = st.family_stratified_paired_bootstrap(d, fam, samples=300, seed=2)
    r2 = rs.family_stratified_paired_bootstrap(d, fam, samples=300, seed=2)
    assert np.array_equal(r1.samples, r2.samples)
    assert st.positive_sequence_ess(d) == pytest.approx(rs.positive_sequence_ess(d))
