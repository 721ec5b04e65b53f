"""Traffic-summary predictors: history-only examples, ridge heads, group
coefficients on a routed topology, npz artifact round trip; differential
against the reference predictor when its tree is installed under
baseline/_ref."""

import importlib
from pathlib import Path
import sys

import numpy as np
import pytest

from revealaiccl_b200.research import traffic_predictor as tp
from revealaiccl_b200.topology.loader import load_topology_info
from revealaiccl_b200.traffic.long_horizon import LongHorizonTrafficConfig, generate_long_horizon_sequence

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _seqs(n=4, length=160):
    return [generate_long_horizon_sequence(LongHorizonTrafficConfig(family=f, seed=s, num_nodes=n,
                                                                    sequence_length=length, calibration_candidates=1))
            for f, s in (("regime_switching_long", 1), ("hotspot_random_walk", 2))]


def test_ridge_recovers_linear_map_and_round_trips():
    rng = np.random.default_rng(0)
    X = rng.normal(size=(200, 5))
    X[:, 3] = 2.0  # constant column keeps scale 1
    W = rng.normal(size=(5, 3))
    Y = X @ W + 0.5
    r = tp.RidgeMultiOutput(alpha=1e-9).fit(X, Y)
    assert np.allclose(r.predict(X), Y, atol=1e-6)
    assert r.x_scale[3] == 1.0
    r2 = tp.RidgeMultiOutput.from_state(r.state("h"), "h")
    assert np.allclose(r2.predict(X), r.predict(X))
    with pytest.raises(RuntimeError):
        tp.RidgeMultiOutput().predict(X)


def test_examples_are_history_only():
    seqs = _seqs()
    ex = tp.build_history_examples(seqs, group_coefficients=np.zeros((0, 4, 4)), history_window=32,
                                   recent_steps=4, min_history=8)
    assert len(ex) == 2 * (160 - 8)
    e = ex[10]
    t = e["step"]
    mats = np.asarray(seqs[0].matrices, dtype=float)
    hist = mats[max(0, t - 32):t]
    off = ~np.eye(4, dtype=bool)
    assert e["history_last_step"] == t - 1
    assert np.allclose(e["moment_features"], np.concatenate([hist.mean(0)[off], hist.var(0)[off]]))
    assert np.allclose(e["target"], tp.summary_vector(tp.traffic_summary(mats[t], np.zeros((0, 4, 4)))))
    # changing X_t changes the target but no feature
    seqs[0].matrices[t] = seqs[0].matrices[t] + 1 - np.eye(4, dtype=np.int64)
    ex2 = tp.build_history_examples(seqs, group_coefficients=np.zeros((0, 4, 4)), history_window=32,
                                    recent_steps=4, min_history=8)
    assert np.array_equal(ex2[10]["moment_features"], e["moment_features"])
    assert np.array_equal(ex2[10]["recent_features"], e["recent_features"])
    assert not np.array_equal(ex2[10]["target"], e["target"])


def test_suite_fit_predict_save_load(tmp_path):
    topo = load_topology_info("Rear8GPU_NoSwitch_Test")
    coeff = tp.deterministic_group_coefficients(topo)
    assert coeff.shape == (len(topo.shared_constraints), topo.V, topo.V) and coeff.sum() > 0
    seqs = _seqs(n=topo.V, length=96)
    ex = tp.build_history_examples(seqs, group_coefficients=coeff, history_window=16, recent_steps=3, min_history=4)
    suite = tp.TrafficPredictorSuite(topo.V, coeff.shape[0]).fit(ex)
    pred = suite.predict(ex)
    assert set(pred) == {"target", "constant", "previous", "moment_only", "recent_history", "oracle_current_summary"}
    assert pred["moment_only"]["continuous"].shape == (len(ex), suite.target_dim)
    path = str(tmp_path / "suite.npz")
    suite.save(path)
    again = tp.TrafficPredictorSuite.load(path).predict(ex)
    assert np.allclose(again["recent_history"]["continuous"], pred["recent_history"]["continuous"])
    assert np.array_equal(again["moment_only"]["hotspot"], pred["moment_only"]["hotspot"])


def _ref(name):
    if not (REF_ROOT / "rlccl").exists():
        return None
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    try:
        return importlib.import_module(name)
    except Exception:
        return None


@pytest.mark.parametrize("topo_name", ["Rear4GPU", "Heterogeneous_6GPU_Ring", "Heterogeneous_32GPU_4Server"])
def test_matches_reference(topo_name, tmp_path):
    ref = _ref("rlccl.models.traffic_predictor")
    if ref is None:
        pytest.skip("reference tree not installed under baseline/_ref")
    topo = load_topology_info(topo_name)
    mine = tp.deterministic_group_coefficients(topo)
    assert np.array_equal(mine, ref.deterministic_group_coefficients(topo))
    seqs = _seqs(n=topo.V, length=64)
    kw = dict(group_coefficients=mine, history_window=16, recent_steps=3, min_history=4)
    a, b = tp.build_history_examples(seqs, **kw), ref.build_history_examples(seqs, **kw)
    assert len(a) == len(b)
    for x, y in zip(a, b):
        assert x.keys() == y.keys()
        for k in x:
            assert np.array_equal(np.asarray(x[k]), np.asarray(y[k])), k
    pa = tp.TrafficPredictorSuite(topo.V, mine.shape[0]).fit(a).predict(a)
    sb = ref.TrafficPredictorSuite(topo.V, mine.shape[0]).fit(b)
    pb = sb.predict(b)
    for k in pa:
        assert np.allclose(pa[k]["continuous"], pb[k]["continuous"], rtol=1e-9, atol=1e-9)
        assert np.array_equal(pa[k]["hotspot"], pb[k]["hotspot"])
    path = str(tmp_path / "ref_suite.npz")
    sb.save(path)  # a reference artifact loads here
    pc = tp.TrafficPredictorSuite.load(path).predict(a)
    assert np.allclose(pc["moment_only"]["continuous"], pb["moment_only"]["continuous"])
