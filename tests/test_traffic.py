"""Traffic process generator, moment validation, sliding estimator and context
views; differential against the reference generator when its tree is
installed under baseline/_ref."""

import importlib
from pathlib import Path
import sys

import numpy as np
import pytest

from revealaiccl_b200.traffic.moments import (SlidingMomentEstimator, mean_only_context, relative_l2_error,
                                             validate_sequence_moment_bounds, zero_moment_context)
from revealaiccl_b200.traffic.process import FAMILIES, TrafficProcessConfig, generate_traffic_sequence

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _cfg(family, seed=3, n=4):
    return TrafficProcessConfig(num_nodes=n, sequence_length=24, window_size=8, mean_level=3.0, std_level=1.5,
                                max_entry=8, epsilon_mean=0.35, epsilon_var=0.6, family=family, seed=seed)


@pytest.mark.parametrize("family", FAMILIES)
def test_generated_sequences_meet_their_bounds(family):
    seq = generate_traffic_sequence(_cfg(family))
    assert len(seq.matrices) == 24
    for m in seq.matrices:
        assert m.dtype == np.int64 and np.all(np.diag(m) == 0) and m.min() >= 0 and m.max() <= 8
    assert validate_sequence_moment_bounds(seq)["passed"]
    assert seq.metadata["validation"]["num_windows"] == 24 - 8 + 1


def _ref_module(name):
    if not (REF_ROOT / "rlccl").exists():
        return None
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    try:
        return importlib.import_module(name)
    except Exception:
        return None


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("seed", [0, 7])
def test_generator_matches_reference(family, seed):
    ref = _ref_module("rlccl.traffic.process_generator")
    if ref is None:
        pytest.skip("reference tree not installed under baseline/_ref")
    c = _cfg(family, seed)
    rc = ref.TrafficProcessConfig(**{k: getattr(c, k) for k in ("num_nodes", "sequence_length", "window_size",
                                                                "mean_level", "std_level", "max_entry",
                                                                "epsilon_mean", "epsilon_var", "family", "seed")})
    mine, theirs = generate_traffic_sequence(c), ref.generate_traffic_sequence(rc)
    assert len(mine.matrices) == len(theirs.matrices)
    for a, b in zip(mine.matrices, theirs.matrices):
        assert np.array_equal(a, b)


def test_estimator_is_history_only_and_round_trips():
    seq = generate_traffic_sequence(_cfg("smooth_ar"))
    est = SlidingMomentEstimator(4, window_size=5, min_history=3)
    cold = est.get_context(seq.matrices[0], seq.mean_ref, seq.var_ref)
    assert cold.history_length == 0 and not cold.is_warm and np.allclose(cold.mean_matrix, seq.mean_ref)
    for m in seq.matrices[:7]:
        est.update(m)
    ctx = est.get_context(seq.matrices[7], seq.mean_ref, seq.var_ref)
    hist = np.stack(seq.matrices[2:7]).astype(float)
    expect = hist.mean(0)
    np.fill_diagonal(expect, 0)
    assert ctx.history_length == 5 and ctx.is_warm and ctx.confidence == 1.0
    assert np.allclose(ctx.mean_matrix, expect)
    assert np.all(np.abs(ctx.current_send_z) <= est.z_clip)
    assert ctx.mean_drift == pytest.approx(relative_l2_error(expect, seq.mean_ref, est.eps))
    again = est.get_context(seq.matrices[7], seq.mean_ref, seq.var_ref)
    assert again.history_length == 5  # reading the context does not append
    est2 = SlidingMomentEstimator(4, window_size=5, min_history=3)
    est2.load_state_dict(est.state_dict())
    assert np.allclose(est2.get_context(seq.matrices[7], seq.mean_ref, seq.var_ref).var_matrix, ctx.var_matrix)
    m0, z0 = mean_only_context(ctx), zero_moment_context(ctx)
    assert np.allclose(m0.mean_matrix, ctx.mean_matrix) and not np.any(m0.var_matrix) and m0.var_drift == 0
    assert not np.any(z0.mean_matrix) and z0.confidence == 0 and not z0.is_warm


# --------------------------------------------------------------------------
# long-horizon processes (rlccl/traffic/long_horizon_generator.py)
# --------------------------------------------------------------------------
from revealaiccl_b200.traffic import long_horizon as lh  # noqa: E402


def _json(x):
    import json
    return json.loads(json.dumps(x, default=lambda o: o.tolist() if hasattr(o, "tolist") else str(o)))


@pytest.mark.parametrize("family", lh.LONG_HORIZON_FAMILIES)
def test_long_horizon_structure(family):
    cfg = lh.LongHorizonTrafficConfig(family=family, seed=5, sequence_length=600)
    seq = lh.generate_long_horizon_sequence(cfg)
    stack = np.stack(seq.matrices)
    assert stack.shape == (600, 4, 4) and stack.min() >= 0 and stack.max() <= cfg.max_entry
    assert not np.any(np.diagonal(stack, axis1=1, axis2=2))
    md = seq.metadata
    # each matrix carries rint(S_t) units unless every pair is at its cap
    want = np.clip(np.rint(md["total_traffic_pre_integer"]), 0, cfg.max_entry * 12).astype(int)
    assert np.array_equal(stack.sum(axis=(1, 2)), want)
    assert md["spatial_distribution_validation"]["diagonal_nonzero_count"] == 0
    assert md["spatial_distribution_validation"]["maximum_sum_error"] < 1e-12
    assert md["multi_scale_constraints"]["long"]["num_windows"] == 600 - 512 + 1
    assert md["constraint_status"] in ("passed", "best_effort")
    assert len(md["latent_regime"]) == len(md["spatial_mode"]) == 600
    again = lh.generate_long_horizon_sequence(cfg)
    assert all(np.array_equal(a, b) for a, b in zip(seq.matrices, again.matrices))
    if family == "rare_shock_recovery":
        assert md["shock_records"] and any(md["shock_flags"])


def test_long_horizon_allocator_respects_caps_and_ties():
    rng = np.random.default_rng(0)
    p = np.full((3, 3), 1 / 6)
    np.fill_diagonal(p, 0)
    m, raw, clipped = lh.allocate_integer(100.0, p, 4, rng)  # more units than 6 pairs x cap 4
    assert m.sum() == 24 and m.max() == 4 and np.all(np.diag(m) == 0)
    m2, _, _ = lh.allocate_integer(3.0, p, 4, np.random.default_rng(1))
    assert m2.sum() == 3 and m2.max() == 1
    assert np.allclose(raw, 100.0 * p) and clipped.max() == 4


def test_same_moment_group_shares_targets():
    g = lh.generate_same_moment_group(lh.LongHorizonTrafficConfig(family="same_moments_different_dynamics",
                                                                  sequence_length=300))
    assert set(g) == set(lh.SAME_MOMENT_VARIANTS)
    for v, seq in g.items():
        assert seq.sequence_id == f"same_moments_different_dynamics-{v}-seed42"
        assert seq.metadata["reference_total_mean"] == 2.0 * 12
    with pytest.raises(ValueError):
        lh.generate_same_moment_group(lh.LongHorizonTrafficConfig())


@pytest.mark.parametrize("family", lh.LONG_HORIZON_FAMILIES)
@pytest.mark.parametrize("extra", [{}, {"num_nodes": 5, "spatial_mode": "sparse_support"},
                                   {"num_nodes": 6, "spatial_mode": "cross_group_concentration"}])
def test_long_horizon_matches_reference(family, extra):
    ref = _ref_module("rlccl.traffic.long_horizon_generator")
    if ref is None:
        pytest.skip("reference tree not installed under baseline/_ref")
    kw = dict(family=family, seed=11, sequence_length=300, **extra)
    mine = lh.generate_long_horizon_sequence(lh.LongHorizonTrafficConfig(**kw))
    theirs = ref.generate_long_horizon_sequence(ref.LongHorizonTrafficConfig(**kw))
    assert mine.sequence_id == theirs.sequence_id
    assert len(mine.matrices) == len(theirs.matrices)
    for a, b in zip(mine.matrices, theirs.matrices):
        assert np.array_equal(a, b)
    assert _json(mine.metadata) == _json(theirs.metadata)
