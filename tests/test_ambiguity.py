"""Empirical ambiguity sets: reconciliation honours every observation
constraint (exact entries, partial-shard lower bounds, source / destination
totals), moment bands admit the uniform witness, selectors are deterministic,
the singleton control at ratio 1; differential against the reference module
when its tree is installed under baseline/_ref."""

import importlib
from pathlib import Path
import sys

import numpy as np
import pytest

from revealaiccl_b200.topology.loader import load_topology_info
from revealaiccl_b200.uncertainty import ambiguity as A

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _case(seed, mode, ratio=0.5):
    topo = load_topology_info("Rear4GPU")
    rng = np.random.default_rng(seed)
    n = topo.V

    def mat():
        m = rng.integers(0, 5, size=(n, n))
        np.fill_diagonal(m, 0)
        return m

    hist = [mat() for _ in range(32)]
    truth = mat()
    mask = rng.random((n, n)) < 0.4
    np.fill_diagonal(mask, True)
    obs = np.where(mask, truth, 0)
    if mode == "partial_shards":
        part = np.minimum(truth, rng.integers(0, 3, size=(n, n)))
        np.fill_diagonal(part, 0)
        obs = np.where(mask, truth, part)
    if ratio == 1.0:
        mask, obs = np.ones((n, n), bool), truth
    src = truth.sum(1) if "source" in mode else None
    dst = truth.sum(0) if "destination" in mode else None
    kw = dict(history_matrices=tuple(hist), history_offsets=tuple(range(-32, 0)), observed_matrix=obs, entry_mask=mask,
              mode=mode, stage=1, ratio=ratio, source_totals=src, destination_totals=dst, topology=topo,
              construction_seed=5, history_cutoff=40)
    return topo, hist, truth, kw


@pytest.mark.parametrize("mode", ["random_entries", "source_totals_first", "source_destination_totals_first",
                                  "partial_shards"])
def test_reconciliation_respects_observation(mode):
    topo, hist, truth, kw = _case(1, mode)
    view = A.AmbiguityConstructionView(normalizer=A.fit_descriptor_normalizer(hist, topo), **kw)
    amb = A.build_empirical_ambiguity_set(view, calibration_radius=0.3)
    mask, obs = kw["entry_mask"], kw["observed_matrix"]
    for m in amb.support_matrices:
        assert np.array_equal(m[mask], obs[mask]) and m.max() <= A.MAX_ENTRY and not np.diag(m).any()
        if mode == "partial_shards":
            assert np.all(m >= obs)
        if kw["source_totals"] is not None:
            assert np.array_equal(m.sum(1), kw["source_totals"])
        if kw["destination_totals"] is not None:
            assert np.array_equal(m.sum(0), kw["destination_totals"])
    assert amb.validate_probability_weights(amb.uniform_witness)
    assert np.all(amb.lower_bounds <= amb.descriptor_vectors.min(0) + 1e-12)
    with pytest.raises(ValueError):
        amb.validate_probability_weights(np.eye(len(amb.support_matrices))[0] * 2)


def test_selectors_and_singleton():
    topo, hist, truth, kw = _case(2, "source_totals_first")
    view = A.AmbiguityConstructionView(normalizer=A.fit_descriptor_normalizer(hist, topo), **kw)
    amb = A.build_empirical_ambiguity_set(view, calibration_radius=0.2)
    for method in ("worst_recent_cases", "boundary_scenarios", "minimax_subset"):
        s1 = A.select_support(amb, method=method, k=5)
        s2 = A.select_support(amb, method=method, k=5)
        assert s1.selected_indices == s2.selected_indices and len(set(s1.selected_indices)) == 5
    full = A.select_support(amb, method="minimax_subset", k=32)
    assert A.support_covering_radius(amb, full) == 0.0
    assert A.support_covering_radius(amb, A.select_support(amb, method="minimax_subset", k=2)) > 0.0
    with pytest.raises(ValueError):
        A.select_support(amb, method="random_empirical", k=2)
    orc = A.oracle_support_upper_bound(amb, truth=truth, k=3)
    assert orc.uses_oracle and orc.selected_indices[0] == -1
    assert A.truth_nearest_descriptor_distance(amb, orc, truth) == 0.0
    _, _, truth1, kw1 = _case(3, "random_entries", ratio=1.0)
    single = A.build_empirical_ambiguity_set(
        A.AmbiguityConstructionView(normalizer=A.fit_descriptor_normalizer(hist, topo), **kw1), calibration_radius=0.3)
    assert single.singleton_control and len(single.support_matrices) == 1
    assert np.array_equal(single.support_matrices[0], truth1)


def test_view_rejects_bad_inputs():
    topo, hist, _, kw = _case(4, "random_entries")
    nz = A.fit_descriptor_normalizer(hist, topo)
    with pytest.raises(ValueError):
        A.AmbiguityConstructionView(normalizer=nz, **dict(kw, history_offsets=tuple(range(-31, 1))))
    with pytest.raises(ValueError):
        A.AmbiguityConstructionView(normalizer=nz, **dict(kw, history_cutoff=10))
    bad = kw["observed_matrix"].copy()
    bad[0, 1] = 9
    with pytest.raises(ValueError):
        A.AmbiguityConstructionView(normalizer=nz, **dict(kw, observed_matrix=bad))


@pytest.mark.parametrize("mode", ["random_entries", "source_totals_first", "source_destination_totals_first",
                                  "partial_shards"])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_matches_reference(mode, seed):
    if not (REF_ROOT / "rlccl").exists():
        pytest.skip("reference tree not installed under baseline/_ref")
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    R = importlib.import_module("rlccl.uncertainty.ambiguity")
    topo, hist, truth, kw = _case(10 + seed, mode)
    out = {}
    for name, M in (("ref", R), ("mine", A)):
        view = M.AmbiguityConstructionView(normalizer=M.fit_descriptor_normalizer(hist, topo), **kw)
        amb = M.build_empirical_ambiguity_set(view, calibration_radius=0.3)
        sel = [M.select_support(amb, method=m, k=k, replicate_seed=7).selected_indices
               for m in ("random_empirical", "worst_recent_cases", "boundary_scenarios", "minimax_subset")
               for k in (1, 6)]
        out[name] = (amb, sel, amb.observation_constraint_fingerprint,
                     M.oracle_support_upper_bound(amb, truth=truth, k=4).selected_indices)
    a, b = out["ref"], out["mine"]
    assert all(np.array_equal(x, y) for x, y in zip(a[0].support_matrices, b[0].support_matrices))
    assert np.allclose(a[0].upper_bounds, b[0].upper_bounds) and np.allclose(a[0].variance_high, b[0].variance_high)
    assert a[1:] == b[1:]
