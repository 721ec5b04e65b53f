"""Phase-3B ambiguity study: the preregistered design, the observation model,
calibration, validation selection, the family-stratified bootstrap, the
six-condition gate, and a toy end-to-end run whose summary is rebuilt from its
written raw tables; differential against the reference module when its tree is
installed under baseline/_ref."""

import importlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

from revealaiccl_b200.topology.loader import load_rear4_topology
from revealaiccl_b200.uncertainty import ambiguity_study as S
from revealaiccl_b200.uncertainty.observation import PublicTopologyView

REF_ROOT = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _ref_module():
    if not (REF_ROOT / "rlccl").exists():
        pytest.skip("reference tree not installed under baseline/_ref")
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    return importlib.import_module("rlccl.uncertainty.ambiguity_experiment")


def _topo():
    return PublicTopologyView.from_topology_info(load_rear4_topology()[0])


def test_design_has_75_sequences_in_five_splits():
    specs = S.build_sequence_specs()
    assert len(specs) == 75 and len({s.sequence_id for s in specs}) == 75
    counts = {sp: sum(s.split == sp for s in specs) for sp in ("fit", "validation", "calibration", "test")}
    assert counts == {"fit": 30, "validation": 15, "calibration": 15, "test": 15}
    s = specs[7]
    assert s.seed == s.base_seed + S.FAMILIES.index(s.family) * 1_000_000 + s.sequence_index * 10_000
    ids = S.case_identities(specs, S.StudyScale.named("formal"))
    assert len(ids) == 72_000  # 45 evaluated sequences x 16 checkpoints x 5 modes x 5 ratios x 4 K


@pytest.mark.parametrize("mode", S.REVEAL_MODES)
def test_observation_model(mode):
    topo = _topo()
    rng = np.random.default_rng(3)
    m = rng.integers(0, 6, size=(4, 4))
    np.fill_diagonal(m, 0)
    obs0, f0 = S.observe(m, mode=mode, ratio=0.0, seed=11, topology=topo)
    obs1, f1 = S.observe(m, mode=mode, ratio=1.0, seed=11, topology=topo)
    assert f0 == 0.0 and f1 == 1.0 and bool(obs1.entry_mask.all())
    assert np.array_equal(np.asarray(obs1.observed_matrix), m)
    half, fh = S.observe(m, mode=mode, ratio=0.5, seed=11, topology=topo)
    again, _ = S.observe(m, mode=mode, ratio=0.5, seed=11, topology=topo)
    assert np.array_equal(np.asarray(half.entry_mask), np.asarray(again.entry_mask))  # seeded
    known = np.asarray(half.entry_mask)
    assert np.array_equal(np.asarray(half.observed_matrix)[known], m[known])
    assert (half.source_totals is not None) == (mode in ("source_totals_first", "source_destination_totals_first"))
    assert (half.destination_totals is not None) == (mode == "source_destination_totals_first")


def test_exceedance_and_calibration_radius():
    lo, hi, sc = np.zeros(3), np.ones(3), np.full(3, 0.5)
    assert S.exceedance_score(lo, hi, [0.5, 0.2, 1.0], sc) == 0.0
    assert S.exceedance_score(lo, hi, [1.5, 0.2, -0.25], sc) == pytest.approx(1.0)
    rows = [{"sequence_id": f"s{i}", "family": "a" if i < 5 else "b", "score": float(j + i)}
            for i in range(10) for j in range(10)]
    per = [float(np.quantile(np.arange(10) + i, 0.9, method="higher")) for i in range(10)]
    assert S.calibration_radius(rows) == float(np.quantile(per, 0.9, method="higher"))
    assert S.calibration_radius(rows, exclude_family="b") == float(np.quantile(per[:5], 0.9, method="higher"))


def test_validation_selection_and_ties():
    rows = [{"sequence_id": f"s{i}", "method": m, "requested_k": 8, "reveal_ratio": 0.5,
             "nearest_rms_distance": {"random_empirical": 1.0, "worst_recent_cases": 0.5, "boundary_scenarios": 0.5,
                                      "minimax_subset": 0.7}[m]} for i in range(3) for m in S.ORDINARY_METHODS]
    method, means = S.select_method(rows)
    assert method == "boundary_scenarios" and means["worst_recent_cases"] == 0.5  # tie -> tie order
    with pytest.raises(ValueError):
        S.select_method(rows + [dict(rows[0], method="oracle_support_upper_bound")])


def test_bootstrap_and_gate():
    deltas = [{"sequence_id": f"s{f}{i}", "family": f"f{f}", "base_seed": 342 + 100 * i, "paired_delta": 0.1 + 0.01 * f}
              for f in range(5) for i in range(3)]
    b = S.family_bootstrap(deltas, replicates=500)
    assert b["ci_lower"] <= b["mean_delta"] <= b["ci_upper"] and b["sequence_count"] == 15
    assert S.family_bootstrap(deltas, replicates=500) == b  # seeded
    fams = {f"f{f}": 0.9 for f in range(5)}
    ev = {"selected_joint_coverage": 0.9, "selected_joint_coverage_by_family": fams,
          "paired_delta_ci95": [0.01, 0.2], "paired_delta_by_base_seed": {"342": 0.1, "442": 0.1, "542": 0.1},
          "paired_delta_by_family": fams, "lofo_aggregate_delta": 0.1, "lofo_delta_by_family": fams,
          "lofo_relative_degradation_by_family": {k: 0.0 for k in fams}, "total_tail_events": 20,
          "total_tail_hits": 18, "group_tail_events": 20, "group_tail_hits": 15, "hotspot_events": 20,
          "hotspot_hits": 16, "selected_mean_physical_normalized_width": 0.5,
          "ordinary_invalid_or_empty_rate": {m: 0.0 for m in S.ORDINARY_METHODS}, "ratio1_singleton_coverage": 1.0,
          "all_timings_finite": True, "integrity_checks_complete": True, "integrity_checks_passed": True}
    assert S.evaluate_gate(ev).data_status == "PASS"
    assert S.evaluate_gate(dict(ev, total_tail_events=5)).data_status == "HOLD"
    assert S.evaluate_gate(dict(ev, paired_delta_ci95=[-0.01, 0.2])).failed_conditions == (2,)


def test_toy_run_writes_artifacts_that_rebuild_the_summary(tmp_path):
    summary = S.run_study("toy", out_dir=tmp_path)
    assert summary["data_status"] in ("PASS", "FAIL", "HOLD") and summary["test_cases"] > 0
    manifest = json.loads((tmp_path / "manifest.json").read_text())
    assert set(manifest["artifacts"]) >= {"raw_calibration.csv", "raw_test.csv", "summary.json"}
    rebuilt = S.recompute_summary(S.read_raw_tables(tmp_path), bootstrap_replicates=200)
    for key in ("calibration_radius", "selected_method", "data_status", "failed_conditions", "bootstrap"):
        assert rebuilt[key] == summary[key], key


@pytest.mark.parametrize("mode", S.REVEAL_MODES)
@pytest.mark.parametrize("ratio", [0.0, 0.25, 0.75, 1.0])
def test_observation_matches_reference(mode, ratio):
    R = _ref_module()
    topo = _topo()
    spec_ref = R.build_formal_sequence_specs()[4]
    rng = np.random.default_rng(17)
    m = rng.integers(0, 6, size=(4, 4))
    np.fill_diagonal(m, 0)
    seed = S.observation_seed(4, 96, S.REVEAL_MODES.index(mode))
    assert seed == R.reveal_seed(4, 96, S.REVEAL_MODES.index(mode))
    ref, rf = R._formal_observation(m, spec=spec_ref, checkpoint=96, topology=topo, mode=mode, ratio=ratio,
                                    seed=seed)
    mine, mf = S.observe(m, mode=mode, ratio=ratio, seed=seed, topology=topo)
    assert rf == mf
    assert np.array_equal(np.asarray(ref.entry_mask), np.asarray(mine.entry_mask))
    assert np.array_equal(np.asarray(ref.observed_matrix), np.asarray(mine.observed_matrix))


def test_statistics_match_reference():
    R = _ref_module()
    assert [s.sequence_id for s in R.build_formal_sequence_specs()] == [s.sequence_id for s in S.build_sequence_specs()]
    lo, hi, sc = np.zeros(5), np.ones(5), np.full(5, 0.3)
    v = np.array([1.4, -0.2, 0.5, 0.9, 1.01])
    assert S.exceedance_score(lo, hi, v, sc) == R.calibration_exceedance_score(lo, hi, v, sc)
    deltas = [{"sequence_id": f"s{f}{i}", "family": f"f{f}", "base_seed": 342 + 100 * i,
               "paired_delta": float(np.sin(7 * f + i))} for f in range(5) for i in range(3)]
    a = S.family_bootstrap(deltas, replicates=2000)
    b = R.family_stratified_sequence_bootstrap(deltas, replicates=2000)
    assert (a["mean_delta"], a["ci_lower"], a["ci_upper"]) == (b.mean_delta, b.ci_lower, b.ci_upper)
