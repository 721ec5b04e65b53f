"""Recourse study (robust-prefix planning with repair on reveal): every
method runs legal episodes whose event ledger validates and rebuilds them,
the lower bound is a lower bound, and a tampered ledger is refused."""

import numpy as np
import pytest

from revealaiccl_b200.scheduling import recourse_study as R


@pytest.fixture(scope="module")
def specs():
    return R.toy_specs(families=("regime_switching_long",), base_seeds=(642,), checkpoints=(40,),
                       reveal_modes=("partial_shards", "source_totals_first"))


def test_every_method_runs_a_consistent_episode(specs):
    for spec in specs:
        results = {m: R.run_episode(spec, m) for m in R.METHODS}
        lb = results["full_information_lower_bound"].completion_slots
        for m, r in results.items():
            assert r.legality, m
            R.validate_event_ledger(r.events)
            again = R.recompute_episode(r.events)
            assert (again["completion_slots"], again["executed_actions"]) == (r.completion_slots, r.executed_actions)
            if ROLE_EXEC(m):
                assert r.completion_slots >= lb, (m, r.completion_slots, lb)
        # waiting for the last stage cannot act before it
        assert results["wait_until_known"].first_action_slot >= 4 * (len(spec.ratios) - 1)


def ROLE_EXEC(m):
    return R.ROLES[m][2]


def test_study_summary_and_tampered_ledger(specs, tmp_path):
    res = R.run_study(specs)
    s = res["summary"]
    assert s["episodes"] == len(specs) and s["all_legal"]
    assert set(s["completion_mean"]) == set(R.METHODS)
    R.write_study(res, tmp_path)
    assert (tmp_path / "episodes.csv").exists() and (tmp_path / "summary.json").exists()
    r = R.run_episode(specs[0], "scenario_robust_prefix")
    bad = [dict(e) for e in r.events]
    for e in bad:
        if e["kind"] == "batch_committed":
            e["state_version_after"] += 1
            break
    with pytest.raises(R.LedgerError):
        R.validate_event_ledger(bad)
    with pytest.raises(R.LedgerError):
        R.validate_event_ledger(bad[1:])
