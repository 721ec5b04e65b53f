"""Paired Early-vs-Delayed statistics (bench/paired.py) against a direct
re-computation and the reference analyzer's gate logic."""

import json

import numpy as np
import pytest

from revealaiccl_b200.bench import paired


def test_bootstrap_median_matches_direct_recipe():
    rng = np.random.default_rng(5)
    x = rng.normal(0.3, 1.0, size=97)
    out = paired.bootstrap_median(x)
    g = np.random.default_rng(20260814)
    med = np.median(g.choice(x, size=(10_000, x.size), replace=True), axis=1)
    assert out["median"] == pytest.approx(float(np.median(x)))
    assert out["ci95_lower"] == pytest.approx(float(np.percentile(med, 2.5)))
    assert out["ci95_upper"] == pytest.approx(float(np.percentile(med, 97.5)))
    assert out["ci95_lower"] <= out["median"] <= out["ci95_upper"]


def test_distribution_and_grouped():
    d = paired.distribution([1.0, 2.0, 3.0, 4.0])
    assert d["count"] == 4 and d["p50"] == 2.5 and d["max"] == 4.0
    g = paired.grouped([-1.0, 2.0, 3.0])
    assert g["positive"] == 2 and g["non_positive"] == 1 and g["median_positive"]


def test_gate_positive_and_negative(tmp_path):
    rows = [{"seed": s, "family": f, "delta": 1.0 + 0.1 * j, "pass": True}
            for s in (0, 1, 2) for f in ("a", "b") for j in range(5)]
    res = paired.analyze_pairs(rows)
    assert res["gate"]["pass"] and res["primary_delta"]["ci95_lower"] > 0
    bad = [dict(r, delta=-r["delta"]) if r["seed"] == 1 else r for r in rows]
    res2 = paired.analyze_pairs(bad)
    assert not res2["gate"]["all_seed_medians_positive"] and not res2["gate"]["pass"]
    rows[0]["pass"] = False
    assert not paired.analyze_pairs(rows)["gate"]["correctness"]
    corpus = tmp_path / "c.json"
    corpus.write_text(json.dumps({"protocol": {"seeds": [0, 1, 2], "families": ["a", "b"]},
                                  "pairs": [dict(r, delta_ms=r["delta"]) for r in bad]}))
    paired.main([str(corpus), "--output-dir", str(tmp_path / "out")])
    assert (tmp_path / "out" / "paired_results.json").exists()
    assert (tmp_path / "out" / "paired_summary.csv").read_text().startswith("scope,name,n")
