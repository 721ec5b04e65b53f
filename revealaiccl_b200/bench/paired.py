"""Paired Early-vs-Delayed statistics: distributions, bootstrap median CI and the
progressive-gain gate.

Same estimator and gate as the reference's formal analyzers
(scripts/analyze_r4_f0_full_moe.py:24-92, scripts/run_r2_f0_integrated.py:99-109):

* ``distribution`` — count / mean / p50 / p95 / p99 / max;
* ``bootstrap_median`` — percentile bootstrap of the median of the paired
  deltas, 10,000 resamples with replacement from a seeded NumPy generator
  (seed 20260814), 2.5 / 97.5 percentiles;
* ``gate`` — the progressive gain passes when the paired median and the CI
  lower bound are positive, every seed's median is positive and every
  correctness flag holds.

``Delta = T_delayed - T_early`` (positive: the progressive early arm is faster).

    python -m revealaiccl_b200.bench.paired corpus.json --output-dir out/
"""

from __future__ import annotations

import argparse
import csv
import hashlib
import json
from pathlib import Path
from typing import Any, Iterable, Mapping, Sequence

import numpy as np

BOOTSTRAP_SEED = 20260814
BOOTSTRAP_REPLICATES = 10_000


def distribution(values: Iterable[float]) -> dict[str, Any]:
    data = np.asarray(list(values), dtype=np.float64)
    if data.size == 0:
        return {"count": 0, "mean": None, "p50": None, "p95": None, "p99": None, "max": None}
    return {"count": int(data.size), "mean": float(data.mean()), "p50": float(np.percentile(data, 50)),
            "p95": float(np.percentile(data, 95)), "p99": float(np.percentile(data, 99)),
            "max": float(data.max())}


def bootstrap_median(values: Sequence[float], *, replicates: int = BOOTSTRAP_REPLICATES,
                     seed: int = BOOTSTRAP_SEED) -> dict[str, Any]:
    data = np.asarray(values, dtype=np.float64)
    if data.size == 0:
        raise ValueError("bootstrap of an empty sample")
    rng = np.random.default_rng(seed)
    samples = rng.choice(data, size=(replicates, data.size), replace=True)
    medians = np.median(samples, axis=1)
    return {"n": int(data.size), "median": float(np.median(data)),
            "ci95_lower": float(np.percentile(medians, 2.5)),
            "ci95_upper": float(np.percentile(medians, 97.5)),
            "replicates": int(replicates), "seed": int(seed)}


def grouped(values: Sequence[float]) -> dict[str, Any]:
    out = distribution(values)
    vals = list(values)
    out["positive"] = sum(v > 0 for v in vals)
    out["non_positive"] = sum(v <= 0 for v in vals)
    out["positive_fraction"] = out["positive"] / len(vals) if vals else 0.0
    out["median_positive"] = bool(vals) and float(np.median(vals)) > 0
    return out


def analyze_pairs(rows: Sequence[Mapping[str, Any]], *, key: str = "delta",
                  seeds: Sequence[Any] | None = None, families: Sequence[str] | None = None,
                  correctness: Mapping[str, bool] | None = None) -> dict[str, Any]:
    """rows: one record per pair with ``key`` (Delta), ``seed``, ``family`` and ``pass``."""
    deltas = [float(r[key]) for r in rows]
    seeds = list(seeds) if seeds is not None else sorted({r.get("seed") for r in rows}, key=str)
    families = list(families) if families is not None else sorted({str(r.get("family")) for r in rows})
    per_seed = {str(s): grouped([float(r[key]) for r in rows if r.get("seed") == s]) for s in seeds}
    per_family = {f: grouped([float(r[key]) for r in rows if str(r.get("family")) == f]) for f in families}
    primary = bootstrap_median(deltas)
    corr = dict(correctness or {})
    corr.setdefault("paired_equivalence_100pct", all(bool(r.get("pass", True)) for r in rows))
    gate = {
        "paired_median_positive": primary["median"] > 0,
        "bootstrap_ci95_lower_positive": primary["ci95_lower"] > 0,
        "all_seed_medians_positive": bool(per_seed) and all(v["median_positive"] for v in per_seed.values()
                                                           if v["count"]),
        "correctness": all(corr.values()),
    }
    gate["pass"] = all(gate.values())
    return {"primary_delta": primary, "corpus_delta_distribution": grouped(deltas), "per_seed_delta": per_seed,
            "per_family_delta": per_family, "correctness": corr, "gate": gate}


def write_report(result: Mapping[str, Any], output_dir: Path, stem: str = "paired") -> Path:
    output_dir.mkdir(parents=True, exist_ok=True)
    out = output_dir / f"{stem}_results.json"
    out.write_text(json.dumps(result, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    with open(output_dir / f"{stem}_summary.csv", "w", newline="", encoding="utf-8") as f:
        w = csv.writer(f)
        w.writerow(["scope", "name", "n", "positive", "non_positive", "p50", "p95", "p99", "max"])
        for scope, key in (("seed", "per_seed_delta"), ("family", "per_family_delta")):
            for name, v in result[key].items():
                w.writerow([scope, name, v["count"], v["positive"], v["non_positive"], v["p50"], v["p95"], v["p99"],
                            v["max"]])
    return out


def sha256_file(path: Path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="revealaiccl_b200.bench.paired")
    ap.add_argument("input", type=Path, help="corpus JSON with a 'pairs' list")
    ap.add_argument("--output-dir", type=Path, required=True)
    ap.add_argument("--key", default="delta_ms")
    args = ap.parse_args(argv)
    corpus = json.loads(args.input.read_text(encoding="utf-8"))
    proto = corpus.get("protocol", {})
    result = analyze_pairs(corpus["pairs"], key=args.key, seeds=proto.get("seeds"), families=proto.get("families"),
                           correctness=corpus.get("correctness"))
    result["source"] = {"path": str(args.input), "sha256": sha256_file(args.input)}
    out = write_report(result, args.output_dir)
    print(json.dumps({"output": str(out), "sha256": sha256_file(out), "gate": result["gate"],
                      "primary": result["primary_delta"]}))


if __name__ == "__main__":
    main()
