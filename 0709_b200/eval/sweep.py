"""One-variable GSM8K sweeps over the serial ATLAS generator.

    python -m 0709_b200.eval.sweep fallback --drafter-model M --target-model T --data-file test.jsonl \
        --output-dir out --thresholds none -1.0 -0.75 -0.5 -0.25 --path-alpha 0.5
    python -m 0709_b200.eval.sweep path-weights --drafter-model M --target-model T --data-file test.jsonl \
        --output-dir out --alphas 0 0.25 0.5 0.75 1

``fallback`` changes only the weighted path-score fallback threshold (``none`` = fallback
off); the path weights stay the normalized exponential ``exp(-alpha * i)`` of ``--path-alpha``
and the first-token trigger is off.  ``path-weights`` changes only ``alpha``, with both
fallback triggers off.  Every other flag goes unchanged to ``eval.gsm8k`` for every run, so
the runs differ in exactly one variable.  Each run writes its own directory
(``threshold_<v>`` / ``alpha_<v>``); the sweep writes ``experiment.json`` (the changed
variable, the fixed settings, each run's arguments) and ``results.json`` / ``results.csv``
(accuracy, speed and fallback rate per run).  ``--dry-run`` writes only ``experiment.json``.

Parity: reference scripts/run_gsm8k_serial_fallback_sweep.py and
scripts/run_gsm8k_serial_path_weight_sweep.py (the same two experiments; here the runs are
in-process calls of the GSM8K driver rather than subprocesses).
"""

from __future__ import annotations

import argparse
import csv
import json
import math
import sys
from pathlib import Path

from . import gsm8k
from .common import exponential_path_weights, optional_float, read_jsonl


def value_tag(v: float | None) -> str:
    """Directory-safe name of a sweep value: ``none``, ``m0p5`` for -0.5, ``0p25`` for 0.25."""
    if v is None:
        return "none"
    text = format(float(v), "g")
    return text.replace("-", "m").replace(".", "p")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="One-variable serial GSM8K sweep; other flags go to eval.gsm8k.",
                                allow_abbrev=False)
    p.add_argument("experiment", choices=["fallback", "path-weights"])
    p.add_argument("--drafter-model", required=True)
    p.add_argument("--target-model", default=None, help="in-process target (or pass --target-url through)")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--backend", choices=["atlas_serial", "atlas"], default="atlas_serial")
    p.add_argument("--thresholds", nargs="+", type=optional_float, default=[None, -1.0, -0.75, -0.5, -0.25],
                   help="fallback: path-score thresholds ('none' = fallback off)")
    p.add_argument("--path-alpha", type=float, default=0.5, help="fallback: the fixed path-weight decay")
    p.add_argument("--alphas", nargs="+", type=float, default=[0.0, 0.25, 0.5, 0.75, 1.0],
                   help="path-weights: the decays to run")
    p.add_argument("--dry-run", action="store_true", help="write experiment.json and the run arguments only")
    return p


def _opt(v: float | None) -> str:
    return "none" if v is None else format(float(v), ".17g")


def plan(args, passthrough: list[str]) -> tuple[dict, list[tuple[float | None, Path, list[str]]]]:
    """The experiment record and, per run, (value, directory, gsm8k arguments)."""
    k_d = gsm8k.build_parser().parse_known_args(["--backend", "ar", "--model", "x", "--data-file", "x",
                                                 "--output-dir", "x", *passthrough])[0]
    root = Path(args.output_dir)
    base = ["--backend", args.backend, "--model", args.drafter_model, *passthrough]
    if args.target_model:
        base += ["--target-model", args.target_model]
    runs = []
    if args.experiment == "fallback":
        values = list(args.thresholds)
        if len(set(values)) != len(values):
            raise SystemExit("--thresholds contains duplicate values")
        for t in values:
            runs.append((t, root / f"threshold_{value_tag(t)}",
                         base + ["--path-weight-alpha", _opt(args.path_alpha), "--fallback-threshold", _opt(t),
                                 "--first-token-threshold", "none"]))
        record = {"experiment": "serial_gsm8k_fallback_threshold_sweep", "changed_variable": "fallback_threshold",
                  "first_token_threshold": None, "fixed_path_alpha": args.path_alpha,
                  "fixed_path_score_weights": list(exponential_path_weights(k_d.d, args.path_alpha)),
                  "fixed_fallback_ar_tokens": k_d.fallback_ar_tokens}
    else:
        values = [float(a) for a in args.alphas]
        if any(not math.isfinite(a) or a < 0.0 for a in values):
            raise SystemExit("every --alphas value must be finite and non-negative")
        if len(set(values)) != len(values):
            raise SystemExit("--alphas contains duplicate values")
        for a in values:
            runs.append((a, root / f"alpha_{value_tag(a)}",
                         base + ["--path-weight-alpha", _opt(a), "--fallback-threshold", "none",
                                 "--first-token-threshold", "none"]))
        record = {"experiment": "serial_gsm8k_path_weight_sweep", "changed_variable": "path_weight_alpha",
                  "fallback_threshold": None, "first_token_threshold": None,
                  "weights_by_alpha": {_opt(a): list(exponential_path_weights(k_d.d, a)) for a in values}}
    record["runs"] = [{"value": v, "output_dir": str(d), "gsm8k_args": [*a, "--output-dir", str(d)]}
                      for v, d, a in runs]
    return record, [(v, d, [*a, "--output-dir", str(d)]) for v, d, a in runs]


def result_row(variable: str, value, run_dir: Path) -> dict:
    """One run's row: the swept value, accuracy, speed and fallback figures (the serial generator's
    own drafter / target / overall rates where the run used it)."""
    summary = json.loads((run_dir / "summary.json").read_text())
    preds = read_jsonl(run_dir / "predictions.jsonl")
    rounds = sum(int(r.get("rounds", 0)) for r in preds)
    fallback = sum(int(r.get("fallback_rounds", 0)) for r in preds)
    speed = summary.get("serial_speed") or {}
    n = summary.get("count") or 0
    row = {variable: value}
    if variable == "fallback_threshold":
        row["fallback_enabled"] = value is not None
    row.update({"count": n, "correct": summary.get("correct"), "accuracy": summary.get("accuracy"),
                "generated_tokens": summary.get("generated_tokens"), "fallback_rounds": fallback, "rounds": rounds,
                "fallback_rate": fallback / rounds if rounds else None,
                "fallback_appended_tokens": speed.get("fallback_appended_tokens"),
                "end_to_end_tokens_per_second": summary.get("end_to_end_tokens_per_second"),
                "serial_overall_tokens_per_second": speed.get("overall_tokens_per_second"),
                "serial_drafter_tokens_per_second": speed.get("drafter_tokens_per_second"),
                "serial_target_tokens_per_second": speed.get("target_tokens_per_second"),
                "elapsed_s": summary.get("elapsed_s"),
                "mean_elapsed_s_per_example": summary["elapsed_s"] / n if n and summary.get("elapsed_s") else None})
    return row


def main(argv=None) -> int:
    args, passthrough = build_parser().parse_known_args(sys.argv[1:] if argv is None else argv)
    record, runs = plan(args, passthrough)
    root = Path(args.output_dir)
    root.mkdir(parents=True, exist_ok=True)
    (root / "experiment.json").write_text(json.dumps(record, indent=2) + "\n")
    if args.dry_run:
        for _, _, a in runs:
            print("python -m 0709_b200.eval.gsm8k " + " ".join(a))
        return 0
    variable = record["changed_variable"]
    rows = []
    for value, run_dir, a in runs:
        print(f"=== {variable}={_opt(value)} -> {run_dir}", flush=True)
        rc = gsm8k.main(a)
        if rc:
            return rc
        rows.append(result_row(variable, value, run_dir))
    (root / "results.json").write_text(json.dumps(rows, indent=2) + "\n")
    with (root / "results.csv").open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(rows[0]))
        w.writeheader()
        w.writerows(rows)
    print(json.dumps({"results": str(root / "results.csv"), "runs": len(rows)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
