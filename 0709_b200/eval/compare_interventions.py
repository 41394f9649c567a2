"""Pair a ``target_best`` GSM8K run with a ``first_route`` run and attribute the difference.

    python -m 0709_b200.eval.compare_interventions --target-best out/best --first-route out/first --json-out cmp.json

Both inputs are ``eval.gsm8k`` output directories (or their ``predictions.jsonl``).  The two
runs must cover the same samples with the same prompts (question, gold answer, model, backend,
prompt length and prompt-token hash) and, where recorded, the same request seeds and the
policies their names say; otherwise the comparison stops with the first difference.  The
report holds each run's aggregated target-intervention statistics and the paired outcome:
samples the target's choice helped (target_best right, first_route wrong) or hurt, the net
gain and an exact McNemar p-value (``utils.interventions.paired_target_quality``).

Parity: reference tools/compare_gsm8k_target_intervention.py (pairing, alignment guards,
report); the statistics are this package's ``utils.interventions``.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Any, Mapping, Sequence

from ..utils.interventions import aggregate_prediction_interventions, paired_target_quality
from .common import read_jsonl

ALIGN_KEYS = ("question", "gold", "model", "backend", "prompt_tokens")


def load_run(path: Path) -> tuple[list[dict], dict, Path]:
    """(prediction rows, summary or {}, predictions path) of a run directory or file."""
    pred = path / "predictions.jsonl" if path.is_dir() else path
    if not pred.exists():
        raise SystemExit(f"{pred}: no predictions")
    summ = pred.parent / "summary.json"
    return read_jsonl(pred), (json.loads(summ.read_text()) if summ.exists() else {}), pred


def run_policy(summary: Mapping[str, Any]) -> str | None:
    return (summary.get("settings") or {}).get("route_selection_policy")


def validate_alignment(best: Sequence[Mapping[str, Any]], first: Sequence[Mapping[str, Any]]) -> dict:
    """Checks that the two runs are the same samples; returns what could be checked."""
    bi, fi = [int(r["index"]) for r in best], [int(r["index"]) for r in first]
    if len(set(bi)) != len(bi) or len(set(fi)) != len(fi):
        raise ValueError("a predictions file holds an index twice")
    if set(bi) != set(fi):
        raise ValueError("the two runs cover different samples")
    b_by, f_by = {int(r["index"]): r for r in best}, {int(r["index"]): r for r in first}
    checked = {"prompt_hash": 0, "generation_seed": 0}
    for i in sorted(b_by):
        b, f = b_by[i], f_by[i]
        for key in ALIGN_KEYS:
            if b.get(key) != f.get(key):
                raise ValueError(f"sample {i} differs in {key}: {b.get(key)!r} vs {f.get(key)!r}")
        for key, name in (("prompt_token_ids_sha256", "prompt_hash"), ("generation_seed", "generation_seed")):
            if key in b and key in f:
                if b[key] != f[key]:
                    raise ValueError(f"sample {i} differs in {key}")
                checked[name] += 1
    return {"samples": len(bi), "fields_checked": list(ALIGN_KEYS), "prompt_hash_checked": checked["prompt_hash"],
            "generation_seed_checked": checked["generation_seed"]}


def compare(best_path: Path, first_path: Path) -> dict:
    best, best_summary, bp = load_run(best_path)
    first, first_summary, fp = load_run(first_path)
    pb, pf = run_policy(best_summary), run_policy(first_summary)
    if pb is not None and pb != "target_best":
        raise ValueError(f"--target-best run reports policy {pb!r}")
    if pf is not None and pf != "first_route":
        raise ValueError(f"--first-route run reports policy {pf!r}")
    return {
        "comparison": "paired_target_best_vs_first_route",
        "target_best_predictions": str(bp), "first_route_predictions": str(fp),
        "policies": {"target_best": pb, "first_route": pf, "policy_metadata_missing": pb is None or pf is None},
        "alignment": validate_alignment(best, first),
        "target_best_intervention": aggregate_prediction_interventions(best),
        "first_route_intervention": aggregate_prediction_interventions(first),
        "paired_quality": paired_target_quality(best, first),
        "interpretation": {"helped": "target_best correct and first_route wrong",
                           "hurt": "target_best wrong and first_route correct",
                           "net_correct_gain": "helped - hurt",
                           "causal_unit": "the paired final answer; rounds after the first differing token do "
                                          "not line up"},
    }


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="Paired target_best vs first_route GSM8K comparison.")
    p.add_argument("--target-best", type=Path, required=True, help="target_best run directory or predictions.jsonl")
    p.add_argument("--first-route", type=Path, required=True, help="first_route run directory or predictions.jsonl")
    p.add_argument("--json-out", type=Path, default=None)
    args = p.parse_args(sys.argv[1:] if argv is None else argv)
    text = json.dumps(compare(args.target_best, args.first_route), indent=2, sort_keys=True) + "\n"
    print(text, end="")
    if args.json_out:
        args.json_out.write_text(text)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
