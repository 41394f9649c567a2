"""Target-intervention statistics over generation traces (quality evaluation).

For every ``select`` round the selected route is compared with two baselines:
the first route of the verify payload (what a Target with no selection power
would commit) and the Drafter's top route by current-prefix path
log-probability (draft rank 1).  Fallback rounds count as Target actions.
Per-generation summaries aggregate over rounds; per-dataset aggregates sum the
per-generation counters; ``paired_target_quality`` compares paired outcomes of
a ``target_best`` and a ``first_route`` run with an exact McNemar test.

The output field names follow the reference's evaluator
(src/atlas_0709/eval_interventions.py:217-510) so its JSON consumers work on
these results; the computation is this module's own.
"""

from __future__ import annotations

import math
from collections import Counter
from typing import Any, Mapping, Sequence

INTERVENTION_SCHEMA_VERSION = 1
TARGET_ACTION = "selected_away_from_first_route_or_fallback"
ROUTE_INTERVENTION = "selected_away_from_current_prefix_draft_top"


def _get(obj: object, key: str, default: Any = None) -> Any:
    return obj.get(key, default) if isinstance(obj, Mapping) else getattr(obj, key, default)


def _num(x: object) -> float | None:
    try:
        v = float(x)  # type: ignore[arg-type]
    except (TypeError, ValueError):
        return None
    return v if math.isfinite(v) else None


def _tokens(score: Mapping[str, Any]) -> list[int]:
    t = score.get("token_ids")
    return [int(v) for v in t] if isinstance(t, (list, tuple)) else []


def draft_path_score(score: Mapping[str, Any]) -> tuple[float | None, str | None]:
    """Drafter path log-prob conditioned on this round's prefix, and where it came from.

    Preference: the explicit ``draft_path_logprob``; else the sum of
    ``draft_token_logprobs``; else the legacy cumulative ``draft_logprob``
    (whose baseline may predate the prefix after forest reuse).
    """
    v = _num(score.get("draft_path_logprob"))
    if v is not None:
        return v, "draft_path_logprob"
    toks = score.get("draft_token_logprobs")
    if isinstance(toks, (list, tuple)) and toks:
        vals = [_num(x) for x in toks]
        if all(x is not None for x in vals):
            return math.fsum(vals), "sum(draft_token_logprobs)"  # type: ignore[arg-type]
    v = _num(score.get("draft_logprob"))
    return (v, "legacy_draft_logprob") if v is not None else (None, None)


def draft_first_token_score(score: Mapping[str, Any]) -> float | None:
    """The Drafter's first-token log-prob (``first_token_logprob`` is the Target's and is not used)."""
    toks = score.get("draft_token_logprobs")
    if isinstance(toks, (list, tuple)) and toks:
        return _num(toks[0])
    return _num(score.get("draft_first_token_logprob"))


def _lower(a: float | None, b: float | None) -> bool | None:
    return None if a is None or b is None else a < b


def _delta(a: float | None, b: float | None) -> float | None:
    return None if a is None or b is None else a - b


def round_intervention(trace: object) -> dict[str, Any]:
    decision = str(_get(trace, "decision", "select"))
    out: dict[str, Any] = {"round_index": int(_get(trace, "round_index", -1)), "decision": decision,
                           "fallback": decision == "fallback_ar", "route_comparison_available": False}
    sel_id = _get(trace, "selected_route_id")
    scores = [dict(s) for s in (_get(trace, "target_scores", []) or []) if isinstance(s, Mapping)]
    if decision != "select" or sel_id is None or not scores:
        return out
    by_id = {int(s["route_id"]): s for s in scores}
    sel = by_id.get(int(sel_id))
    if sel is None:
        return out
    # Draft ranking: path log-prob descending, payload order breaks ties; missing scores rank last.
    order = sorted(range(len(scores)),
                   key=lambda i: (-(draft_path_score(scores[i])[0] if draft_path_score(scores[i])[0] is not None
                                    else -math.inf), i))
    ranked = [scores[i] for i in order]
    top, first = ranked[0], scores[0]
    rank = 1 + next(i for i, s in enumerate(ranked) if int(s["route_id"]) == int(sel_id))
    st, tt, ft = _tokens(sel), _tokens(top), _tokens(first)
    s_path, s_src = draft_path_score(sel)
    t_path, t_src = draft_path_score(top)
    s_d1, t_d1 = draft_first_token_score(sel), draft_first_token_score(top)
    s_t1, t_t1 = _num(sel.get("first_token_logprob")), _num(top.get("first_token_logprob"))
    s_tt, t_tt = _num(sel.get("target_logprob")), _num(top.get("target_logprob"))
    out.update({
        "route_comparison_available": True,
        "selected_route_id": int(sel_id),
        "draft_top_route_id": int(top["route_id"]),
        "first_route_id": int(first["route_id"]),
        "selected_differs_from_draft_top": int(sel_id) != int(top["route_id"]),
        "selected_differs_from_first_route": int(sel_id) != int(first["route_id"]),
        "draft_rank": rank,
        "selected_first_token_id": st[0] if st else None,
        "draft_top_first_token_id": tt[0] if tt else None,
        "first_token_changed": bool(st and tt and st[0] != tt[0]),
        "first_route_first_token_changed": bool(st and ft and st[0] != ft[0]),
        "selected_draft_path_logprob": s_path,
        "draft_top_path_logprob": t_path,
        "selected_draft_path_logprob_source": s_src,
        "draft_top_path_logprob_source": t_src,
        "current_prefix_draft_path_comparison": (s_src not in (None, "legacy_draft_logprob")
                                                 and t_src not in (None, "legacy_draft_logprob")),
        "draft_path_logprob_delta": _delta(s_path, t_path),
        "lower_total_draft_probability": _lower(s_path, t_path),
        "draft_first_token_comparison_available": _lower(s_d1, t_d1) is not None,
        "selected_draft_first_token_logprob": s_d1,
        "draft_top_first_token_logprob": t_d1,
        "draft_first_token_logprob_delta": _delta(s_d1, t_d1),
        "lower_first_token_draft_probability": _lower(s_d1, t_d1),
        "lower_first_token_target_probability": _lower(s_t1, t_t1),
        "target_first_token_logprob_delta": _delta(s_t1, t_t1),
        "lower_total_target_probability": _lower(s_tt, t_tt),
        "target_total_logprob_delta": _delta(s_tt, t_tt),
    })
    return out


def _rate(num: int, den: int) -> float | None:
    return num / den if den else None


def summarize_generation_interventions(rounds: Sequence[object]) -> dict[str, Any]:
    """Per-generation summary of Target actions and route interventions."""
    det = [round_intervention(r) for r in rounds]
    comp = [d for d in det if d["route_comparison_available"]]
    fb = sum(d["fallback"] for d in det)
    n_first = sum(d["selected_differs_from_first_route"] for d in comp)
    n_top = sum(d["selected_differs_from_draft_top"] for d in comp)
    n_tok = sum(d["first_token_changed"] for d in comp)
    n_ftok = sum(d["first_route_first_token_changed"] for d in comp)
    n_low = sum(d["lower_total_draft_probability"] is True for d in comp)
    d1 = [d for d in comp if d["draft_first_token_comparison_available"]]
    n_low1 = sum(d["lower_first_token_draft_probability"] is True for d in d1)
    hist = Counter(str(d["draft_rank"]) for d in comp)
    moved = [d["draft_rank"] for d in comp if d["selected_differs_from_draft_top"]]
    return {
        "schema_version": INTERVENTION_SCHEMA_VERSION,
        "definition": ("Causal Target action is selection away from first_route or fallback; probability "
                       "displacement is selection away from the Drafter top path conditioned on the current "
                       "round prefix"),
        "target_action_definition": TARGET_ACTION,
        "route_intervention_definition": ROUTE_INTERVENTION,
        "legacy_score_policy": "legacy draft_logprob is used only when current-prefix path fields are absent",
        "round_count": len(det),
        "select_rounds": len(comp),
        "fallback_rounds": fb,
        "target_action_rounds": n_first + fb,
        "target_action_rate": _rate(n_first + fb, len(det)),
        "first_route_intervention_rounds": n_first,
        "first_route_intervention_rate": _rate(n_first, len(comp)),
        "route_intervention_rounds": n_top,
        "route_intervention_rate": _rate(n_top, len(comp)),
        "first_token_changed_rounds": n_tok,
        "first_route_first_token_changed_rounds": n_ftok,
        "lower_total_draft_probability_rounds": n_low,
        "current_prefix_draft_path_comparison_rounds": sum(d["current_prefix_draft_path_comparison"] for d in comp),
        "draft_first_token_comparison_rounds": len(d1),
        "draft_first_token_comparison_coverage": _rate(len(d1), len(comp)),
        "lower_first_token_draft_probability_rounds": n_low1,
        "draft_rank_histogram": dict(sorted(hist.items(), key=lambda kv: int(kv[0]))),
        "max_intervened_draft_rank": max(moved) if moved else None,
        "any_target_action": n_first + fb > 0,
        "any_first_route_intervention": n_first > 0,
        "any_route_intervention": n_top > 0,
        "any_fallback": fb > 0,
        "any_first_token_changed": n_tok > 0,
        "any_first_route_first_token_changed": n_ftok > 0,
        "any_lower_total_draft_probability": n_low > 0,
        "any_lower_first_token_draft_probability": n_low1 > 0,
        "rounds": det,
    }


def prediction_intervention(row: Mapping[str, Any]) -> Mapping[str, Any] | None:
    """The per-sample summary stored in an evaluation row (top level or under ``metadata``)."""
    for holder in (row, row.get("metadata") if isinstance(row.get("metadata"), Mapping) else None):
        if holder is not None and isinstance(holder.get("target_intervention"), Mapping):
            return holder["target_intervention"]
    return None


_SUMMED = ("round_count", "select_rounds", "fallback_rounds", "target_action_rounds",
           "first_route_intervention_rounds", "route_intervention_rounds", "first_token_changed_rounds",
           "first_route_first_token_changed_rounds", "lower_total_draft_probability_rounds",
           "current_prefix_draft_path_comparison_rounds", "draft_first_token_comparison_rounds",
           "lower_first_token_draft_probability_rounds")


def aggregate_prediction_interventions(rows: Sequence[Mapping[str, Any]]) -> dict[str, Any]:
    """Sum the per-sample summaries of an evaluation run."""
    stats = [s for s in (prediction_intervention(r) for r in rows) if s is not None]
    tot = {k: sum(int(s.get(k, 0)) for s in stats) for k in _SUMMED}
    hist: Counter[str] = Counter()
    for s in stats:
        h = s.get("draft_rank_histogram", {})
        if isinstance(h, Mapping):
            hist.update({str(k): int(v) for k, v in h.items()})
    n_action = sum(bool(s.get("any_target_action")) for s in stats)
    n_route = sum(bool(s.get("any_route_intervention")) for s in stats)
    return {
        "schema_version": INTERVENTION_SCHEMA_VERSION,
        "target_action_definition": TARGET_ACTION,
        "route_intervention_definition": ROUTE_INTERVENTION,
        "sample_count": len(rows),
        "samples_with_statistics": len(stats),
        "sample_coverage": _rate(len(stats), len(rows)),
        "samples_with_target_action": n_action,
        "sample_target_action_rate": _rate(n_action, len(stats)),
        "samples_with_first_route_intervention": sum(bool(s.get("any_first_route_intervention")) for s in stats),
        "samples_with_route_intervention": n_route,
        "sample_route_intervention_rate": _rate(n_route, len(stats)),
        **{k: tot[k] for k in ("round_count", "select_rounds", "fallback_rounds", "target_action_rounds")},
        "target_action_rate": _rate(tot["target_action_rounds"], tot["round_count"]),
        "first_route_intervention_rounds": tot["first_route_intervention_rounds"],
        "first_route_intervention_rate": _rate(tot["first_route_intervention_rounds"], tot["select_rounds"]),
        "route_intervention_rounds": tot["route_intervention_rounds"],
        "route_intervention_rate": _rate(tot["route_intervention_rounds"], tot["select_rounds"]),
        **{k: tot[k] for k in ("first_token_changed_rounds", "first_route_first_token_changed_rounds",
                               "lower_total_draft_probability_rounds",
                               "current_prefix_draft_path_comparison_rounds",
                               "draft_first_token_comparison_rounds")},
        "draft_first_token_comparison_coverage": _rate(tot["draft_first_token_comparison_rounds"],
                                                       tot["select_rounds"]),
        "lower_first_token_draft_probability_rounds": tot["lower_first_token_draft_probability_rounds"],
        "draft_rank_histogram": dict(sorted(hist.items(), key=lambda kv: int(kv[0]))),
    }


def mcnemar_exact_p_value(helped: int, hurt: int) -> float | None:
    """Two-sided exact McNemar test: binomial(n = helped + hurt, 1/2) tail, doubled, capped at 1."""
    n = int(helped) + int(hurt)
    if n == 0:
        return None
    k = min(int(helped), int(hurt))
    tail = sum(math.comb(n, i) for i in range(k + 1))
    return min(1.0, 2.0 * tail / float(2 ** n))


def paired_target_quality(target_best_rows: Sequence[Mapping[str, Any]],
                          first_route_rows: Sequence[Mapping[str, Any]]) -> dict[str, Any]:
    """Paired outcome comparison; rows must cover the same sample indices with the same question/gold/model."""
    best = {int(r["index"]): r for r in target_best_rows}
    first = {int(r["index"]): r for r in first_route_rows}
    if len(best) != len(target_best_rows) or len(first) != len(first_route_rows):
        raise ValueError("a sample index appears twice in the predictions (duplicate)")
    if set(best) != set(first):
        raise ValueError(f"paired sample indices differ: missing_target_best={sorted(set(first) - set(best))[:10]}, "
                         f"missing_first_route={sorted(set(best) - set(first))[:10]}")
    pairs = []
    for i in sorted(best):
        for key in ("question", "gold", "model"):
            if best[i].get(key) != first[i].get(key):
                raise ValueError(f"sample {i} has mismatched {key}")
        pairs.append((best[i], first[i]))

    def outcome(subset):
        helped = sum(bool(b.get("correct")) and not bool(f.get("correct")) for b, f in subset)
        hurt = sum(bool(f.get("correct")) and not bool(b.get("correct")) for b, f in subset)
        return helped, hurt

    helped, hurt = outcome(pairs)
    both_ok = sum(bool(b.get("correct")) and bool(f.get("correct")) for b, f in pairs)

    def impact(flag: str, need_draft_first: bool = False) -> dict[str, Any]:
        with_stats = [(b, f, prediction_intervention(b)) for b, f in pairs]
        with_stats = [x for x in with_stats if x[2] is not None]
        metric = [x for x in with_stats
                  if not need_draft_first or int(x[2].get("draft_first_token_comparison_rounds", 0)) > 0]
        chosen = [(b, f) for b, f, s in metric if bool(s.get(flag))]
        h, u = outcome(chosen)
        return {"samples_with_statistics": len(with_stats), "samples_with_comparable_metric": len(metric),
                "sample_count": len(chosen), "helped": h, "hurt": u, "net_correct_gain": h - u}

    n = len(pairs)
    return {
        "schema_version": INTERVENTION_SCHEMA_VERSION,
        "pair_count": n,
        "target_best_correct": both_ok + helped,
        "first_route_correct": both_ok + hurt,
        "target_best_accuracy": _rate(both_ok + helped, n),
        "first_route_accuracy": _rate(both_ok + hurt, n),
        "accuracy_delta": _rate(helped - hurt, n),
        "helped": helped,
        "hurt": hurt,
        "net_correct_gain": helped - hurt,
        "both_correct": both_ok,
        "both_wrong": n - helped - hurt - both_ok,
        "response_changed": sum(b.get("response") != f.get("response") for b, f in pairs),
        "mcnemar_exact_two_sided_p": mcnemar_exact_p_value(helped, hurt),
        "impact_by_target_best_intervention": {
            "any_target_action": impact("any_target_action"),
            "selected_away_from_first_route": impact("any_first_route_intervention"),
            "route_selected_below_draft_top": impact("any_route_intervention"),
            "first_token_changed": impact("any_first_token_changed"),
            "first_route_first_token_changed": impact("any_first_route_first_token_changed"),
            "lower_total_draft_probability": impact("any_lower_total_draft_probability"),
            "lower_first_token_draft_probability": impact("any_lower_first_token_draft_probability", True),
            "fallback_ar": impact("any_fallback"),
        },
    }
