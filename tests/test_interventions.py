"""Intervention statistics: per-round comparisons, aggregation, exact McNemar, paired quality."""

from __future__ import annotations

import math

import pytest

from conftest import mod


def sc(rid, toks, *, path=None, draft_toks=None, legacy=None, target=-1.0, tfirst=-0.5):
    d = {"route_id": rid, "token_ids": toks, "target_logprob": target, "first_token_logprob": tfirst}
    if path is not None:
        d["draft_path_logprob"] = path
    if draft_toks is not None:
        d["draft_token_logprobs"] = draft_toks
    if legacy is not None:
        d["draft_logprob"] = legacy
    return d


def test_round_summary_counts_route_intervention_and_fallback():
    iv = mod("utils.interventions")
    rounds = [
        {"round_index": 0, "decision": "select", "selected_route_id": 7,
         "target_scores": [sc(3, [1, 2], draft_toks=[-0.1, -0.2], target=-3.0, tfirst=-1.0),
                           sc(7, [5, 6], draft_toks=[-0.5, -0.9], target=-0.4, tfirst=-0.1)]},
        {"round_index": 1, "decision": "fallback_ar", "selected_route_id": 3, "target_scores": []},
        {"round_index": 2, "decision": "select", "selected_route_id": 3,
         "target_scores": [sc(3, [9], draft_toks=[-0.1]), sc(4, [8], draft_toks=[-0.2])]},
    ]
    s = iv.summarize_generation_interventions(rounds)
    assert s["round_count"] == 3 and s["select_rounds"] == 2 and s["fallback_rounds"] == 1
    assert s["route_intervention_rounds"] == 1 and s["first_route_intervention_rounds"] == 1
    assert s["target_action_rounds"] == 2 and math.isclose(s["target_action_rate"], 2 / 3)
    assert s["draft_rank_histogram"] == {"1": 1, "2": 1} and s["max_intervened_draft_rank"] == 2
    r0 = s["rounds"][0]
    assert r0["first_token_changed"] and r0["lower_total_draft_probability"]
    assert r0["selected_draft_path_logprob_source"] == "sum(draft_token_logprobs)"
    assert math.isclose(r0["draft_path_logprob_delta"], (-1.4) - (-0.3))
    assert r0["lower_first_token_draft_probability"] and not r0["lower_first_token_target_probability"]
    assert s["any_fallback"] and s["any_route_intervention"]


def test_draft_path_source_preference():
    iv = mod("utils.interventions")
    assert iv.draft_path_score(sc(1, [1], path=-0.3, draft_toks=[-5.0], legacy=-9.0)) == (-0.3, "draft_path_logprob")
    assert iv.draft_path_score(sc(1, [1], draft_toks=[-0.5, -0.25], legacy=-9.0))[0] == -0.75
    assert iv.draft_path_score(sc(1, [1], legacy=-2.0)) == (-2.0, "legacy_draft_logprob")
    assert iv.draft_path_score(sc(1, [1])) == (None, None)
    # Non-finite per-token values fall through to the legacy score.
    assert iv.draft_path_score(sc(1, [1], draft_toks=[float("nan")], legacy=-1.0))[1] == "legacy_draft_logprob"
    # The Target's first-token field never stands in for the Drafter's.
    assert iv.draft_first_token_score(sc(1, [1], tfirst=-0.1)) is None


def test_legacy_scores_are_not_current_prefix_comparisons():
    iv = mod("utils.interventions")
    s = iv.summarize_generation_interventions([
        {"round_index": 0, "decision": "select", "selected_route_id": 2,
         "target_scores": [sc(1, [1], legacy=-0.1), sc(2, [2], legacy=-0.2)]}])
    assert s["current_prefix_draft_path_comparison_rounds"] == 0
    assert s["draft_first_token_comparison_rounds"] == 0 and s["draft_first_token_comparison_coverage"] == 0.0


def test_aggregate_sums_counters_and_histograms():
    iv = mod("utils.interventions")
    a = iv.summarize_generation_interventions([
        {"round_index": 0, "decision": "select", "selected_route_id": 2,
         "target_scores": [sc(1, [1], path=-0.1), sc(2, [2], path=-0.2)]}])
    b = iv.summarize_generation_interventions([{"round_index": 0, "decision": "fallback_ar", "target_scores": []}])
    rows = [{"target_intervention": a}, {"metadata": {"target_intervention": b}}, {"other": 1}]
    agg = iv.aggregate_prediction_interventions(rows)
    assert agg["sample_count"] == 3 and agg["samples_with_statistics"] == 2
    assert agg["round_count"] == 2 and agg["fallback_rounds"] == 1 and agg["select_rounds"] == 1
    assert agg["draft_rank_histogram"] == {"2": 1}
    assert agg["samples_with_target_action"] == 2 and agg["samples_with_route_intervention"] == 1


@pytest.mark.parametrize("helped,hurt", [(5, 0), (3, 3), (10, 2), (1, 7), (40, 25)])
def test_mcnemar_matches_binomial_test(helped, hurt):
    iv = mod("utils.interventions")
    from scipy.stats import binomtest

    ref = binomtest(min(helped, hurt), helped + hurt, 0.5).pvalue
    assert math.isclose(iv.mcnemar_exact_p_value(helped, hurt), min(1.0, ref), rel_tol=1e-9)
    assert iv.mcnemar_exact_p_value(0, 0) is None


def test_paired_quality_counts_and_alignment_guards():
    iv = mod("utils.interventions")
    stats_yes = {"any_target_action": True, "any_route_intervention": True, "draft_first_token_comparison_rounds": 1,
                 "any_lower_first_token_draft_probability": True}
    best = [
        {"index": 0, "question": "q0", "gold": "1", "model": "m", "correct": True, "response": "a",
         "target_intervention": stats_yes},
        {"index": 1, "question": "q1", "gold": "2", "model": "m", "correct": False, "response": "b"},
        {"index": 2, "question": "q2", "gold": "3", "model": "m", "correct": True, "response": "c"},
    ]
    first = [
        {"index": 0, "question": "q0", "gold": "1", "model": "m", "correct": False, "response": "x"},
        {"index": 1, "question": "q1", "gold": "2", "model": "m", "correct": True, "response": "b"},
        {"index": 2, "question": "q2", "gold": "3", "model": "m", "correct": True, "response": "c"},
    ]
    r = iv.paired_target_quality(best, first)
    assert (r["helped"], r["hurt"], r["both_correct"], r["both_wrong"]) == (1, 1, 1, 0)
    assert r["response_changed"] == 1 and r["mcnemar_exact_two_sided_p"] == 1.0
    imp = r["impact_by_target_best_intervention"]
    assert imp["any_target_action"]["helped"] == 1 and imp["any_target_action"]["samples_with_statistics"] == 1
    assert imp["lower_first_token_draft_probability"]["sample_count"] == 1
    with pytest.raises(ValueError, match="mismatched gold"):
        iv.paired_target_quality(best, [dict(first[0], gold="9"), first[1], first[2]])
    with pytest.raises(ValueError, match="indices differ"):
        iv.paired_target_quality(best, first[:2])
    with pytest.raises(ValueError, match="duplicate"):
        iv.paired_target_quality(best + [best[0]], first)
