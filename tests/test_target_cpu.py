"""Target verify service on CPU: compaction into the prefix, scoring, selection policies, sampling, truncation."""

from __future__ import annotations

import math

import pytest
import torch

from conftest import mod

PAGE = 4


@pytest.fixture(scope="module")
def tw():
    llama = mod("models.llama")
    return llama.random_weights(llama.get_config("tiny-target"), seed=2, dtype=torch.float32)


def verifier(tw, **kw):
    engine = mod("runtime.engine")
    target = mod("runtime.target")
    e = engine.LlamaEngine(tw, num_pages=256, page_size=PAGE, max_positions=512)
    return target.TargetVerifier(e, k=kw.pop("k", 3), d=kw.pop("d", 3), **kw)


def payload(rid, toks, draft=None):
    types = mod("types")
    dl = tuple(draft) if draft is not None else tuple([-0.5] * len(toks))
    return types.VerifyRoutePayload(route_id=rid, token_ids=tuple(toks), draft_logprob=sum(dl), draft_token_logprobs=dl)


def score(rid, toks, target, *, draft=(-1.0,), sel=None, first=None):
    types = mod("types")
    return types.TargetRouteScore(route_id=rid, token_ids=tuple(toks), target_logprob=target,
                                  draft_logprob=sum(draft), token_logprobs=(), first_token_logprob=first,
                                  selection_score=sel, draft_token_logprobs=tuple(draft))


def greedy_logits(tw, toks):
    return mod("models.llama").reference_forward(tw, toks)


def test_selected_nodes_are_compacted_into_the_committed_prefix(tw):
    tv = verifier(tw, route_selection_policy="first_route")
    prompt = list(range(20, 37))
    tv.prefill(prompt)
    # Route 0 shares no node with routes 1 and 2 beyond the first token, so its
    # nodes are not the first ones of the trie: the commit must move KV.
    routes = [payload(0, [7, 8, 9]), payload(1, [7, 5, 6]), payload(2, [3, 4, 1])]
    res = tv.verify_payloads(prefix_token_ids=prompt, routes=[routes[1], routes[0], routes[2]])
    assert res.decision == "select" and res.selected_route_id == 1
    assert tv.prefix_token_ids == tuple(prompt + [7, 5, 6])
    # The next-token logits kept for the new prefix match a fresh recompute.
    torch.testing.assert_close(tv.prefix_logits, greedy_logits(tw, prompt + [7, 5, 6])[-1], rtol=1e-4, atol=1e-4)
    # A second round after a commit whose nodes were moved still sees correct KV.
    tv.verify_payloads(prefix_token_ids=list(tv.prefix_token_ids),
                       routes=[payload(5, [2, 2, 2]), payload(6, [2, 3, 3]), payload(7, [9, 9, 9])])
    want = greedy_logits(tw, prompt + [7, 5, 6, 2, 2, 2])[-1]
    torch.testing.assert_close(tv.prefix_logits, want, rtol=1e-4, atol=1e-4)
    tv.seq.validate()


def test_scores_use_shared_parent_logits(tw):
    tv = verifier(tw)
    prompt = list(range(50, 61))
    tv.prefill(prompt)
    tree = tv.run_tree([[4, 5, 6], [4, 5, 9], [4, 7, 7]])
    lp = tree["path_logprobs"]
    assert lp[0][0] == lp[1][0] == lp[2][0]  # same first token, same prefix row
    assert lp[0][1] == lp[1][1]              # same parent node for the second token
    ref = torch.log_softmax(greedy_logits(tw, prompt + [4, 5]), -1)
    assert math.isclose(lp[1][2], float(ref[-1, 9]), rel_tol=1e-4, abs_tol=1e-5)
    assert tree["node_count"] == 6


def test_first_route_policy_ignores_scores_and_rejects_thresholds(tw):
    tv = verifier(tw, route_selection_policy="first_route")
    sel, meta = tv._select_route_with_metadata([score(4, [1], -9.0), score(2, [2], -0.1)])
    assert sel.route_id == 4 and meta["route_sampling_enabled"] is False
    with pytest.raises(ValueError, match="first_route"):
        verifier(tw, route_selection_policy="first_route", fallback_threshold=-1.0)


def test_target_best_tie_break_order(tw):
    tv = verifier(tw)
    # Equal selection scores: higher draft path log-prob wins, then the lower route id.
    a = score(5, [1, 2], -1.0, draft=(-0.2, -0.2))
    b = score(3, [1, 3], -1.0, draft=(-0.1, -0.2))
    c = score(1, [1, 4], -1.0, draft=(-0.1, -0.2))
    sel, _ = tv._select_route_with_metadata([a, b, c])
    assert sel.route_id == 1
    # The draft path score is the current-prefix per-token sum, not the legacy cumulative score.
    d = mod("types").TargetRouteScore(route_id=9, token_ids=(1,), target_logprob=-1.0, draft_logprob=50.0,
                                      draft_token_logprobs=(-3.0,))
    sel, _ = tv._select_route_with_metadata([a, d])
    assert sel.route_id == 5


def test_policy_and_temperature_validation(tw):
    with pytest.raises(ValueError, match="route_selection_policy"):
        verifier(tw, route_selection_policy="best")
    for bad in (0.0, -1.0, float("nan"), float("inf")):
        with pytest.raises(ValueError, match="temperature"):
            verifier(tw, route_selection_policy="target_sample", route_sampling_temperature=bad)


def test_target_sample_is_seeded_and_payload_order_independent(tw):
    tv = verifier(tw, route_selection_policy="target_sample")
    scores = [score(i, [i, i + 1], -0.5 * i, draft=(-0.3, -0.3)) for i in range(4)]
    picks = {tv._sample_route(scores, 11, r)[0].route_id for r in range(40)}
    assert len(picks) > 1  # the draw varies with the round
    for r in range(10):
        a, ma = tv._sample_route(scores, 7, r)
        b, mb = tv._sample_route(list(reversed(scores)), 7, r)
        assert a.route_id == b.route_id and ma["route_sampling_uniform"] == mb["route_sampling_uniform"]
        assert ma["route_sampling_selected_cdf_low"] <= ma["route_sampling_uniform"] < ma["route_sampling_selected_cdf_high"]
    probs = [c["probability"] for c in ma["route_sampling_ordered_candidates"]]
    assert math.isclose(sum(probs), 1.0, rel_tol=1e-12)
    with pytest.raises(ValueError, match="route_sampling_seed"):
        tv._select_route_with_metadata(scores, route_sampling_seed=None, route_sampling_round=1)
    with pytest.raises(ValueError, match="non-negative"):
        tv._sample_route(scores, 1, -1)


def test_selected_path_truncated_by_budget_and_eos(tw):
    target = mod("runtime.target")
    tr = target.TargetVerifier._truncate_selected_path
    assert tr(token_ids=(5, 6, 7), node_ids=(0, 1, 2), max_tokens=2, eos_token_id=None) == ((5, 6), (0, 1))
    assert tr(token_ids=(5, 6, 7), node_ids=(0, 4, 9), max_tokens=None, eos_token_id=6) == ((5, 6), (0, 4))
    with pytest.raises(ValueError, match="positive"):
        tr(token_ids=(5,), node_ids=(0,), max_tokens=0, eos_token_id=None)


def test_fallback_reasons_checked_in_order(tw):
    tv = verifier(tw, fallback_threshold=-1.0, first_token_threshold=-0.5)
    assert tv._fallback_reason(score(1, [1], -0.2, first=-0.9)) == "first_token_below_threshold"
    assert tv._fallback_reason(score(1, [1], -3.0, first=-0.1)) == "path_score_below_threshold"
    assert tv._fallback_reason(score(1, [1], -0.2, first=-0.1)) is None


def test_score_weights_are_normalized_and_validated(tw):
    target = mod("runtime.target")
    w = target.validate_score_weights([0.9, 0.6, 0.3, 0.2])
    assert math.isclose(sum(w), 1.0) and w[0] > w[-1]
    with pytest.raises(ValueError):
        target.validate_score_weights([0.5, -0.1])
    tv = verifier(tw, d=2, score_weights=[3, 1])
    s = tv._score_routes([payload(0, [1, 2])], [(1, 2)], [[-1.0, -2.0]])[0]
    assert math.isclose(s.selection_score, 0.75 * -1.0 + 0.25 * -2.0) and s.target_logprob == -3.0


def test_intervention_metadata_in_verify_result(tw):
    tv = verifier(tw, k=2, d=2)
    prompt = list(range(80, 90))
    tv.prefill(prompt)
    res = tv.verify_payloads(prefix_token_ids=prompt,
                             routes=[payload(0, [1, 2], draft=(-0.1, -0.1)), payload(1, [3, 4], draft=(-2.0, -2.0))])
    md = res.metadata
    assert md["route_count"] == 2
    assert any("intervention" in key or "draft" in key for key in md), sorted(md)


def test_linear_verify_matches_deduplicated_tree(tw):
    tv = verifier(tw)
    prompt = list(range(60, 73))
    tv.prefill(prompt)
    paths = [[4, 5, 6], [4, 5, 9], [1, 7, 7]]
    a = tv.run_tree(paths)
    b = tv.run_tree(paths, deduplicate=False)
    assert b["node_count"] == 9 and a["node_count"] == 7
    for ra, rb in zip(a["path_logprobs"], b["path_logprobs"]):
        for x, y in zip(ra, rb):
            assert abs(x - y) < 1e-4


def test_pending_fallback_token_is_resolved_by_the_next_verify(tw):
    """After a fallback the last AR token's forward is deferred; the next verify runs it as
    the trie root.  Scores, the committed path's KV and the prefix logits match a recompute."""
    tv = verifier(tw, route_selection_policy="first_route")
    prompt = list(range(30, 47))
    tv.prefill(prompt)
    tv.fallback_threshold = 1e9
    tv.route_selection_policy = "target_best"
    res = tv.verify_payloads(prefix_token_ids=prompt, routes=[payload(i, [i + 1, 2, 3]) for i in range(3)],
                             fallback_max_tokens=4)
    assert res.decision == "fallback_ar" and len(res.fallback_token_ids) == 4
    ar = list(res.fallback_token_ids)
    # The target's greedy tokens.
    toks = list(prompt)
    for _ in range(4):
        toks.append(int(greedy_logits(tw, toks)[-1].argmax()))
    assert ar == toks[len(prompt):]
    assert tv._pending_token == ar[-1]
    # Next round selects: the pending token rides along as the trie root.
    tv.fallback_threshold = None
    tv.route_selection_policy = "first_route"
    prefix = prompt + ar
    routes = [payload(0, [9, 8, 7]), payload(1, [9, 8, 1]), payload(2, [4, 4, 4])]
    res2 = tv.verify_payloads(prefix_token_ids=prefix, routes=routes)
    assert res2.decision == "select" and res2.selected_route_id == 0
    assert tv._pending_token is None
    ref = torch.log_softmax(greedy_logits(tw, prefix + [9, 8, 7]), dim=-1)
    want = [float(ref[len(prefix) - 1 + j, t]) for j, t in enumerate([9, 8, 7])]
    got = list(res2.scores[0].token_logprobs)
    assert got == pytest.approx(want, abs=1e-4)
    torch.testing.assert_close(tv.prefix_logits, greedy_logits(tw, prefix + [9, 8, 7])[-1], rtol=1e-4, atol=1e-4)
    # And one more round on top sees correct KV for every committed token.
    tv.verify_payloads(prefix_token_ids=list(tv.prefix_token_ids),
                       routes=[payload(5, [1, 2, 3]), payload(6, [1, 2, 4]), payload(7, [6, 6, 6])])
    torch.testing.assert_close(tv.prefix_logits, greedy_logits(tw, prefix + [9, 8, 7, 1, 2, 3])[-1],
                               rtol=1e-4, atol=1e-4)
    tv.seq.validate()


def test_pending_fallback_token_flushes_on_demand(tw):
    tv = verifier(tw)
    prompt = list(range(60, 71))
    tv.prefill(prompt)
    tv.fallback_threshold = 1e9
    res = tv.verify_payloads(prefix_token_ids=prompt, routes=[payload(i, [i + 1, 2, 3]) for i in range(3)],
                             fallback_max_tokens=2)
    assert tv._pending_token is not None
    # Reading the prefix logits (or a linear verify) runs the pending forward on its own.
    want = greedy_logits(tw, prompt + list(res.fallback_token_ids))[-1]
    torch.testing.assert_close(tv.prefix_logits, want, rtol=1e-4, atol=1e-4)
    assert tv._pending_token is None


def test_fallback_with_zero_token_budget_keeps_metadata(tw):
    tv = verifier(tw)
    prompt = list(range(70, 81))
    tv.prefill(prompt)
    tv.fallback_threshold = 1e9
    res = tv.verify_payloads(prefix_token_ids=prompt, routes=[payload(i, [i + 1, 2, 3]) for i in range(3)],
                             fallback_max_tokens=0)
    assert res.decision == "fallback_ar" and res.fallback_token_ids == ()
    assert res.metadata["prefix_len_before"] == len(prompt) and res.metadata["node_count"] > 0
