"""Drafter candidate sampling and frontier selection order (CPU)."""

from __future__ import annotations

import torch

from conftest import mod


def ctx(seed=0, prefix=(1, 2, 3), do_sample=True, temperature=1.0):
    s = mod("runtime.sampling")
    return s.DrafterSamplingContext(s.DrafterSamplingConfig(do_sample, seed, temperature), tuple(prefix))


def test_semantic_key_is_invariant_to_prefix_route_split():
    a = ctx(prefix=(1, 2, 3, 4, 5))
    b = ctx(prefix=(1, 2, 3))
    assert a.seed_for_parent(()) == b.seed_for_parent((4, 5))
    assert a.seed_for_parent((6,)) == b.seed_for_parent((4, 5, 6))
    assert b.seed_for_parent((4,)) != b.seed_for_parent((5,))


def test_sampling_reproducible_and_seed_sensitive():
    s = mod("runtime.sampling")
    logits = torch.randn(3, 500, generator=torch.Generator().manual_seed(0))
    paths = [(1,), (2,), (3,)]
    a = s.batch_parent_token_candidates(logits, k=4, sampling=ctx(seed=7), relative_parent_paths=paths)
    b = s.batch_parent_token_candidates(logits, k=4, sampling=ctx(seed=7), relative_parent_paths=paths)
    c = s.batch_parent_token_candidates(logits, k=4, sampling=ctx(seed=8), relative_parent_paths=paths)
    assert torch.equal(a[1], b[1]) and torch.equal(a[0], b[0])
    assert not torch.equal(a[1], c[1])
    # Distinct tokens per parent (sampling without replacement).
    assert all(len(set(row.tolist())) == 4 for row in a[1])


def test_sampling_independent_of_batch_order():
    s = mod("runtime.sampling")
    logits = torch.randn(3, 300, generator=torch.Generator().manual_seed(1))
    paths = [(1,), (2, 2), (3,)]
    a_lp, a_ids = s.batch_parent_token_candidates(logits, k=3, sampling=ctx(), relative_parent_paths=paths)
    perm = [2, 0, 1]
    b_lp, b_ids = s.batch_parent_token_candidates(logits[perm], k=3, sampling=ctx(),
                                                  relative_parent_paths=[paths[i] for i in perm])
    assert torch.equal(a_ids[perm], b_ids) and torch.equal(a_lp[perm], b_lp)


def test_recorded_logprobs_are_untempered():
    s = mod("runtime.sampling")
    logits = torch.randn(2, 200, generator=torch.Generator().manual_seed(2))
    lp, ids = s.batch_parent_token_candidates(logits, k=3, sampling=ctx(temperature=0.3),
                                              relative_parent_paths=[(), (9,)])
    ref = torch.log_softmax(logits, -1).gather(-1, ids)
    torch.testing.assert_close(lp, ref)


def test_greedy_mode_is_plain_topk():
    s = mod("runtime.sampling")
    logits = torch.randn(4, 100, generator=torch.Generator().manual_seed(3))
    lp, ids = s.batch_parent_token_candidates(logits, k=2, sampling=ctx(do_sample=False),
                                              relative_parent_paths=[()] * 4)
    ref = torch.topk(torch.log_softmax(logits, -1), 2)
    assert torch.equal(ids, ref.indices)
    lp2, ids2 = s.batch_parent_token_candidates(logits, k=2, sampling=None, relative_parent_paths=[()] * 4)
    assert torch.equal(ids, ids2)


def test_keyed_uniform_is_in_open_unit_interval_and_deterministic():
    s = mod("runtime.sampling")
    keys = torch.tensor([0, 1, 2 ** 62, 123456789], dtype=torch.int64)
    u = s.keyed_uniform(keys, 1000)
    assert bool(((u > 0) & (u < 1)).all())
    assert torch.equal(u, s.keyed_uniform(keys, 1000))
    assert 0.45 < float(u.mean()) < 0.55


def test_device_order_matches_host_order_under_full_ties():
    sel = mod("runtime.selection")
    types = mod("types")
    g = torch.Generator().manual_seed(4)
    cands = []
    for i in range(30):
        cands.append(types.PendingCandidate(
            parent_route_id=int(torch.randint(0, 4, (1,), generator=g)),
            stage1_root_id=int(torch.randint(0, 3, (1,), generator=g)),
            pending_token_id=int(torch.randint(0, 6, (1,), generator=g)),
            rank_in_parent=int(torch.randint(0, 3, (1,), generator=g)),
            cumulative_logprob=float(torch.randint(0, 3, (1,), generator=g)) * -0.5,
        ))
    host = sel.global_topk_candidates(cands, 30)
    key = lambda c: (-c.cumulative_logprob, c.parent_route_id, c.rank_in_parent, c.pending_token_id)  # noqa: E731
    assert [key(c) for c in host] == sorted(key(c) for c in cands)
    fields = {
        "pending_token_ids": torch.tensor([c.pending_token_id for c in cands]),
        "ranks_in_parent": torch.tensor([c.rank_in_parent for c in cands]),
        "parent_route_ids": torch.tensor([c.parent_route_id for c in cands]),
        "cumulative_logprobs": torch.tensor([c.cumulative_logprob for c in cands], dtype=torch.float64),
        "stage1_root_ids": torch.tensor([c.stage1_root_id for c in cands]),
    }
    batch = type("B", (), {**fields, "candidate_count": len(cands)})()
    order = sel.stable_candidate_order(batch).tolist()
    assert [key(cands[i]) for i in order] == [key(c) for c in host]
    order_r = sel.stable_candidate_order(batch, include_stage1_root=True).tolist()
    keyr = lambda c: (c.stage1_root_id, *key(c))  # noqa: E731
    assert [keyr(cands[i]) for i in order_r] == sorted(keyr(c) for c in cands)
