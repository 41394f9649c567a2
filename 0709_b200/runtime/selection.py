"""Deterministic ranking of a frontier depth's candidates.

The selection order is part of the contract (greedy equivalence and
reproducible drafts depend on it): higher cumulative draft log-prob first,
then smaller parent route id, then smaller rank inside the parent's top-k,
then smaller token id.  Stage-1 trees keep the best ``k`` over the whole
frontier; stage-2 forests keep the best ``k`` of every stage-1 root, roots in
ascending id order.

Host ranking sorts the (at most k^3) candidates once by that key -- with the
stage-1 root as a leading key for forests, so every root's block is
contiguous and its quota is taken in one pass.

``stable_candidate_order`` ranks candidate tensors on their own device without
a chain of sorts: the rank of candidate ``i`` is the number of candidates that
precede it under the order (candidate index breaks exact ties, so the ranks
form a permutation), computed from one pairwise comparison matrix.  For the
few dozen candidates of a depth that is a handful of elementwise kernels
whose cost does not grow with the number of sort keys.

Reference order: src/atlas_0709/flashinfer_paged/utils.py:28-123.
"""

from __future__ import annotations

from typing import Sequence

import torch

from ..types import PendingCandidate


def rank_key(c: PendingCandidate) -> tuple:
    return (-float(c.cumulative_logprob), int(c.parent_route_id), int(c.rank_in_parent), int(c.pending_token_id))


def global_topk_candidates(candidates: Sequence[PendingCandidate], num_selected: int) -> list[PendingCandidate]:
    """The best ``num_selected`` candidates overall, in selection order."""
    n = int(num_selected)
    if n < 1:
        raise ValueError(f"cannot select {num_selected} candidates")
    return sorted(candidates, key=rank_key)[:n]


def best_per_root(candidates: Sequence[PendingCandidate], per_root: int,
                  roots: Sequence[int]) -> list[PendingCandidate]:
    """The best ``per_root`` candidates of each root in ``roots`` (ascending), concatenated."""
    n = int(per_root)
    if n < 1:
        raise ValueError(f"cannot select {per_root} candidates per root")
    ranked = sorted(candidates, key=lambda c: (int(c.stage1_root_id), *rank_key(c)))
    picks: dict[int, list[PendingCandidate]] = {}
    for c in ranked:
        got = picks.setdefault(int(c.stage1_root_id), [])
        if len(got) < n:
            got.append(c)
    out: list[PendingCandidate] = []
    for r in sorted({int(x) for x in roots}):
        if r not in picks:
            raise ValueError(f"no candidates were produced under stage-1 root {r}")
        out.extend(picks[r])
    return out


def stable_candidate_order(candidates, *, include_stage1_root: bool = False) -> torch.Tensor:
    """Candidate indices in selection order, computed on the candidates' device.

    ``candidates`` has tensors ``cumulative_logprobs``, ``parent_route_ids``,
    ``ranks_in_parent``, ``pending_token_ids`` (and ``stage1_root_ids`` when
    ``include_stage1_root``), one entry per candidate.
    """
    score = candidates.cumulative_logprobs.to(torch.float64).reshape(-1)
    n = int(score.numel())
    dev = score.device
    idx = torch.arange(n, device=dev)
    keys = [-score, candidates.parent_route_ids, candidates.ranks_in_parent, candidates.pending_token_ids, idx]
    if include_stage1_root:
        keys.insert(0, candidates.stage1_root_ids)
    # before[j, i]: candidate j precedes candidate i (lexicographic over the keys).
    before = torch.zeros((n, n), dtype=torch.bool, device=dev)
    tied = torch.ones((n, n), dtype=torch.bool, device=dev)
    for key in keys:
        v = key.reshape(-1).to(dev)
        v = v.to(torch.float64) if v.is_floating_point() else v.to(torch.int64)
        before |= tied & (v[:, None] < v[None, :])
        tied &= v[:, None] == v[None, :]
    order = torch.empty(n, dtype=torch.long, device=dev)
    order[before.sum(dim=0)] = idx
    return order
