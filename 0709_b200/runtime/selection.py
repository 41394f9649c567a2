"""Deterministic frontier selection.

Candidates are ranked by ``(score desc, parent route asc, rank-in-parent asc,
token asc)``; forest selection groups by stage-1 root (ascending) first and
keeps ``k`` per root.  The device path ranks with a chain of stable sorts,
least significant key first, so exact ties resolve exactly as the host order
does and the result never leaves the device before the single packed
materialization (reference: src/atlas_0709/flashinfer_paged/utils.py:28-123).
"""

from __future__ import annotations

from collections import defaultdict
from typing import Iterable, Sequence

import torch

from ..types import PendingCandidate, PendingCandidateBatch


def _order_key(c: PendingCandidate) -> tuple:
    return (-c.cumulative_logprob, c.parent_route_id, c.rank_in_parent, c.pending_token_id)


def global_topk_candidates(candidates: Sequence[PendingCandidate], num_selected: int) -> list[PendingCandidate]:
    if num_selected <= 0:
        raise ValueError("num_selected must be positive")
    return sorted(candidates, key=_order_key)[: int(num_selected)]


def group_candidates_by_stage1_root(candidates: Iterable[PendingCandidate]) -> dict[int, list[PendingCandidate]]:
    grouped: dict[int, list[PendingCandidate]] = defaultdict(list)
    for c in candidates:
        grouped[int(c.stage1_root_id)].append(c)
    return dict(grouped)


def stable_candidate_order(candidates: PendingCandidateBatch, *, include_stage1_root: bool = False) -> torch.Tensor:
    """Permutation of candidate indices in selection order (stays on the candidates' device)."""
    n = candidates.candidate_count
    dev = candidates.pending_token_ids.device
    order = torch.arange(n, device=dev, dtype=torch.long)
    keys: list[tuple[torch.Tensor, bool]] = [
        (candidates.pending_token_ids, False),
        (candidates.ranks_in_parent, False),
        (candidates.parent_route_ids, False),
        (candidates.cumulative_logprobs, True),
    ]
    if include_stage1_root:
        keys.append((candidates.stage1_root_ids, False))
    for values, descending in keys:
        perm = torch.argsort(values.index_select(0, order), dim=0, descending=descending, stable=True)
        order = order.index_select(0, perm)
    return order


def global_topk_candidate_indices(candidates: PendingCandidateBatch, *, num_selected: int) -> torch.Tensor:
    if num_selected <= 0:
        raise ValueError("num_selected must be positive")
    order = stable_candidate_order(candidates)
    return order[: min(int(num_selected), candidates.candidate_count)]


def per_root_topk_candidate_indices(
    candidates: PendingCandidateBatch,
    *,
    num_selected: int,
    root_candidate_counts: Sequence[tuple[int, int]],
) -> torch.Tensor:
    if num_selected <= 0:
        raise ValueError("num_selected must be positive")
    counts = sorted((int(r), int(c)) for r, c in root_candidate_counts)
    if sum(c for _, c in counts) != candidates.candidate_count:
        raise ValueError("root candidate counts do not cover the candidate batch")
    order = stable_candidate_order(candidates, include_stage1_root=True)
    parts: list[torch.Tensor] = []
    off = 0
    for _, c in counts:
        parts.append(order[off: off + min(int(num_selected), c)])
        off += c
    return torch.cat(parts) if parts else order[:0]


def topk_pairs_to_python(token_ids: torch.Tensor, token_logprobs: torch.Tensor) -> list[tuple[int, float]]:
    """A top-k result as host (token, log-prob) pairs: one wait, two small copies, no packing kernels."""
    if token_ids.shape != token_logprobs.shape:
        raise ValueError("token ids and logprobs must have matching shapes")
    ids = token_ids.detach().reshape(-1).cpu().tolist()
    lps = token_logprobs.detach().reshape(-1).cpu().tolist()
    return [(int(t), float(lp)) for t, lp in zip(ids, lps)]
