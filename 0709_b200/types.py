"""Shared value types of the speculative-decoding runtime.

The field names mirror the reference's public result objects so that result
JSON, RPC payloads and evaluators stay interchangeable
(reference: src/atlas_0709/types.py:77-120, src/atlas_0709/flashinfer_paged/types.py:16-150).
The implementation is independent: routes carry a handle into the native page
pool instead of SGLang request rows.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Mapping, NamedTuple, Sequence

import torch


class DecodePhase(str, Enum):
    """Which stage a frontier step extends: the stage-1 tree or the stage-2 forest."""

    STAGE1 = "stage1"
    STAGE2 = "stage2"


@dataclass(frozen=True)
class PrefixKVView:
    """Committed prefix seen by every live route (length only; pages live in the pool)."""

    committed_length: int

    def fork(self) -> "RouteKVView":
        return RouteKVView(prefix=self, node_ids=())


@dataclass(frozen=True)
class RouteKVView:
    """Logical KV of a route: the committed prefix plus the tree nodes it has materialized."""

    prefix: PrefixKVView
    node_ids: tuple[int, ...] = ()

    def fork(self) -> "RouteKVView":
        return RouteKVView(prefix=self.prefix, node_ids=tuple(self.node_ids))

    def append_node(self, node_id: int) -> "RouteKVView":
        return RouteKVView(prefix=self.prefix, node_ids=(*self.node_ids, int(node_id)))

    @property
    def length(self) -> int:
        return int(self.prefix.committed_length) + len(self.node_ids)


@dataclass
class RouteState:
    """A live route: a materialized node path plus one pending (not yet decoded) token.

    ``token_logprobs`` holds the drafter log-probabilities of the route's tokens
    relative to the current committed prefix; a frontier route includes its
    pending token, a completed route exactly its materialized path.
    """

    route_id: int
    stage1_root_id: int
    parent_route_id: int | None
    materialized_leaf_node_id: int | None
    pending_token_id: int
    cumulative_logprob: float
    stage1_depth: int
    stage2_depth: int
    kv_view: RouteKVView
    token_logprobs: tuple[float, ...] = ()

    def total_materialized_depth(self) -> int:
        return int(self.stage1_depth) + int(self.stage2_depth)


class PendingCandidate(NamedTuple):
    """One proposed child of a frontier route (immutable; a tuple so that a depth's few dozen
    candidates are cheap to build on the host between two drafter forwards)."""

    parent_route_id: int
    stage1_root_id: int
    pending_token_id: int
    cumulative_logprob: float
    rank_in_parent: int = 0
    parent_logprob: float = 0.0


@dataclass(frozen=True)
class FrontierSelectionStats:
    candidate_count: int = 0
    selected_count: int = 0
    host_materialization_batches: int = 0
    host_materialization_elements: int = 0
    host_transfer_batches: int = 0
    host_transfer_elements: int = 0
    selection_device: str = "cpu"
    new_node_ids_source: str = "unknown"


@dataclass(frozen=True)
class DraftPrefixState:
    token_tuple: tuple[int, ...]
    prefix_kv_view: PrefixKVView
    next_token_logits: torch.Tensor
    committed_length: int
    # Greedy top-k children of the prefix selected inside the extend forward's graph (see
    # ``FrontierDecodeOutput.candidates``), or None.
    candidates: Any = None

    @property
    def token_ids(self) -> torch.Tensor:
        """The committed prefix as an int64 tensor (built on request: prefixes are long)."""
        return torch.tensor(self.token_tuple, dtype=torch.long)


@dataclass(frozen=True)
class FrontierDecodeOutput:
    route_ids: torch.Tensor
    next_token_logits: torch.Tensor
    new_node_ids: torch.Tensor | Sequence[int]
    new_node_ids_cpu: tuple[int, ...] | None = None
    attention_ms: float = 0.0
    model_ms: float = 0.0
    kv_append_ms: float = 0.0
    metadata: Mapping[str, Any] = field(default_factory=dict)
    # Greedy top-k children of every row selected inside the forward's graph (an object with
    # ``get() -> (ids [n, k], log-probs [n, k])`` and ``words``), or None.
    candidates: Any = None


@dataclass(frozen=True)
class FrontierStepOutput:
    decoded_routes: list[RouteState]
    next_routes: list[RouteState]
    candidates: list[PendingCandidate]
    selected_candidates: list[PendingCandidate]
    decode_output: FrontierDecodeOutput
    selection_stats: FrontierSelectionStats = field(default_factory=FrontierSelectionStats)


@dataclass(frozen=True)
class BuildDepthsOutput:
    completed_routes: list[RouteState]
    next_frontier_routes: list[RouteState]
    last_logits: torch.Tensor
    steps: list[FrontierStepOutput]


@dataclass(frozen=True)
class PrefixState:
    token_ids: tuple[int, ...]
    next_token_logits: torch.Tensor
    committed_length: int
    metadata: Mapping[str, Any] = field(default_factory=dict)


@dataclass(frozen=True)
class VerifyRoutePayload:
    route_id: int
    token_ids: tuple[int, ...]
    draft_logprob: float
    draft_token_logprobs: tuple[float, ...] = ()


@dataclass(frozen=True)
class TargetRouteScore:
    route_id: int
    token_ids: tuple[int, ...]
    target_logprob: float
    draft_logprob: float
    token_logprobs: tuple[float, ...] = ()
    first_token_logprob: float | None = None
    selection_score: float | None = None
    score_weights: tuple[float, ...] = ()
    draft_token_logprobs: tuple[float, ...] = ()

    @property
    def draft_first_token_logprob(self) -> float | None:
        if not self.draft_token_logprobs:
            return None
        return float(self.draft_token_logprobs[0])

    @property
    def draft_path_logprob(self) -> float:
        """Drafter path log-probability relative to the current prefix."""
        if self.draft_token_logprobs:
            return float(sum(self.draft_token_logprobs))
        return float(self.draft_logprob)

    @property
    def effective_selection_score(self) -> float:
        if self.selection_score is None:
            return float(self.target_logprob)
        return float(self.selection_score)


@dataclass(frozen=True)
class TargetVerifyResult:
    selected_route_id: int | None
    scores: list[TargetRouteScore]
    metadata: Mapping[str, Any] = field(default_factory=dict)
    decision: str = "select"
    fallback_token_ids: tuple[int, ...] = ()
    fallback_reason: str | None = None

    @property
    def selected_score(self) -> TargetRouteScore:
        if self.selected_route_id is None:
            raise KeyError("a fallback_ar result commits target tokens, not a route")
        for score in self.scores:
            if score.route_id == self.selected_route_id:
                return score
        raise KeyError(self.selected_route_id)


def verify_payload_from_mapping(item: Mapping[str, Any]) -> VerifyRoutePayload:
    """Parse one ``routes[]`` entry of a ``/verify`` request."""
    raw = item.get("draft_token_logprobs")
    if raw is None:
        draft_token_logprobs: tuple[float, ...] = ()
    elif isinstance(raw, (list, tuple)):
        draft_token_logprobs = tuple(float(v) for v in raw)
    else:
        raise ValueError("draft_token_logprobs, when present, is a list of numbers")
    return VerifyRoutePayload(
        route_id=int(item["route_id"]),
        token_ids=tuple(int(t) for t in item["token_ids"]),
        draft_logprob=float(item.get("draft_logprob", 0.0)),
        draft_token_logprobs=draft_token_logprobs,
    )
