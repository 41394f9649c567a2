"""Stage-1 tree and stage-2 forest construction over a frontier model backend.

Parity: reference src/atlas_0709/flashinfer_paged/builders.py:31-261.
- stage-1 tree: ``k`` routes, global top-k per depth (batch-k decode);
- stage-2 forest: ``k`` children per completed stage-1 route (``k^2`` routes),
  per-root top-k per depth (batch-k^2 decode);
- ``select_routes_by_stage1_root`` keeps the selected root's ``k`` routes.
"""

from __future__ import annotations

from typing import Any, Sequence

import torch

from ..types import BuildDepthsOutput, DecodePhase, DraftPrefixState, FrontierStepOutput, PendingCandidate, RouteState
from .frontier import (
    FrontierModelBackend,
    GlobalTopKSelection,
    PerStage1RootTopKSelection,
    advance_frontier_one_token,
    collect_pending_candidates,
)
from .sampling import DrafterSamplingContext, batch_parent_token_candidates, single_parent_token_candidates
from .selection import topk_pairs_to_python
from .store import KVTreeStore


def initialize_stage1_routes(
    draft_prefix_state: DraftPrefixState,
    *,
    k: int,
    route_store: KVTreeStore,
    sampling: DrafterSamplingContext | None = None,
) -> list[RouteState]:
    lp, ids = single_parent_token_candidates(draft_prefix_state.next_token_logits, k=k, sampling=sampling)
    routes: list[RouteState] = []
    for tok, tlp in topk_pairs_to_python(ids, lp):
        rid = route_store.allocate_route_id()
        routes.append(
            route_store.register_route(
                RouteState(
                    route_id=rid,
                    stage1_root_id=rid,
                    parent_route_id=None,
                    materialized_leaf_node_id=None,
                    pending_token_id=tok,
                    cumulative_logprob=tlp,
                    stage1_depth=0,
                    stage2_depth=0,
                    kv_view=draft_prefix_state.prefix_kv_view.fork(),
                    token_logprobs=(float(tlp),),
                )
            )
        )
    return routes


def build_tree_one_depth(
    active_routes: Sequence[RouteState],
    *,
    k: int,
    route_store: KVTreeStore,
    model_backend: FrontierModelBackend,
    attention_backend: Any = None,
    phase: DecodePhase = DecodePhase.STAGE1,
    sampling: DrafterSamplingContext | None = None,
) -> FrontierStepOutput:
    if len(active_routes) != k:
        raise ValueError(f"build_tree_one_depth expects {k} active routes, got {len(active_routes)}")
    return advance_frontier_one_token(
        active_routes,
        k=k,
        route_store=route_store,
        model_backend=model_backend,
        selection_policy=GlobalTopKSelection(phase=phase),
        attention_backend=attention_backend,
        sampling=sampling,
    )


def _depths(step_fn, active_routes, depth: int, **kw) -> BuildDepthsOutput:
    if depth <= 0:
        raise ValueError("depth must be positive")
    steps: list[FrontierStepOutput] = []
    frontier = list(active_routes)
    for _ in range(depth):
        step = step_fn(frontier, **kw)
        steps.append(step)
        frontier = step.next_routes
    last = steps[-1]
    return BuildDepthsOutput(
        completed_routes=last.decoded_routes,
        next_frontier_routes=last.next_routes,
        last_logits=last.decode_output.next_token_logits,
        steps=steps,
    )


def build_tree_depths(
    active_routes: Sequence[RouteState],
    *,
    depth: int,
    k: int,
    route_store: KVTreeStore,
    model_backend: FrontierModelBackend,
    attention_backend: Any = None,
    phase: DecodePhase = DecodePhase.STAGE1,
    sampling: DrafterSamplingContext | None = None,
) -> BuildDepthsOutput:
    return _depths(
        build_tree_one_depth,
        active_routes,
        depth,
        k=k,
        route_store=route_store,
        model_backend=model_backend,
        attention_backend=attention_backend,
        phase=phase,
        sampling=sampling,
    )


def initialize_forest_routes(
    stage1_routes: Sequence[RouteState],
    stage1_last_logits: torch.Tensor,
    *,
    k: int,
    route_store: KVTreeStore,
    sampling: DrafterSamplingContext | None = None,
) -> list[RouteState]:
    if len(stage1_routes) != int(stage1_last_logits.shape[0]):
        raise ValueError("stage1_routes and stage1_last_logits must have the same batch size")
    rel = [route_store.materialized_token_path(r) for r in stage1_routes]
    lp, ids = batch_parent_token_candidates(stage1_last_logits, k=k, sampling=sampling, relative_parent_paths=rel)
    kk = int(ids.shape[-1])
    pairs = topk_pairs_to_python(ids, lp)
    out: list[RouteState] = []
    for row, parent in enumerate(stage1_routes):
        for rank in range(kk):
            tok, tlp = pairs[row * kk + rank]
            out.append(
                route_store.register_route(
                    RouteState(
                        route_id=route_store.allocate_route_id(),
                        stage1_root_id=parent.route_id,
                        parent_route_id=parent.route_id,
                        materialized_leaf_node_id=parent.materialized_leaf_node_id,
                        pending_token_id=tok,
                        cumulative_logprob=parent.cumulative_logprob + tlp,
                        stage1_depth=parent.stage1_depth,
                        stage2_depth=0,
                        kv_view=parent.kv_view.fork(),
                        token_logprobs=(*parent.token_logprobs, float(tlp)),
                    )
                )
            )
    return out


def build_forest_one_depth(
    active_routes: Sequence[RouteState],
    *,
    k: int,
    route_store: KVTreeStore,
    model_backend: FrontierModelBackend,
    attention_backend: Any = None,
    sampling: DrafterSamplingContext | None = None,
) -> FrontierStepOutput:
    if len(active_routes) != k * k:
        raise ValueError(f"build_forest_one_depth expects {k * k} active routes, got {len(active_routes)}")
    return advance_frontier_one_token(
        active_routes,
        k=k,
        route_store=route_store,
        model_backend=model_backend,
        selection_policy=PerStage1RootTopKSelection(phase=DecodePhase.STAGE2),
        attention_backend=attention_backend,
        sampling=sampling,
    )


def build_forest_depths(
    active_routes: Sequence[RouteState],
    *,
    depth: int,
    k: int,
    route_store: KVTreeStore,
    model_backend: FrontierModelBackend,
    attention_backend: Any = None,
    sampling: DrafterSamplingContext | None = None,
) -> BuildDepthsOutput:
    return _depths(
        build_forest_one_depth,
        active_routes,
        depth,
        k=k,
        route_store=route_store,
        model_backend=model_backend,
        attention_backend=attention_backend,
        sampling=sampling,
    )


def select_routes_by_stage1_root(routes: Sequence[RouteState], selected_stage1_root_id: int) -> list[RouteState]:
    return [r for r in routes if r.stage1_root_id == selected_stage1_root_id]


def collect_final_pending_candidates(completed_routes, last_logits, *, k: int) -> list[PendingCandidate]:
    return collect_pending_candidates(completed_routes, last_logits, k=k)
