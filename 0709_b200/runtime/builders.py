"""Stage-1 trees and stage-2 forests built from frontier depths.

Everything here is one of two moves over ``KVTreeStore``:

* ``seed``: open ``k`` routes per parent from already decoded logits -- the
  committed prefix's logits for a stage-1 tree (the parent is the prefix), or
  the last logits of the ``k`` completed stage-1 routes for a forest (each
  completed route becomes the stage-1 root of its ``k`` children);
* ``grow``: one frontier depth (``frontier.advance_frontier_one_token``) with
  the tree's or the forest's selection policy, repeated ``depth`` times.

Shapes: a tree keeps ``k`` routes at every depth (batch-``k`` decodes), a
forest ``k^2`` (batch-``k^2`` decodes, best ``k`` per root).

Behaviour matches the reference's builders (src/atlas_0709/flashinfer_paged/builders.py:31-261).
"""

from __future__ import annotations

from typing import Any, Sequence

import torch

from ..types import BuildDepthsOutput, DecodePhase, DraftPrefixState, FrontierStepOutput, RouteState
from .frontier import (BestKOverall, BestKPerRoot, FrontierModelBackend, advance_frontier_one_token,
                       backend_status, propose_children)
from .sampling import DrafterSamplingContext
from .store import KVTreeStore

TREE = BestKOverall()
FOREST = BestKPerRoot()


def initialize_stage1_routes(
    draft_prefix_state: DraftPrefixState,
    *,
    k: int,
    route_store: KVTreeStore,
    sampling: DrafterSamplingContext | None = None,
    model_backend: FrontierModelBackend | None = None,
) -> list[RouteState]:
    """``k`` stage-1 routes seeded from the committed prefix's next-token logits (one pending token each)."""
    cands, _ = propose_children([None], draft_prefix_state.next_token_logits, k=k, sampling=sampling,
                                history=lambda _p: (), status=backend_status(model_backend),
                                readout=getattr(draft_prefix_state, "candidates", None))
    prefix = draft_prefix_state.prefix_kv_view
    return [route_store.new_route(root=None, parent=None, token=c.pending_token_id,
                                  token_logprob=c.cumulative_logprob, prefix=prefix) for c in cands]


def initialize_forest_routes(
    stage1_routes: Sequence[RouteState],
    stage1_last_logits: torch.Tensor,
    *,
    k: int,
    route_store: KVTreeStore,
    sampling: DrafterSamplingContext | None = None,
    model_backend: FrontierModelBackend | None = None,
) -> list[RouteState]:
    """``k`` stage-2 children of every completed stage-1 route; each completed route is their root."""
    if len(stage1_routes) != int(stage1_last_logits.shape[0]):
        raise ValueError(f"{len(stage1_routes)} completed stage-1 routes but {int(stage1_last_logits.shape[0])} "
                         "rows of last logits")
    cands, _ = propose_children(list(stage1_routes), stage1_last_logits, k=k, sampling=sampling,
                                history=route_store.materialized_token_path, status=backend_status(model_backend),
                                root_of=lambda r: r.route_id)
    by_id = {int(r.route_id): r for r in stage1_routes}
    return [route_store.new_route(root=c.stage1_root_id, parent=by_id[c.parent_route_id], token=c.pending_token_id,
                                  token_logprob=c.cumulative_logprob - c.parent_logprob) for c in cands]


def _grow(routes, depth: int, *, k: int, width: int, policy, route_store, model_backend, attention_backend,
          sampling) -> BuildDepthsOutput:
    if int(depth) < 1:
        raise ValueError(f"cannot build {depth} depths")
    steps: list[FrontierStepOutput] = []
    front = list(routes)
    for _ in range(int(depth)):
        if len(front) != width:
            raise ValueError(f"a depth of this build decodes {width} routes; {len(front)} are active")
        step = advance_frontier_one_token(front, k=k, route_store=route_store, model_backend=model_backend,
                                          selection_policy=policy, attention_backend=attention_backend,
                                          sampling=sampling)
        steps.append(step)
        front = step.next_routes
    last = steps[-1]
    return BuildDepthsOutput(completed_routes=last.decoded_routes, next_frontier_routes=last.next_routes,
                             last_logits=last.decode_output.next_token_logits, steps=steps)


def _tree_policy(phase: DecodePhase) -> BestKOverall:
    return TREE if phase == DecodePhase.STAGE1 else BestKOverall(phase=phase)


def build_tree_one_depth(active_routes: Sequence[RouteState], *, k: int, route_store: KVTreeStore,
                         model_backend: FrontierModelBackend, attention_backend: Any = None,
                         phase: DecodePhase = DecodePhase.STAGE1,
                         sampling: DrafterSamplingContext | None = None) -> FrontierStepOutput:
    """One stage-1 depth: decode the ``k`` routes and keep the best ``k`` children overall."""
    return _grow(active_routes, 1, k=k, width=k, policy=_tree_policy(phase), route_store=route_store,
                 model_backend=model_backend, attention_backend=attention_backend, sampling=sampling).steps[0]


def build_tree_depths(active_routes: Sequence[RouteState], *, depth: int, k: int, route_store: KVTreeStore,
                      model_backend: FrontierModelBackend, attention_backend: Any = None,
                      phase: DecodePhase = DecodePhase.STAGE1,
                      sampling: DrafterSamplingContext | None = None) -> BuildDepthsOutput:
    return _grow(active_routes, depth, k=k, width=k, policy=_tree_policy(phase), route_store=route_store,
                 model_backend=model_backend, attention_backend=attention_backend, sampling=sampling)


def build_forest_one_depth(active_routes: Sequence[RouteState], *, k: int, route_store: KVTreeStore,
                           model_backend: FrontierModelBackend, attention_backend: Any = None,
                           sampling: DrafterSamplingContext | None = None) -> FrontierStepOutput:
    """One stage-2 depth: decode the ``k^2`` routes and keep the best ``k`` children per root."""
    return _grow(active_routes, 1, k=k, width=k * k, policy=FOREST, route_store=route_store,
                 model_backend=model_backend, attention_backend=attention_backend, sampling=sampling).steps[0]


def build_forest_depths(active_routes: Sequence[RouteState], *, depth: int, k: int, route_store: KVTreeStore,
                        model_backend: FrontierModelBackend, attention_backend: Any = None,
                        sampling: DrafterSamplingContext | None = None) -> BuildDepthsOutput:
    return _grow(active_routes, depth, k=k, width=k * k, policy=FOREST, route_store=route_store,
                 model_backend=model_backend, attention_backend=attention_backend, sampling=sampling)


def select_routes_by_stage1_root(routes: Sequence[RouteState], selected_stage1_root_id: int) -> list[RouteState]:
    """The routes under one stage-1 root (the forest part that survives a selection)."""
    root = int(selected_stage1_root_id)
    return [r for r in routes if int(r.stage1_root_id) == root]
