"""Logical route/tree topology.

Tracks tree nodes (token, parent, depth, stage-1 root) and live routes. Physical
KV placement is owned by the native page pool (``runtime.kv_pool``); the store
only hands out node ids and route ids and rebases routes after a commit.

Behavioural parity: reference src/atlas_0709/flashinfer_paged/kv.py:21-258
(node materialization, descriptor fork with per-token log-probs, commit, and
promotion that rebases ``stage2_depth -> stage1_depth``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Iterable, Sequence

from ..types import DecodePhase, PendingCandidate, PrefixKVView, RouteKVView, RouteState


@dataclass
class TreeNode:
    node_id: int
    token_id: int
    parent_node_id: int | None
    stage1_root_id: int
    depth: int
    owner_route_id: int | None = None
    committed: bool = False


ReleaseHook = Callable[[Sequence[RouteState], Sequence[RouteState]], None]


class KVTreeStore:
    def __init__(self) -> None:
        self._next_route_id = 1
        self._next_node_id = 1
        self.nodes: dict[int, TreeNode] = {}
        self.routes: dict[int, RouteState] = {}
        self.committed_token_ids: list[int] = []
        self._release_hooks: list[ReleaseHook] = []

    # ---------------------------------------------------------------- ids
    def allocate_route_id(self) -> int:
        rid = self._next_route_id
        self._next_route_id += 1
        return rid

    def allocate_node_id(self) -> int:
        nid = self._next_node_id
        self._next_node_id += 1
        return nid

    def reserve_node_ids(self, count: int) -> list[int]:
        start = self._next_node_id
        self._next_node_id += int(count)
        return list(range(start, start + int(count)))

    def peek_next_node_id(self) -> int:
        return self._next_node_id

    # ------------------------------------------------------------ routes
    def reset_speculative(self) -> None:
        self.nodes.clear()
        self.routes.clear()

    def add_route_release_hook(self, hook: ReleaseHook) -> None:
        self._release_hooks.append(hook)

    def prefix_view(self, committed_length: int | None = None) -> PrefixKVView:
        n = len(self.committed_token_ids) if committed_length is None else int(committed_length)
        return PrefixKVView(committed_length=n)

    def register_route(self, route: RouteState) -> RouteState:
        self.routes[int(route.route_id)] = route
        return route

    def get_route(self, route_id: int) -> RouteState:
        return self.routes[int(route_id)]

    def get_routes(self, route_ids: Iterable[int]) -> list[RouteState]:
        return [self.get_route(r) for r in route_ids]

    def mark_routes_materialized(
        self,
        routes: Sequence[RouteState],
        new_node_ids: Sequence[int],
        phase: DecodePhase,
    ) -> list[RouteState]:
        """Turn each route's pending token into a tree node (its KV was just written)."""
        if len(routes) != len(new_node_ids):
            raise ValueError("routes and new_node_ids must have the same length")
        out: list[RouteState] = []
        for route, raw in zip(routes, new_node_ids):
            nid = int(raw)
            next_depth = route.total_materialized_depth() + 1
            if route.token_logprobs and len(route.token_logprobs) != next_depth:
                raise ValueError(
                    "frontier route token_logprobs must include exactly its pending token: "
                    f"route_id={route.route_id}, logprobs={len(route.token_logprobs)}, "
                    f"next_materialized_depth={next_depth}"
                )
            parent = route.kv_view.node_ids[-1] if route.kv_view.node_ids else None
            self.nodes[nid] = TreeNode(
                node_id=nid,
                token_id=int(route.pending_token_id),
                parent_node_id=parent,
                stage1_root_id=route.stage1_root_id,
                depth=next_depth,
                owner_route_id=route.route_id,
            )
            route.materialized_leaf_node_id = nid
            route.kv_view = route.kv_view.append_node(nid)
            if phase == DecodePhase.STAGE1:
                route.stage1_depth += 1
            elif phase == DecodePhase.STAGE2:
                route.stage2_depth += 1
            else:  # pragma: no cover - enum exhausted
                raise ValueError(f"unsupported decode phase: {phase}")
            self.register_route(route)
            out.append(route)
        return out

    def materialize_route_descriptors(
        self,
        selected: Sequence[PendingCandidate],
        parent_routes: Sequence[RouteState],
    ) -> list[RouteState]:
        """Create one child route per selected candidate, forking its parent's view."""
        parents = {r.route_id: r for r in parent_routes}
        out: list[RouteState] = []
        for cand in selected:
            parent = parents.get(cand.parent_route_id) or self.get_route(cand.parent_route_id)
            if parent.token_logprobs and len(parent.token_logprobs) != parent.total_materialized_depth():
                raise ValueError(
                    "decoded parent token_logprobs must match its materialized path: "
                    f"route_id={parent.route_id}, logprobs={len(parent.token_logprobs)}, "
                    f"materialized_depth={parent.total_materialized_depth()}"
                )
            local = float(cand.cumulative_logprob - cand.parent_logprob)
            child = RouteState(
                route_id=self.allocate_route_id(),
                stage1_root_id=cand.stage1_root_id,
                parent_route_id=parent.route_id,
                materialized_leaf_node_id=parent.materialized_leaf_node_id,
                pending_token_id=int(cand.pending_token_id),
                cumulative_logprob=float(cand.cumulative_logprob),
                stage1_depth=parent.stage1_depth,
                stage2_depth=parent.stage2_depth,
                kv_view=parent.kv_view.fork(),
                token_logprobs=(*parent.token_logprobs, local) if parent.token_logprobs else (),
            )
            out.append(self.register_route(child))
        return out

    def release_routes_without_descendants(
        self, previous_routes: Sequence[RouteState], next_routes: Sequence[RouteState]
    ) -> None:
        """Notify physical backends that parents without selected children can go."""
        for hook in self._release_hooks:
            hook(previous_routes, next_routes)

    # ------------------------------------------------------------- paths
    def tokens_for_node_ids(self, node_ids: Sequence[int]) -> tuple[int, ...]:
        return tuple(self.nodes[int(n)].token_id for n in node_ids)

    def materialized_token_path(self, route: RouteState) -> tuple[int, ...]:
        return self.tokens_for_node_ids(route.kv_view.node_ids)

    def node_path_for_route(self, route: RouteState) -> tuple[int, ...]:
        return tuple(route.kv_view.node_ids)

    def pending_token_path(self, route: RouteState) -> tuple[int, ...]:
        return (*self.materialized_token_path(route), int(route.pending_token_id))

    # ------------------------------------------------------ commit/promote
    def commit_route(self, route: RouteState, max_tokens: int | None = None) -> tuple[int, ...]:
        nodes = self.node_path_for_route(route)
        if max_tokens is not None:
            nodes = nodes[: int(max_tokens)]
        for n in nodes:
            self.nodes[n].committed = True
        tokens = self.tokens_for_node_ids(nodes)
        self.committed_token_ids.extend(tokens)
        return tokens

    def promote_routes_after_commit(
        self,
        committed_route: RouteState,
        routes: Sequence[RouteState],
        new_prefix: PrefixKVView,
    ) -> list[RouteState]:
        """Rebase stage-2 routes of the selected root so they become stage-1 routes."""
        committed = self.node_path_for_route(committed_route)
        out: list[RouteState] = []
        for route in routes:
            nodes = route.kv_view.node_ids
            if nodes[: len(committed)] != committed:
                raise ValueError("cannot promote a route outside the committed branch")
            if route.token_logprobs:
                depth = route.total_materialized_depth()
                if len(route.token_logprobs) not in (depth, depth + 1):
                    raise ValueError(
                        "promoted route token_logprobs do not match its token path: "
                        f"route_id={route.route_id}, logprobs={len(route.token_logprobs)}"
                    )
                route.token_logprobs = tuple(route.token_logprobs[len(committed):])
            suffix = tuple(nodes[len(committed):])
            route.kv_view = RouteKVView(prefix=new_prefix, node_ids=suffix)
            route.materialized_leaf_node_id = suffix[-1] if suffix else None
            route.stage1_depth = route.stage2_depth
            route.stage2_depth = 0
            route.stage1_root_id = route.route_id
            route.parent_route_id = None
            out.append(self.register_route(route))
        return out
