"""Speculative tree state of one drafter session: a node arena plus the live routes.

Nodes are the drafted tokens whose KV has been written.  They live in an
append-only arena of parallel lists (token, parent node, depth, stage-1 root)
addressed by ``node_id - base``; a depth's node ids are reserved in one block
when the drafter launches its decode, and filled in when the step's routes
``grow``.  Nothing is deleted while a round runs: dead branches simply stop
being referenced, and on a commit the arena is cut below the survivors'
oldest node -- a few hundred list entries per round instead of per-node
objects that are created and freed.  Node ids never repeat.

Routes are ``RouteState`` records (the public route type).  The store gives
them ids, grows them by one node, spawns children from selected candidates,
and on a commit moves the committed route's tokens into the prefix and
rebases the surviving stage-2 routes onto it.  Physical KV (pages, tail
copy-on-write) is the native ``RoutePool``'s business; listeners registered
with ``on_spawn`` learn about new children so the pool can fork their views.

Behaviour matches the reference's tree store (src/atlas_0709/flashinfer_paged/kv.py:21-258):
the same ids, per-token draft log-probs relative to the committed prefix,
commit semantics and stage-2 -> stage-1 rebasing.
"""

from __future__ import annotations

from typing import Callable, Iterable, Sequence

from ..types import DecodePhase, PendingCandidate, PrefixKVView, RouteKVView, RouteState

SpawnListener = Callable[[Sequence[RouteState]], None]
_HOLE = -1  # arena slot reserved for a node that has not grown yet


class KVTreeStore:
    def __init__(self) -> None:
        self.committed_token_ids: list[int] = []
        self.routes: dict[int, RouteState] = {}
        self._route_ids = 0
        self._base = 1          # node id of arena slot 0
        self._tok: list[int] = []
        self._parent: list[int] = []
        self._depth: list[int] = []
        self._root: list[int] = []
        self._listeners: list[SpawnListener] = []

    # ------------------------------------------------------------- ids
    def allocate_route_id(self) -> int:
        self._route_ids += 1
        return self._route_ids

    def reserve_node_ids(self, count: int) -> list[int]:
        """Reserve ``count`` consecutive node ids (one decode step's nodes)."""
        first = self._base + len(self._tok)
        n = int(count)
        self._tok.extend([_HOLE] * n)
        self._parent.extend([_HOLE] * n)
        self._depth.extend([0] * n)
        self._root.extend([0] * n)
        return list(range(first, first + n))

    @property
    def arena_size(self) -> int:
        return len(self._tok)

    def on_spawn(self, listener: SpawnListener) -> None:
        self._listeners.append(listener)

    # ------------------------------------------------------------ views
    def prefix_view(self, committed_length: int | None = None) -> PrefixKVView:
        n = len(self.committed_token_ids) if committed_length is None else int(committed_length)
        return PrefixKVView(committed_length=n)

    def node_token(self, node_id: int) -> int:
        tok = self._tok[int(node_id) - self._base]
        if tok == _HOLE:
            raise KeyError(f"node {node_id} was reserved but never grown")
        return tok

    def node_parent(self, node_id: int) -> int | None:
        p = self._parent[int(node_id) - self._base]
        return None if p == _HOLE else p

    def tokens_for_node_ids(self, node_ids: Iterable[int]) -> tuple[int, ...]:
        base, tok = self._base, self._tok
        return tuple(tok[int(n) - base] for n in node_ids)

    def materialized_token_path(self, route: RouteState) -> tuple[int, ...]:
        """Tokens of the route's grown nodes (relative to the committed prefix)."""
        return self.tokens_for_node_ids(route.kv_view.node_ids)

    def pending_token_path(self, route: RouteState) -> tuple[int, ...]:
        """Grown tokens followed by the route's pending token."""
        return (*self.materialized_token_path(route), int(route.pending_token_id))

    # ----------------------------------------------------------- routes
    def new_route(self, *, root: int | None, parent: RouteState | None, token: int, token_logprob: float,
                  prefix: PrefixKVView | None = None) -> RouteState:
        """A route one pending token beyond ``parent`` (or beyond the committed prefix when ``parent`` is None).

        A route without a parent is its own stage-1 root; a child takes ``root``
        (default: its parent's root).
        """
        rid = self.allocate_route_id()
        if parent is None:
            view = (prefix or self.prefix_view()).fork()
            route = RouteState(route_id=rid, stage1_root_id=rid if root is None else int(root), parent_route_id=None,
                               materialized_leaf_node_id=None, pending_token_id=int(token),
                               cumulative_logprob=float(token_logprob), stage1_depth=0, stage2_depth=0, kv_view=view,
                               token_logprobs=(float(token_logprob),))
        else:
            route = RouteState(
                route_id=rid,
                stage1_root_id=int(parent.stage1_root_id if root is None else root),
                parent_route_id=int(parent.route_id),
                materialized_leaf_node_id=parent.materialized_leaf_node_id,
                pending_token_id=int(token),
                cumulative_logprob=float(parent.cumulative_logprob) + float(token_logprob),
                stage1_depth=int(parent.stage1_depth),
                stage2_depth=int(parent.stage2_depth),
                kv_view=parent.kv_view.fork(),
                token_logprobs=(*parent.token_logprobs, float(token_logprob)) if parent.token_logprobs else (),
            )
        self.routes[rid] = route
        return route

    def get_route(self, route_id: int) -> RouteState:
        return self.routes[int(route_id)]

    def grow(self, routes: Sequence[RouteState], node_ids: Sequence[int], phase: DecodePhase) -> list[RouteState]:
        """Each route's pending token became node ``node_ids[i]`` (its KV is written); extend the routes."""
        if len(routes) != len(node_ids):
            raise ValueError(f"{len(routes)} routes grew but {len(node_ids)} node ids were reserved")
        stage2 = phase == DecodePhase.STAGE2
        if not stage2 and phase != DecodePhase.STAGE1:
            raise ValueError(f"unknown decode phase {phase!r}")
        base = self._base
        for route, nid in zip(routes, node_ids):
            depth = int(route.stage1_depth) + int(route.stage2_depth) + 1
            if route.token_logprobs and len(route.token_logprobs) != depth:
                raise ValueError(
                    f"route {route.route_id} carries {len(route.token_logprobs)} draft log-probs; growing it to "
                    f"depth {depth} needs exactly one per token including the pending one")
            slot = int(nid) - base
            if not 0 <= slot < len(self._tok) or self._tok[slot] != _HOLE:
                raise ValueError(f"node id {nid} is not a reserved, unused slot")
            leaf = route.materialized_leaf_node_id
            self._tok[slot] = int(route.pending_token_id)
            self._parent[slot] = _HOLE if leaf is None else int(leaf)
            self._depth[slot] = depth
            self._root[slot] = int(route.stage1_root_id)
            route.materialized_leaf_node_id = int(nid)
            route.kv_view = route.kv_view.append_node(int(nid))
            if stage2:
                route.stage2_depth += 1
            else:
                route.stage1_depth += 1
        return list(routes)

    def spawn(self, picks: Sequence[PendingCandidate], parents: Sequence[RouteState]) -> list[RouteState]:
        """One child route per picked candidate, forked from its (just grown) parent."""
        by_id = {int(r.route_id): r for r in parents}
        children: list[RouteState] = []
        for c in picks:
            parent = by_id.get(int(c.parent_route_id))
            if parent is None:
                parent = self.get_route(c.parent_route_id)
            grown = int(parent.stage1_depth) + int(parent.stage2_depth)
            if parent.token_logprobs and len(parent.token_logprobs) != grown:
                raise ValueError(f"parent route {parent.route_id} has {len(parent.token_logprobs)} draft "
                                 f"log-probs for {grown} grown tokens")
            children.append(self.new_route(root=c.stage1_root_id, parent=parent, token=c.pending_token_id,
                                           token_logprob=float(c.cumulative_logprob) - float(c.parent_logprob)))
        for listener in self._listeners:
            listener(children)
        return children

    # -------------------------------------------------- commit / rebase
    def advance_prefix(self, route: RouteState, survivors: Sequence[RouteState], *,
                       max_tokens: int | None = None) -> tuple[tuple[int, ...], list[RouteState]]:
        """Commit ``route``'s grown tokens and rebase ``survivors`` (its stage-2 descendants) onto them.

        Returns the committed tokens and the rebased routes, which are now
        stage-1 routes of the longer prefix: their node paths, depths and draft
        log-probs lose the committed part, and each becomes its own root.
        Every other route is forgotten and the arena below the survivors'
        oldest node is released.
        """
        path = tuple(route.kv_view.node_ids)
        if max_tokens is not None:
            path = path[: int(max_tokens)]
        tokens = self.tokens_for_node_ids(path)
        self.committed_token_ids.extend(tokens)
        cut = len(path)
        prefix = self.prefix_view()
        for r in survivors:
            nodes = tuple(r.kv_view.node_ids)
            if nodes[:cut] != path:
                raise ValueError(f"route {r.route_id} does not descend from the committed route {route.route_id}")
            if r.token_logprobs:
                grown = int(r.stage1_depth) + int(r.stage2_depth)
                if len(r.token_logprobs) - grown not in (0, 1):
                    raise ValueError(f"route {r.route_id}: {len(r.token_logprobs)} draft log-probs for {grown} "
                                     "grown tokens")
                r.token_logprobs = tuple(r.token_logprobs[cut:])
            rest = nodes[cut:]
            r.kv_view = RouteKVView(prefix=prefix, node_ids=rest)
            r.materialized_leaf_node_id = rest[-1] if rest else None
            r.stage1_depth, r.stage2_depth = int(r.stage2_depth), 0
            r.stage1_root_id = int(r.route_id)
            r.parent_route_id = None
        self._release_below(survivors)
        self.routes = {int(r.route_id): r for r in survivors}
        return tokens, list(survivors)

    def reset_speculative(self) -> None:
        """Forget every route and node (the committed prefix stays)."""
        self.routes.clear()
        self._release_below(())

    def _release_below(self, survivors: Sequence[RouteState]) -> None:
        oldest = min((int(n) for r in survivors for n in r.kv_view.node_ids), default=None)
        cut = len(self._tok) if oldest is None else oldest - self._base
        if cut > 0:
            del self._tok[:cut], self._parent[:cut], self._depth[:cut], self._root[:cut]
            self._base += cut
