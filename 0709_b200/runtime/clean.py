"""Clean controller: the tree/forest/verify race without physical KV.

Backends implement ``prefill(tokens) -> PrefixState`` and
``decode_batch(prefix_token_ids, routes)`` / ``verify_batch(prefix_token_ids,
routes)`` over plain token paths.  ``DeterministicMockBackend`` produces logits
from a hash of the full context, so runs are exactly reproducible on CPU; the
controller re-prefills the Target every round (it has no persistent KV).

Parity: reference src/atlas_0709/controller.py:16-239, backends.py:37-126,
route_store.py:9-113, builders.py:13-195 (clean variants).
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Protocol, Sequence

import torch

from ..types import DecodePhase, PendingCandidate, PrefixState, TargetRouteScore, TargetVerifyResult


@dataclass(frozen=True)
class CleanRoute:
    route_id: int
    stage1_root_id: int
    parent_route_id: int | None
    materialized_tokens: tuple[int, ...]
    pending_token_id: int
    cumulative_logprob: float
    stage1_depth: int
    stage2_depth: int

    @property
    def pending_path(self) -> tuple[int, ...]:
        return (*self.materialized_tokens, int(self.pending_token_id))


@dataclass(frozen=True)
class BatchDecodeOutput:
    route_ids: tuple[int, ...]
    logits: torch.Tensor
    metadata: dict = field(default_factory=dict)


@dataclass(frozen=True)
class BuildResult:
    completed_routes: list[CleanRoute]
    next_frontier_routes: list[CleanRoute]
    last_logits: torch.Tensor


@dataclass(frozen=True)
class RoundTrace:
    round_index: int
    selected_route_id: int
    committed_tokens: tuple[int, ...]
    forest_depth: int
    verify_returned_before_forest_done: bool
    target_scores: tuple[tuple[int, float], ...]


class BatchDecodeBackend(Protocol):
    def prefill(self, prompt_token_ids: Sequence[int]) -> PrefixState: ...

    def decode_batch(self, *, prefix_token_ids: Sequence[int], routes: Sequence[CleanRoute]) -> BatchDecodeOutput: ...


class DeterministicMockBackend:
    """Logits are a pure function of the whole context (position-weighted token sum)."""

    def __init__(self, *, name: str, vocab_size: int = 128, salt: int = 0) -> None:
        self.name = name
        self.vocab_size = int(vocab_size)
        self.salt = int(salt)

    def logits_for_context(self, tokens: Sequence[int]) -> torch.Tensor:
        v = self.vocab_size
        total = sum((i + 1) * int(t) for i, t in enumerate(tokens))
        center = (total + self.salt + 17 * len(tokens)) % v
        ids = torch.arange(v, dtype=torch.float32)
        logits = -0.03 * torch.remainder(torch.abs(ids - center), v)
        for rank in range(min(8, v)):
            logits[(center + rank * 7 + self.salt) % v] += 2.0 - rank * 0.1
        return logits

    def prefill(self, prompt_token_ids: Sequence[int]) -> PrefixState:
        toks = tuple(int(t) for t in prompt_token_ids)
        return PrefixState(toks, self.logits_for_context(toks), len(toks), {"backend": "deterministic_mock", "name": self.name})

    def decode_batch(self, *, prefix_token_ids, routes) -> BatchDecodeOutput:
        base = tuple(int(t) for t in prefix_token_ids)
        rows = [self.logits_for_context((*base, *r.pending_path)) for r in routes]
        return BatchDecodeOutput(tuple(r.route_id for r in routes), torch.stack(rows), {"backend": "deterministic_mock"})

    def verify_batch(self, *, prefix_token_ids, routes) -> TargetVerifyResult:
        prefix = tuple(int(t) for t in prefix_token_ids)
        scores = []
        for r in routes:
            path = r.materialized_tokens[: r.stage1_depth]
            ctx, total = prefix, 0.0
            for t in path:
                lp = torch.log_softmax(self.logits_for_context(ctx), -1)
                total += float(lp[int(t)])
                ctx = (*ctx, int(t))
            scores.append(TargetRouteScore(r.route_id, tuple(path), total, r.cumulative_logprob))
        best = max(scores, key=lambda s: (s.target_logprob, s.draft_logprob, -s.route_id))
        return TargetVerifyResult(best.route_id, scores, {"backend": "deterministic_mock"})


class RouteStore:
    def __init__(self) -> None:
        self._next = 1
        self.routes: dict[int, CleanRoute] = {}

    def reset(self) -> None:
        self.routes.clear()

    def new_id(self) -> int:
        self._next += 1
        return self._next - 1

    def register(self, r: CleanRoute) -> CleanRoute:
        self.routes[r.route_id] = r
        return r

    def get(self, rid: int) -> CleanRoute:
        return self.routes[int(rid)]


def _topk(logits: torch.Tensor, k: int):
    return torch.topk(torch.log_softmax(logits.float(), -1), k=min(int(k), logits.shape[-1]), dim=-1)


def _order(c: PendingCandidate):
    return (-c.cumulative_logprob, c.parent_route_id, c.rank_in_parent)


def _step(routes, *, prefix, k, store: RouteStore, drafter, phase: DecodePhase, per_root: bool):
    out = drafter.decode_batch(prefix_token_ids=prefix, routes=routes)
    decoded = []
    for r in routes:
        s1, s2 = (r.stage1_depth + 1, r.stage2_depth) if phase == DecodePhase.STAGE1 else (r.stage1_depth, r.stage2_depth + 1)
        decoded.append(store.register(CleanRoute(r.route_id, r.stage1_root_id, r.parent_route_id, r.pending_path,
                                                 r.pending_token_id, r.cumulative_logprob, s1, s2)))
    lp, ids = _topk(out.logits, k)
    cands = [
        PendingCandidate(d.route_id, d.stage1_root_id, int(ids[i, j]), d.cumulative_logprob + float(lp[i, j]), j)
        for i, d in enumerate(decoded)
        for j in range(ids.shape[1])
    ]
    if per_root:
        sel = []
        for root in sorted({r.stage1_root_id for r in routes}):
            sel += sorted([c for c in cands if c.stage1_root_id == root], key=_order)[:k]
    else:
        sel = sorted(cands, key=_order)[:k]
    parents = {d.route_id: d for d in decoded}
    nxt = [
        store.register(CleanRoute(store.new_id(), c.stage1_root_id, c.parent_route_id,
                                  parents[c.parent_route_id].materialized_tokens, c.pending_token_id,
                                  c.cumulative_logprob, parents[c.parent_route_id].stage1_depth,
                                  parents[c.parent_route_id].stage2_depth))
        for c in sel
    ]
    return decoded, nxt, out.logits


def build_tree(routes, *, prefix, depth, k, store, drafter) -> BuildResult:
    frontier = list(routes)
    decoded, logits = [], None
    for _ in range(depth):
        decoded, frontier, logits = _step(frontier, prefix=prefix, k=k, store=store, drafter=drafter,
                                          phase=DecodePhase.STAGE1, per_root=False)
    return BuildResult(decoded, frontier, logits)


@dataclass(frozen=True)
class AtlasCleanConfig:
    k: int = 3
    d: int = 4
    max_new_tokens: int = 64
    eos_token_id: int | None = None

    def validate(self) -> None:
        if self.k <= 0 or self.d <= 0 or self.max_new_tokens <= 0:
            raise ValueError("k, d and max_new_tokens must be positive")


@dataclass
class GenerationResult:
    prompt_token_ids: tuple[int, ...]
    generated_token_ids: list[int]
    rounds: list[RoundTrace] = field(default_factory=list)

    @property
    def token_ids(self) -> list[int]:
        return [*self.prompt_token_ids, *self.generated_token_ids]


class AtlasCleanGenerator:
    def __init__(self, *, config: AtlasCleanConfig, drafter, target) -> None:
        config.validate()
        self.config, self.drafter, self.target = config, drafter, target
        self.store = RouteStore()

    def _init_stage1(self, prefix_state: PrefixState) -> list[CleanRoute]:
        lp, ids = _topk(prefix_state.next_token_logits, self.config.k)
        out = []
        for t, l in zip(ids.tolist(), lp.tolist()):
            rid = self.store.new_id()
            out.append(self.store.register(CleanRoute(rid, rid, None, (), int(t), float(l), 0, 0)))
        return out

    def _init_forest(self, stage1: BuildResult) -> list[CleanRoute]:
        lp, ids = _topk(stage1.last_logits, self.config.k)
        out = []
        for i, r in enumerate(stage1.completed_routes):
            for j in range(ids.shape[1]):
                out.append(self.store.register(CleanRoute(self.store.new_id(), r.route_id, r.route_id,
                                                          r.materialized_tokens, int(ids[i, j]),
                                                          r.cumulative_logprob + float(lp[i, j]), r.stage1_depth, 0)))
        return out

    def _promote(self, sel: CleanRoute, routes) -> list[CleanRoute]:
        pre = sel.materialized_tokens[: sel.stage1_depth]
        out = []
        for r in routes:
            if r.materialized_tokens[: len(pre)] != pre:
                raise RuntimeError("only routes under the selected stage-1 route can be promoted")
            out.append(self.store.register(CleanRoute(r.route_id, r.route_id, None, r.materialized_tokens[len(pre):],
                                                      r.pending_token_id, r.cumulative_logprob, r.stage2_depth, 0)))
        return out

    def generate(self, prompt_token_ids: Sequence[int]) -> GenerationResult:
        cfg = self.config
        committed = [int(t) for t in prompt_token_ids]
        generated: list[int] = []
        traces: list[RoundTrace] = []
        self.store.reset()
        with ThreadPoolExecutor(max_workers=2) as pool:
            fd = pool.submit(self.drafter.prefill, tuple(committed))
            ft = pool.submit(self.target.prefill, tuple(committed))
            dstate, _ = fd.result(), ft.result()
        stage1 = build_tree(self._init_stage1(dstate), prefix=committed, depth=cfg.d, k=cfg.k, store=self.store,
                            drafter=self.drafter)
        with ThreadPoolExecutor(max_workers=1) as vp:
            rnd = 0
            while len(generated) < cfg.max_new_tokens:
                fut = vp.submit(self.target.verify_batch, prefix_token_ids=tuple(committed),
                                routes=list(stage1.completed_routes))
                frontier = self._init_forest(stage1)
                done, last, depth = None, None, 0
                while not fut.done() and depth < cfg.d:
                    done, frontier, last = _step(frontier, prefix=committed, k=cfg.k, store=self.store,
                                                 drafter=self.drafter, phase=DecodePhase.STAGE2, per_root=True)
                    depth += 1
                early = depth < cfg.d and fut.done()
                res = fut.result()
                sel = self.store.get(res.selected_route_id)
                path = list(sel.materialized_tokens[: sel.stage1_depth])[: cfg.max_new_tokens - len(generated)]
                if cfg.eos_token_id is not None and cfg.eos_token_id in path:
                    path = path[: path.index(cfg.eos_token_id) + 1]
                generated.extend(path)
                committed.extend(path)
                traces.append(RoundTrace(rnd, res.selected_route_id, tuple(path), depth, early,
                                         tuple((s.route_id, s.target_logprob) for s in res.scores)))
                rnd += 1
                if len(generated) >= cfg.max_new_tokens or (
                    cfg.eos_token_id is not None and cfg.eos_token_id in path
                ):
                    break
                self.target.prefill(tuple(committed))
                nxt = None
                if depth >= cfg.d and done is not None:
                    idx = [i for i, r in enumerate(done) if r.stage1_root_id == sel.route_id]
                    if len(idx) == cfg.k:
                        nxt = BuildResult(self._promote(sel, [done[i] for i in idx]), [], last[idx])
                elif depth < cfg.d:
                    keep = [r for r in frontier if r.stage1_root_id == sel.route_id]
                    if len(keep) == cfg.k:
                        pr = self._promote(sel, keep)
                        nxt = build_tree(pr, prefix=committed, depth=cfg.d - pr[0].stage1_depth, k=cfg.k,
                                         store=self.store, drafter=self.drafter)
                if nxt is None:
                    self.store.reset()
                    nxt = build_tree(self._init_stage1(self.drafter.prefill(committed)), prefix=committed,
                                     depth=cfg.d, k=cfg.k, store=self.store, drafter=self.drafter)
                stage1 = nxt
        return GenerationResult(tuple(int(t) for t in prompt_token_ids), generated, traces)
