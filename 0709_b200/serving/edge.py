"""Asynchronous tree/forest coordinator (the Edge/Drafter side).

Round structure: send the k stage-1 paths to the Target; while it verifies,
expand the k^2 forest one decode step at a time, checking for the verify
result only between steps; then
- ``select`` + completed forest: promote the selected root's k completed
  stage-2 routes (zero-copy) -- they are the next stage-1 tree;
- ``select`` + partial forest: promote the k active stage-2 routes and build
  the remaining tree depths;
- ``fallback_ar``: drop speculative routes, EXTEND the prefix with the Target's
  tokens, build a fresh tree.
Neither side re-prefills its history.  A tree built by a handoff stops one
decode step short: the paths (with the depth-d tokens still pending) are
enough for the verify request, and the step that decodes the depth-d tokens
runs first in the next round, while the Target verifies.  The reference
decodes it before sending; the requests are identical.

Parity: reference src/atlas_0709/distributed_system.py:47-1216 (config,
round traces, result JSON, handoff modes, timeline, warmup and CLI flags).
"""

from __future__ import annotations

import math
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Sequence

import torch

from ..runtime.builders import (
    build_forest_one_depth,
    build_tree_depths,
    build_tree_one_depth,
    initialize_forest_routes,
    initialize_stage1_routes,
    select_routes_by_stage1_root,
)
from ..runtime.drafter import DrafterRuntime
from ..runtime.sampling import DrafterSamplingConfig, DrafterSamplingContext
from ..runtime.store import KVTreeStore
from ..types import BuildDepthsOutput, RouteState
from ..utils.nvtx import nvtx_range
from ..utils.timeline import EdgeBlackboxTimeline, EdgeRoundTimeline, EdgeSpan
from .rpc import selected_route_id_from_response


@dataclass(frozen=True)
class DistributedAtlasConfig:
    k: int = 3
    d: int = 4
    max_new_tokens: int = 64
    eos_token_id: int | None = None
    fallback_ar_tokens: int = 4
    generation_seed: int = 0
    drafter_do_sample: bool = False
    drafter_temperature: float = 1.0
    fixed_forest_depth: int | None = None
    validate_state_alignment: bool = False
    # "overlap": the drafter decodes the rest of the tree and the forest while the
    # target verifies (the reference schedule).  "adaptive": the same, except while
    # the moving average of fallback decisions is >= forest_gate_threshold; then
    # the drafter first waits for the target's decision, and on a fallback spends
    # nothing on a tree and forest that the fallback discards (they would only
    # compete with the target's AR steps for the GPU).  Tokens are identical.
    forest_gate: str = "adaptive"
    forest_gate_threshold: float = 0.75

    def validate(self) -> None:
        if self.k <= 0:
            raise ValueError(f"tree width k={self.k}: need at least one route")
        if self.d <= 0:
            raise ValueError(f"tree depth d={self.d}: need at least one drafted token per route")
        if self.max_new_tokens <= 0:
            raise ValueError(f"max_new_tokens={self.max_new_tokens}: nothing to generate")
        if self.fallback_ar_tokens <= 0:
            raise ValueError(f"fallback_ar_tokens={self.fallback_ar_tokens}: a fallback must commit at least one token")
        t = float(self.drafter_temperature)
        if not math.isfinite(t) or t <= 0.0:
            raise ValueError(f"drafter_temperature {self.drafter_temperature} is not a positive finite number")
        if self.fixed_forest_depth is not None and not 0 <= int(self.fixed_forest_depth) <= int(self.d):
            raise ValueError(f"fixed_forest_depth {self.fixed_forest_depth} is outside 0..d={self.d}")
        if self.forest_gate not in ("overlap", "adaptive"):
            raise ValueError("forest_gate must be 'overlap' or 'adaptive'")
        if not 0.0 < float(self.forest_gate_threshold) <= 1.0:
            raise ValueError("forest_gate_threshold must be in (0, 1]")


@dataclass
class DistributedRoundTrace:
    round_index: int
    selected_route_id: int | None
    committed_tokens: list[int]
    decision: str
    fallback_reason: str | None
    fallback_token_ids: list[int]
    forest_depth: int
    verify_returned_before_forest_done: bool
    target_scores: list[dict[str, object]]
    handoff_mode: str
    reused_stage2_routes: int
    reused_stage2_depth: int
    remaining_tree_depth: int
    committed_kv_tokens: int
    released_route_rows: int
    released_kv_pages: int
    target_unique_tree_nodes: int
    target_unmerged_path_nodes: int
    target_prefix_len_before: int
    target_prefix_len_after: int
    target_decision_metadata: dict[str, object] = field(default_factory=dict)

    def to_dict(self) -> dict[str, object]:
        return {k: getattr(self, k) for k in self.__dataclass_fields__}


@dataclass
class DistributedGenerationResult:
    prompt_token_ids: list[int]
    generated_token_ids: list[int]
    text: str | None
    rounds: list[DistributedRoundTrace] = field(default_factory=list)
    metadata: dict[str, object] = field(default_factory=dict)

    def to_dict(self) -> dict[str, object]:
        return {
            "prompt_token_ids": self.prompt_token_ids,
            "generated_token_ids": self.generated_token_ids,
            "token_ids": [*self.prompt_token_ids, *self.generated_token_ids],
            "text": self.text,
            "rounds": [r.to_dict() for r in self.rounds],
            "metadata": self.metadata,
        }


@dataclass
class DeferredTree:
    """A stage-1 tree whose last depth is not decoded yet.

    ``routes`` carry ``d - 1`` materialized tokens and the depth-``d`` token as
    their pending token (with its draft log-prob), which is all the verify
    request needs.  The step that decodes the pending tokens -- KV for the
    forest and the logits its roots start from -- then runs while the target
    verifies instead of before the request is sent.  The tokens sent are the
    ones a fully decoded tree would send.
    """

    routes: list[RouteState]
    steps: list


@dataclass(frozen=True)
class StageHandoff:
    stage1: BuildDepthsOutput | DeferredTree
    mode: str
    reused_stage2_routes: int
    reused_stage2_depth: int
    remaining_tree_depth: int
    physical_stats: dict[str, int]
    commit_prune_span: EdgeSpan | None = None
    tree_step_spans: tuple[EdgeSpan, ...] = ()


COMPACT_DECISION_KEYS = (
    "selection_policy",
    "route_sampling_enabled",
    "route_sampling_scope",
    "route_sampling_seed",
    "route_sampling_round",
    "route_sampling_temperature",
    "route_sampling_uniform",
    "route_sampling_selected_probability",
    "route_sampling_selected_cdf_low",
    "route_sampling_selected_cdf_high",
    "route_sampling_boundary_margin",
    "route_sampling_ordered_candidates",
    "selected_draft_rank",
    "route0_route_id",
    "draft_top_route_id",
    "selected_route_changed_from_route0",
    "selected_first_token_changed_from_route0",
    "selected_minus_route0_draft_first_token_logprob",
    "selected_minus_route0_draft_logprob",
    "selected_minus_route0_target_selection_score",
    "route_intervention",
    "best_selection_score",
    "best_first_token_logprob",
)


class PagedDistributedAtlasGenerator:
    """Drives one generation: drafter in this thread, Target through ``target_client``."""

    system_name = "atlas_distributed_two_process"

    def __init__(
        self,
        *,
        config: DistributedAtlasConfig,
        drafter: DrafterRuntime,
        target_client: Any,
        tokenizer=None,
    ) -> None:
        config.validate()
        self.config = config
        self.drafter = drafter
        self.target_client = target_client
        self.tokenizer = tokenizer
        self.last_timeline: EdgeBlackboxTimeline | None = None
        self._t0: float | None = None
        # Moving average of fallback decisions (forest_gate="adaptive"); kept across prompts.
        self.fallback_ema = 0.0

    # ------------------------------------------------------------ helpers
    def _now(self) -> float:
        if self._t0 is None:
            raise RuntimeError("the round timeline clock starts with a session; start() one first")
        return time.perf_counter() - self._t0

    def _timed(self, name: str, fn, *args):
        s = self._now()
        out = fn(*args)
        return out, EdgeSpan(name, s, self._now())

    def _sampling_config(self) -> DrafterSamplingConfig:
        c = self.config
        return DrafterSamplingConfig(bool(c.drafter_do_sample), int(c.generation_seed), float(c.drafter_temperature))

    def _sampling(self, committed: Sequence[int]) -> DrafterSamplingContext:
        cfg = self._sampling_config()
        if not cfg.do_sample:
            # Greedy drafting never reads the prefix (it only keys sampling noise): one
            # shared context per configuration instead of a copy of the prefix per call.
            cached = getattr(self, "_greedy_context", None)
            if cached is None or cached.config != cfg:
                cached = DrafterSamplingContext(cfg, ())
                self._greedy_context = cached
            return cached
        return DrafterSamplingContext(cfg, tuple(committed))

    def _should_build_forest_step(self, *, verify_done: bool, forest_depth: int) -> bool:
        if forest_depth >= self.config.d:
            return False
        if self.config.fixed_forest_depth is not None:
            return forest_depth < int(self.config.fixed_forest_depth)
        return not verify_done

    def _should_stop(self, committed_now: Sequence[int], generated: Sequence[int]) -> bool:
        if len(generated) >= self.config.max_new_tokens:
            return True
        eos = self.config.eos_token_id
        return eos is not None and any(int(t) == int(eos) for t in committed_now)

    def _truncate_commit(self, toks: Sequence[int], generated: Sequence[int]) -> list[int]:
        out = [int(t) for t in toks[: self.config.max_new_tokens - len(generated)]]
        eos = self.config.eos_token_id
        if eos is not None:
            for i, t in enumerate(out):
                if t == int(eos):
                    return out[: i + 1]
        return out

    def _route_payloads(self, store: KVTreeStore, routes: Sequence[RouteState], *,
                        pending: bool = False) -> list[dict[str, object]]:
        """Verify payloads; ``pending`` routes contribute their pending token as the last one."""
        out = []
        for r in routes:
            depth = int(r.stage1_depth) + (1 if pending else 0)
            path = store.pending_token_path(r) if pending else store.materialized_token_path(r)
            out.append({
                "route_id": int(r.route_id),
                "token_ids": [int(t) for t in path[:depth]],
                "draft_logprob": float(r.cumulative_logprob),
                "draft_token_logprobs": [float(v) for v in r.token_logprobs[:depth]],
            })
        return out

    def _tree_for_verify(self, active: Sequence[RouteState], *, depth: int, store: KVTreeStore,
                         sampling) -> DeferredTree:
        """Decode ``depth - 1`` tree depths; the last one is left to run during the verify."""
        steps: list = []
        front = list(active)
        for _ in range(int(depth) - 1):
            st = build_tree_one_depth(front, k=self.config.k, route_store=store, model_backend=self.drafter,
                                      sampling=sampling)
            steps.append(st)
            front = st.next_routes
        return DeferredTree(front, steps)

    @staticmethod
    def _find_route(stage1: BuildDepthsOutput, route_id: int) -> RouteState:
        for r in stage1.completed_routes:
            if int(r.route_id) == int(route_id):
                return r
        raise KeyError(f"the target selected route {route_id}, which is not one of this round's stage-1 routes")

    def _verify_call(self, committed, routes, remaining, round_index, fallback_event=None, decision_event=None):
        kw = {}
        if fallback_event is not None and getattr(self.target_client, "supports_early_decision", False):
            def on_decision(decision):
                if decision == "fallback_ar":
                    fallback_event.set()
                if decision_event is not None:
                    decision_event.set()

            kw["on_decision"] = on_decision
        resp = self.target_client.verify(
            prefix_token_ids=committed,
            routes=routes,
            fallback_max_tokens=min(int(self.config.fallback_ar_tokens), int(remaining)),
            selected_path_max_tokens=int(remaining),
            eos_token_id=self.config.eos_token_id,
            route_sampling_seed=int(self.config.generation_seed),
            route_sampling_round=int(round_index),
            **kw,
        )
        return resp, self._now()

    # ----------------------------------------------------------- generate
    def generate(self, prompt_token_ids: Sequence[int]) -> DistributedGenerationResult:
        session = self.start(prompt_token_ids)
        while not session.finished:
            session.step()
        return session.result()

    def start(self, prompt_token_ids: Sequence[int]) -> "AtlasSession":
        """Prefill both sides (concurrently) and build the initial tree; returns a steppable session."""
        s = AtlasSession(self, prompt_token_ids)
        s.begin()
        return s

    def close(self) -> None:
        self._vpool.shutdown(wait=True)

    @property
    def _vpool(self) -> ThreadPoolExecutor:
        pool = getattr(self, "_verify_pool", None)
        if pool is None:
            pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="atlas-verify")
            self._verify_pool = pool
        return pool

    # ------------------------------------------------------------ handoffs
    def _fallback_extend_handoff(self, store: KVTreeStore, tokens: Sequence[int]):
        suffix = [int(t) for t in tokens]
        if not suffix:
            raise ValueError("a fallback round returned no target tokens to extend the drafter with")
        dropped = self.drafter.drop_speculative()
        store.committed_token_ids.extend(suffix)
        self.drafter.append_known_tokens_as_prefix(suffix)
        rs = self._sampling(store.committed_token_ids)
        active = initialize_stage1_routes(self.drafter.prefix_state(), k=self.config.k, route_store=store, sampling=rs,
                                          model_backend=self.drafter)
        stage1 = self._tree_for_verify(active, depth=self.config.d, store=store, sampling=rs)
        return stage1, {
            "committed_kv_tokens": len(suffix),
            "retained_routes": 0,
            "released_route_rows": dropped["released_route_rows"],
            "released_kv_pages": dropped["released_kv_pages"],
        }

    def _handoff_after_verify(
        self,
        *,
        store: KVTreeStore,
        selected_stage1_route: RouteState,
        forest_depth: int,
        forest_frontier: Sequence[RouteState],
        forest_completed: Sequence[RouteState] | None,
        forest_last_logits: torch.Tensor | None,
        sampling: DrafterSamplingContext,
    ) -> StageHandoff:
        cfg = self.config
        root = int(selected_stage1_route.route_id)
        clock = self._now if self._t0 is not None else time.perf_counter
        if forest_depth >= cfg.d:
            if forest_completed is None or forest_last_logits is None:
                raise RuntimeError("the forest reached depth d but its last routes or logits were not kept")
            idx = [i for i, r in enumerate(forest_completed) if int(r.stage1_root_id) == root]
            if len(idx) != cfg.k:
                raise RuntimeError(
                    "the finished forest should hold k routes under the selected root: "
                    f"expected={cfg.k}, got={len(idx)}"
                )
            s0 = clock()
            promoted, phys = self.drafter.commit_stage1_and_promote(
                committed_route=selected_stage1_route, retained_routes=[forest_completed[i] for i in idx]
            )
            span = EdgeSpan("edge_commit_prune", s0, clock())
            sel = torch.tensor(idx, dtype=torch.long, device=forest_last_logits.device)
            return StageHandoff(
                stage1=BuildDepthsOutput(promoted, [], forest_last_logits.index_select(0, sel), []),
                mode="completed_forest_reused",
                reused_stage2_routes=len(promoted),
                reused_stage2_depth=cfg.d,
                remaining_tree_depth=0,
                physical_stats=phys,
                commit_prune_span=span,
            )
        retained = select_routes_by_stage1_root(forest_frontier, root)
        if len(retained) != cfg.k:
            raise RuntimeError(
                "the unfinished forest should hold k frontier routes under the selected root: "
                f"expected={cfg.k}, got={len(retained)}"
            )
        s0 = clock()
        promoted, phys = self.drafter.commit_stage1_and_promote(
            committed_route=selected_stage1_route, retained_routes=retained
        )
        span = EdgeSpan("edge_commit_prune", s0, clock())
        depths = {int(r.stage1_depth) for r in promoted}
        if depths != {int(forest_depth)}:
            raise RuntimeError(
                f"promoted route depth does not match completed forest depth: route_depths={sorted(depths)}, "
                f"forest_depth={forest_depth}"
            )
        remaining = cfg.d - int(forest_depth)
        steps = []
        spans: list[EdgeSpan] = []
        front = list(promoted)
        # The last depth is decoded during the next verify (see DeferredTree).
        for i in range(remaining - 1):
            s1 = clock()
            st = build_tree_one_depth(front, k=cfg.k, route_store=store, model_backend=self.drafter, sampling=sampling)
            spans.append(EdgeSpan(f"edge_post_prune_tree_step_{i + 1}", s1, clock()))
            steps.append(st)
            front = st.next_routes
        return StageHandoff(
            stage1=DeferredTree(front, steps),
            mode="partial_forest_pruned_then_build_tree",
            reused_stage2_routes=len(promoted),
            reused_stage2_depth=int(forest_depth),
            remaining_tree_depth=remaining,
            physical_stats=phys,
            commit_prune_span=span,
            tree_step_spans=tuple(spans),
        )

    # ---------------------------------------------------------- validators
    @staticmethod
    def _validate_target_prefix_lengths(meta: dict, before: int, after: int) -> None:
        ob, oa = int(meta.get("prefix_len_before", -1)), int(meta.get("prefix_len_after", -1))
        if ob != before or oa != after:
            raise RuntimeError(
                f"Target committed-prefix length diverged from the coordinator: target={ob}->{oa}, "
                f"coordinator={before}->{after}"
            )

    def _validate_drafter_prefix_state(self, store: KVTreeStore, committed, routes) -> None:
        exp = [int(t) for t in committed]
        if list(self.drafter.prefix_token_ids) != exp or list(store.committed_token_ids) != exp:
            raise RuntimeError("the drafter's committed tokens no longer match the coordinator's")
        if int(self.drafter.route_pool.prefix_len) != len(exp):
            raise RuntimeError(
                f"the drafter's page pool holds a different committed length than the coordinator: "
                f"slots={int(self.drafter.route_pool.prefix_len)}, tokens={len(exp)}"
            )
        for r in routes:
            if self.drafter.route_pool.has_route(int(r.route_id)):
                self.drafter.validate_route_physical_state(r)


class AtlasSession:
    """One generation advanced one speculative round per ``step()``."""

    def __init__(self, gen: PagedDistributedAtlasGenerator, prompt_token_ids: Sequence[int]) -> None:
        self.gen = gen
        self.prompt = [int(t) for t in prompt_token_ids]
        self.committed = list(self.prompt)
        self.generated: list[int] = []
        self.traces: list[DistributedRoundTrace] = []
        self.fallback_profiles: list[dict[str, object]] = []
        self.rounds_tl: list[EdgeRoundTimeline] = []
        self.finished = False
        self.round_index = 0
        self.store = KVTreeStore()
        self.gated_rounds = 0

    def begin(self) -> None:
        g, cfg = self.gen, self.gen.config
        self.health = g.target_client.health()
        self.target_meta = dict(self.health.get("metadata", {}))
        g._t0 = time.perf_counter()
        g.drafter.bind_store(self.store)
        self.pre_frontier = self.pre_completed = self.pre_logits = None
        self.pre_depth = 0
        self.pre_spans: list[EdgeSpan] = []
        s0 = g._sampling(self.committed)
        tfut = g._vpool.submit(g._timed, "cloud_prompt_blackbox", g.target_client.prefill, list(self.committed))
        _, self.edge_prefill = g._timed("edge_prompt_prefill", g.drafter.prefill, self.committed)
        self.store.committed_token_ids = list(self.committed)
        t_tree = g._now()
        active = initialize_stage1_routes(g.drafter.prefix_state(), k=cfg.k, route_store=self.store, sampling=s0,
                                          model_backend=g.drafter)
        self.stage1 = build_tree_depths(
            active, depth=cfg.d, k=cfg.k, route_store=self.store, model_backend=g.drafter, sampling=s0
        )
        self.initial_tree = EdgeSpan("edge_initial_stage1_tree", t_tree, g._now())
        if cfg.fixed_forest_depth is None and not tfut.done():
            self.pre_frontier = initialize_forest_routes(
                self.stage1.completed_routes, self.stage1.last_logits, k=cfg.k, route_store=self.store, sampling=s0,
                model_backend=g.drafter,
            )
            while not tfut.done() and self.pre_depth < cfg.d:
                t0 = g._now()
                st = build_forest_one_depth(
                    self.pre_frontier, k=cfg.k, route_store=self.store, model_backend=g.drafter, sampling=s0
                )
                self.pre_depth += 1
                self.pre_spans.append(EdgeSpan(f"edge_forest_step_{self.pre_depth}", t0, g._now()))
                self.pre_completed = st.decoded_routes
                self.pre_logits = st.decode_output.next_token_logits
                self.pre_frontier = st.next_routes
        _, self.cloud_prefill = tfut.result()

    def step(self) -> DistributedRoundTrace:
        """One round: verify in the worker while the forest grows; then hand off."""
        if self.finished:
            raise RuntimeError("session already finished")
        g, cfg, store = self.gen, self.gen.config, self.store
        committed, generated = self.committed, self.generated
        rs = g._sampling(committed)
        p_round = len(committed)
        deferred = self.stage1 if isinstance(self.stage1, DeferredTree) else None
        if deferred is not None:
            payload = g._route_payloads(store, deferred.routes, pending=True)
        else:
            payload = g._route_payloads(store, self.stage1.completed_routes)
        v_submit = g._now()
        remaining = cfg.max_new_tokens - len(generated)
        # Set by the target (in-process transports) once it has decided to fall back:
        # the forest of this round is then discarded, so growing it further would
        # only compete with the target's AR forwards.
        fb_decided = threading.Event()
        decided = threading.Event()
        gated = (cfg.forest_gate == "adaptive" and cfg.fixed_forest_depth is None
                 and g.fallback_ema >= float(cfg.forest_gate_threshold))
        if gated:
            # Nothing overlaps the verify of a gated round: run it on this thread
            # (no hand-off to the worker and back).
            self.gated_rounds += 1
            vfut = Future()
            vfut.set_result(g._verify_call(list(committed), payload, remaining, self.round_index, fb_decided,
                                           decided))
        else:
            vfut = g._vpool.submit(g._verify_call, list(committed), payload, remaining, self.round_index,
                                   fb_decided, decided)
            vfut.add_done_callback(lambda _f: decided.set())
        # A gated round that falls back builds nothing: the fallback drops this tree.
        skip = gated and fb_decided.is_set()
        tree_spans: list[EdgeSpan] = []
        if deferred is not None and not skip:
            t0 = g._now()
            with nvtx_range("edge_tree_last_depth"):
                st = build_tree_one_depth(deferred.routes, k=cfg.k, route_store=store, model_backend=g.drafter,
                                          sampling=rs)
            self.stage1 = BuildDepthsOutput(st.decoded_routes, st.next_routes, st.decode_output.next_token_logits,
                                            [*deferred.steps, st])
            tree_spans.append(EdgeSpan("edge_tree_last_depth", t0, g._now()))
        if skip:
            f_depth, f_done, f_logits, f_spans, f_front = 0, None, None, [], []
        elif self.round_index == 0 and self.pre_frontier is not None:
            f_depth, f_done, f_logits = self.pre_depth, self.pre_completed, self.pre_logits
            f_spans, f_front = list(self.pre_spans), self.pre_frontier
        else:
            f_depth, f_done, f_logits, f_spans = 0, None, None, list(tree_spans)
            f_front = initialize_forest_routes(
                self.stage1.completed_routes, self.stage1.last_logits, k=cfg.k, route_store=store, sampling=rs,
                model_backend=g.drafter,
            )
        while not skip and g._should_build_forest_step(verify_done=vfut.done() or fb_decided.is_set(),
                                                       forest_depth=f_depth):
            t0 = g._now()
            with nvtx_range(f"edge_forest_depth_{f_depth + 1}"):
                st = build_forest_one_depth(f_front, k=cfg.k, route_store=store, model_backend=g.drafter,
                                            sampling=rs)
            f_depth += 1
            f_spans.append(EdgeSpan(f"edge_forest_step_{f_depth}", t0, g._now()))
            f_done, f_logits, f_front = st.decoded_routes, st.decode_output.next_token_logits, st.next_routes
        early = f_depth < cfg.d and vfut.done()
        resp, v_done = vfut.result()
        vspan = EdgeSpan("cloud_verify_blackbox", v_submit, v_done)
        tmeta = dict(resp.get("metadata", {}))
        prof = tmeta.get("fallback_ar_profile")
        if isinstance(prof, dict):
            self.fallback_profiles.append({"round_index": self.round_index, **prof})
        decision = str(resp.get("decision", "select"))
        g.fallback_ema = 0.7 * g.fallback_ema + 0.3 * (1.0 if decision == "fallback_ar" else 0.0)
        sel_id: int | None = None
        reason: str | None = None
        fb_tokens: list[int] = []
        mode = "stopped"
        reused = reused_depth = remaining_depth = 0
        phys = {"committed_kv_tokens": 0, "released_route_rows": 0, "released_kv_pages": 0}
        handoff_span: EdgeSpan | None = None
        post_spans: list[EdgeSpan] = []
        if decision == "fallback_ar":
            fb_tokens = [int(t) for t in resp.get("fallback_token_ids", [])]
            reason = None if resp.get("fallback_reason") is None else str(resp.get("fallback_reason"))
            if len(fb_tokens) > remaining:
                raise RuntimeError(
                    "the target's fallback overran the token budget: "
                    f"returned={len(fb_tokens)}, remaining={remaining}"
                )
            now = list(fb_tokens)
            generated.extend(now)
            committed.extend(now)
            stop = not now or g._should_stop(now, generated)
            mode = "fallback_ar_stopped" if stop else "fallback_ar_extend_prefix_kv"
            if not stop:
                t0 = g._now()
                with nvtx_range("edge_fallback_extend_then_build_tree"):
                    self.stage1, phys = g._fallback_extend_handoff(store, now)
                handoff_span = EdgeSpan("edge_fallback_extend_then_build_tree", t0, g._now())
        elif decision == "select":
            sel_id = selected_route_id_from_response(resp)
            sel = g._find_route(self.stage1, sel_id)
            full = list(store.materialized_token_path(sel)[: cfg.d])
            now = g._truncate_commit(full, generated)
            generated.extend(now)
            committed.extend(now)
            stop = not now or g._should_stop(now, generated)
            if not stop:
                if now != full:
                    raise RuntimeError("the commit was truncated, so the forest built on the full route cannot be promoted")
                h = g._handoff_after_verify(
                    store=store,
                    selected_stage1_route=sel,
                    forest_depth=f_depth,
                    forest_frontier=f_front,
                    forest_completed=f_done,
                    forest_last_logits=f_logits,
                    sampling=g._sampling(committed),
                )
                handoff_span, post_spans = h.commit_prune_span, list(h.tree_step_spans)
                self.stage1, mode = h.stage1, h.mode
                reused, reused_depth, remaining_depth = h.reused_stage2_routes, h.reused_stage2_depth, h.remaining_tree_depth
                phys = h.physical_stats
        else:
            raise RuntimeError(f"the target answered with decision {decision!r}, expected select or fallback_ar")
        if cfg.validate_state_alignment:
            g._validate_target_prefix_lengths(tmeta, p_round, len(committed))
            if not stop:
                live = (self.stage1.routes if isinstance(self.stage1, DeferredTree)
                        else [*self.stage1.completed_routes, *self.stage1.next_frontier_routes])
                g._validate_drafter_prefix_state(store, committed, live)
        trace = DistributedRoundTrace(
            round_index=self.round_index,
            selected_route_id=sel_id,
            committed_tokens=[int(t) for t in now],
            decision=decision,
            fallback_reason=reason,
            fallback_token_ids=list(fb_tokens),
            forest_depth=f_depth,
            verify_returned_before_forest_done=early,
            target_scores=list(resp.get("scores", [])),
            handoff_mode=mode,
            reused_stage2_routes=reused,
            reused_stage2_depth=reused_depth,
            remaining_tree_depth=remaining_depth,
            committed_kv_tokens=int(phys["committed_kv_tokens"]),
            released_route_rows=int(phys["released_route_rows"]),
            released_kv_pages=int(phys["released_kv_pages"]),
            target_unique_tree_nodes=int(tmeta.get("node_count", 0)),
            target_unmerged_path_nodes=int(tmeta.get("unmerged_path_node_count", 0)),
            target_prefix_len_before=int(tmeta.get("prefix_len_before", len(committed) - len(now))),
            target_prefix_len_after=int(tmeta.get("prefix_len_after", len(committed))),
            target_decision_metadata={k: tmeta[k] for k in COMPACT_DECISION_KEYS if k in tmeta},
        )
        self.traces.append(trace)
        self.rounds_tl.append(
            EdgeRoundTimeline(
                round_index=self.round_index,
                verify_blackbox=vspan,
                forest_steps=f_spans,
                post_prune_tree_steps=post_spans,
                handoff=handoff_span,
                forest_depth=f_depth,
                accepted_tokens=len(now),
                generated_tokens=len(generated),
                handoff_mode=mode,
                verify_returned_before_forest_done=early,
            )
        )
        self.round_index += 1
        if stop:
            self.finished = True
        return trace

    def result(self) -> DistributedGenerationResult:
        g, cfg = self.gen, self.gen.config
        elapsed = g._now()
        timeline = EdgeBlackboxTimeline(
            self.edge_prefill, self.cloud_prefill, self.initial_tree, self.rounds_tl, elapsed, len(self.generated)
        )
        g.last_timeline = timeline
        fb_rounds = sum(t.decision == "fallback_ar" for t in self.traces)
        return DistributedGenerationResult(
            prompt_token_ids=list(self.prompt),
            generated_token_ids=list(self.generated),
            text=g.tokenizer.decode(self.committed) if g.tokenizer is not None else None,
            rounds=self.traces,
            metadata={
                "system": g.system_name,
                "drafter_backend": "b200_native_paged_decode",
                "target_backend": self.target_meta.get("backend", "b200_native_masked_tree_verify"),
                "target_transport": str(self.health.get("transport", "http")),
                "target_health": self.health,
                "k": cfg.k,
                "d": cfg.d,
                "max_new_tokens": cfg.max_new_tokens,
                "fallback_ar_tokens": int(cfg.fallback_ar_tokens),
                "generation_seed": int(cfg.generation_seed),
                "drafter_sampling": g._sampling_config().to_dict(),
                "fixed_forest_depth": cfg.fixed_forest_depth,
                "validate_state_alignment": bool(cfg.validate_state_alignment),
                "rebuild_drafter_prefix_after_commit": False,
                "rebuild_drafter_prefix_after_fallback": False,
                "fallback_drafter_handoff": "single_multi_token_extend",
                "target_fallback_ar_profiles": self.fallback_profiles,
                "rebuild_target_prefix_after_commit": False,
                "cross_round_stage2_kv_reuse": True,
                "cross_round_target_kv_reuse": True,
                "target_selection_policy": self.target_meta.get("selection_policy"),
                "target_route_selection_policy": self.target_meta.get("route_selection_policy"),
                "route_tail_page_cow": True,
                "branch_safe_page_size": True,
                "forest_cancel_granularity": "between_decode_steps",
                "forest_gate": cfg.forest_gate,
                "forest_gate_threshold": float(cfg.forest_gate_threshold),
                "forest_gated_rounds": self.gated_rounds,
                "rounds": len(self.traces),
                "fallback_rounds": fb_rounds,
                "fallback_rate": fb_rounds / len(self.traces) if self.traces else None,
                "edge_blackbox_timeline": timeline.summary(),
                "drafter_hot_path_counters": g.drafter.hot_path_counters(),
            },
        )
