"""Target verifier: one deduplicated, ancestor-masked tree forward per round.

A persistent session holds the committed prefix in a page list of the native
pool.  ``verify_payloads`` builds the prefix trie of the k stage-1 paths (the
native ``build_tree``), writes the unique nodes' KV to scratch positions
``P..P+N-1`` of the same page list in one forward whose attention reads the
prefix once for all nodes and masks the node region by ancestry, scores every
path from the node logits with optional front-loaded weights, selects a route
(best of k, seeded route-level sampling, or the first route), and then either
compacts the selected nodes' KV in place into positions ``P..P+d-1`` (one
multi-layer move kernel) or, on low confidence, runs greedy AR decoding whose
argmax chain stays on the device.

Parity: reference src/atlas_0709/target_runtime.py:33-935 (validation,
selection, sampling audit, intervention metadata, truncation, fallback
reasons and order, commit semantics, runtime metadata).
"""

from __future__ import annotations

import hashlib
import json
import math
import time
from typing import Sequence

import numpy as np
import torch

from ..ops import _native
from ..utils.transfer import KernelError, ids_to_device, read_back
from ..utils.nvtx import nvtx_range
from ..types import PrefixState, TargetRouteScore, TargetVerifyResult, VerifyRoutePayload
from .drafter import PrefixPageMirror
from .engine import LlamaEngine, row_bucket

ROUTE_SAMPLE_DOMAIN = "atlas0709-target-route-sample-v1"


def validate_score_weights(weights: Sequence[float] | None) -> tuple[float, ...] | None:
    if weights is None:
        return None
    vals = tuple(float(v) for v in weights)
    if not vals:
        return None
    if any(v < 0.0 for v in vals):
        raise ValueError("every path score weight must be non-negative")
    total = sum(vals)
    if total <= 0.0:
        raise ValueError("the path score weights sum to zero; at least one must be positive")
    return tuple(v / total for v in vals)


def token_path_hash(token_ids: Sequence[int]) -> str:
    payload = json.dumps([int(t) for t in token_ids], separators=(",", ":")).encode("utf-8")
    return hashlib.sha256(payload).hexdigest()


class TargetVerifier:
    def __init__(
        self,
        engine: LlamaEngine,
        *,
        k: int = 3,
        d: int = 4,
        page_pool=None,
        score_weights: Sequence[float] | None = None,
        fallback_threshold: float | None = None,
        first_token_threshold: float | None = None,
        fallback_ar_tokens: int = 4,
        profile_fallback_ar: bool = False,
        route_selection_policy: str = "target_best",
        route_sampling_temperature: float = 1.0,
        model_name: str = "random-init",
        prefill_chunk_size: int = 8192,
    ) -> None:
        self.engine = engine
        self.k = int(k)
        self.d = int(d)
        if self.k <= 0 or self.d <= 0:
            raise ValueError(f"the target verifies k routes of depth d, both at least 1 (got k={k}, d={d})")
        self.host = _native.host()
        # The engine's last page is the trash page for padded graph rows.
        self.page_pool = page_pool if page_pool is not None else self.host.PagePool(engine.num_pages - 1, engine.page_size)
        self.seq = self.host.RoutePool(self.page_pool)
        self.device = engine.device
        self.page_size = engine.page_size
        self.mirror = PrefixPageMirror(engine.num_pages, self.device)
        if hasattr(engine, "register_mirror"):
            engine.register_mirror(self.mirror)
        self.score_weights = validate_score_weights(score_weights)
        self.fallback_threshold = None if fallback_threshold is None else float(fallback_threshold)
        self.first_token_threshold = None if first_token_threshold is None else float(first_token_threshold)
        self.fallback_ar_tokens = int(fallback_ar_tokens)
        if self.fallback_ar_tokens <= 0:
            raise ValueError("the fallback AR budget (fallback_ar_tokens) must be positive")
        self.profile_fallback_ar = bool(profile_fallback_ar)
        policy = str(route_selection_policy).strip().lower()
        if policy not in {"target_best", "target_sample", "first_route"}:
            raise ValueError(f"unknown route_selection_policy {route_selection_policy!r} "
                             "(choose target_best, target_sample or first_route)")
        self.route_selection_policy = policy
        temp = float(route_sampling_temperature)
        if not math.isfinite(temp) or temp <= 0.0:
            raise ValueError(f"route_sampling_temperature {route_sampling_temperature} is not a positive finite number")
        self.route_sampling_temperature = temp
        if policy == "first_route" and (self.fallback_threshold is not None or self.first_token_threshold is not None):
            raise ValueError(
                "the first_route policy always commits route 0, so it cannot be combined with fallback thresholds"
            )
        self.model_name = model_name
        self.prefill_chunk_size = int(prefill_chunk_size)
        self.prefix_token_ids: tuple[int, ...] = ()
        self._prefix_logits: torch.Tensor | None = None
        # Last committed token whose forward has not run yet (after a fallback AR): its
        # KV slot is committed, its KV and the prefix logits come with the next forward.
        self._pending_token: int | None = None
        self._committed_verify_rounds = 0
        self._last_fallback_ar_profile: dict[str, object] | None = None

    def release(self) -> None:
        """End the session: every page returns to the (possibly shared) pool."""
        self.seq.clear()
        self.mirror.host = []
        self.prefix_token_ids = ()
        self._prefix_logits = None
        self._pending_token = None

    # -------------------------------------------------------------- prefill
    def _sync(self) -> None:
        self.mirror.sync(self.seq.prefix_pages())

    @torch.inference_mode()
    def prefill(self, prompt_token_ids: Sequence[int]) -> PrefixState:
        toks = tuple(int(t) for t in prompt_token_ids)
        if not toks:
            raise ValueError("cannot prefill the target with an empty prompt")
        self.seq.clear()
        self.mirror.host = []
        slots, _ = self.seq.append_prefix(len(toks))
        self._sync()
        logits = self.engine.prefill_sequence(
            ids_to_device(toks, self.device),
            start_pos=0,
            slots=slots.to(self.device),
            pages=self.mirror.view(),
            chunk_size=self.prefill_chunk_size,
        )
        self.prefix_token_ids = toks
        self._prefix_logits = logits
        self._pending_token = None
        self._committed_verify_rounds = 0
        self._last_fallback_ar_profile = None
        return PrefixState(
            token_ids=toks, next_token_logits=logits, committed_length=len(toks), metadata=self.runtime_metadata()
        )

    # --------------------------------------------------------------- verify
    @torch.inference_mode()
    def verify_payloads(
        self,
        *,
        prefix_token_ids: Sequence[int],
        routes: Sequence[VerifyRoutePayload],
        fallback_max_tokens: int | None = None,
        selected_path_max_tokens: int | None = None,
        eos_token_id: int | None = None,
        route_sampling_seed: int | None = None,
        route_sampling_round: int | None = None,
        on_decision=None,
    ) -> TargetVerifyResult:
        """Verify the routes; ``on_decision(decision)`` (optional) is called as soon as the
        decision is known, before the fallback AR tokens are generated or the path is committed."""
        prefix = tuple(prefix_token_ids)  # element-wise == also accepts numpy integers
        if self._prefix_logits is None and self._pending_token is None:
            self.prefill([int(t) for t in prefix])
        elif prefix != self.prefix_token_ids:
            raise RuntimeError(
                "the request's committed prefix differs from the one whose KV the target holds (it never re-prefills silently): "
                f"request_len={len(prefix)}, target_len={len(self.prefix_token_ids)}"
            )
        paths, depth = self._validate_routes(routes)
        p_committed = len(self.prefix_token_ids)
        try:
            with nvtx_range("target_tree_verify"):
                tree = self.run_tree(paths)
        except KernelError:
            # Nothing is scored, selected or committed: drop the nodes' scratch slots.
            self.seq.set_prefix_len(p_committed)
            self._sync()
            raise
        scores = self._score_routes(routes, paths, tree["path_logprobs"])
        best = max(scores, key=self._best_key)
        selected, sampling_meta = self._select_route_with_metadata(
            scores, route_sampling_seed=route_sampling_seed, route_sampling_round=route_sampling_round
        )
        reason = self._fallback_reason(selected)
        p_before = len(self.prefix_token_ids)
        if on_decision is not None:
            on_decision("fallback_ar" if reason is not None else "select")
        meta: dict[str, object] = {}

        def build_metadata() -> None:
            meta.update(self._verify_metadata(routes, depth, tree, p_before, scores, best, selected, sampling_meta))

        if reason is not None:
            limit = self.fallback_ar_tokens if fallback_max_tokens is None else min(
                int(fallback_max_tokens), self.fallback_ar_tokens
            )
            # The response metadata is assembled while the AR steps run on the GPU.
            with nvtx_range("target_fallback_ar"):
                generated = self._generate_fallback_ar(max_tokens=limit, eos_token_id=eos_token_id,
                                                       while_running=build_metadata)
            if not meta:  # no AR step ran (a budget of zero tokens)
                build_metadata()
            return TargetVerifyResult(
                selected_route_id=None,
                scores=scores,
                decision="fallback_ar",
                fallback_token_ids=tuple(generated),
                fallback_reason=reason,
                metadata={
                    **meta,
                    "prefix_len_after": int(len(self.prefix_token_ids)),
                    "target_kv_commit": "fallback_ar_in_place",
                    "target_reprefill_after_verify": False,
                    "fallback_triggered": True,
                    "fallback_reason": reason,
                    "fallback_token_count": int(len(generated)),
                    "fallback_ar_profile": self._last_fallback_ar_profile,
                },
            )
        build_metadata()
        idx = next(i for i, r in enumerate(routes) if int(r.route_id) == int(selected.route_id))
        node_path = tree["node_paths"][idx]
        committed_path, committed_nodes = self._truncate_selected_path(
            token_ids=paths[idx], node_ids=node_path, max_tokens=selected_path_max_tokens, eos_token_id=eos_token_id
        )
        self._commit_selected_path(committed_path, committed_nodes, tree["logits"])
        return TargetVerifyResult(
            selected_route_id=selected.route_id,
            scores=scores,
            metadata={
                **meta,
                "prefix_len_after": int(len(self.prefix_token_ids)),
                "target_kv_commit": "selected_tree_path_in_place",
                "target_reprefill_after_verify": False,
                "fallback_triggered": False,
                "selected_route_id": int(selected.route_id),
                "selected_selection_score": float(selected.effective_selection_score),
                "selected_path_committed_tokens": int(len(committed_path)),
                "selected_path_was_truncated": bool(len(committed_path) != len(paths[idx])),
            },
        )

    def _verify_metadata(self, routes, depth, tree, p_before, scores, best, selected, sampling_meta) -> dict:
        """Response metadata of one verify (state as of before its commit)."""
        return {
            **self.runtime_metadata(),
            "route_count": len(routes),
            "path_depth": int(depth),
            "node_count": int(tree["node_count"]),
            "unmerged_path_node_count": int(len(routes) * depth),
            "kv_len": int(p_before + tree["node_count"]),
            "prefix_len_before": int(p_before),
            "selection_policy": self._selection_policy_name(),
            "selection_score_name": (
                "weighted_target_logprob" if self.score_weights is not None else "target_logprob"
            ),
            "fallback_threshold": self.fallback_threshold,
            "first_token_threshold": self.first_token_threshold,
            "fallback_ar_tokens": int(self.fallback_ar_tokens),
            **sampling_meta,
            **self._route_intervention_metadata(scores, selected),
            "best_route_id": int(best.route_id),
            "best_selection_score": float(best.effective_selection_score),
            "best_first_token_logprob": (
                None if best.first_token_logprob is None else float(best.first_token_logprob)
            ),
        }

    def _validate_routes(self, routes: Sequence[VerifyRoutePayload]) -> tuple[list[tuple[int, ...]], int]:
        if not routes:
            raise ValueError("a verify request carried no routes")
        if len(routes) != self.k:
            raise ValueError(f"this target verifies k={self.k} routes per request, got {len(routes)}")
        ids = [int(r.route_id) for r in routes]
        if len(set(ids)) != len(ids):
            raise ValueError("two routes of the request share a route_id")
        paths = [tuple(int(t) for t in r.token_ids) for r in routes]
        for r, p in zip(routes, paths):
            if r.draft_token_logprobs and len(r.draft_token_logprobs) != len(p):
                raise ValueError(
                    "a route's draft_token_logprobs must be omitted or hold one value per token: "
                    f"route_id={int(r.route_id)}, values={len(r.draft_token_logprobs)}, depth={len(p)}"
                )
        lengths = {len(p) for p in paths}
        if len(lengths) != 1:
            raise ValueError(f"the routes of one request must be equally long; lengths {sorted(lengths)}")
        depth = next(iter(lengths))
        if depth <= 0:
            raise ValueError("a verify route needs at least one token")
        if depth != self.d:
            raise ValueError(f"this target verifies routes of depth d={self.d}, got depth {depth}")
        return paths, depth

    # ------------------------------------------------------- tree forward
    @staticmethod
    def linear_tree(paths: Sequence[Sequence[int]]):
        """The same outputs as ``build_tree`` with no prefix sharing: every route keeps
        its own chain of nodes (block-diagonal causal mask).  Used by the linear
        verify baseline (reference src/atlas_0709/flashinfer_full_verify.py:742-784)."""
        r, d = len(paths), len(paths[0])
        n = r * d
        tokens = torch.tensor([int(t) for p in paths for t in p], dtype=torch.int64)
        depths = torch.arange(d, dtype=torch.int32).repeat(r)
        parents = torch.arange(n, dtype=torch.int32) - 1
        parents[::d] = -1
        node_paths = torch.arange(n, dtype=torch.int32).reshape(r, d)
        w = (n + 63) // 64
        masks = np.zeros((n, w), dtype=np.uint64)
        for i in range(n):
            for a in range(i - i % d, i + 1):
                masks[i, a // 64] |= np.uint64(1) << np.uint64(a % 64)
        return tokens, parents, depths, node_paths, torch.from_numpy(masks.view(np.int64))

    @torch.inference_mode()
    def run_tree(self, paths: Sequence[Sequence[int]], *, deduplicate: bool = True) -> dict[str, object]:
        """One masked forward over the deduplicated trie; returns logits and path log-probs.

        ``deduplicate=False`` runs every route's tokens as its own chain (linear verify baseline).
        """
        if self._pending_token is not None:
            if deduplicate:
                return self._run_tree_with_pending(paths)
            self._flush_pending()
        if deduplicate:
            tokens, parents, depths, node_paths, masks = self.host.build_tree(
                torch.tensor([list(p) for p in paths], dtype=torch.int64)
            )
        else:
            tokens, parents, depths, node_paths, masks = self.linear_tree(paths)
        n = int(tokens.numel())
        p = len(self.prefix_token_ids)
        scratch = self.seq.reserve_scratch(p + n)
        # Path log-probs: token t of route r is scored by the prefix row (t == 0) or by its
        # parent node's row; the gather's indices go to the device before the forward.
        r_, d_ = node_paths.shape
        rows = torch.full((r_, d_), -1, dtype=torch.long)
        rows[:, 1:] = node_paths[:, :-1].long()
        gidx = self._stage_gather(rows, torch.tensor([list(x) for x in paths], dtype=torch.long), prefix_row=True)
        self._sync()
        logits = self.engine.run_rows(
            row_bucket(n),
            tail_stride=1,
            aux=gidx["aux"],
            mask_words=int(masks.shape[1]),
            prefix_pages=self.mirror.dev,
            tokens=tokens.numpy(),
            positions=depths.numpy() + p,
            slots=scratch.numpy(),
            shared_len=p,
            n_shared_pages=len(self.mirror.host),
            mask_base=p,
            row_full=np.full(n, p),
            row_len=np.full(n, p + n),
            row_mask=masks.numpy(),
        )
        lp = self.gather_logprobs(logits, gidx, self.engine.static_batch(row_bucket(n), 1, int(masks.shape[1])))
        return {
            "logits": logits,
            "node_count": n,
            "node_paths": node_paths.tolist(),
            "parents": parents.tolist(),
            "path_logprobs": lp,
        }

    def _run_tree_with_pending(self, paths: Sequence[Sequence[int]]) -> dict[str, object]:
        """``run_tree`` when the last prefix token's forward is still pending.

        That token becomes the root of the trie (every path is prefixed with it),
        at its own position and KV slot: the masked forward writes its KV, its row
        gives the prefix logits, and the routes' first tokens are scored by that
        row -- one forward instead of a one-row forward followed by the verify.
        Its key is read as a masked node (the tensor-core pass covers the keys
        before it), since this forward writes it.
        """
        lead = int(self._pending_token)
        tokens, parents, depths, node_paths, masks = self.host.build_tree(
            torch.tensor([[lead, *p] for p in paths], dtype=torch.int64)
        )
        n = int(tokens.numel())
        p = len(self.prefix_token_ids)
        base = p - 1  # the lead token's position
        scratch = self.seq.reserve_scratch(p + n - 1)
        slots = torch.cat((self.seq.slots_for_positions(base, 1), scratch))
        # Token t of a route is scored by its parent's row: the lead row for t == 0.
        gidx = self._stage_gather(node_paths[:, :-1].long(), torch.tensor([list(x) for x in paths], dtype=torch.long),
                                  prefix_row=False)
        self._sync()
        logits = self.engine.run_rows(
            row_bucket(n),
            tail_stride=1,
            aux=gidx["aux"],
            mask_words=int(masks.shape[1]),
            prefix_pages=self.mirror.dev,
            tokens=tokens.numpy(),
            positions=depths.numpy() + base,
            slots=slots.numpy(),
            shared_len=base,
            n_shared_pages=len(self.mirror.host),
            mask_base=base,
            row_full=np.full(n, base),
            row_len=np.full(n, base + n),
            row_mask=masks.numpy(),
        )
        lp = self.gather_logprobs(logits, gidx, self.engine.static_batch(row_bucket(n), 1, int(masks.shape[1])))
        self._prefix_logits = logits[0].detach().clone()
        self._pending_token = None
        real = node_paths[:, 1:] - 1  # node i >= 1 of this trie is node i - 1 of the routes' trie
        return {
            "logits": logits[1:],
            "node_count": n - 1,
            "node_paths": real.tolist(),
            "parents": [int(x) - 1 if int(x) > 0 else -1 for x in parents[1:].tolist()],
            "path_logprobs": lp,
        }

    @torch.inference_mode()
    def _flush_pending(self) -> None:
        """Run the pending token's one-row forward (KV and prefix logits) on its own."""
        if self._pending_token is None:
            return
        p = len(self.prefix_token_ids)
        q = p - 1
        slot = self.seq.slots_for_positions(q, 1).numpy()
        logits = self.engine.run_rows(
            1,
            prefix_pages=self.mirror.dev,
            tokens=np.array([self._pending_token]),
            positions=[q],
            slots=slot,
            shared_len=q,
            n_shared_pages=len(self.mirror.host),
            mask_base=q,
            row_full=[q + 1],
            row_len=[q + 1],
        )
        self._prefix_logits = logits[0].detach().clone()
        self._pending_token = None

    @staticmethod
    def _stage_gather(rows: torch.Tensor, toks: torch.Tensor, *, prefix_row: bool) -> dict:
        """Indices of a path log-prob gather (host tensors ``rows``, ``toks`` of one shape).  They
        travel in the forward's own input copy (the static batch's auxiliary words), so the
        gather after the forward waits for nothing on the host.  With ``prefix_row`` the prefix
        logits are row -1."""
        r = (rows + 1 if prefix_row else rows).reshape(-1).numpy()
        t = toks.reshape(-1).numpy()
        return {"aux": np.concatenate((r, t)).astype(np.int32), "n": int(r.size), "shape": tuple(rows.shape),
                "prefix_row": prefix_row}

    def gather_logprobs(self, logits: torch.Tensor, g: dict, sb) -> list[list[float]]:
        """Log-probs of the staged tokens under the staged rows of ``logits`` (see ``_stage_gather``);
        ``sb`` is the static batch whose forward carried the indices."""
        if g["prefix_row"]:
            assert self._prefix_logits is not None
            allrows = torch.cat((self._prefix_logits.reshape(1, -1).float(), logits.float()), dim=0)
        else:
            allrows = logits.float()
        n = g["n"]
        r, t = sb.aux[:n], sb.aux[n: 2 * n]
        if allrows.is_cuda:
            from ..ops.cuda_ops import shared_ops

            vals = shared_ops(allrows.device).gather_logprobs(allrows, r, t).reshape(g["shape"])
        else:
            r, t = r.long(), t.long()
            lse = torch.logsumexp(allrows, dim=-1)
            vals = (allrows[r, t] - lse[r]).reshape(g["shape"]).float()
        # The one transfer of the verify also brings back the device error flag.
        (host,) = read_back([vals], self.status_flag(), where="target tree verify")
        return host.astype(np.float64).tolist()

    def status_flag(self) -> torch.Tensor | None:
        """The target device's kernel error flag (None for op tables that raise directly)."""
        return getattr(self.engine.ops, "err", None)

    def warm_graphs(self) -> None:
        """Capture the verify bucket (up to k*d nodes) and the AR bucket up front."""
        n = self.k * self.d
        self.engine.warm_graph(row_bucket(n), tail_stride=1, mask_words=(n + 63) // 64, prefix_pages=self.mirror.dev)
        self.engine.warm_graph(1, tail_stride=1, mask_words=1, prefix_pages=self.mirror.dev)

    # -------------------------------------------------------------- scoring
    def _weights_for_depth(self, depth: int) -> tuple[float, ...] | None:
        if self.score_weights is None:
            return None
        if len(self.score_weights) != int(depth):
            raise ValueError(
                f"{len(self.score_weights)} path score weights for routes of depth {depth}"
            )
        return self.score_weights

    def _score_routes(self, routes, paths, path_lp) -> list[TargetRouteScore]:
        out: list[TargetRouteScore] = []
        for route, path, lps in zip(routes, paths, path_lp):
            lps = [float(v) for v in lps]
            total = sum(lps)
            w = self._weights_for_depth(len(lps))
            sel = total if w is None else sum(a * b for a, b in zip(w, lps))
            out.append(
                TargetRouteScore(
                    route_id=int(route.route_id),
                    token_ids=tuple(path),
                    target_logprob=total,
                    draft_logprob=float(route.draft_logprob),
                    token_logprobs=tuple(lps),
                    first_token_logprob=lps[0],
                    selection_score=sel,
                    score_weights=() if w is None else tuple(w),
                    draft_token_logprobs=tuple(float(v) for v in route.draft_token_logprobs),
                )
            )
        return out

    @staticmethod
    def _best_key(s: TargetRouteScore):
        return (s.effective_selection_score, s.draft_path_logprob, -s.route_id)

    def _selection_policy_name(self) -> str:
        if self.route_selection_policy == "first_route":
            return "diagnostic_first_payload_route"
        if self.route_selection_policy == "target_sample":
            return (
                "sample_target_route_logprob_distribution"
                if self.score_weights is None
                else "sample_weighted_target_route_score_distribution"
            )
        return "best_of_n_target_path_logprob" if self.score_weights is None else "best_of_n_weighted_target_path_logprob"

    def _sampling_disabled(self) -> dict[str, object]:
        return {
            "route_sampling_enabled": False,
            "route_sampling_scope": "verified_route_level_only",
            "route_sampling_seed": None,
            "route_sampling_round": None,
            "route_sampling_temperature": float(self.route_sampling_temperature),
        }

    def _select_route_with_metadata(self, scores, *, route_sampling_seed=None, route_sampling_round=None):
        if not scores:
            raise ValueError("no route scores to choose from")
        if self.route_selection_policy == "first_route":
            return scores[0], self._sampling_disabled()
        if self.route_selection_policy == "target_sample":
            return self._sample_route(scores, route_sampling_seed, route_sampling_round)
        return max(scores, key=self._best_key), self._sampling_disabled()

    def _sample_route(self, scores, seed, rnd):
        """Seeded route-level draw (host-side, bit-exact replay).

        Candidates are put in a canonical order (token path, draft score,
        selection score, route id) so the draw does not depend on payload order;
        the uniform is derived from SHA-256 of the domain, seed and round.
        """
        if seed is None or rnd is None:
            raise ValueError(
                "the target_sample policy needs route_sampling_seed and route_sampling_round in every verify request"
            )
        rnd = int(rnd)
        if rnd < 0:
            raise ValueError("route_sampling_round is a round index and must be non-negative")
        seed = int(seed)
        ordered = sorted(
            scores,
            key=lambda s: (tuple(s.token_ids), float(s.draft_path_logprob), s.effective_selection_score, int(s.route_id)),
        )
        temp = self.route_sampling_temperature
        logits = [s.effective_selection_score / temp for s in ordered]
        if any(math.isnan(v) for v in logits):
            raise ValueError("a target route score is NaN; no sampling distribution exists")
        pos_inf = [math.isinf(v) and v > 0 for v in logits]
        if any(pos_inf):
            cnt = sum(pos_inf)
            probs = [1.0 / cnt if f else 0.0 for f in pos_inf]
        else:
            finite = [v for v in logits if math.isfinite(v)]
            if not finite:
                probs = [1.0 / len(ordered)] * len(ordered)
            else:
                mx = max(finite)
                ws = [0.0 if v == -math.inf else math.exp(v - mx) for v in logits]
                tot = sum(ws)
                probs = [w / tot for w in ws]
        material = f"{ROUTE_SAMPLE_DOMAIN}:{seed}:{rnd}".encode("utf-8")
        bits = int.from_bytes(hashlib.sha256(material).digest()[:8], "big")
        u = (bits + 0.5) / float(1 << 64)
        chosen, lo, hi, acc = len(ordered) - 1, 0.0, 1.0, 0.0
        for i, pr in enumerate(probs):
            nxt = acc + pr
            if u < nxt or i == len(ordered) - 1:
                chosen, lo = i, acc
                hi = nxt if i < len(ordered) - 1 else 1.0
                break
            acc = nxt
        return ordered[chosen], {
            "route_sampling_enabled": True,
            "route_sampling_scope": "verified_route_level_only",
            "route_sampling_seed": seed,
            "route_sampling_round": rnd,
            "route_sampling_temperature": temp,
            "route_sampling_uniform": float(u),
            "route_sampling_selected_probability": float(probs[chosen]),
            "route_sampling_selected_cdf_low": float(lo),
            "route_sampling_selected_cdf_high": float(hi),
            "route_sampling_boundary_margin": float(min(u - lo, hi - u)),
            "route_sampling_ordered_candidates": [
                {"route_id": int(s.route_id), "token_path_hash": token_path_hash(s.token_ids), "probability": float(pr)}
                for s, pr in zip(ordered, probs)
            ],
        }

    def _route_intervention_metadata(self, scores, selected) -> dict[str, object]:
        if not scores:
            raise ValueError("intervention metadata needs at least one route score")
        route0 = scores[0]
        order = sorted(enumerate(scores), key=lambda p: (-float(p[1].draft_path_logprob), int(p[0])))
        ranks = {int(s.route_id): i for i, (_, s) in enumerate(order, start=1)}
        top = order[0][1]

        def summary(s: TargetRouteScore) -> dict[str, object]:
            return {
                "route_id": int(s.route_id),
                "token_path_hash": token_path_hash(s.token_ids),
                "first_token_id": int(s.token_ids[0]),
                "draft_rank": int(ranks[int(s.route_id)]),
                "draft_first_token_logprob": s.draft_first_token_logprob,
                "draft_path_logprob": float(s.draft_path_logprob),
                "legacy_cumulative_draft_logprob": float(s.draft_logprob),
                "target_first_token_logprob": None if s.first_token_logprob is None else float(s.first_token_logprob),
                "target_logprob": float(s.target_logprob),
                "target_selection_score": float(s.effective_selection_score),
            }

        def delta(a, b):
            return None if a is None or b is None else float(a) - float(b)

        def compare(base: TargetRouteScore) -> dict[str, object]:
            return {
                "route_changed": tuple(selected.token_ids) != tuple(base.token_ids),
                "first_token_changed": int(selected.token_ids[0]) != int(base.token_ids[0]),
                "draft_first_token_logprob_delta": delta(
                    selected.draft_first_token_logprob, base.draft_first_token_logprob
                ),
                "draft_path_logprob_delta": float(selected.draft_path_logprob) - float(base.draft_path_logprob),
                "legacy_cumulative_draft_logprob_delta": float(selected.draft_logprob) - float(base.draft_logprob),
                "target_first_token_logprob_delta": delta(selected.first_token_logprob, base.first_token_logprob),
                "target_path_logprob_delta": float(selected.target_logprob) - float(base.target_logprob),
                "target_selection_score_delta": selected.effective_selection_score - base.effective_selection_score,
            }

        v0, vt = compare(route0), compare(top)
        return {
            "route_intervention": {
                "baseline": "route0",
                "draft_token_logprobs_available": bool(all(s.draft_token_logprobs for s in scores)),
                "route0_is_draft_top": int(route0.route_id) == int(top.route_id),
                "route0": summary(route0),
                "draft_top": summary(top),
                "selected": summary(selected),
                "selected_vs_route0": v0,
                "selected_vs_draft_top": vt,
            },
            "selected_draft_rank": int(ranks[int(selected.route_id)]),
            "route0_route_id": int(route0.route_id),
            "draft_top_route_id": int(top.route_id),
            "selected_route_changed_from_route0": bool(v0["route_changed"]),
            "selected_first_token_changed_from_route0": bool(v0["first_token_changed"]),
            "selected_minus_route0_draft_first_token_logprob": v0["draft_first_token_logprob_delta"],
            "selected_minus_route0_draft_logprob": float(v0["draft_path_logprob_delta"]),
            "selected_minus_route0_target_selection_score": float(v0["target_selection_score_delta"]),
        }

    @staticmethod
    def _truncate_selected_path(*, token_ids, node_ids, max_tokens, eos_token_id):
        if len(token_ids) != len(node_ids) or not token_ids:
            raise ValueError("a committed path needs as many node ids as tokens, and at least one")
        limit = len(token_ids) if max_tokens is None else min(len(token_ids), int(max_tokens))
        if limit <= 0:
            raise ValueError("selected_path_max_tokens must be positive when given")
        toks = [int(t) for t in token_ids[:limit]]
        if eos_token_id is not None:
            for i, t in enumerate(toks):
                if t == int(eos_token_id):
                    toks = toks[: i + 1]
                    break
        return tuple(toks), tuple(int(n) for n in node_ids[: len(toks)])

    def _fallback_reason(self, selected: TargetRouteScore) -> str | None:
        if (
            self.first_token_threshold is not None
            and selected.first_token_logprob is not None
            and float(selected.first_token_logprob) < self.first_token_threshold
        ):
            return "first_token_below_threshold"
        if self.fallback_threshold is not None and selected.effective_selection_score < self.fallback_threshold:
            return "path_score_below_threshold"
        return None

    # --------------------------------------------------------------- commit
    @torch.inference_mode()
    def _commit_selected_path(self, token_ids, node_ids, logits: torch.Tensor) -> None:
        if len(token_ids) != len(node_ids) or not node_ids:
            raise ValueError("a committed path needs as many node ids as tokens, and at least one")
        p = len(self.prefix_token_ids)
        moves = [(p + int(n), p + j) for j, n in enumerate(node_ids) if int(n) != j]
        if moves:
            src = torch.tensor([a for a, _ in moves], dtype=torch.int64)
            dst = torch.tensor([b for _, b in moves], dtype=torch.int64)
            src_slots = torch.cat([self.seq.slots_for_positions(int(a), 1) for a in src])
            dst_slots = torch.cat([self.seq.slots_for_positions(int(b), 1) for b in dst])
            self.engine.move_slots(src_slots, dst_slots)
        self.seq.set_prefix_len(p + len(node_ids))
        self._sync()
        self.prefix_token_ids = (*self.prefix_token_ids, *(int(t) for t in token_ids))
        self._prefix_logits = logits[int(node_ids[-1])].detach().clone()
        self._committed_verify_rounds += 1

    # ------------------------------------------------------------ fallback
    def _profile_sync(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    @torch.inference_mode()
    def _generate_fallback_ar(self, *, max_tokens: int, eos_token_id: int | None, while_running=None) -> list[int]:
        """Greedy AR from the committed prefix; ``while_running`` (optional) is called after
        every step is enqueued and before the host waits for the tokens."""
        self._flush_pending()
        if self._prefix_logits is None:
            raise RuntimeError("fallback AR needs a prefilled target (no prefix logits yet)")
        steps = int(max_tokens)
        if steps <= 0:
            return []
        prof = self.profile_fallback_ar
        t_setup = time.perf_counter()
        p = len(self.prefix_token_ids)
        slots = self.seq.reserve_scratch(p + steps)
        self._sync()
        if prof:
            self._profile_sync()
        setup_s = time.perf_counter() - t_setup
        dev = self.device
        toks = torch.empty(steps, dtype=torch.int32, device=dev)
        all_logits: list[torch.Tensor] = []
        cur = self._prefix_logits.reshape(1, -1)
        t_model = time.perf_counter()
        if cur.is_cuda:
            from ..ops.cuda_ops import shared_ops

            sops = shared_ops(dev)

            def argmax_into(row: torch.Tensor, t: int) -> None:
                _, ids = sops.topk_logprobs(row, 1)
                toks[t: t + 1] = ids.reshape(-1).to(torch.int32)
        else:

            def argmax_into(row: torch.Tensor, t: int) -> None:
                toks[t: t + 1] = torch.argmax(row, dim=-1).to(torch.int32)

        slots_np = slots.numpy()
        n_pages = len(self.mirror.host)
        for t in range(steps):
            argmax_into(cur, t)
            if t == steps - 1:
                break  # the last token's forward runs with the next verify (or on demand)
            cur = self.engine.run_rows(
                1,
                prefix_pages=self.mirror.dev,
                tokens=toks[t: t + 1],
                positions=[p + t],
                slots=slots_np[t: t + 1],
                shared_len=p + t,
                n_shared_pages=n_pages,
                mask_base=p + t,
                row_full=[p + t + 1],
                row_len=[p + t + 1],
            )
            all_logits.append(cur)
        if while_running is not None:
            while_running()
        try:
            (host_toks,) = read_back([toks], self.status_flag(), where="target fallback AR")
        except KernelError:
            self.seq.set_prefix_len(p)
            self._sync()
            raise
        generated = [int(x) for x in host_toks.tolist()]
        if prof:
            self._profile_sync()
        model_s = time.perf_counter() - t_model
        keep = len(generated)
        if eos_token_id is not None:
            for i, t in enumerate(generated):
                if t == int(eos_token_id):
                    keep = i + 1
                    break
        generated = generated[:keep]
        self.seq.set_prefix_len(p + keep)
        self._sync()
        if keep == steps:
            self._pending_token = int(generated[-1])
            self._prefix_logits = None
        else:
            self._prefix_logits = all_logits[keep - 1][0].detach().clone()
        self.prefix_token_ids = (*self.prefix_token_ids, *generated)
        self._committed_verify_rounds += 1
        self._last_fallback_ar_profile = (
            {
                "enabled": True,
                "wrapper_was_cached": True,
                "wrapper_setup_seconds": setup_s,
                "decode_plan_seconds": 0.0,
                "model_forward_seconds": model_s,
                "token_count": len(generated),
            }
            if prof
            else None
        )
        return generated

    # ------------------------------------------------------------- metadata
    def runtime_metadata(self) -> dict[str, object]:
        from .metadata import runtime_info

        cfg = getattr(self.engine, "model_cfg", self.engine.cfg)
        tp = getattr(self.engine, "tp", None)
        return {
            "backend": "b200_native_masked_tree_verify",
            "framework": runtime_info(self.device),
            "tensor_parallel": 1 if tp is None else int(tp.world),
            "tensor_parallel_comm": None if tp is None else tp.mode,
            "model": self.model_name,
            "model_vocab_size": int(cfg.vocab_size),
            "paged_kv": True,
            "custom_mask": True,
            "ancestor_mask_words": "per-node 64-bit words over the node region only",
            "rope_applied": True,
            "semantic_correctness_required": True,
            "page_size": int(self.page_size),
            "dtype": str(self.engine.dtype).replace("torch.", ""),
            "device": str(self.device),
            "persistent_target_paged_kv": True,
            "deduplicated_tree_nodes": True,
            "selection_policy": self._selection_policy_name(),
            "route_selection_policy": self.route_selection_policy,
            "route_sampling_scope": "verified_route_level_only",
            "route_sampling_temperature": float(self.route_sampling_temperature),
            "fallback_ar_sampling": "greedy_argmax",
            "score_weights": None if self.score_weights is None else [float(v) for v in self.score_weights],
            "fallback_threshold": self.fallback_threshold,
            "first_token_threshold": self.first_token_threshold,
            "fallback_ar_tokens": int(self.fallback_ar_tokens),
            "profile_fallback_ar": self.profile_fallback_ar,
            "committed_verify_rounds": self._committed_verify_rounds,
            "committed_prefix_length": len(self.prefix_token_ids),
            "k": self.k,
            "d": self.d,
        }

    @property
    def prefix_logits(self) -> torch.Tensor | None:
        self._flush_pending()
        return self._prefix_logits
