"""Serial tree -> verify baseline (no forest, no overlap, no stage-2 reuse).

Same drafter, target, scoring and fallback as the async coordinator, so
quality comparisons isolate the scheduling.  Phase timers synchronize the
device at phase boundaries.  Parity: reference src/atlas_0709/serial_system.py:18-326.
"""

from __future__ import annotations

import time
from typing import Sequence

import torch

from ..runtime.builders import build_tree_depths, initialize_stage1_routes
from ..runtime.store import KVTreeStore
from .edge import COMPACT_DECISION_KEYS, DistributedGenerationResult, DistributedRoundTrace, PagedDistributedAtlasGenerator
from .rpc import selected_route_id_from_response


def _sync(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


class SerialAtlasGenerator(PagedDistributedAtlasGenerator):
    system_name = "atlas_serial_tree_verify"

    def generate(self, prompt_token_ids: Sequence[int]) -> DistributedGenerationResult:
        cfg = self.config
        dev = self.drafter.device
        committed = [int(t) for t in prompt_token_ids]
        generated: list[int] = []
        traces: list[DistributedRoundTrace] = []
        fallback_profiles: list[dict[str, object]] = []
        health = self.target_client.health()
        target_meta = dict(health.get("metadata", {}))
        store = KVTreeStore()
        self.drafter.bind_store(store)

        t = time.perf_counter()
        self.target_client.prefill(committed)
        target_prefill_s = time.perf_counter() - t
        t = time.perf_counter()
        self.drafter.prefill(committed)
        store.committed_token_ids = list(committed)
        _sync(dev)
        drafter_prefill_s = time.perf_counter() - t

        drafter_s = target_s = fb_append_s = 0.0
        fb_appended = 0
        last_verify_s = None
        round_index = 0
        total_start = time.perf_counter()
        while len(generated) < cfg.max_new_tokens:
            rs = self._sampling(committed)
            t = time.perf_counter()
            active = initialize_stage1_routes(self.drafter.prefix_state(), k=cfg.k, route_store=store, sampling=rs,
                                              model_backend=self.drafter)
            stage1 = build_tree_depths(
                active, depth=cfg.d, k=cfg.k, route_store=store, model_backend=self.drafter, sampling=rs
            )
            _sync(dev)
            drafter_s += time.perf_counter() - t
            remaining = cfg.max_new_tokens - len(generated)
            t = time.perf_counter()
            resp = self.target_client.verify(
                prefix_token_ids=committed,
                routes=self._route_payloads(store, stage1.completed_routes),
                fallback_max_tokens=min(int(cfg.fallback_ar_tokens), int(remaining)),
                selected_path_max_tokens=int(remaining),
                eos_token_id=cfg.eos_token_id,
                route_sampling_seed=int(cfg.generation_seed),
                route_sampling_round=int(round_index),
            )
            last_verify_s = time.perf_counter() - t
            target_s += last_verify_s
            tmeta = dict(resp.get("metadata", {}))
            prof = tmeta.get("fallback_ar_profile")
            if isinstance(prof, dict):
                fallback_profiles.append({"round_index": round_index, **prof})
            decision = str(resp.get("decision", "select"))
            sel_id: int | None = None
            reason: str | None = None
            fb: list[int] = []
            if decision == "fallback_ar":
                fb = [int(x) for x in resp.get("fallback_token_ids", [])]
                reason = None if resp.get("fallback_reason") is None else str(resp.get("fallback_reason"))
                if not fb:
                    raise RuntimeError("a fallback round returned no target tokens")
                if len(fb) > remaining:
                    raise RuntimeError(
                        f"the target's fallback overran the token budget: "
                        f"returned={len(fb)}, remaining={remaining}"
                    )
                now = list(fb)
                mode = "serial_fallback_ar_append_persistent_kv"
            elif decision == "select":
                sel_id = selected_route_id_from_response(resp)
                sel = self._find_route(stage1, sel_id)
                full = list(store.materialized_token_path(sel)[: cfg.d])
                now = self._truncate_commit(full, generated)
                if not now:
                    raise RuntimeError("the target selected a route but nothing was left to commit")
                mode = "serial_tree_only_persistent_kv"
            else:
                raise RuntimeError(f"the target answered with decision {decision!r}, expected select or fallback_ar")
            generated.extend(now)
            committed.extend(now)
            stop = self._should_stop(now, generated)
            t = time.perf_counter()
            phys = {"committed_kv_tokens": 0, "released_route_rows": 0, "released_kv_pages": 0}
            if decision == "select":
                if now == full and not stop:
                    _, phys = self.drafter.commit_stage1_and_promote(committed_route=sel, retained_routes=[])
                    self.drafter.prefix_next_token_logits = stage1.last_logits[
                        [i for i, r in enumerate(stage1.completed_routes) if r.route_id == sel_id]
                    ]
                    store.reset_speculative()
            elif not stop:
                dropped = self.drafter.drop_speculative()
                store.committed_token_ids.extend(now)
                self.drafter.append_known_tokens_as_prefix(now)
                phys = {
                    "committed_kv_tokens": len(now),
                    "released_route_rows": dropped["released_route_rows"],
                    "released_kv_pages": dropped["released_kv_pages"],
                }
            _sync(dev)
            ho = time.perf_counter() - t
            drafter_s += ho
            if decision == "fallback_ar":
                fb_append_s += ho
                fb_appended += len(now)
            traces.append(
                DistributedRoundTrace(
                    round_index=round_index,
                    selected_route_id=sel_id,
                    committed_tokens=list(now),
                    decision=decision,
                    fallback_reason=reason,
                    fallback_token_ids=list(fb),
                    forest_depth=0,
                    verify_returned_before_forest_done=False,
                    target_scores=list(resp.get("scores", [])),
                    handoff_mode=mode,
                    reused_stage2_routes=0,
                    reused_stage2_depth=0,
                    remaining_tree_depth=0,
                    committed_kv_tokens=int(phys["committed_kv_tokens"]),
                    released_route_rows=int(phys["released_route_rows"]),
                    released_kv_pages=int(phys["released_kv_pages"]),
                    target_unique_tree_nodes=int(tmeta.get("node_count", 0)),
                    target_unmerged_path_nodes=int(tmeta.get("unmerged_path_node_count", 0)),
                    target_prefix_len_before=int(tmeta.get("prefix_len_before", len(committed) - len(now))),
                    target_prefix_len_after=int(tmeta.get("prefix_len_after", len(committed))),
                    target_decision_metadata={k: tmeta[k] for k in COMPACT_DECISION_KEYS if k in tmeta},
                )
            )
            round_index += 1
            if stop:
                break
        total_s = time.perf_counter() - total_start
        n = len(generated)
        fb_rounds = sum(tr.decision == "fallback_ar" for tr in traces)
        return DistributedGenerationResult(
            prompt_token_ids=[int(x) for x in prompt_token_ids],
            generated_token_ids=generated,
            text=self.tokenizer.decode(committed) if self.tokenizer is not None else None,
            rounds=traces,
            metadata={
                "system": self.system_name,
                "execution_mode": "serial_tree_verify",
                "async": False,
                "build_forest": False,
                "prefill_overlap": False,
                "verify_overlap": False,
                "serial_phase_order": "drafter_build_tree_then_target_verify",
                "drafter_backend": "b200_native_paged_decode",
                "target_backend": target_meta.get("backend"),
                "target_transport": str(health.get("transport", "http")),
                "target_health": health,
                "k": cfg.k,
                "d": cfg.d,
                "max_new_tokens": cfg.max_new_tokens,
                "fallback_ar_tokens": int(cfg.fallback_ar_tokens),
                "generation_seed": int(cfg.generation_seed),
                "drafter_sampling": self._sampling_config().to_dict(),
                "drafter_prefill_elapsed_s": drafter_prefill_s,
                "target_prefill_elapsed_s": target_prefill_s,
                "rebuild_drafter_prefix_after_commit": False,
                "cross_round_drafter_prefix_kv_reuse": True,
                "cross_round_stage2_kv_reuse": False,
                "cross_round_target_kv_reuse": True,
                "target_selection_policy": target_meta.get("selection_policy"),
                "target_route_selection_policy": target_meta.get("route_selection_policy"),
                "last_verify_elapsed_s": last_verify_s,
                "generated_tokens": n,
                "rounds": len(traces),
                "fallback_rounds": fb_rounds,
                "fallback_rate": fb_rounds / len(traces) if traces else None,
                "fallback_drafter_append_mode": "single_multi_token_extend",
                "target_fallback_ar_profiles": fallback_profiles,
                "fallback_appended_tokens": fb_appended,
                "fallback_append_elapsed_s": fb_append_s,
                "fallback_append_tokens_per_second": fb_appended / fb_append_s if fb_append_s else None,
                "drafter_elapsed_s": drafter_s,
                "target_elapsed_s": target_s,
                "total_elapsed_s": total_s,
                "drafter_tokens_per_second": n / drafter_s if drafter_s else None,
                "target_tokens_per_second": n / target_s if target_s else None,
                "overall_tokens_per_second": n / total_s if total_s else None,
                "throughput_token_definition": "committed_generated_tokens",
                "throughput_excludes_target_prompt_prefill": True,
                "throughput_excludes_drafter_prompt_prefill": True,
                "route_tail_page_cow": True,
            },
        )
