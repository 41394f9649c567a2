"""Drafter-only autoregressive baseline on the same paged runtime.

Batch-1 greedy (or keyed-sampling) decoding through ``k=1`` tree steps, so it
exercises exactly the drafter path the speculative generator uses.
Parity: reference src/atlas_0709/flashinfer_ar.py:18-126.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from ..runtime.builders import build_tree_one_depth, initialize_stage1_routes
from ..runtime.drafter import DrafterRuntime
from ..runtime.sampling import DrafterSamplingConfig, DrafterSamplingContext
from ..runtime.store import KVTreeStore


@dataclass(frozen=True)
class ARResult:
    generated_token_ids: list[int]
    finish_reason: str
    metadata: dict[str, object]


class PagedGreedyARGenerator:
    def __init__(self, *, drafter: DrafterRuntime) -> None:
        self.drafter = drafter

    @torch.inference_mode()
    def generate(self, prompt_token_ids: Sequence[int], *, max_new_tokens: int, eos_token_id: int | None = None,
                 do_sample: bool = False, generation_seed: int = 0, temperature: float = 1.0) -> ARResult:
        if not prompt_token_ids:
            raise ValueError("prompt_token_ids cannot be empty")
        if max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        cfg = DrafterSamplingConfig(bool(do_sample), int(generation_seed), float(temperature))
        sampling = DrafterSamplingContext(cfg, tuple(int(t) for t in prompt_token_ids))
        store = KVTreeStore()
        self.drafter.bind_store(store)
        self.drafter.prefill(prompt_token_ids)
        routes = initialize_stage1_routes(self.drafter.prefix_state(), k=1, route_store=store, sampling=sampling)
        out: list[int] = []
        reason = "length"
        while len(out) < int(max_new_tokens):
            tok = int(routes[0].pending_token_id)
            out.append(tok)
            if eos_token_id is not None and tok == int(eos_token_id):
                reason = "eos"
                break
            if len(out) >= int(max_new_tokens):
                break
            step = build_tree_one_depth(routes, k=1, route_store=store, model_backend=self.drafter, sampling=sampling)
            # Commit the decoded token so the route's private tail stays one page deep.
            routes, _ = self.drafter.commit_stage1_and_promote(
                committed_route=step.decoded_routes[0], retained_routes=step.next_routes
            )
        self.drafter.drop_speculative()
        return ARResult(out, reason, {
            "backend": "b200_native_paged_sampled_ar" if do_sample else "b200_native_paged_greedy_ar",
            "batch_size": 1,
            "paged_kv": True,
            "page_size": self.drafter.page_size,
            **cfg.to_dict(),
            "generation_seed": int(generation_seed),
        })
