"""Drafter-only autoregressive baseline on the same paged runtime (batch 1).

Decoding is a stream over one route: the route's pending token is the next
output token; to produce the one after it, the route takes one frontier depth
with ``k = 1`` (decode, best child) and the decoded token is committed at once,
so the route never holds more than one private token and every forward reads
the shared prefix pages -- exactly the drafter path the speculative generator
uses, with greedy or keyed sampling.

Result fields and metadata keys follow the reference's AR baseline
(src/atlas_0709/flashinfer_ar.py:18-126).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, Sequence

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

    def _token_stream(self, prompt: Sequence[int], sampling: DrafterSamplingContext) -> Iterator[int]:
        """Yield output tokens one at a time; the next one is decoded only when asked for."""
        dr = self.drafter
        store = KVTreeStore()
        dr.bind_store(store)
        dr.prefill(prompt)
        (route,) = initialize_stage1_routes(dr.prefix_state(), k=1, route_store=store, sampling=sampling,
                                            model_backend=dr)
        try:
            while True:
                tok = int(route.pending_token_id)
                yield tok
                step = build_tree_one_depth([route], k=1, route_store=store, model_backend=dr, sampling=sampling)
                (route,), _ = dr.commit_stage1_and_promote(committed_route=step.decoded_routes[0],
                                                           retained_routes=step.next_routes)
                if sampling.config.do_sample:
                    # Keys hash the committed prefix plus the path after it: the token just
                    # committed joins the prefix, as the route store's relative paths now start
                    # after it.
                    sampling = DrafterSamplingContext(sampling.config, (*sampling.committed_token_ids, tok))
        finally:
            dr.drop_speculative()

    @torch.inference_mode()
    def generate(self, prompt_token_ids: Sequence[int], *, max_new_tokens: int, eos_token_id: int | None = None,
                 do_sample: bool = False, generation_seed: int = 0, temperature: float = 1.0) -> ARResult:
        prompt = [int(t) for t in prompt_token_ids]
        if not prompt:
            raise ValueError("the AR baseline needs a non-empty prompt")
        budget = int(max_new_tokens)
        if budget < 1:
            raise ValueError(f"max_new_tokens must be at least 1, got {max_new_tokens}")
        cfg = DrafterSamplingConfig(bool(do_sample), int(generation_seed), float(temperature))
        out: list[int] = []
        finish = "length"
        stream = self._token_stream(prompt, DrafterSamplingContext(cfg, tuple(prompt)))
        try:
            for tok in stream:
                out.append(tok)
                if eos_token_id is not None and tok == int(eos_token_id):
                    finish = "eos"
                    break
                if len(out) == budget:
                    break
        finally:
            stream.close()
        return ARResult(out, finish, {
            "backend": "b200_native_paged_sampled_ar" if do_sample else "b200_native_paged_greedy_ar",
            "batch_size": 1,
            "paged_kv": True,
            "page_size": self.drafter.page_size,
            **cfg.to_dict(),
            "generation_seed": int(generation_seed),
        })
