"""No-KV recompute backend for the clean controller (correctness only).

Every call recomputes whole padded sequences with the fp32-accumulating
oracle forward, so it needs no KV state at all; it is the independent check
for the paged runtimes.  Parity: reference src/atlas_0709/hf_backend.py:11-155
(HFRecomputeBatchBackend), here on this package's own model definition.
"""

from __future__ import annotations

from typing import Sequence

import torch

from ..models.llama import LlamaWeights, reference_forward
from ..types import PrefixState, TargetRouteScore, TargetVerifyResult
from .clean import BatchDecodeOutput


class RecomputeBatchBackend:
    def __init__(self, weights: LlamaWeights, *, name: str = "recompute") -> None:
        self.w = weights
        self.name = name

    def _last_logits(self, tokens: Sequence[int]) -> torch.Tensor:
        return reference_forward(self.w, list(tokens))[-1]

    def prefill(self, prompt_token_ids: Sequence[int]) -> PrefixState:
        toks = tuple(int(t) for t in prompt_token_ids)
        return PrefixState(toks, self._last_logits(toks), len(toks), {"backend": "recompute_batch", "name": self.name})

    def decode_batch(self, *, prefix_token_ids, routes) -> BatchDecodeOutput:
        base = [int(t) for t in prefix_token_ids]
        rows = [self._last_logits(base + list(r.pending_path)) for r in routes]
        return BatchDecodeOutput(tuple(r.route_id for r in routes), torch.stack(rows),
                                 {"backend": "recompute_batch", "batch_size": len(routes)})

    def verify_batch(self, *, prefix_token_ids, routes) -> TargetVerifyResult:
        base = [int(t) for t in prefix_token_ids]
        scores = []
        for r in routes:
            path = list(r.materialized_tokens[: r.stage1_depth])
            logits = reference_forward(self.w, base + path)
            lp = torch.log_softmax(logits.float(), -1)
            toks = [lp[len(base) - 1 + i, t].item() for i, t in enumerate(path)]
            scores.append(TargetRouteScore(r.route_id, tuple(path), float(sum(toks)), r.cumulative_logprob,
                                           token_logprobs=tuple(toks), first_token_logprob=toks[0]))
        best = max(scores, key=lambda s: (s.target_logprob, s.draft_logprob, -s.route_id))
        return TargetVerifyResult(best.route_id, scores, {"backend": "recompute_batch"})
