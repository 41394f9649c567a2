"""Drafter candidate generation: greedy top-k or keyed Gumbel-top-k sampling.

Sampling draws ``k`` distinct children per parent with the Gumbel-top-k
construction (Kool, van Hoof and Welling, "Stochastic Beams and Where to Find
Them", ICML 2019).  The noise for vocabulary entry ``v`` is a pure function of
a 63-bit key and ``v`` (a SplitMix64-style integer mix, Steele, Lea and Flood,
OOPSLA 2014), so a candidate set depends only on the request seed and the
complete absolute token history of its parent -- not on batch order, batch
size or how much speculative forest work ran.  The same function runs in the
fused CUDA top-k kernel and here in PyTorch.

Recorded candidate scores are always the untempered model log-probabilities.

Behavioural parity: reference src/atlas_0709/flashinfer_paged/sampling.py:16-156
(semantic-prefix keyed, reproducible, batch-order independent sampling).
The key derivation differs (incremental BLAKE2b over the history with the
length appended last, so the committed prefix is hashed once per round).
"""

from __future__ import annotations

import hashlib
import math
import struct
from dataclasses import dataclass, field
from typing import Sequence

import torch

_DOMAIN = b"atlas-b200-drafter-history-key-v1\0"
KEY_MASK = (1 << 63) - 1
_M64 = (1 << 64) - 1


@dataclass(frozen=True)
class DrafterSamplingConfig:
    do_sample: bool = False
    seed: int = 0
    temperature: float = 1.0

    def validate(self) -> None:
        t = float(self.temperature)
        if not math.isfinite(t) or t <= 0.0:
            raise ValueError(f"drafter sampling temperature {self.temperature} is not a positive finite number")

    def to_dict(self) -> dict[str, object]:
        return {
            "do_sample": bool(self.do_sample),
            "seed": int(self.seed),
            "temperature": float(self.temperature),
            "candidate_sampling": (
                "semantic_prefix_gumbel_topk_without_replacement" if self.do_sample else "model_logprob_topk"
            ),
            "rng_key": ("request_seed_and_complete_semantic_parent_token_prefix" if self.do_sample else None),
        }


@dataclass(frozen=True)
class DrafterSamplingContext:
    """Binds request sampling to the committed prefix of the current round."""

    config: DrafterSamplingConfig
    committed_token_ids: tuple[int, ...]
    _prefix_state: object = field(default=None, repr=False, compare=False)

    def __post_init__(self) -> None:
        self.config.validate()
        if not isinstance(self.committed_token_ids, tuple):
            object.__setattr__(self, "committed_token_ids", tuple(int(t) for t in self.committed_token_ids))

    def _prefix_hash(self):
        """Hash state of (domain, seed, committed prefix); built on first use -- greedy
        drafting never needs it, and the prefix grows to thousands of tokens."""
        h = self._prefix_state
        if h is None:
            h = hashlib.blake2b(digest_size=8)
            h.update(_DOMAIN)
            h.update(struct.pack("<Q", int(self.config.seed) & _M64))
            h.update(_pack_tokens(self.committed_token_ids))
            object.__setattr__(self, "_prefix_state", h)
        return h

    def seed_for_parent(self, relative_parent_path: Sequence[int]) -> int:
        """63-bit key for the parent whose absolute history is prefix + relative path."""
        rel = tuple(int(t) for t in relative_parent_path)
        h = self._prefix_hash().copy()
        h.update(_pack_tokens(rel))
        h.update(struct.pack("<Q", len(self.committed_token_ids) + len(rel)))
        return int.from_bytes(h.digest(), "little") & KEY_MASK


def _pack_tokens(tokens: Sequence[int]) -> bytes:
    for t in tokens:
        if t < 0 or t > KEY_MASK:
            raise ValueError(f"token id {t} does not fit the 63-bit sampling key")
    return struct.pack(f"<{len(tokens)}Q", *tokens)


# ------------------------------------------------------------------ noise
_MIX1 = 0xBF58476D1CE4E5B9
_MIX2 = 0x94D049BB133111EB
_GOLDEN = 0x9E3779B97F4A7C15


def _to_i64(x: int) -> int:
    x &= _M64
    return x - (1 << 64) if x >= (1 << 63) else x


def _lsr(x: torch.Tensor, s: int) -> torch.Tensor:
    """Logical right shift of int64 lanes."""
    return torch.bitwise_and(torch.bitwise_right_shift(x, s), (1 << (64 - s)) - 1)


def keyed_uniform(keys: torch.Tensor, vocab: int) -> torch.Tensor:
    """Uniform(0,1) fp32 noise u[b, v] = mix(key_b + (v + 1) * golden) (exact integer math).

    ``keys`` is an int64 tensor of 63-bit keys, shape [B].  The top 24 bits of
    the mixed word give ``(m + 0.5) / 2**24``, which is exactly representable
    in fp32 and never 0 or 1.
    """
    v = torch.arange(1, vocab + 1, dtype=torch.int64, device=keys.device)
    x = keys.to(torch.int64)[:, None] + v[None, :] * _to_i64(_GOLDEN)
    x = torch.bitwise_xor(x, _lsr(x, 30)) * _to_i64(_MIX1)
    x = torch.bitwise_xor(x, _lsr(x, 27)) * _to_i64(_MIX2)
    x = torch.bitwise_xor(x, _lsr(x, 31))
    m = _lsr(x, 40).to(torch.float32)
    return (m + 0.5) * (1.0 / 16777216.0)


def gumbel_from_uniform(u: torch.Tensor) -> torch.Tensor:
    return -torch.log(-torch.log(u))


def batch_parent_token_candidates(
    logits: torch.Tensor,
    *,
    k: int,
    sampling: DrafterSamplingContext | None,
    relative_parent_paths: Sequence[Sequence[int]],
) -> tuple[torch.Tensor, torch.Tensor]:
    """Return (untempered log-probs, token ids), each [B, k], one distinct set per parent."""
    if k <= 0:
        raise ValueError("k must be positive")
    rows = logits.unsqueeze(0) if logits.ndim == 1 else logits
    if rows.ndim != 2:
        raise ValueError(f"logits must be [vocab] or [rows, vocab], not {tuple(logits.shape)}")
    batch, vocab = int(rows.shape[0]), int(rows.shape[1])
    if len(relative_parent_paths) != batch:
        raise ValueError(f"{len(relative_parent_paths)} parent paths for {batch} rows of logits")
    kk = min(int(k), vocab)
    do_sample = sampling is not None and sampling.config.do_sample
    keys = None
    if do_sample:
        keys = torch.tensor([sampling.seed_for_parent(p) for p in relative_parent_paths], dtype=torch.int64)
    if rows.is_cuda and kk <= 8:
        # Fused log-softmax + top-k (greedy or keyed Gumbel) kernel, one block per row.
        from ..ops.cuda_ops import shared_ops

        temp = float(sampling.config.temperature) if do_sample else 1.0
        return shared_ops(rows.device).topk_logprobs(
            rows, kk, None if keys is None else keys.to(rows.device, non_blocking=True), temp
        )
    logprobs = torch.log_softmax(rows.float(), dim=-1)
    if not do_sample:
        vals, ids = torch.topk(logprobs, k=kk, dim=-1)
        return vals, ids
    keys = keys.to(rows.device)
    noise = gumbel_from_uniform(keyed_uniform(keys, vocab))
    proposal = rows.float() / float(sampling.config.temperature) + noise
    ids = torch.topk(proposal, k=kk, dim=-1).indices
    return logprobs.gather(-1, ids), ids


def single_parent_token_candidates(
    logits: torch.Tensor,
    *,
    k: int,
    sampling: DrafterSamplingContext | None,
    relative_parent_path: Sequence[int] = (),
) -> tuple[torch.Tensor, torch.Tensor]:
    rows = logits.unsqueeze(0) if logits.ndim == 1 else logits
    if int(rows.shape[0]) != 1:
        raise ValueError("single_parent_token_candidates takes one row of logits")
    vals, ids = batch_parent_token_candidates(
        rows, k=k, sampling=sampling, relative_parent_paths=(tuple(relative_parent_path),)
    )
    return vals[0], ids[0]
