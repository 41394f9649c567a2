"""Llama forward executor over a paged KV cache.

One engine owns a model's weights, its KV cache
``[layers, pages, 2, kv_heads, page_size, head_dim]`` and a rotary table.
``forward`` runs any batch of rows (drafter routes, target tree nodes, an AR
token, a prefill chunk): each row has a token, a position, the KV slot it
writes, and an attention descriptor row.  On CUDA devices every op is an
sm_100a kernel from the ``atlas_cuda`` extension (the forward raises if the
extension is missing); on CPU the PyTorch ops in ``ops.torch_ops`` run.

Parity: reference src/atlas_0709/flashinfer_full_verify.py:1065-1231 (manual
Llama layer loop with RoPE, suffix KV write and paged attention) and the
SGLang decode forward the drafter uses (fp/flashinfer_backends.py:89-132).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..models.llama import LlamaWeights, rope_table
from ..ops import torch_ops
from ..ops.attn_desc import AttnDesc, single_sequence_desc


def kv_bytes_per_token(cfg) -> int:
    return cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2


@dataclass
class ForwardStats:
    calls: int = 0
    rows: int = 0
    prefill_tokens: int = 0


class LlamaEngine:
    def __init__(
        self,
        weights: LlamaWeights,
        *,
        num_pages: int,
        page_size: int = 16,
        max_positions: int = 32768,
        ops=None,
    ) -> None:
        self.w = weights
        self.cfg = weights.config
        self.device = weights.device
        self.dtype = weights.dtype
        self.page_size = int(page_size)
        self.num_pages = int(num_pages)
        c = self.cfg
        self.kv = torch.zeros(
            (c.num_layers, self.num_pages, 2, c.num_kv_heads, self.page_size, c.head_dim),
            dtype=self.dtype,
            device=self.device,
        )
        self.rope = rope_table(c, max_positions, device=self.device)
        self.scale = 1.0 / math.sqrt(c.head_dim)
        if ops is None:
            if self.device.type == "cuda":
                from ..ops import cuda_ops

                ops = cuda_ops.CudaOps(self)
            else:
                ops = torch_ops
        self.ops = ops
        self.stats = ForwardStats()

    # ------------------------------------------------------------------
    @torch.inference_mode()
    def forward(
        self,
        tokens: torch.Tensor,
        positions: torch.Tensor,
        slots: torch.Tensor,
        desc: AttnDesc,
        *,
        logits_rows: torch.Tensor | None = None,
        causal_start: int | None = None,
    ) -> torch.Tensor:
        """Run all layers for ``M`` rows; return fp32 logits for ``logits_rows`` (default: all)."""
        o = self.ops
        c = self.cfg
        self.stats.calls += 1
        self.stats.rows += int(tokens.numel())
        h = o.embed(tokens, self.w.embed)
        for li, lw in enumerate(self.w.layers):
            x = o.rmsnorm(h, lw.attn_norm, c.rms_eps, self.dtype)
            qkv = o.linear(x, lw.wqkv)
            q = o.rope_qkv_append(qkv, self.rope, positions, slots, self.kv[li], c.num_heads, c.num_kv_heads)
            if causal_start is None:
                a = o.attention(q, self.kv[li], desc, self.scale)
            else:
                a = o.attention_causal(q, self.kv[li], desc, causal_start, self.scale) if hasattr(
                    o, "attention_causal"
                ) else o.attention(q, self.kv[li], desc, self.scale)
            h = o.linear_residual(a, lw.wo, h)
            x = o.rmsnorm(h, lw.mlp_norm, c.rms_eps, self.dtype)
            act = o.gate_up_silu(x, lw.wgu)
            h = o.linear_residual(act, lw.wd, h)
        if logits_rows is not None:
            h = h.index_select(0, logits_rows.long())
        x = o.rmsnorm(h, self.w.final_norm, c.rms_eps, self.dtype)
        return o.lm_head(x, self.w.lm_head)

    # ------------------------------------------------------------------
    def prefill_sequence(
        self,
        tokens: torch.Tensor,
        *,
        start_pos: int,
        slots: torch.Tensor,
        pages: torch.Tensor,
        chunk_size: int = 8192,
    ) -> torch.Tensor:
        """Causal prefill of ``tokens`` at positions ``start_pos..`` in one page list.

        Runs in chunks of ``chunk_size``; returns the fp32 logits of the last token.
        """
        n = int(tokens.numel())
        if n == 0:
            raise ValueError("prefill needs at least one token")
        dev = self.device
        logits = None
        self.stats.prefill_tokens += n
        for c0 in range(0, n, int(chunk_size)):
            c1 = min(n, c0 + int(chunk_size))
            pos = torch.arange(start_pos + c0, start_pos + c1, dtype=torch.int32, device=dev)
            desc = single_sequence_desc(pages, pos + 1, shared_len=start_pos + c0)
            last = torch.tensor([c1 - c0 - 1], dtype=torch.long, device=dev)
            logits = self.forward(
                tokens[c0:c1], pos, slots[c0:c1], desc, logits_rows=last, causal_start=start_pos + c0
            )
        assert logits is not None
        return logits[0]

    def copy_pages(self, copies: torch.Tensor) -> None:
        if copies.numel():
            self.ops.kv_copy_pages(self.kv, copies.to(self.device))

    def move_slots(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        if src.numel():
            self.ops.kv_move_slots(self.kv, src.to(self.device), dst.to(self.device))
