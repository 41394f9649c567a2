"""Llama engine over block-scaled fp8 weights (the 70B-on-one-GPU target).

Same paged KV, graphs and attention as ``LlamaEngine``; the projections run
the fp8 tcgen05 GEMM.  Activations are quantized per token per 128 columns
right where they are produced: RMSNorm writes e4m3 + scales directly
(``rmsnorm_fp8``), the attention output and the SiLU·mul output go through
``quant_fp8``.  KV cache, attention, residual stream (fp32) and LM head stay
in bf16/fp16.  On CPU the fp32 emulation in ``models.fp8`` runs.
"""

from __future__ import annotations

import torch

from ..models import fp8 as fp8m
from ..ops import torch_ops
from .engine import LlamaEngine


class Fp8LlamaEngine(LlamaEngine):
    def __init__(self, weights: fp8m.Fp8LlamaWeights, **kw) -> None:
        super().__init__(weights, **kw)  # type: ignore[arg-type]

    @torch.inference_mode()
    def forward(self, tokens, positions, slots, desc, *, logits_rows=None, causal_start=None):
        o = self.ops
        c = self.cfg
        self.stats.calls += 1
        self.stats.rows += int(tokens.numel())
        cuda = self.device.type == "cuda"
        h = o.embed(tokens, self.w.embed)
        m = h.shape[0]
        for li, lw in enumerate(self.w.layers):
            if cuda:
                xq, sa = o.rmsnorm_fp8(h, lw.attn_norm, c.rms_eps)
                qkv = o.gemm_fp8(xq, sa, lw.wqkv, torch.empty((m, c.qkv_size), dtype=self.dtype, device=h.device),
                                 o.ext.EPI_STORE)
            else:
                qkv = fp8m.fp8_matmul_ref(torch_ops.rmsnorm(h, lw.attn_norm, c.rms_eps, torch.float32),
                                          lw.wqkv).to(self.dtype)
            q = o.rope_qkv_append(qkv, self.rope, positions, slots, self.kv[li], c.num_heads, c.num_kv_heads)
            if causal_start is not None and hasattr(o, "attention_causal"):
                a = o.attention_causal(q, self.kv[li], desc, causal_start, self.scale)
            else:
                a = o.attention(q, self.kv[li], desc, self.scale)
            if cuda:
                aq, sa = o.quant_fp8(a)
                o.gemm_fp8(aq, sa, lw.wo, h, o.ext.EPI_RESIDUAL)
                xq, sa = o.rmsnorm_fp8(h, lw.mlp_norm, c.rms_eps)
                act = torch.empty((m, c.intermediate_size), dtype=self.dtype, device=h.device)
                o.gemm_fp8(xq, sa, lw.wgu, act, o.ext.EPI_SILU)
                dq, sa = o.quant_fp8(act)
                o.gemm_fp8(dq, sa, lw.wd, h, o.ext.EPI_RESIDUAL)
            else:
                h += fp8m.fp8_matmul_ref(a, lw.wo)
                gu = fp8m.fp8_matmul_ref(torch_ops.rmsnorm(h, lw.mlp_norm, c.rms_eps, torch.float32), lw.wgu)
                g = gu.reshape(m, -1, 2, 64)[:, :, 0].reshape(m, -1)
                u = gu.reshape(m, -1, 2, 64)[:, :, 1].reshape(m, -1)
                act = (torch.nn.functional.silu(g) * u).to(self.dtype)
                h += fp8m.fp8_matmul_ref(act, lw.wd)
        if logits_rows is not None:
            h = h.index_select(0, logits_rows.long())
        x = o.rmsnorm(h, self.w.final_norm, c.rms_eps, self.dtype)
        return o.lm_head(x, self.w.lm_head)
