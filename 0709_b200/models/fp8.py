"""Block-scaled fp8 (e4m3) weights for the Llama target.

Weights are quantized per 128x128 block (one fp32 scale per block, amax/448)
and activations per token per 128 columns (1x128), the DeepSeek-V3 style
block scaling used for the single-GPU 70B target.  The projection weights
(QKV, O, gate/up, down) are fp8; embedding, norms and the LM head stay in the
activation dtype.  Quantization happens once at load (here, from seeded
random bf16 weights), so ``random_weights_fp8`` and ``quantize_weights``
describe the same model as the bf16 ``random_weights`` up to fp8 rounding.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .llama import LayerWeights, LlamaConfig, LlamaWeights, interleave_gate_up

E4M3_MAX = 448.0
BLOCK = 128


@dataclass
class Fp8Tensor:
    q: torch.Tensor      # [M, K] float8_e4m3fn
    scale: torch.Tensor  # [ceil(M/128), K/128] fp32

    @property
    def shape(self) -> torch.Size:
        return self.q.shape

    def dequantize(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        m, k = self.q.shape
        s = self.scale.repeat_interleave(BLOCK, 0)[:m].repeat_interleave(BLOCK, 1)[:, :k]
        return (self.q.float() * s).to(dtype)

    @property
    def nbytes(self) -> int:
        return self.q.numel() + self.scale.numel() * 4


def quantize_blockwise(w: torch.Tensor) -> Fp8Tensor:
    """[M, K] (K % 128 == 0) -> e4m3 values and per-128x128-block scales."""
    m, k = w.shape
    if k % BLOCK:
        raise ValueError(f"K={k} is not a multiple of {BLOCK}")
    mb = (m + BLOCK - 1) // BLOCK
    pad = mb * BLOCK - m
    wf = w.float()
    if pad:
        wf = torch.cat((wf, wf.new_zeros(pad, k)))
    blocks = wf.reshape(mb, BLOCK, k // BLOCK, BLOCK)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = amax.clamp_min(1e-10) / E4M3_MAX
    q = (blocks / scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).reshape(mb * BLOCK, k)[:m]
    return Fp8Tensor(q.to(torch.float8_e4m3fn).contiguous(), scale.contiguous())


def quantize_activations(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[N, K] -> (e4m3 [N, K], scales [K/128, N]) with one scale per token per 128 columns."""
    n, k = x.shape
    xf = x.float().reshape(n, k // BLOCK, BLOCK)
    scale = xf.abs().amax(-1).clamp_min(1e-10) * (1.0 / E4M3_MAX)
    # amax * (1/448) and x * (1 / scale): the kernels' arithmetic.
    q = (xf * (1.0 / scale)[..., None]).clamp(-E4M3_MAX, E4M3_MAX).reshape(n, k).to(torch.float8_e4m3fn)
    return q, scale.t().contiguous()


def dequantize_activations(xq: torch.Tensor, sa: torch.Tensor) -> torch.Tensor:
    n, k = xq.shape
    return xq.float() * sa[:, :n].t().repeat_interleave(BLOCK, 1)[:, :k]


def fp8_matmul_ref(x: torch.Tensor, w: Fp8Tensor) -> torch.Tensor:
    """fp32 reference of the kernel: quantized activations times quantized weights, block scales applied."""
    xq, sa = quantize_activations(x)
    return dequantize_activations(xq, sa) @ w.dequantize().t()


@dataclass
class Fp8Layer:
    attn_norm: torch.Tensor
    wqkv: Fp8Tensor
    wo: Fp8Tensor
    mlp_norm: torch.Tensor
    wgu: Fp8Tensor
    wd: Fp8Tensor


@dataclass
class Fp8LlamaWeights:
    config: LlamaConfig
    embed: torch.Tensor
    layers: list[Fp8Layer]
    final_norm: torch.Tensor
    lm_head: torch.Tensor

    @property
    def dtype(self) -> torch.dtype:
        return self.embed.dtype

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def nbytes(self) -> int:
        n = self.embed.numel() * self.embed.element_size()
        if self.lm_head is not self.embed:
            n += self.lm_head.numel() * self.lm_head.element_size()
        for l in self.layers:
            n += l.wqkv.nbytes + l.wo.nbytes + l.wgu.nbytes + l.wd.nbytes
        return n


def quantize_layer(lw: LayerWeights) -> Fp8Layer:
    return Fp8Layer(lw.attn_norm, quantize_blockwise(lw.wqkv), quantize_blockwise(lw.wo), lw.mlp_norm,
                    quantize_blockwise(lw.wgu), quantize_blockwise(lw.wd))


def quantize_weights(w: LlamaWeights) -> Fp8LlamaWeights:
    return Fp8LlamaWeights(w.config, w.embed, [quantize_layer(l) for l in w.layers], w.final_norm, w.lm_head)


def random_weights_fp8(cfg: LlamaConfig, *, seed: int = 0, dtype: torch.dtype = torch.bfloat16,
                       device: str | torch.device = "cpu") -> Fp8LlamaWeights:
    """fp8 quantization of ``random_weights(cfg, seed=seed, dtype=dtype)``, one layer in memory at a time."""
    dev = torch.device(device)
    counter = [0]

    def normal(*shape: int) -> torch.Tensor:
        g = torch.Generator(device=dev)
        g.manual_seed((int(seed) * 1_000_003 + counter[0]) & ((1 << 63) - 1))
        counter[0] += 1
        t = torch.empty(*shape, dtype=dtype, device=dev)
        t.normal_(0.0, cfg.init_std, generator=g)
        return t

    h = cfg.hidden_size
    ones = lambda n: torch.ones(n, dtype=dtype, device=dev)  # noqa: E731
    embed = normal(cfg.vocab_size, h)
    layers = []
    for _ in range(cfg.num_layers):
        gate = normal(cfg.intermediate_size, h)
        up = normal(cfg.intermediate_size, h)
        full = LayerWeights(ones(h), normal(cfg.qkv_size, h), normal(h, cfg.q_size), ones(h),
                            interleave_gate_up(gate, up), normal(h, cfg.intermediate_size))
        del gate, up
        layers.append(quantize_layer(full))
        del full
    lm = embed if cfg.tie_word_embeddings else normal(cfg.vocab_size, h)
    return Fp8LlamaWeights(cfg, embed, layers, ones(h), lm)


def fp8_reference_forward(w: Fp8LlamaWeights, tokens: list[int]) -> torch.Tensor:
    """Causal fp32 forward of the fp8 model (activations quantized as the kernels do); returns [T, V] logits."""
    from .llama import apply_rope, rmsnorm_ref, rope_table

    cfg = w.config
    t = len(tokens)
    table = rope_table(cfg, t, device=w.device)
    pos = torch.arange(t, device=w.device)
    h = w.embed[torch.tensor(tokens, device=w.device)].float()
    hq, hk, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    mask = torch.full((t, t), float("-inf"), device=w.device).triu(1)
    for l in w.layers:
        x = rmsnorm_ref(h, l.attn_norm, cfg.rms_eps)
        qkv = fp8_matmul_ref(x, l.wqkv).to(w.dtype).float()
        q = qkv[:, :cfg.q_size].reshape(t, hq, hd)
        k = qkv[:, cfg.q_size:cfg.q_size + cfg.kv_size].reshape(t, hk, hd)
        v = qkv[:, cfg.q_size + cfg.kv_size:].reshape(t, hk, hd)
        q = apply_rope(q, table, pos)
        k = apply_rope(k, table, pos)
        k = k.repeat_interleave(hq // hk, 1)
        v = v.repeat_interleave(hq // hk, 1)
        att = torch.einsum("qhd,khd->hqk", q, k) / hd ** 0.5 + mask
        a = torch.einsum("hqk,khd->qhd", att.softmax(-1), v).reshape(t, hq * hd).to(w.dtype)
        h = h + fp8_matmul_ref(a, l.wo)
        x = rmsnorm_ref(h, l.mlp_norm, cfg.rms_eps)
        gu = fp8_matmul_ref(x, l.wgu)
        g, u = gu.reshape(t, -1, 2, 64)[:, :, 0].reshape(t, -1), gu.reshape(t, -1, 2, 64)[:, :, 1].reshape(t, -1)
        act = (torch.nn.functional.silu(g) * u).to(w.dtype)
        h = h + fp8_matmul_ref(act, l.wd)
    x = rmsnorm_ref(h, w.final_norm, cfg.rms_eps)
    return x @ w.lm_head.float().t()
