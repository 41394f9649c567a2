"""Llama-architecture models: configs, seeded random-init weights, and an eager oracle.

Weights are stored in the layouts the sm_100a kernels consume:
- ``wqkv``  [(Hq + 2*Hkv) * hd, H]  (q rows, then k rows, then v rows);
- ``wo``    [H, Hq * hd];
- ``wgu``   [2 * F, H] gate/up rows interleaved in blocks of ``GU_BLOCK`` so one
  128-row GEMM tile holds 64 gate rows and the matching 64 up rows and its
  epilogue can emit ``silu(gate) * up`` directly;
- ``wd``    [H, F];
- RMSNorm gains and the embedding/LM-head tables.

``reference_forward`` is the fp32 oracle used by the numerics tests: plain
PyTorch, contiguous K/V, an explicit boolean visibility mask.

The reference runs the same architecture as Hugging Face Llama modules plus a manual
forward around FlashInfer (src/atlas_0709/flashinfer_full_verify.py:259-335 rotary
embedding, :1066-1122 AR decode, :1183-1231 masked tree verify) and checks it against
transformers' own logits (:1263-1346); here the checkpoint layout is converted once at load
(``models/loader.py``) and the oracle plays the role of that check.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Sequence

import torch

GU_BLOCK = 64


@dataclass(frozen=True)
class RopeScaling:
    """Llama-3 frequency scaling (factor, low/high frequency factors, original context)."""

    factor: float = 8.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192


@dataclass(frozen=True)
class LlamaConfig:
    name: str
    num_layers: int
    hidden_size: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rope_theta: float = 500000.0
    rope_scaling: RopeScaling | None = field(default_factory=RopeScaling)
    rms_eps: float = 1e-5
    tie_word_embeddings: bool = False
    init_std: float = 0.02

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def group(self) -> int:
        return self.num_heads // self.num_kv_heads

    def param_count(self) -> int:
        per_layer = (
            self.qkv_size * self.hidden_size
            + self.hidden_size * self.q_size
            + 3 * self.hidden_size * self.intermediate_size
            + 2 * self.hidden_size
        )
        emb = self.vocab_size * self.hidden_size
        return self.num_layers * per_layer + emb * (1 if self.tie_word_embeddings else 2) + self.hidden_size

    def validate(self) -> None:
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for rotary embeddings")
        if self.intermediate_size % GU_BLOCK:
            raise ValueError(f"intermediate_size must be a multiple of {GU_BLOCK}")


PRESETS: dict[str, LlamaConfig] = {
    # CPU plumbing configuration: tiny drafter and target.
    "tiny-drafter": LlamaConfig("tiny-drafter", 2, 256, 4, 2, 64, 512, 1024, rope_theta=10000.0, rope_scaling=None),
    "tiny-target": LlamaConfig("tiny-target", 4, 256, 4, 2, 64, 512, 1024, rope_theta=10000.0, rope_scaling=None),
    # Small head_dim-128 models for GPU tests (the CUDA attention kernel needs head_dim 128).
    "small-drafter": LlamaConfig("small-drafter", 2, 512, 8, 2, 128, 1024, 4096),
    "small-target": LlamaConfig("small-target", 3, 512, 8, 2, 128, 1024, 4096),
    # Splits over up to 8 tensor-parallel ranks (8 KV heads, FFN 8 x 512).
    "small-tp-target": LlamaConfig("small-tp-target", 4, 1024, 16, 8, 128, 4096, 8192),
    # Llama-3.2-1B shape as declared by the benchmark (head_dim 128, so q_proj is 2048 -> 4096).
    "llama-1b": LlamaConfig(
        "llama-1b", 16, 2048, 32, 8, 128, 8192, 128256, rope_scaling=RopeScaling(factor=32.0), tie_word_embeddings=True
    ),
    "llama-8b": LlamaConfig("llama-8b", 32, 4096, 32, 8, 128, 14336, 128256),
    "llama-70b": LlamaConfig("llama-70b", 80, 8192, 64, 8, 128, 28672, 128256),
}


def get_config(name: str, **overrides) -> LlamaConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    cfg = PRESETS[name]
    return replace(cfg, **overrides) if overrides else cfg


# ----------------------------------------------------------------- rotary
def rope_inv_freq(cfg: LlamaConfig) -> torch.Tensor:
    """Per-pair inverse frequencies in float64, with Llama-3 scaling when configured."""
    half = cfg.head_dim // 2
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(half, dtype=torch.float64) * 2.0 / cfg.head_dim))
    rs = cfg.rope_scaling
    if rs is None:
        return inv
    low_wl = rs.original_max_position_embeddings / rs.low_freq_factor
    high_wl = rs.original_max_position_embeddings / rs.high_freq_factor
    wl = 2.0 * math.pi / inv
    out = torch.where(wl > low_wl, inv / rs.factor, inv)
    smooth = (rs.original_max_position_embeddings / wl - rs.low_freq_factor) / (
        rs.high_freq_factor - rs.low_freq_factor
    )
    mid = (1.0 - smooth) * out / rs.factor + smooth * out
    is_mid = (wl >= high_wl) & (wl <= low_wl)
    return torch.where(is_mid, mid, out)


def rope_table(cfg: LlamaConfig, max_positions: int, device=None) -> torch.Tensor:
    """fp32 table [max_positions, head_dim]: cos in [:, :half], sin in [:, half:]."""
    inv = rope_inv_freq(cfg)
    pos = torch.arange(int(max_positions), dtype=torch.float64)
    ang = pos[:, None] * inv[None, :]
    return torch.cat((torch.cos(ang), torch.sin(ang)), dim=-1).to(torch.float32).to(device)


def apply_rope(x: torch.Tensor, table: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on [M, heads, hd] in fp32 using a ``rope_table``."""
    half = x.shape[-1] // 2
    cs = table[positions.long()]
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)


# ---------------------------------------------------------------- weights
@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    wqkv: torch.Tensor
    wo: torch.Tensor
    mlp_norm: torch.Tensor
    wgu: torch.Tensor
    wd: torch.Tensor


@dataclass
class LlamaWeights:
    config: LlamaConfig
    embed: torch.Tensor
    layers: list[LayerWeights]
    final_norm: torch.Tensor
    lm_head: torch.Tensor

    @property
    def dtype(self) -> torch.dtype:
        return self.embed.dtype

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def nbytes(self) -> int:
        seen: set[int] = set()
        total = 0
        for t in self.tensors():
            if t.data_ptr() in seen:
                continue
            seen.add(t.data_ptr())
            total += t.numel() * t.element_size()
        return total

    def tensors(self) -> list[torch.Tensor]:
        out = [self.embed, self.final_norm, self.lm_head]
        for lw in self.layers:
            out += [lw.attn_norm, lw.wqkv, lw.wo, lw.mlp_norm, lw.wgu, lw.wd]
        return out


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = GU_BLOCK) -> torch.Tensor:
    f, h = gate.shape
    g = gate.reshape(f // block, block, h)
    u = up.reshape(f // block, block, h)
    return torch.stack((g, u), dim=1).reshape(2 * f, h)


def split_gate_up(wgu: torch.Tensor, block: int = GU_BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    two_f, h = wgu.shape
    x = wgu.reshape(two_f // (2 * block), 2, block, h)
    return x[:, 0].reshape(-1, h), x[:, 1].reshape(-1, h)


def random_weights(
    cfg: LlamaConfig,
    *,
    seed: int = 0,
    dtype: torch.dtype = torch.float16,
    device: str | torch.device = "cpu",
    layers: Sequence[int] | None = None,
) -> LlamaWeights:
    """Seeded random init: N(0, init_std) matrices, unit RMSNorm gains.

    Generated directly on ``device`` (one generator per tensor, keyed by the
    seed and the tensor's index), so the 8B/70B shapes initialize in seconds.
    """
    cfg.validate()
    dev = torch.device(device)
    counter = [0]

    def normal(*shape: int) -> torch.Tensor:
        g = torch.Generator(device=dev)
        g.manual_seed((int(seed) * 1_000_003 + counter[0]) & ((1 << 63) - 1))
        counter[0] += 1
        t = torch.empty(*shape, dtype=dtype, device=dev)
        t.normal_(0.0, cfg.init_std, generator=g)
        return t

    def ones(n: int) -> torch.Tensor:
        return torch.ones(n, dtype=dtype, device=dev)

    h = cfg.hidden_size
    embed = normal(cfg.vocab_size, h)
    idx = range(cfg.num_layers) if layers is None else layers
    lws: list[LayerWeights] = []
    for _ in idx:
        gate = normal(cfg.intermediate_size, h)
        up = normal(cfg.intermediate_size, h)
        lws.append(
            LayerWeights(
                attn_norm=ones(h),
                wqkv=normal(cfg.qkv_size, h),
                wo=normal(h, cfg.q_size),
                mlp_norm=ones(h),
                wgu=interleave_gate_up(gate, up),
                wd=normal(h, cfg.intermediate_size),
            )
        )
    lm_head = embed if cfg.tie_word_embeddings else normal(cfg.vocab_size, h)
    return LlamaWeights(cfg, embed, lws, ones(h), lm_head)


def weights_to(w: LlamaWeights, *, dtype=None, device=None) -> LlamaWeights:
    def cv(t: torch.Tensor) -> torch.Tensor:
        return t.to(device=device or t.device, dtype=dtype or t.dtype)

    embed = cv(w.embed)
    lm = embed if w.lm_head is w.embed else cv(w.lm_head)
    layers = [
        LayerWeights(cv(l.attn_norm), cv(l.wqkv), cv(l.wo), cv(l.mlp_norm), cv(l.wgu), cv(l.wd)) for l in w.layers
    ]
    return LlamaWeights(w.config, embed, layers, cv(w.final_norm), lm)


# ----------------------------------------------------------------- oracle
def rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


@torch.no_grad()
def reference_forward(
    w: LlamaWeights,
    tokens: Sequence[int] | torch.Tensor,
    *,
    positions: Sequence[int] | torch.Tensor | None = None,
    visible: torch.Tensor | None = None,
) -> torch.Tensor:
    """fp32 logits [T, V] for ``tokens`` attending per the boolean ``visible`` [T, T] mask.

    Defaults: positions 0..T-1 and a causal mask.  A tree is expressed by the
    positions (prefix length + depth) and an ancestor mask.
    """
    cfg = w.config
    toks = torch.as_tensor(tokens, dtype=torch.long, device=w.device).reshape(-1)
    t = int(toks.numel())
    pos = torch.arange(t, device=w.device) if positions is None else torch.as_tensor(positions, device=w.device)
    if visible is None:
        visible = torch.tril(torch.ones(t, t, dtype=torch.bool, device=w.device))
    table = rope_table(cfg, int(pos.max()) + 1, device=w.device)
    hd = cfg.head_dim
    x = w.embed[toks].float()
    scale = 1.0 / math.sqrt(hd)
    for lw in w.layers:
        a = rmsnorm_ref(x, lw.attn_norm, cfg.rms_eps)
        qkv = a @ lw.wqkv.float().t()
        q = qkv[:, : cfg.q_size].reshape(t, cfg.num_heads, hd)
        k = qkv[:, cfg.q_size: cfg.q_size + cfg.kv_size].reshape(t, cfg.num_kv_heads, hd)
        v = qkv[:, cfg.q_size + cfg.kv_size:].reshape(t, cfg.num_kv_heads, hd)
        q = apply_rope(q, table, pos)
        k = apply_rope(k, table, pos)
        k = k.repeat_interleave(cfg.group, dim=1)
        v = v.repeat_interleave(cfg.group, dim=1)
        s = torch.einsum("qhd,khd->hqk", q, k) * scale
        s = s.masked_fill(~visible[None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("hqk,khd->qhd", p, v).reshape(t, cfg.q_size)
        x = x + o @ lw.wo.float().t()
        m = rmsnorm_ref(x, lw.mlp_norm, cfg.rms_eps)
        gate, up = split_gate_up(lw.wgu.float())
        act = torch.nn.functional.silu(m @ gate.t()) * (m @ up.t())
        x = x + act @ lw.wd.float().t()
    x = rmsnorm_ref(x, w.final_norm, cfg.rms_eps)
    return x @ w.lm_head.float().t()
