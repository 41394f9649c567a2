"""Megatron-style sharding of a Llama model over a tensor-parallel group.

Column-parallel: the fused QKV projection (each rank keeps ``heads/tp`` query
heads and ``kv_heads/tp`` KV heads, laid out q|k|v locally) and the
interleaved gate/up projection (``ffn/tp`` rows of each).  Row-parallel: the
output projection and the down projection (matching column slices), whose
partial outputs are summed across ranks.  Vocabulary-parallel: the LM head
(``vocab/tp`` rows per rank; the logits are gathered on the root rank).  The
embedding table and the RMSNorm gains are replicated.

``random_weights_tp`` draws exactly the tensors ``random_weights`` draws for
the whole model (same seeds, same order) and keeps this rank's slices, so a
TP model is the same logical model as the single-GPU one.  The reference has
no tensor parallelism (SGLang ``tp_size=1``, fp/sglang_runtime.py:36).
"""

from __future__ import annotations

from dataclasses import replace

import torch

from ..models.llama import GU_BLOCK, LayerWeights, LlamaConfig, LlamaWeights, interleave_gate_up, split_gate_up


def check_tp(cfg: LlamaConfig, tp: int) -> None:
    if tp < 1:
        raise ValueError("tp must be positive")
    if cfg.num_kv_heads % tp or cfg.num_heads % tp:
        raise ValueError(f"{cfg.name}: {cfg.num_heads} q / {cfg.num_kv_heads} kv heads do not split over tp={tp}")
    if cfg.intermediate_size % (tp * GU_BLOCK):
        raise ValueError(f"{cfg.name}: FFN {cfg.intermediate_size} does not split over tp={tp} in {GU_BLOCK}-row blocks")
    if cfg.vocab_size % tp:
        raise ValueError(f"{cfg.name}: vocabulary {cfg.vocab_size} does not split over tp={tp}")


def local_config(cfg: LlamaConfig, tp: int) -> LlamaConfig:
    """Per-rank shapes (heads, FFN rows); vocabulary stays the full size (embedding is replicated)."""
    check_tp(cfg, tp)
    if tp == 1:
        return cfg
    return replace(cfg, name=f"{cfg.name}/tp{tp}", num_heads=cfg.num_heads // tp,
                   num_kv_heads=cfg.num_kv_heads // tp, intermediate_size=cfg.intermediate_size // tp)


def _qkv_rows(cfg: LlamaConfig, rank: int, tp: int) -> torch.Tensor:
    hd = cfg.head_dim
    hq, hk = cfg.num_heads // tp, cfg.num_kv_heads // tp
    q = torch.arange(rank * hq * hd, (rank + 1) * hq * hd)
    k = cfg.q_size + torch.arange(rank * hk * hd, (rank + 1) * hk * hd)
    v = cfg.q_size + cfg.kv_size + torch.arange(rank * hk * hd, (rank + 1) * hk * hd)
    return torch.cat((q, k, v))


def shard_layer(cfg: LlamaConfig, lw: LayerWeights, rank: int, tp: int) -> LayerWeights:
    if tp == 1:
        return lw
    rows = _qkv_rows(cfg, rank, tp).to(lw.wqkv.device)
    qs = cfg.q_size // tp
    f = cfg.intermediate_size // tp
    gate, up = split_gate_up(lw.wgu)
    return LayerWeights(
        attn_norm=lw.attn_norm,
        wqkv=lw.wqkv.index_select(0, rows).contiguous(),
        wo=lw.wo[:, rank * qs:(rank + 1) * qs].contiguous(),
        mlp_norm=lw.mlp_norm,
        wgu=interleave_gate_up(gate[rank * f:(rank + 1) * f], up[rank * f:(rank + 1) * f]).contiguous(),
        wd=lw.wd[:, rank * f:(rank + 1) * f].contiguous(),
    )


def shard_lm_head(cfg: LlamaConfig, lm_head: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    v = cfg.vocab_size // tp
    return lm_head[rank * v:(rank + 1) * v].contiguous()


def shard_weights(w: LlamaWeights, rank: int, tp: int) -> LlamaWeights:
    """Slice full weights (any device) into rank ``rank``'s shard; ``config`` becomes the local config."""
    cfg = w.config
    check_tp(cfg, tp)
    layers = [shard_layer(cfg, lw, rank, tp) for lw in w.layers]
    return LlamaWeights(local_config(cfg, tp), w.embed, layers, w.final_norm, shard_lm_head(cfg, w.lm_head, rank, tp))


def random_weights_tp(cfg: LlamaConfig, *, rank: int, tp: int, seed: int = 0, dtype: torch.dtype = torch.float16,
                      device: str | torch.device = "cpu") -> LlamaWeights:
    """This rank's shard of ``random_weights(cfg, seed=seed)``, drawing one full layer at a time."""
    check_tp(cfg, tp)
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
        layers.append(shard_layer(cfg, full, rank, tp))
        del full
    lm = embed if cfg.tie_word_embeddings else normal(cfg.vocab_size, h)
    return LlamaWeights(local_config(cfg, tp), embed, layers, ones(h), shard_lm_head(cfg, lm, rank, tp))
