"""Model resolution and Hugging Face-format checkpoint I/O.

``resolve_model(spec)`` accepts a preset name (``llama-8b``, seeded random-init
weights) or a directory holding ``config.json`` plus ``*.safetensors`` in the
Hugging Face Llama naming (``model.layers.N.self_attn.q_proj.weight`` ...).
Loading fuses q/k/v into ``wqkv`` and interleaves gate/up rows for the fused
SiLU epilogue; ``save_hf_checkpoint`` writes the inverse layout, so random-init
weights can be handed to other runtimes.

Parity: the reference loads Hugging Face checkpoints through transformers
(src/atlas_0709/flashinfer_full_verify.py:402-413); this reads the same files
without building a transformers model.
"""

from __future__ import annotations

import json
import os
from pathlib import Path

import torch

from .llama import LayerWeights, LlamaConfig, LlamaWeights, RopeScaling, get_config, interleave_gate_up, random_weights, split_gate_up

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def config_from_hf(d: dict, name: str = "hf") -> LlamaConfig:
    heads = int(d["num_attention_heads"])
    hidden = int(d["hidden_size"])
    rs = d.get("rope_scaling") or None
    scaling = None
    if isinstance(rs, dict) and rs.get("rope_type", rs.get("type")) == "llama3":
        scaling = RopeScaling(
            factor=float(rs.get("factor", 8.0)),
            low_freq_factor=float(rs.get("low_freq_factor", 1.0)),
            high_freq_factor=float(rs.get("high_freq_factor", 4.0)),
            original_max_position_embeddings=int(rs.get("original_max_position_embeddings", 8192)),
        )
    return LlamaConfig(
        name=name,
        num_layers=int(d["num_hidden_layers"]),
        hidden_size=hidden,
        num_heads=heads,
        num_kv_heads=int(d.get("num_key_value_heads", heads)),
        head_dim=int(d.get("head_dim") or hidden // heads),
        intermediate_size=int(d["intermediate_size"]),
        vocab_size=int(d["vocab_size"]),
        rope_theta=float(d.get("rope_theta", 10000.0)),
        rope_scaling=scaling,
        rms_eps=float(d.get("rms_norm_eps", 1e-5)),
        tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
        init_std=float(d.get("initializer_range", 0.02)),
    )


def config_to_hf(cfg: LlamaConfig) -> dict:
    out = {
        "architectures": ["LlamaForCausalLM"],
        "model_type": "llama",
        "hidden_size": cfg.hidden_size,
        "intermediate_size": cfg.intermediate_size,
        "num_hidden_layers": cfg.num_layers,
        "num_attention_heads": cfg.num_heads,
        "num_key_value_heads": cfg.num_kv_heads,
        "head_dim": cfg.head_dim,
        "vocab_size": cfg.vocab_size,
        "rope_theta": cfg.rope_theta,
        "rms_norm_eps": cfg.rms_eps,
        "tie_word_embeddings": cfg.tie_word_embeddings,
        "initializer_range": cfg.init_std,
        "max_position_embeddings": 131072,
        "hidden_act": "silu",
    }
    if cfg.rope_scaling is not None:
        rs = cfg.rope_scaling
        out["rope_scaling"] = {
            "rope_type": "llama3",
            "factor": rs.factor,
            "low_freq_factor": rs.low_freq_factor,
            "high_freq_factor": rs.high_freq_factor,
            "original_max_position_embeddings": rs.original_max_position_embeddings,
        }
    return out


def load_hf_checkpoint(path: str | os.PathLike, *, dtype: torch.dtype = torch.float16,
                       device: str | torch.device = "cpu") -> LlamaWeights:
    from safetensors import safe_open

    root = Path(path)
    cfg = config_from_hf(json.loads((root / "config.json").read_text()), name=root.name)
    tensors: dict[str, torch.Tensor] = {}
    files = sorted(root.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no *.safetensors under {root}")
    for f in files:
        with safe_open(str(f), framework="pt", device="cpu") as h:
            for k in h.keys():
                tensors[k] = h.get_tensor(k)

    def t(name: str) -> torch.Tensor:
        return tensors[name].to(device=device, dtype=dtype)

    layers = []
    for i in range(cfg.num_layers):
        pre = f"model.layers.{i}."
        wqkv = torch.cat((t(pre + "self_attn.q_proj.weight"), t(pre + "self_attn.k_proj.weight"),
                          t(pre + "self_attn.v_proj.weight")), dim=0).contiguous()
        layers.append(
            LayerWeights(
                attn_norm=t(pre + "input_layernorm.weight"),
                wqkv=wqkv,
                wo=t(pre + "self_attn.o_proj.weight").contiguous(),
                mlp_norm=t(pre + "post_attention_layernorm.weight"),
                wgu=interleave_gate_up(t(pre + "mlp.gate_proj.weight"), t(pre + "mlp.up_proj.weight")).contiguous(),
                wd=t(pre + "mlp.down_proj.weight").contiguous(),
            )
        )
    embed = t("model.embed_tokens.weight").contiguous()
    lm = embed if cfg.tie_word_embeddings or "lm_head.weight" not in tensors else t("lm_head.weight").contiguous()
    return LlamaWeights(cfg, embed, layers, t("model.norm.weight"), lm)


def save_hf_checkpoint(w: LlamaWeights, path: str | os.PathLike) -> None:
    """Write Hugging Face Llama naming (config.json + model.safetensors)."""
    from safetensors.torch import save_file

    root = Path(path)
    root.mkdir(parents=True, exist_ok=True)
    (root / "config.json").write_text(json.dumps(config_to_hf(w.config), indent=2))
    out = {name: t.detach().contiguous().cpu() for name, t in hf_state_dict(w).items()}
    save_file(out, str(root / "model.safetensors"))


def hf_state_dict(w: LlamaWeights) -> dict[str, torch.Tensor]:
    """The weights under Hugging Face Llama names (views of ``w`` where the layout allows)."""
    cfg = w.config
    out: dict[str, torch.Tensor] = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.final_norm}
    if not cfg.tie_word_embeddings:
        out["lm_head.weight"] = w.lm_head
    q, kv = cfg.q_size, cfg.kv_size
    for i, lw in enumerate(w.layers):
        pre = f"model.layers.{i}."
        gate, up = split_gate_up(lw.wgu)
        out.update({
            pre + "input_layernorm.weight": lw.attn_norm,
            pre + "post_attention_layernorm.weight": lw.mlp_norm,
            pre + "self_attn.q_proj.weight": lw.wqkv[:q],
            pre + "self_attn.k_proj.weight": lw.wqkv[q:q + kv],
            pre + "self_attn.v_proj.weight": lw.wqkv[q + kv:],
            pre + "self_attn.o_proj.weight": lw.wo,
            pre + "mlp.gate_proj.weight": gate,
            pre + "mlp.up_proj.weight": up,
            pre + "mlp.down_proj.weight": lw.wd,
        })
    return out


def resolve_model(spec: str, *, dtype: str | torch.dtype = "float16", device: str | torch.device = "cpu",
                  seed: int = 0) -> LlamaWeights:
    """Preset name -> seeded random init; directory -> checkpoint load."""
    dt = DTYPES[dtype] if isinstance(dtype, str) else dtype
    if os.path.isdir(spec):
        return load_hf_checkpoint(spec, dtype=dt, device=device)
    return random_weights(get_config(spec), seed=seed, dtype=dt, device=device)
