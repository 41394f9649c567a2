"""Shared pieces of the evaluation drivers: JSONL I/O with resume, generator construction.

Counterparts in the reference's GSM8K driver: JSONL rows and resume
(scripts/gsm8k_eval.py:62-89), the AR / ATLAS / serial generator factories (:186-315).
"""

from __future__ import annotations

import hashlib
import json
import math
import time
from dataclasses import replace
from pathlib import Path
from typing import Any, Iterable, Mapping, Sequence

import torch


def read_jsonl(path: str | Path) -> list[dict[str, Any]]:
    out = []
    with Path(path).open(encoding="utf-8") as f:
        for n, line in enumerate(f, 1):
            if line.strip():
                try:
                    out.append(json.loads(line))
                except json.JSONDecodeError as exc:
                    raise RuntimeError(f"{path}:{n}: invalid JSON: {exc}") from exc
    return out


def append_jsonl(path: str | Path, row: Mapping[str, Any]) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    with p.open("a", encoding="utf-8") as f:
        f.write(json.dumps(row, ensure_ascii=False, sort_keys=True) + "\n")


def done_indices(path: str | Path) -> set[int]:
    p = Path(path)
    return {int(r["index"]) for r in read_jsonl(p)} if p.exists() else set()


def token_ids_sha256(ids: Sequence[int]) -> str:
    return hashlib.sha256(json.dumps([int(t) for t in ids], separators=(",", ":")).encode()).hexdigest()


def optional_float(v: str) -> float | None:
    if v.strip().lower() in {"none", "off", "disabled"}:
        return None
    x = float(v)
    if not math.isfinite(x):
        raise ValueError("value must be finite or none/off/disabled")
    return x


def non_negative_float(v: str) -> float:
    x = float(v)
    if not math.isfinite(x) or x < 0.0:
        raise ValueError("value must be finite and non-negative")
    return x


def exponential_path_weights(depth: int, alpha: float) -> tuple[float, ...]:
    """Path-score weights ``w[i] = exp(-alpha * i)`` over the ``depth`` route tokens, normalized
    to sum to one (the reference's ``--path-weight-alpha``, scripts/gsm8k_eval.py:49-56)."""
    if depth <= 0:
        raise ValueError("depth must be positive")
    raw = [math.exp(-float(alpha) * i) for i in range(int(depth))]
    total = sum(raw)
    return tuple(x / total for x in raw)


# Settings of the reference's SGLang/FlashInfer runtimes (memory fraction, scheduler limits,
# NCCL port, FlashInfer workspace) with no counterpart here: accepted so that reference command
# lines run, and ignored.
_INERT_FLAGS = (("--mem-fraction-static", float), ("--max-running-requests", int), ("--max-total-tokens", int),
                ("--nccl-port", int), ("--target-workspace-mb", int))


def add_runtime_compat_flags(p) -> None:
    for flag, typ in _INERT_FLAGS:
        p.add_argument(flag, type=typ, default=None,
                       help="No-op, kept so reference command lines run (a setting of the reference's "
                            "SGLang/FlashInfer runtime with no counterpart here).")
    p.add_argument("--use-packed-custom-mask", action="store_true",
                   help="No-op: the tree mask is always the attention kernel's packed ancestor bitmask.")
    p.add_argument("--trust-remote-code", action="store_true", help="No-op: checkpoints are read as safetensors.")
    p.add_argument("--gpu-id", type=int, default=None, help="CUDA device index (same as --device cuda:N)")
    p.add_argument("--prefill-chunk-size", type=int, default=8192, help="tokens per prefill forward (both models)")
    p.add_argument("--target-timeout", type=float, default=600.0, help="seconds per remote target call")
    p.add_argument("--warmup-runs", type=int, default=1,
                   help="untimed generations of the first pending prompt before the recorded ones")


def add_generation_flags(p) -> None:
    p.add_argument("--backend", choices=["ar", "atlas", "atlas_serial"], required=True)
    p.add_argument("--model", required=True, help="AR model, or the ATLAS drafter (preset or checkpoint dir)")
    add_atlas_flags(p)


def add_atlas_flags(p) -> None:
    """Model, tree, target-policy and drafter-sampling flags shared by every driver."""
    p.add_argument("--target-model", default=None, help="in-process target (preset or checkpoint dir)")
    p.add_argument("--target-url", default=None, help="remote target server (HTTP)")
    p.add_argument("--tokenizer", default=None, help="tokenizer.json or its directory (bytes if absent)")
    p.add_argument("--max-new-tokens", type=int, default=512)
    p.add_argument("--eos-token-id", type=int, default=None)
    p.add_argument("--dtype", choices=["float16", "bfloat16", "float32"], default="float16")
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--context-length", type=int, default=4096)
    p.add_argument("--k", type=int, default=3)
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--path-score-weights", default="0.45,0.30,0.17,0.08")
    p.add_argument("--fallback-threshold", type=optional_float, default=-0.5)
    p.add_argument("--first-token-threshold", type=optional_float, default=-0.7)
    p.add_argument("--fallback-ar-tokens", type=int, default=4)
    p.add_argument("--route-selection-policy", choices=["target_best", "target_sample", "first_route"],
                   default="target_best")
    p.add_argument("--generation-seed", type=int, default=0)
    p.add_argument("--path-weight-alpha", type=non_negative_float, default=None,
                   help="normalized exponential weights exp(-alpha * i); overrides --path-score-weights")
    p.add_argument("--route-sampling-temperature", type=float, default=1.0,
                   help="target route temperature of the target_sample policy (in-process target)")
    p.add_argument("--drafter-do-sample", action="store_true",
                   help="semantic-prefix keyed drafter sampling instead of greedy top-k")
    p.add_argument("--drafter-temperature", type=float, default=1.0, help="proposal temperature with sampling")
    p.add_argument("--fixed-forest-depth", type=int, default=None,
                   help="build exactly this many forest depths per round (async backend; replay runs)")
    p.add_argument("--validate-state-alignment", action="store_true",
                   help="check the drafter, target and coordinator prefixes after every handoff")
    p.add_argument("--seed", type=int, default=0, help="seed of random-init presets")
    p.add_argument("--device", default=None)
    p.add_argument("--resume", action="store_true")
    add_runtime_compat_flags(p)


def make_generate(args):
    """Return ``generate(prompt_ids) -> (token ids, metadata, rounds)`` for the chosen backend."""
    from ..models.loader import resolve_model
    from ..runtime.drafter import DrafterRuntime
    from ..runtime.engine import LlamaEngine

    if args.device:
        dev = torch.device(args.device)
    elif getattr(args, "gpu_id", None) is not None:
        dev = torch.device("cuda", int(args.gpu_id))
    else:
        dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    chunk = int(getattr(args, "prefill_chunk_size", 8192) or 8192)
    ctx = int(args.context_length) + int(args.max_new_tokens) + 8 * args.k * args.d + 64
    pages = 2 * math.ceil(ctx / args.page_size) + 64

    def engine(spec, seed):
        return LlamaEngine(resolve_model(spec, dtype=args.dtype, device=dev, seed=seed), num_pages=pages,
                           page_size=args.page_size, max_positions=ctx + 64)

    drafter = DrafterRuntime(engine(args.model, args.seed), prefill_chunk_size=chunk)
    do_sample = bool(getattr(args, "drafter_do_sample", False))
    temperature = float(getattr(args, "drafter_temperature", 1.0))
    if args.backend == "ar":
        from ..serving.ar import PagedGreedyARGenerator

        gen = PagedGreedyARGenerator(drafter=drafter)

        def run(ids, seed=None):
            r = gen.generate(ids, max_new_tokens=args.max_new_tokens, eos_token_id=args.eos_token_id,
                             do_sample=do_sample, temperature=temperature,
                             generation_seed=args.generation_seed if seed is None else int(seed))
            return r.generated_token_ids, dict(r.metadata), []

        return run
    from ..serving.edge import DistributedAtlasConfig, PagedDistributedAtlasGenerator
    from ..serving.rpc import InProcessTargetClient, RemoteTargetClient
    from ..serving.serial import SerialAtlasGenerator
    from ..runtime.target import TargetVerifier

    if args.target_url:
        client = RemoteTargetClient(args.target_url, timeout=float(getattr(args, "target_timeout", 600.0)))
    else:
        if not args.target_model:
            raise SystemExit("ATLAS backends need --target-model or --target-url")
        if getattr(args, "path_weight_alpha", None) is not None:
            weights = list(exponential_path_weights(args.d, args.path_weight_alpha))
        else:
            weights = [float(x) for x in args.path_score_weights.split(",")] if args.path_score_weights else None
        tv = TargetVerifier(engine(args.target_model, args.seed + 1), k=args.k, d=args.d, score_weights=weights,
                            fallback_threshold=args.fallback_threshold,
                            first_token_threshold=args.first_token_threshold,
                            fallback_ar_tokens=args.fallback_ar_tokens,
                            route_selection_policy=args.route_selection_policy,
                            route_sampling_temperature=float(getattr(args, "route_sampling_temperature", 1.0)),
                            model_name=str(args.target_model), prefill_chunk_size=chunk)
        if dev.type == "cuda":
            tv.warm_graphs()
        client = InProcessTargetClient(tv)
    if dev.type == "cuda":
        drafter.warm_graphs(args.k, args.fallback_ar_tokens)
    cls = SerialAtlasGenerator if args.backend == "atlas_serial" else PagedDistributedAtlasGenerator
    cfg = DistributedAtlasConfig(k=args.k, d=args.d, max_new_tokens=args.max_new_tokens,
                                 eos_token_id=args.eos_token_id, fallback_ar_tokens=args.fallback_ar_tokens,
                                 generation_seed=args.generation_seed,
                                 drafter_do_sample=do_sample, drafter_temperature=temperature,
                                 fixed_forest_depth=(None if args.backend == "atlas_serial"
                                                     else getattr(args, "fixed_forest_depth", None)),
                                 validate_state_alignment=bool(getattr(args, "validate_state_alignment", False)))
    gen = cls(config=cfg, drafter=drafter, target_client=client)

    def run(ids, seed=None):
        """One request; ``seed`` (default ``--generation-seed``) keys the drafter's sampling and
        the target's route sampling for this request only."""
        gen.config = replace(cfg, generation_seed=args.generation_seed if seed is None else int(seed))
        r = gen.generate(ids)
        return r.generated_token_ids, dict(r.metadata), list(r.rounds)

    return run


def warm_up(generate, ids, runs: int) -> None:
    """Untimed generations before the recorded ones (graph capture, allocator, clocks).  Every
    ``generate`` call starts from its own prefill of both models, so nothing carries over."""
    for _ in range(max(0, int(runs))):
        generate(ids)


def timed(fn, *a):
    t0 = time.perf_counter()
    out = fn(*a)
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    return out, time.perf_counter() - t0


def rows_summary(rows: Iterable[Mapping[str, Any]]) -> dict[str, Any]:
    rows = list(rows)
    toks = sum(int(r.get("generated_tokens", 0)) for r in rows)
    secs = sum(float(r.get("elapsed_s", 0.0)) for r in rows)
    return {"samples": len(rows), "generated_tokens": toks, "elapsed_s": secs,
            "tokens_per_s": toks / secs if secs > 0 else None}
