"""Target verify server: ``python -m 0709_b200.serving.target_server --model llama-8b --port 18090``.

Flags follow the reference Target server (src/atlas_0709/target_server.py:19-93):
k, d, prefix length, page size, path-score weights, fallback thresholds,
fallback AR tokens, route-selection policy and temperature.  ``--model`` takes
a preset name (seeded random-init weights) or a Hugging Face checkpoint
directory.  FlashInfer-specific flags are accepted and ignored (the attention
here is this package's own kernel).
"""

from __future__ import annotations

import argparse
import math

import torch

from ..models.loader import resolve_model
from ..runtime.engine import LlamaEngine
from ..runtime.target import TargetVerifier
from .rpc import TargetServerApp, serve_target


def parse_score_weights(raw: str | None) -> tuple[float, ...] | None:
    if raw is None or not raw.strip():
        return None
    vals = tuple(float(p.strip()) for p in raw.split(",") if p.strip())
    return vals or None


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Run the target verify server.")
    p.add_argument("--model", required=True, help="Preset name (random init) or checkpoint directory.")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, required=True)
    p.add_argument("--k", type=int, default=3)
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--prefix-len", type=int, default=8192, help="Longest committed prefix to provision KV for.")
    p.add_argument("--repeat-token-id", type=int, default=42)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--dtype", choices=["float16", "bfloat16", "float32"], default="float16")
    p.add_argument("--device", default="cuda")
    p.add_argument("--seed", type=int, default=0, help="Seed for random-init presets.")
    p.add_argument("--max-new-tokens-capacity", type=int, default=4096,
                   help="Generated tokens to provision KV for beyond --prefix-len.")
    p.add_argument("--workspace-mb", type=int, default=128, help="Accepted for compatibility; unused.")
    p.add_argument("--flashinfer-backend", default="auto", choices=["auto"],
                   help="No-op, kept so reference command lines run: attention is this package's own kernel, "
                        "so there is no FlashInfer backend to choose (only 'auto' is accepted).")
    p.add_argument("--use-packed-custom-mask", action="store_true",
                   help="No-op, kept so reference command lines run: the tree mask is always the kernel's own "
                        "packed ancestor bitmask.")
    p.add_argument("--trust-remote-code", action="store_true", help="Accepted for compatibility; unused.")
    p.add_argument("--path-score-weights", default=None,
                   help="Comma-separated per-token weights, e.g. 0.45,0.30,0.17,0.08 (normalized).")
    p.add_argument("--fallback-threshold", type=float, default=None)
    p.add_argument("--first-token-threshold", type=float, default=None)
    p.add_argument("--fallback-ar-tokens", type=int, default=4)
    p.add_argument("--profile-fallback-ar", action="store_true")
    p.add_argument("--route-selection-policy", choices=["target_best", "target_sample", "first_route"],
                   default="target_best")
    p.add_argument("--route-sampling-temperature", type=float, default=1.0)
    p.add_argument("--verbose", action="store_true", help="Log every HTTP request.")
    p.add_argument("--sessions", type=int, default=1,
                   help="Serve up to this many concurrent sessions (requests carry session_id; POST /release ends one).")
    return p


def build_backend(args: argparse.Namespace) -> TargetVerifier:
    device = torch.device(args.device if torch.cuda.is_available() or not args.device.startswith("cuda") else "cpu")
    w = resolve_model(args.model, dtype=args.dtype, device=device, seed=args.seed)
    ctx = int(args.prefix_len) + int(args.max_new_tokens_capacity) + 4 * int(args.k) * int(args.d) + 64
    pages = 2 * math.ceil(ctx / args.page_size) + 64
    engine = LlamaEngine(w, num_pages=pages, page_size=args.page_size, max_positions=ctx + 64)
    tv = TargetVerifier(
        engine,
        k=args.k,
        d=args.d,
        score_weights=parse_score_weights(args.path_score_weights),
        fallback_threshold=args.fallback_threshold,
        first_token_threshold=args.first_token_threshold,
        fallback_ar_tokens=args.fallback_ar_tokens,
        profile_fallback_ar=args.profile_fallback_ar,
        route_selection_policy=args.route_selection_policy,
        route_sampling_temperature=args.route_sampling_temperature,
        model_name=args.model,
    )
    if device.type == "cuda":
        tv.warm_graphs()
    return tv


def build_multi_session_app(args: argparse.Namespace):
    """One engine and page pool shared by up to ``--sessions`` target sessions."""
    from .. import ops  # noqa: F401
    from ..ops import _native
    from .sessions import MultiSessionTargetApp

    device = torch.device(args.device if torch.cuda.is_available() or not args.device.startswith("cuda") else "cpu")
    w = resolve_model(args.model, dtype=args.dtype, device=device, seed=args.seed)
    ctx = int(args.prefix_len) + int(args.max_new_tokens_capacity) + 4 * int(args.k) * int(args.d) + 64
    pages = int(args.sessions) * (2 * math.ceil(ctx / args.page_size) + 64)
    engine = LlamaEngine(w, num_pages=pages, page_size=args.page_size, max_positions=ctx + 64)
    pool = _native.host().PagePool(engine.num_pages - 1, args.page_size)

    def make(sid: str) -> TargetVerifier:
        tv = TargetVerifier(engine, k=args.k, d=args.d, page_pool=pool,
                            score_weights=parse_score_weights(args.path_score_weights),
                            fallback_threshold=args.fallback_threshold,
                            first_token_threshold=args.first_token_threshold,
                            fallback_ar_tokens=args.fallback_ar_tokens, profile_fallback_ar=args.profile_fallback_ar,
                            route_selection_policy=args.route_selection_policy,
                            route_sampling_temperature=args.route_sampling_temperature, model_name=args.model)
        if device.type == "cuda":
            tv.warm_graphs()
        return tv

    return MultiSessionTargetApp(make, max_sessions=int(args.sessions))


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    if int(args.sessions) > 1:
        app = build_multi_session_app(args)
    else:
        app = TargetServerApp(build_backend(args))
    app.verbose = bool(args.verbose)
    serve_target(app, host=args.host, port=args.port)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
