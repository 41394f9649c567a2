"""Edge (drafter + coordinator) command line: ``python -m 0709_b200.serving.distributed_system``.

Runs the asynchronous tree/forest generator against a Target reached over
HTTP (``--target-url``) or hosted in this process (``--target-model``, on
``--target-device``).  Flags follow the reference Edge CLI
(src/atlas_0709/distributed_system.py:975-1071); SGLang pool-sizing flags are
accepted and mapped onto the native page pool.  Writes the result JSON and
optional timeline SVG/JSON.
"""

from __future__ import annotations

import argparse
import json
import math
import time
from pathlib import Path

import torch

from ..models.loader import resolve_model
from ..runtime.drafter import DrafterRuntime
from ..runtime.engine import LlamaEngine
from ..utils.timeline import write_timeline_json, write_timeline_svg
from .edge import DistributedAtlasConfig, PagedDistributedAtlasGenerator
from .prompts import decode, load_tokenizer, parse_token_ids, required_context_length
from .rpc import InProcessTargetClient, RemoteTargetClient


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Run the drafter/coordinator process.")
    p.add_argument("--drafter-model", required=True, help="Preset name (random init) or checkpoint directory.")
    p.add_argument("--target-url", default=None, help="Example: http://127.0.0.1:18090")
    p.add_argument("--target-model", default=None, help="Host the target in this process instead of over HTTP.")
    p.add_argument("--target-device", default=None)
    p.add_argument("--tokenizer", default=None, help="tokenizer.json (or its directory) for text prompts.")
    p.add_argument("--prompt", default="ATLAS distributed generation.")
    p.add_argument("--prompt-token-ids", default=None)
    p.add_argument("--prefix-len", type=int, default=None)
    p.add_argument("--repeat-token-id", type=int, default=None)
    p.add_argument("--k", type=int, default=3)
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--fixed-forest-depth", type=int, default=None)
    p.add_argument("--forest-gate", choices=["overlap", "adaptive"], default="adaptive",
                   help="overlap: always grow the forest during the verify (reference schedule); adaptive: wait for "
                        "the target's decision while most recent rounds fell back.")
    p.add_argument("--forest-gate-threshold", type=float, default=0.75)
    p.add_argument("--validate-state-alignment", action="store_true")
    p.add_argument("--max-new-tokens", type=int, default=16)
    p.add_argument("--eos-token-id", type=int, default=None)
    p.add_argument("--fallback-ar-tokens", type=int, default=4)
    p.add_argument("--generation-seed", type=int, default=0)
    p.add_argument("--drafter-do-sample", action="store_true")
    p.add_argument("--drafter-temperature", type=float, default=1.0)
    p.add_argument("--dtype", default="float16")
    p.add_argument("--context-length", type=int, default=None)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--prefill-chunk-size", type=int, default=8192)
    p.add_argument("--mem-fraction-static", type=float, default=0.75, help="Accepted for compatibility; unused.")
    p.add_argument("--max-running-requests", type=int, default=256, help="Accepted for compatibility; unused.")
    p.add_argument("--max-total-tokens", type=int, default=65536, help="Drafter KV pool size in tokens.")
    p.add_argument("--warmup-runs", type=int, default=1)
    p.add_argument("--gpu-id", type=int, default=0)
    p.add_argument("--nccl-port", type=int, default=29500, help="Accepted for compatibility; unused.")
    p.add_argument("--timeout", type=float, default=600.0)
    p.add_argument("--trust-remote-code", action="store_true", help="Accepted for compatibility; unused.")
    p.add_argument("--seed", type=int, default=0, help="Seed for random-init presets.")
    # Target options when hosted in process.
    p.add_argument("--path-score-weights", default=None)
    p.add_argument("--fallback-threshold", type=float, default=None)
    p.add_argument("--first-token-threshold", type=float, default=None)
    p.add_argument("--route-selection-policy", default="target_best")
    p.add_argument("--json-out", default=None)
    p.add_argument("--timeline-svg", default=None)
    p.add_argument("--timeline-json", default=None)
    p.add_argument("--timeline-width", type=int, default=1600)
    return p


def make_target_client(args, ctx: int):
    if args.target_url:
        return RemoteTargetClient(args.target_url, timeout=args.timeout)
    if not args.target_model:
        raise SystemExit("give --target-url or --target-model")
    from ..runtime.target import TargetVerifier
    from .target_server import parse_score_weights

    dev = torch.device(args.target_device or (f"cuda:{args.gpu_id}" if torch.cuda.is_available() else "cpu"))
    w = resolve_model(args.target_model, dtype=args.dtype, device=dev, seed=args.seed + 1)
    eng = LlamaEngine(w, num_pages=2 * math.ceil(ctx / args.page_size) + 64, page_size=args.page_size,
                      max_positions=ctx + 64)
    tv = TargetVerifier(eng, k=args.k, d=args.d, score_weights=parse_score_weights(args.path_score_weights),
                        fallback_threshold=args.fallback_threshold, first_token_threshold=args.first_token_threshold,
                        fallback_ar_tokens=args.fallback_ar_tokens, route_selection_policy=args.route_selection_policy,
                        model_name=args.target_model)
    if dev.type == "cuda":
        tv.warm_graphs()
    return InProcessTargetClient(tv)


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    if args.warmup_runs < 0:
        raise SystemExit("--warmup-runs is a count and cannot be negative")
    tok = load_tokenizer(args.tokenizer)
    prompt = parse_token_ids(args.prompt_token_ids, tokenizer=tok, prompt=args.prompt, prefix_len=args.prefix_len,
                             repeat_token_id=args.repeat_token_id)
    warm_tokens = max(2 * args.d, args.page_size + 2 * args.d) if args.warmup_runs else 0
    ctx = required_context_length(len(prompt), max_new_tokens=max(args.max_new_tokens, warm_tokens), depth=args.d)
    if args.context_length is not None:
        ctx = max(ctx, int(args.context_length))
    dev = torch.device(f"cuda:{args.gpu_id}" if torch.cuda.is_available() else "cpu")
    wd = resolve_model(args.drafter_model, dtype=args.dtype, device=dev, seed=args.seed)
    pages = max(math.ceil(args.max_total_tokens / args.page_size), 2 * math.ceil(ctx / args.page_size) + 64)
    drafter = DrafterRuntime(LlamaEngine(wd, num_pages=pages, page_size=args.page_size, max_positions=ctx + 64),
                             prefill_chunk_size=args.prefill_chunk_size)
    if dev.type == "cuda":
        drafter.warm_graphs(args.k, args.fallback_ar_tokens)
    client = make_target_client(args, ctx)

    def config(max_new: int, eos) -> DistributedAtlasConfig:
        return DistributedAtlasConfig(
            k=args.k, d=args.d, max_new_tokens=max_new, eos_token_id=eos, fallback_ar_tokens=args.fallback_ar_tokens,
            generation_seed=args.generation_seed, drafter_do_sample=args.drafter_do_sample,
            drafter_temperature=args.drafter_temperature, fixed_forest_depth=args.fixed_forest_depth,
            validate_state_alignment=args.validate_state_alignment, forest_gate=args.forest_gate,
            forest_gate_threshold=args.forest_gate_threshold)

    warm_s = 0.0
    for i in range(args.warmup_runs):
        t0 = time.perf_counter()
        PagedDistributedAtlasGenerator(config=config(warm_tokens, None), drafter=drafter,
                                       target_client=client).generate(prompt)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        warm_s += time.perf_counter() - t0
        print(f"[warmup] run {i + 1}/{args.warmup_runs} done", flush=True)
    gen = PagedDistributedAtlasGenerator(config=config(args.max_new_tokens, args.eos_token_id), drafter=drafter,
                                         target_client=client)
    res = gen.generate(prompt)
    res.text = decode(tok, res.prompt_token_ids + res.generated_token_ids)
    res.metadata.update({"warmup_runs": args.warmup_runs, "warmup_generated_tokens_per_run": warm_tokens,
                         "warmup_elapsed_s": warm_s, "warmup_excluded_from_timeline": True})
    text = json.dumps(res.to_dict(), ensure_ascii=False, indent=2, sort_keys=True)
    print(text)
    if args.json_out:
        Path(args.json_out).write_text(text + "\n", encoding="utf-8")
    if args.timeline_svg:
        write_timeline_svg(args.timeline_svg, gen.last_timeline, width=args.timeline_width)
    if args.timeline_json:
        write_timeline_json(args.timeline_json, gen.last_timeline)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
