"""Greedy (or seeded-sampling) equivalence check of the asynchronous generator.

    python -m 0709_b200.serving.check_equivalence --drafter-model llama-1b --target-url http://127.0.0.1:18109 \
        --prompt-token-ids 1,2,3 --forest-depths live,0,2,4 --repeats 2 --json-out eq.json

With one route per round (k = 1), a target that always commits the first route and never falls
back, the asynchronous ATLAS generator must commit exactly the drafter's own autoregressive
tokens: greedy, or with ``--drafter-do-sample`` the same semantic-prefix keyed samples.  The
check runs every prompt under every forest schedule (``live``: the forest grows until the
verify returns; an integer: exactly that many forest depths per round, a replayable
diagnostic) ``--repeats`` times, with the cross-model state validated after every handoff, and
compares each run's tokens with the drafter's paged AR on the same prompt.  The target is a
running server (``--target-url``, which must report the first-route policy with both
fallback triggers off) or an in-process one (``--target-model``).  Writes a JSON report and
exits 1 on any mismatch.

Parity: reference tools/check_async_greedy_equivalence.py:27-455 (flags, the first-route and
no-fallback preconditions, schedules, repeats, the report).  The reference's SGLang settings
are accepted and ignored.
"""

from __future__ import annotations

import argparse
import json
import math
import random
import sys

import numpy as np
import torch

_INERT = (("--mem-fraction-static", float), ("--max-running-requests", int), ("--max-total-tokens", int),
          ("--nccl-port", int))


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="k=1 first-route ATLAS vs the drafter's own paged AR, token for token.",
                                allow_abbrev=False)
    p.add_argument("--drafter-model", required=True, help="preset (seeded random init) or checkpoint directory")
    p.add_argument("--target-url", default=None, help="running target server (first_route, fallback off)")
    p.add_argument("--target-model", default=None, help="in-process target instead of --target-url")
    p.add_argument("--prompt", action="append", default=None, help="prompt text; repeat for several cases")
    p.add_argument("--prompt-token-ids", action="append", default=None, help="comma-separated ids; repeatable")
    p.add_argument("--tokenizer", default=None, help="tokenizer.json for --prompt (UTF-8 bytes without one)")
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--forest-depths", default="live", help="comma-separated: 'live' or integers in [0, d]")
    p.add_argument("--max-new-tokens", type=int, default=64)
    p.add_argument("--repeats", type=int, default=2)
    p.add_argument("--eos-token-id", type=int, default=None)
    p.add_argument("--dtype", choices=["float16", "bfloat16", "float32"], default="float16")
    p.add_argument("--context-length", type=int, default=4096)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--prefill-chunk-size", type=int, default=4096)
    p.add_argument("--device", default=None)
    p.add_argument("--gpu-id", type=int, default=None)
    p.add_argument("--target-timeout", type=float, default=600.0)
    p.add_argument("--seed", type=int, default=0, help="generation seed (and the seed of random-init presets)")
    p.add_argument("--drafter-do-sample", action="store_true")
    p.add_argument("--drafter-temperature", type=float, default=1.0)
    p.add_argument("--deterministic-algorithms", action="store_true",
                   help="ask PyTorch to reject its known nondeterministic operations")
    for flag, typ in _INERT:
        p.add_argument(flag, type=typ, default=None, help="No-op (a setting of the reference's SGLang runtime).")
    p.add_argument("--trust-remote-code", action="store_true", help="No-op (checkpoints are read as safetensors).")
    p.add_argument("--json-out", required=True)
    return p


def parse_schedules(text: str, d: int) -> list[int | None]:
    out: list[int | None] = []
    for part in (x.strip().lower() for x in text.split(",")):
        if not part:
            continue
        out.append(None if part in ("live", "none") else int(part))
    if not out or any(v is not None and not 0 <= v <= d for v in out):
        raise SystemExit(f"--forest-depths takes 'live' or integers in [0, {d}]")
    return out


def prompts_of(args) -> list[list[int]]:
    from .prompts import encode, load_tokenizer

    cases = [[int(x) for x in s.split(",") if x.strip()] for s in (args.prompt_token_ids or [])]
    if args.prompt:
        tok = load_tokenizer(args.tokenizer)
        cases += [encode(tok, s) for s in args.prompt]
    if not cases:
        cases = [[1, 2, 3, 4, 5, 6, 7, 8]]
    if any(not c for c in cases):
        raise SystemExit("a prompt encoded to no tokens")
    return cases


def check_target_policy(metadata: dict) -> None:
    if metadata.get("route_selection_policy") != "first_route":
        raise SystemExit("the target must run with --route-selection-policy first_route")
    if metadata.get("fallback_threshold") is not None or metadata.get("first_token_threshold") is not None:
        raise SystemExit("the target must run with both fallback triggers off")


def run(args) -> dict:
    from ..models.loader import resolve_model
    from ..runtime.drafter import DrafterRuntime
    from ..runtime.engine import LlamaEngine
    from .ar import PagedGreedyARGenerator
    from .edge import DistributedAtlasConfig, PagedDistributedAtlasGenerator
    from .rpc import InProcessTargetClient, RemoteTargetClient

    if args.d <= 0 or args.max_new_tokens <= 0 or args.repeats <= 0:
        raise SystemExit("d, max-new-tokens and repeats must be positive")
    if not math.isfinite(args.drafter_temperature) or args.drafter_temperature <= 0.0:
        raise SystemExit("drafter-temperature must be finite and positive")
    if bool(args.target_url) == bool(args.target_model):
        raise SystemExit("give exactly one of --target-url and --target-model")
    schedules = parse_schedules(args.forest_depths, args.d)
    random.seed(args.seed)
    np.random.seed(args.seed)
    torch.manual_seed(args.seed)
    if args.deterministic_algorithms:
        torch.use_deterministic_algorithms(True)
    if args.device:
        dev = torch.device(args.device)
    elif args.gpu_id is not None:
        dev = torch.device("cuda", args.gpu_id)
    else:
        dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    ctx = int(args.context_length) + int(args.max_new_tokens) + 8 * args.d + 64
    pages = 2 * math.ceil(ctx / args.page_size) + 64

    def engine(spec, seed):
        return LlamaEngine(resolve_model(spec, dtype=args.dtype, device=dev, seed=seed), num_pages=pages,
                           page_size=args.page_size, max_positions=ctx + 64)

    if args.target_url:
        client = RemoteTargetClient(args.target_url, timeout=args.target_timeout)
    else:
        from ..runtime.target import TargetVerifier

        client = InProcessTargetClient(TargetVerifier(engine(args.target_model, args.seed + 1), k=1, d=args.d,
                                                      route_selection_policy="first_route",
                                                      prefill_chunk_size=args.prefill_chunk_size,
                                                      model_name=str(args.target_model)))
    health = client.health()
    check_target_policy(dict(health.get("metadata", {})))
    drafter = DrafterRuntime(engine(args.drafter_model, args.seed), prefill_chunk_size=args.prefill_chunk_size)
    sample = dict(do_sample=bool(args.drafter_do_sample), generation_seed=int(args.seed),
                  temperature=float(args.drafter_temperature))
    cases = []
    for pi, prompt in enumerate(prompts_of(args)):
        ref = PagedGreedyARGenerator(drafter=drafter).generate(prompt, max_new_tokens=args.max_new_tokens,
                                                               eos_token_id=args.eos_token_id, **sample)
        want = list(ref.generated_token_ids)
        for fd in schedules:
            cfg = DistributedAtlasConfig(k=1, d=args.d, max_new_tokens=args.max_new_tokens,
                                         eos_token_id=args.eos_token_id, generation_seed=int(args.seed),
                                         drafter_do_sample=bool(args.drafter_do_sample),
                                         drafter_temperature=float(args.drafter_temperature),
                                         fixed_forest_depth=fd, validate_state_alignment=True, forest_gate="overlap")
            for rep in range(int(args.repeats)):
                gen = PagedDistributedAtlasGenerator(config=cfg, drafter=drafter, target_client=client)
                got = list(gen.generate(prompt).generated_token_ids)
                first = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b),
                             None if len(got) == len(want) else min(len(got), len(want)))
                cases.append({"prompt_index": pi, "prompt_len": len(prompt),
                              "forest_schedule": "live" if fd is None else fd, "repeat": rep,
                              "equal": first is None, "first_mismatch": first, "tokens": len(got),
                              "atlas_tokens": got if first is not None else None,
                              "ar_tokens": want if first is not None else None})
    passed = all(c["equal"] for c in cases)
    return {"passed": passed, "cases": cases, "checked": len(cases), "d": args.d, "k": 1,
            "drafter_do_sample": bool(args.drafter_do_sample), "forest_schedules": args.forest_depths,
            "target_transport": health.get("transport", "http"), "device": str(dev),
            "reproducibility": {"seed": args.seed, "deterministic_algorithms": bool(args.deterministic_algorithms)}}


def main(argv=None) -> int:
    args = build_parser().parse_args(sys.argv[1:] if argv is None else argv)
    report = run(args)
    with open(args.json_out, "w") as f:
        json.dump(report, f, indent=2)
    print(json.dumps({"passed": report["passed"], "checked": report["checked"]}))
    return 0 if report["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
