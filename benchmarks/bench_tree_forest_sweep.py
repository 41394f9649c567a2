#!/usr/bin/env python
"""Tree / forest vs batch AR over several (k, d) pairs, with the reference's command line.

    python benchmarks/bench_tree_forest_sweep.py --model llama-1b --target-model llama-8b \
        --prefix-len 8192 --pairs 3 4 --pairs 4 5 --warmup 3 --iters 10

For every ``--pairs K D`` on one prefilled drafter, each timed as ``--warmup`` untimed then
``--iters`` timed runs (CUDA events, mean and min):

* ``batch1_ar_{D}_tokens``, ``batch{K}_ar_{D}_tokens``, ``batch{K*K}_ar_{D}_tokens``: batch AR
  from the prefix (every route keeps its own greedy child);
* ``atlas_tree_k{K}_d{D}``: the stage-1 tree (global top-k per depth);
* ``atlas_forest_k{K}_d{D}``: the k^2-route forest grown from a finished tree (the tree untimed).

With ``--target-model``, the target also runs, per pair, the full-model arms of
``bench_full_verify.py`` (AR1, linear and masked verify of K synthetic routes of depth D, with
the alignment check against one-row append decoding unless ``--skip-logit-alignment-check``).

Parity: reference benchmarks/bench_flashinfer_paged_tree_forest.py:47-666 (flags :60-97, the
per-pair arms :554-620, target verify :423-491).  Its SGLang memory and scheduler settings and
FlashInfer switches are accepted and ignored.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)


def sibling(name: str):
    spec = importlib.util.spec_from_file_location(name, os.path.join(HERE, f"{name}.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


iso = sibling("bench_isolated_components")
fv = sibling("bench_full_verify")
pkg = iso.pkg

_INERT = (("--mem-fraction-static", float), ("--max-running-requests", int), ("--max-total-tokens", int),
          ("--nccl-port", int), ("--verify-workspace-mb", int))


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Batch AR vs ATLAS tree/forest over (k, d) pairs, optional target verify.")
    p.add_argument("--model", required=True, help="drafter preset or checkpoint directory")
    p.add_argument("--target-model", default=None, help="also run the target's full-model verify arms per pair")
    p.add_argument("--prompt", default="ATLAS staged decode benchmark.")
    p.add_argument("--prompt-token-ids", default=None, help="comma-separated ids (overrides --prompt)")
    p.add_argument("--tokenizer", default=None, help="tokenizer.json for --prompt (UTF-8 bytes without one)")
    p.add_argument("--prefix-len", type=int, default=None, help="repeat / cut the prompt to this many tokens")
    p.add_argument("--repeat-token-id", type=int, default=None, help="prefix = this token, --prefix-len times")
    p.add_argument("--prefill-chunk-size", type=int, default=8192)
    p.add_argument("--pairs", nargs=2, type=int, action="append", metavar=("K", "D"))
    p.add_argument("--dtype", default="float16")
    p.add_argument("--device", default="cuda")
    p.add_argument("--gpu-id", type=int, default=None)
    p.add_argument("--context-length", type=int, default=8192)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--seed", type=int, default=0, help="seed of random-init presets")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--verify-warmup", type=int, default=None)
    p.add_argument("--verify-iters", type=int, default=None)
    for flag, typ in _INERT:
        p.add_argument(flag, type=typ, default=None, help="No-op (a setting of the reference's SGLang/FlashInfer "
                                                          "runtime with no counterpart here).")
    p.add_argument("--flashinfer-backend", default="auto", help="No-op (attention is this package's own kernel).")
    p.add_argument("--use-packed-custom-mask", action="store_true", help="No-op (the mask is always packed).")
    p.add_argument("--skip-logit-alignment-check", action="store_true")
    p.add_argument("--fail-on-logit-mismatch", action="store_true")
    p.add_argument("--alignment-atol", type=float, default=1.0)
    p.add_argument("--alignment-rtol", type=float, default=0.05)
    p.add_argument("--trust-remote-code", action="store_true", help="No-op (checkpoints are read as safetensors).")
    p.add_argument("--json-out", default=None)
    return p


def prompt_tokens(args, vocab: int) -> list[int]:
    if args.prompt_token_ids:
        base = [int(x) for x in args.prompt_token_ids.split(",") if x.strip()]
    elif args.repeat_token_id is not None:
        base = [int(args.repeat_token_id) % vocab]
    else:
        prompts = pkg("serving.prompts")
        base = [t % vocab for t in prompts.encode(prompts.load_tokenizer(args.tokenizer), args.prompt)]
    if not base:
        raise SystemExit("the prompt is empty")
    n = int(args.prefix_len) if args.prefix_len else len(base)
    return (base * ((n + len(base) - 1) // len(base)))[:n]


def required_context(prompt_len: int, pairs) -> int:
    """Positions a pair needs after the prompt: the deepest forest route (2 d) plus slack."""
    return prompt_len + max(2 * d for _, d in pairs) + 64


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    pairs = [tuple(x) for x in (args.pairs or [[3, 4]])]
    loader = pkg("models.loader")
    engine_mod, drafter_mod, store_mod = pkg("runtime.engine"), pkg("runtime.drafter"), pkg("runtime.store")
    dev = torch.device(args.device if args.gpu_id is None else f"cuda:{args.gpu_id}")
    if dev.type == "cuda" and dev.index is not None:
        torch.cuda.set_device(dev)
    cuda = dev.type == "cuda"
    dw = loader.resolve_model(args.model, dtype=args.dtype, device=dev, seed=args.seed)
    prompt = prompt_tokens(args, dw.config.vocab_size)
    need = required_context(len(prompt), pairs)
    ctx = max(int(args.context_length), need)
    ps = int(args.page_size)
    pages = 2 * (ctx // ps) + 64 + 4 * max(k * k * d for k, d in pairs)
    report: dict = {"metadata": {"model": args.model, "target_model": args.target_model, "prompt_len": len(prompt),
                                 "page_size": ps, "requested_context_length": args.context_length,
                                 "effective_context_length": ctx, "required_context_length": need,
                                 "warmup": args.warmup, "iters": args.iters, "dtype": args.dtype,
                                 "device": str(dev), "paged_kv": True}, "pairs": []}
    dr = drafter_mod.DrafterRuntime(engine_mod.LlamaEngine(dw, num_pages=pages, page_size=ps, max_positions=ctx),
                                    prefill_chunk_size=args.prefill_chunk_size)
    store = store_mod.KVTreeStore()
    dr.bind_store(store)
    if cuda:
        dr.warm_graphs(max(k for k, _ in pairs))
    dr.prefill(prompt)

    def measure(fn, warmup: int, iters: int, setup=None) -> dict:
        ms = []
        for i in range(int(warmup) + int(iters)):
            call = setup() if setup is not None else fn
            t = iso.timed(call, cuda)[0]
            dr.drop_speculative()
            if i >= int(warmup):
                ms.append(t)
        return {"mean_ms": round(statistics.fmean(ms), 4), "min_ms": round(min(ms), 4), "iters": len(ms)}

    for k, d in pairs:
        arms = iso.DrafterArms(dr, store, k, d)
        r: dict = {"k": k, "d": d}
        r[f"batch1_ar_{d}_tokens"] = measure(lambda: arms.batch_ar(1), args.warmup, args.iters)
        r[f"batch{k}_ar_{d}_tokens"] = measure(lambda: arms.batch_ar(k), args.warmup, args.iters)
        r[f"atlas_tree_k{k}_d{d}"] = measure(arms.tree, args.warmup, args.iters)
        r[f"batch{k * k}_ar_{d}_tokens"] = measure(lambda: arms.batch_ar(k * k), args.warmup, args.iters)
        r[f"atlas_forest_k{k}_d{d}"] = measure(None, args.warmup, args.iters, setup=arms.forest_after_tree)
        r["tree_over_batch_k"] = round(r[f"atlas_tree_k{k}_d{d}"]["mean_ms"] / r[f"batch{k}_ar_{d}_tokens"]["mean_ms"], 4)
        r["forest_over_batch_k2"] = round(r[f"atlas_forest_k{k}_d{d}"]["mean_ms"]
                                          / r[f"batch{k * k}_ar_{d}_tokens"]["mean_ms"], 4)
        report["pairs"].append(r)
    dr.engine.ops.check()
    del dr, dw
    if cuda:
        torch.cuda.empty_cache()

    if args.target_model:
        vw = args.verify_warmup if args.verify_warmup is not None else args.warmup
        vi = args.verify_iters if args.verify_iters is not None else args.iters
        for r in report["pairs"]:
            fv_args = fv.build_parser().parse_args(
                ["--model", args.target_model, "--k", str(r["k"]), "--d", str(r["d"]), "--prefix-len",
                 str(len(prompt)), "--prompt-token-ids", ",".join(map(str, prompt)), "--page-size", str(ps),
                 "--dtype", args.dtype, "--device", str(dev), "--seed", str(args.seed + 1), "--warmup", str(vw),
                 "--iters", str(vi), "--alignment-atol", str(args.alignment_atol), "--alignment-rtol",
                 str(args.alignment_rtol)]
                + (["--skip-logit-alignment-check"] if args.skip_logit_alignment_check else [])
                + (["--fail-on-logit-mismatch"] if args.fail_on_logit_mismatch else []))
            r["target"] = fv.run(fv_args)
            if cuda:
                torch.cuda.empty_cache()
    line = json.dumps(report)
    print(line, flush=True)
    if args.json_out:
        with open(args.json_out, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
