#!/usr/bin/env python
"""Target side on one GPU: the reference's own verify backend vs this framework's, same weights.

    python benchmarks/bench_reference_target.py --prefix 1024 4096 8192 16384

Reference arm: the unmodified ``DirectFlashInferMaskedTreeVerifyBackend`` of
the installed reference package (``baseline/_ref``; Hugging Face transformers
Llama modules plus FlashInfer's masked paged prefill and paged decode) driven
through its public ``prefill`` / ``verify_payloads`` API.  Ours:
``TargetVerifier`` over ``LlamaEngine`` (tcgen05 GEMMs, paged tree attention,
graphed forwards).

Both arms run the same random-init Llama-3.1-8B-shaped fp16 weights: this
framework generates them and writes them as a Hugging Face checkpoint
(``models.loader.save_hf_checkpoint`` plus a stub tokenizer, which the
reference's loader requires but never uses for ids); the reference loads that
checkpoint with transformers.  The prefill logits of both arms are compared as
a cross-check that the two models are the same.

Protocol (the reference's own, benchmarks/bench_atlas_0709_isolated_components.py:1204-1233):
every iteration prefills the prompt, synchronizes, then times ONE
``verify_payloads`` call with the host clock between device synchronizations
-- the call includes the masked tree forward, scoring, selection and the
selected path's KV commit.  Cases: k routes of depth d=4 with no shared
tokens (k=3: 12 tree nodes; k=12: 48 nodes), in two regimes:

* ``select``: first-route policy, no thresholds (verify + commit);
* ``fallback``: every route below the threshold, 4 fallback AR tokens (the
  config-2 fallback round; ours also runs the last token's forward, which it
  normally defers to the next verify, inside the timed region).

Prints one JSON line.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
REF = os.path.join(ROOT, "baseline", "_ref")


def pkg(name):
    return importlib.import_module(f"0709_b200.{name}")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama-8b")
    p.add_argument("--prefix", type=int, nargs="+", default=[1024, 4096, 8192, 16384])
    p.add_argument("--k", type=int, nargs="+", default=[3, 12])
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--ckpt-dir", default="/tmp/atlas_ref_target_ckpt")
    p.add_argument("--seed", type=int, default=2)
    p.add_argument("--skip-reference", action="store_true")
    p.add_argument("--json-out", default=None)
    return p.parse_args()


def write_stub_tokenizer(path: str) -> None:
    """A one-entry word-level tokenizer: enough for ``AutoTokenizer.from_pretrained``."""
    from tokenizers import Tokenizer, models
    from transformers import PreTrainedTokenizerFast

    tok = PreTrainedTokenizerFast(tokenizer_object=Tokenizer(models.WordLevel({"<unk>": 0}, unk_token="<unk>")),
                                  unk_token="<unk>")
    tok.save_pretrained(path)


def synthetic_routes(types, k: int, d: int, base: int, vocab: int):
    """``k`` routes of ``d`` distinct tokens each (no shared prefix: k*d tree nodes)."""
    out = []
    for r in range(k):
        toks = tuple(int((base + 17 + r * d + j) % vocab) for j in range(d))
        out.append(types.VerifyRoutePayload(route_id=r + 1, token_ids=toks, draft_logprob=-float(r)))
    return out


def host_timed(fn) -> float:
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    return (time.perf_counter() - t0) * 1e3


def measure(prefill, verify, warmup: int, iters: int) -> dict:
    for _ in range(warmup):
        prefill()
        verify()
    samples = []
    for _ in range(iters):
        prefill()
        samples.append(host_timed(verify))
    return {"mean_ms": round(statistics.mean(samples), 3), "median_ms": round(statistics.median(samples), 3),
            "min_ms": round(min(samples), 3)}


def run_ours(args, w, prompts, dev) -> tuple[dict, dict]:
    engine = pkg("runtime.engine")
    target = pkg("runtime.target")
    types = pkg("types")
    vocab = w.config.vocab_size
    p_max = max(args.prefix)
    out, logits = {}, {}
    for k in args.k:
        for regime in ("select", "fallback"):
            kw = (dict(route_selection_policy="first_route") if regime == "select"
                  else dict(fallback_threshold=1e9, fallback_ar_tokens=4))
            eng = engine.LlamaEngine(w, num_pages=(p_max + 1024) // 16 + 512, page_size=16,
                                     max_positions=p_max + 1024)
            tv = target.TargetVerifier(eng, k=k, d=args.d, **kw)
            tv.warm_graphs()
            for P in args.prefix:
                prompt = prompts[P]
                routes = synthetic_routes(types, k, args.d, prompt[-1], vocab)

                def prefill():
                    res = tv.prefill(prompt)
                    if P not in logits:
                        logits[P] = res.next_token_logits.float().reshape(-1).clone()

                def verify():
                    res = tv.verify_payloads(prefix_token_ids=prompt, routes=routes)
                    assert res.decision == ("select" if regime == "select" else "fallback_ar")
                    if regime == "fallback":
                        tv.prefix_logits  # noqa: B018  (runs the deferred last-token forward)

                out[f"k{k}_{regime}_P{P}"] = measure(prefill, verify, args.warmup, args.iters)
            eng.ops.check()
            del tv, eng
            torch.cuda.empty_cache()
    return out, logits


def run_reference(args, prompts, ckpt) -> tuple[dict, dict]:
    sys.path.insert(0, REF)
    rt = importlib.import_module("atlas_0709.target_runtime")
    fv = importlib.import_module("atlas_0709.flashinfer_full_verify")
    out, logits = {}, {}
    for k in args.k:
        for regime in ("select", "fallback"):
            kw = (dict(route_selection_policy="first_route") if regime == "select"
                  else dict(fallback_threshold=1e9, fallback_ar_tokens=4))
            cfg = fv.FlashInferFullVerifyConfig(k=k, d=args.d, page_size=16, dtype="float16", device="cuda")
            backend = rt.DirectFlashInferMaskedTreeVerifyBackend(model_path=ckpt, config=cfg, **kw)
            vocab = backend.model.config.vocab_size
            for P in args.prefix:
                prompt = prompts[P]
                routes = [rt.VerifyRoutePayload(route_id=r.route_id, token_ids=r.token_ids,
                                                draft_logprob=r.draft_logprob)
                          for r in synthetic_routes(pkg("types"), k, args.d, prompt[-1], vocab)]

                def prefill():
                    res = backend.prefill(prompt)
                    if P not in logits:
                        logits[P] = res.next_token_logits.float().reshape(-1).clone()

                def verify():
                    res = backend.verify_payloads(prefix_token_ids=prompt, routes=routes)
                    assert res.decision == ("select" if regime == "select" else "fallback_ar")

                out[f"k{k}_{regime}_P{P}"] = measure(prefill, verify, args.warmup, args.iters)
            del backend
            torch.cuda.empty_cache()
    return out, logits


def main() -> int:
    args = parse()
    if not torch.cuda.is_available():
        raise SystemExit("CUDA is required")
    dev = torch.device("cuda", 0)
    llama = pkg("models.llama")
    clocks = pkg("utils.clocks")
    cfg = llama.get_config(args.model)
    w = llama.random_weights(cfg, seed=args.seed, dtype=torch.float16, device=dev)
    g = torch.Generator().manual_seed(0)
    prompts = {P: torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist() for P in args.prefix}
    line: dict = {"model": f"{args.model} (random init, fp16)", "d": args.d, "k": args.k, "prefix": args.prefix,
                  "protocol": "prefill, sync, host-timed verify_payloads (tree forward, scoring, selection, KV "
                              "commit; fallback: + 4 AR tokens), sync; mean/median over iters"}
    with clocks.ClockSampler(0) as cs_ours:
        ours, ours_logits = run_ours(args, w, prompts, dev)
    line["ours"] = ours
    line["ours_clocks"] = cs_ours.summary()
    if not args.skip_reference:
        if not os.path.isdir(os.path.join(REF, "atlas_0709")):
            line["reference"] = {"unavailable": f"reference package not installed under {REF}"}
        else:
            ckpt = args.ckpt_dir
            if not os.path.exists(os.path.join(ckpt, "model.safetensors")):
                pkg("models.loader").save_hf_checkpoint(w, ckpt)
                write_stub_tokenizer(ckpt)
            del w
            torch.cuda.empty_cache()
            with clocks.ClockSampler(0) as cs_ref:
                ref, ref_logits = run_reference(args, prompts, ckpt)
            line["reference"] = ref
            line["reference_clocks"] = cs_ref.summary()
            line["speedup_ours_vs_reference"] = {
                key: round(ref[key]["median_ms"] / ours[key]["median_ms"], 3) for key in ours if key in ref}
            line["prefill_logits_check"] = {
                str(P): {"max_abs_diff": round(float((ours_logits[P] - ref_logits[P].to(dev)).abs().max()), 4),
                         "top1_equal": int(ours_logits[P].argmax()) == int(ref_logits[P].argmax())}
                for P in args.prefix if P in ours_logits and P in ref_logits}
    s = json.dumps(line)
    print(s, flush=True)
    if args.json_out:
        with open(args.json_out, "w") as f:
            f.write(s + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
