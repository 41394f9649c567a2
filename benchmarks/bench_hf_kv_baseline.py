#!/usr/bin/env python
"""Ordinary Hugging Face KV-cache decode of the ATLAS component shapes (a library baseline).

    python benchmarks/bench_hf_kv_baseline.py --drafter-model llama-1b --target-model llama-8b \
        --prefix-len 8192 --k 3 --d 4 --warmup 3 --iters 10

Nothing of this framework runs in the timed regions: the models are transformers'
``LlamaForCausalLM`` (presets carry this package's seeded random weights under Hugging Face
names, checkpoint directories load as they are) and the cache is
transformers' ``DynamicCache``, one copy of the prefix per batch row, reordered along the
batch after each selection.  It gives the numbers the paged, shared-prefix runtime is to be
compared with:

* drafter: batch-1 / batch-k / batch-k^2 greedy AR of d tokens, the stage-1 tree (global
  top-k over the k x k children of each depth) and the stage-2 forest (k children per tree
  route, then per-root top-k for d depths);
* target (``--target-model``, default the drafter): batch-1 decode of 1 and of d tokens,
  batch-k AR of d tokens, and the verify append of k paths of d tokens onto a batch-k cache.

Each sample starts from a freshly prefilled cache (prefill untimed) unless ``--stateful-cache``
reuses one cache across samples.  Times are CUDA-event (or wall, on CPU) medians and means.

Parity: reference benchmarks/bench_hf_kv_components.py:22-663 (arms :263-443, flags :29-60);
the result keys follow its names so the two reports line up.
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


def pkg(name):
    return importlib.import_module(f"0709_b200.{name}")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Hugging Face DynamicCache decode of the ATLAS component shapes "
                                            "(not a shared-KV benchmark).")
    p.add_argument("--drafter-model", required=True, help="preset (seeded random init) or HF checkpoint directory")
    p.add_argument("--target-model", default=None, help="default: the drafter model")
    p.add_argument("--k", type=int, default=3)
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--prompt", default="ATLAS clean component speed benchmark.")
    p.add_argument("--prompt-token-ids", default=None)
    p.add_argument("--tokenizer", default=None, help="tokenizer.json for --prompt (UTF-8 bytes without one)")
    p.add_argument("--prefix-len", type=int, default=8192)
    p.add_argument("--repeat-token-id", type=int, default=42, help="a negative value uses --prompt")
    p.add_argument("--dtype", choices=["float16", "bfloat16", "float32"], default="float16")
    p.add_argument("--device", default="cuda")
    p.add_argument("--seed", type=int, default=0, help="seed of random-init presets (target: seed + 1)")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--trust-remote-code", action="store_true", help="passed to transformers")
    p.add_argument("--stateful-cache", action="store_true",
                   help="reuse and extend one cache across samples (faster to run, not a fair comparison)")
    p.add_argument("--json-out", default=None)
    return p


def prompt_tokens(args, vocab: int) -> list[int]:
    if args.prompt_token_ids:
        base = [int(x) for x in args.prompt_token_ids.split(",") if x.strip()]
    elif args.repeat_token_id is not None and args.repeat_token_id >= 0:
        base = [int(args.repeat_token_id)]
    else:
        prompts = pkg("serving.prompts")
        base = prompts.encode(prompts.load_tokenizer(args.tokenizer), args.prompt)
    base = [t % vocab for t in base]
    if not base:
        raise SystemExit("the prompt is empty")
    n = int(args.prefix_len)
    return (base * ((n + len(base) - 1) // len(base)))[:n]


def load_hf(spec: str, *, dtype: torch.dtype, device: torch.device, seed: int, trust: bool):
    """transformers' Llama: loaded from a checkpoint directory, or built for a preset and given
    this package's seeded weights (drawn on ``device``, as the engines draw presets) in memory."""
    from transformers import AutoModelForCausalLM, LlamaConfig, LlamaForCausalLM

    if os.path.isdir(spec):
        return AutoModelForCausalLM.from_pretrained(spec, dtype=dtype, trust_remote_code=trust).to(device).eval()
    loader, llama = pkg("models.loader"), pkg("models.llama")
    w = llama.random_weights(llama.get_config(spec), seed=seed, dtype=dtype, device=device)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            model = LlamaForCausalLM(LlamaConfig(**loader.config_to_hf(w.config)))
    finally:
        torch.set_default_dtype(prev)
    model.load_state_dict(loader.hf_state_dict(w), strict=not w.config.tie_word_embeddings)
    return model.eval()


class Stats:
    def __init__(self, device: torch.device) -> None:
        self.cuda = device.type == "cuda"

    def time(self, fn) -> float:
        if not self.cuda:
            t0 = time.perf_counter()
            fn()
            return (time.perf_counter() - t0) * 1e3
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    def measure(self, setup, run, warmup: int, iters: int, stateful: bool) -> dict:
        """``run(state)`` timed ``iters`` times after ``warmup``; a fresh ``setup()`` per sample
        (untimed) unless ``stateful``, where one state is reused and extended."""
        state = setup() if stateful else None
        ms = []
        for i in range(int(warmup) + int(iters)):
            s = state if stateful else setup()
            t = self.time(lambda: run(s))
            if i >= int(warmup):
                ms.append(t)
        return {"median_ms": round(statistics.median(ms), 4), "mean_ms": round(statistics.fmean(ms), 4),
                "samples_ms": [round(x, 4) for x in ms]}


class HFArms:
    """The component workloads on one transformers model and its ``DynamicCache``."""

    def __init__(self, model, prompt: list[int], device: torch.device) -> None:
        self.model, self.prompt, self.device = model, prompt, device

    @torch.inference_mode()
    def prefill(self, batch: int):
        ids = torch.tensor([self.prompt] * int(batch), dtype=torch.long, device=self.device)
        out = self.model(input_ids=ids, use_cache=True)
        return out.past_key_values, out.logits[:, -1].float()

    @torch.inference_mode()
    def step(self, past, ids: torch.Tensor):
        """Decode one token per row ([b] ids); returns the rows' next-token logits."""
        out = self.model(input_ids=ids.reshape(-1, 1), past_key_values=past, use_cache=True)
        return out.logits[:, -1].float()

    @torch.inference_mode()
    def ar(self, state, steps: int) -> None:
        past, ids = state
        for _ in range(int(steps)):
            ids = self.step(past, ids).argmax(-1)

    @staticmethod
    def children(logits: torch.Tensor, scores: torch.Tensor, k: int):
        """Every row's k best children: (token [b, k], cumulative score [b, k])."""
        lp, tok = torch.topk(torch.log_softmax(logits, -1), int(k), dim=-1)
        return tok, scores[:, None] + lp

    @torch.inference_mode()
    def tree_state(self, k: int):
        past, logits = self.prefill(k)
        lp, tok = torch.topk(torch.log_softmax(logits[:1], -1), int(k), dim=-1)
        return past, tok.reshape(-1), lp.reshape(-1)

    @torch.inference_mode()
    def tree(self, state, k: int, depth: int):
        """Global top-k over the k x k children per depth, the cache reordered to the parents."""
        past, ids, scores = state
        for _ in range(int(depth)):
            tok, sc = self.children(self.step(past, ids), scores, k)
            scores, flat = torch.topk(sc.reshape(-1), int(k))
            parents = flat // int(k)
            ids = tok.reshape(-1)[flat]
            past.reorder_cache(parents)
        return past, ids, scores

    @torch.inference_mode()
    def forest_state(self, k: int, depth: int):
        """A finished tree (its pending tokens decoded), each route expanded to its k children."""
        past, ids, scores = self.tree(self.tree_state(k), k, depth)
        tok, sc = self.children(self.step(past, ids), scores, k)
        past.reorder_cache(torch.arange(int(k), device=self.device).repeat_interleave(int(k)))
        return past, tok.reshape(-1), sc.reshape(-1)

    @torch.inference_mode()
    def forest(self, state, k: int, depth: int) -> None:
        """Per-root top-k: the k^2 rows stay grouped by root (k rows each), each root keeps the
        k best of its k x k children."""
        past, ids, scores = state
        k = int(k)
        for _ in range(int(depth)):
            tok, sc = self.children(self.step(past, ids), scores, k)  # [k*k, k]
            scores, pick = torch.topk(sc.reshape(k, k * k), k, dim=1)  # per root
            rows = (torch.arange(k, device=self.device)[:, None] * k + pick // k).reshape(-1)
            ids = tok.reshape(k * k, k)[rows, (pick % k).reshape(-1)]
            scores = scores.reshape(-1)
            past.reorder_cache(rows)

    @torch.inference_mode()
    def verify_state(self, k: int, depth: int):
        past, logits = self.prefill(k)
        _, tok = torch.topk(logits, int(depth), dim=-1)
        return past, tok

    @torch.inference_mode()
    def verify(self, state) -> None:
        past, tok = state
        self.model(input_ids=tok, past_key_values=past, use_cache=True)


def run(args) -> dict:
    dev = torch.device(args.device)
    dt = getattr(torch, args.dtype)
    k, d = int(args.k), int(args.d)
    if k <= 0 or d <= 0:
        raise SystemExit("k and d must be positive")
    st = Stats(dev)
    W, I, S = args.warmup, args.iters, args.stateful_cache
    out: dict = {"backend": "hf_kv_ordinary_batch", "shared_kv_optimized": False, "masked_verify": False,
                 "drafter_model": args.drafter_model, "target_model": args.target_model or args.drafter_model,
                 "k": k, "d": d, "dtype": args.dtype, "device": str(dev), "warmup": W, "iters": I,
                 "stateful_cache": bool(S), "prefill_excluded_from_timing": True}
    m = load_hf(args.drafter_model, dtype=dt, device=dev, seed=args.seed, trust=args.trust_remote_code)
    prompt = prompt_tokens(args, m.config.vocab_size)
    out["prefix_len"] = len(prompt)
    a = HFArms(m, prompt, dev)

    def ar_setup(b):
        def setup():
            past, logits = a.prefill(b)
            return past, logits.argmax(-1)
        return setup

    dr = {}
    dr[f"batch1_ar_{d}_tokens"] = st.measure(ar_setup(1), lambda s: a.ar(s, d), W, I, S)
    dr[f"batch{k}_ar_{d}_tokens"] = st.measure(ar_setup(k), lambda s: a.ar(s, d), W, I, S)
    dr[f"build_tree_stage1_k{k}_d{d}"] = st.measure(lambda: a.tree_state(k), lambda s: a.tree(s, k, d), W, I, S)
    dr[f"batch{k * k}_ar_{d}_tokens"] = st.measure(ar_setup(k * k), lambda s: a.ar(s, d), W, I, S)
    dr[f"build_forest_stage2_k2_{k * k}_d{d}"] = st.measure(lambda: a.forest_state(k, d),
                                                             lambda s: a.forest(s, k, d), W, I, S)
    med = {n: v["median_ms"] for n, v in dr.items()}
    tree, forest = med[f"build_tree_stage1_k{k}_d{d}"], med[f"build_forest_stage2_k2_{k * k}_d{d}"]
    dr["ratios_median"] = {"tree_over_batch1_ar": tree / med[f"batch1_ar_{d}_tokens"],
                           "tree_over_batchk_ar": tree / med[f"batch{k}_ar_{d}_tokens"],
                           "forest_over_batch1_ar": forest / med[f"batch1_ar_{d}_tokens"],
                           "forest_over_batchk2_ar": forest / med[f"batch{k * k}_ar_{d}_tokens"]}
    out["drafter"] = dr
    if args.target_model and args.target_model != args.drafter_model:
        del a, m
        if dev.type == "cuda":
            torch.cuda.empty_cache()
        m = load_hf(args.target_model, dtype=dt, device=dev, seed=args.seed + 1, trust=args.trust_remote_code)
        a = HFArms(m, prompt, dev)
    tg = {}
    tg["target_batch1_decode_1_token"] = st.measure(ar_setup(1), lambda s: a.ar(s, 1), W, I, S)
    tg[f"target_batch1_ar_{d}_tokens"] = st.measure(ar_setup(1), lambda s: a.ar(s, d), W, I, S)
    tg[f"target_batch{k}_ar_{d}_tokens"] = st.measure(ar_setup(k), lambda s: a.ar(s, d), W, I, S)
    tg[f"target_verify_k{k}_paths_d{d}"] = st.measure(lambda: a.verify_state(k, d), a.verify, W, I, S)
    v = tg[f"target_verify_k{k}_paths_d{d}"]["median_ms"]
    tg["ratios_median"] = {"verify_over_decode1": v / tg["target_batch1_decode_1_token"]["median_ms"],
                           "verify_over_batch1_ar": v / tg[f"target_batch1_ar_{d}_tokens"]["median_ms"],
                           "verify_over_batchk_ar": v / tg[f"target_batch{k}_ar_{d}_tokens"]["median_ms"]}
    out["target"] = tg
    return out


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    line = json.dumps(run(args))
    print(line, flush=True)
    if args.json_out:
        with open(args.json_out, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
