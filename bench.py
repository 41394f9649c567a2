#!/usr/bin/env python
"""Headline benchmark: asynchronous tree/forest speculative decoding throughput.

Workload: Llama-3.2-1B-shaped drafter + Llama-3.1-8B-shaped
target, fp16, random-init weights, k=3 d=4, page 16, path weights
0.45/0.30/0.17/0.08, fallback -0.50, first-token -0.70, 4 fallback AR tokens;
synthetic prompts of uniform-random token ids with lengths uniform in
[128, 2048], 256 new tokens each.  One step = one speculative round of the
session (verify || forest, then handoff); when a prompt finishes, the next
prompt's prefill runs inside the following step.  Each rank (one per GPU)
serves its own session with drafter and target on its GPU (data parallel,
weak scaling).

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier and
``torch.cuda.synchronize()``, timed with CUDA events; tokens are summed over
ranks and the time is the max over ranks.  The weights (17 GB) stream through
every step, so the working set is far larger than the 126 MB L2.

``--impl reference`` runs the reference implementation's arm.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import random
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Reference: async GSM8K end to end, k=3 d=4, weights .45/.30/.17/.08, fallback
# -0.5/-0.7, AR4, Llama-3.2-1B + Llama-3.1-8B fp16 on 1xH800: 57.88 tok/s.
BASELINE_TOKENS_PER_S = 57.88
METRIC = "decode tokens/sec (device-timed, max over ranks) at 8B/70B; ms per spec round"


def _pkg(name: str):
    return importlib.import_module(f"0709_b200.{name}")


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=48)
    p.add_argument("--warmup", type=int, default=4)
    p.add_argument("--impl", choices=["atlas", "reference"], default="atlas")
    p.add_argument("--drafter", default="llama-1b")
    p.add_argument("--target", default="llama-8b")
    p.add_argument("--dtype", default="float16")
    p.add_argument("--k", type=int, default=3)
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--prompts", type=int, default=64)
    p.add_argument("--min-prompt", type=int, default=128)
    p.add_argument("--max-prompt", type=int, default=2048)
    p.add_argument("--max-new-tokens", type=int, default=256)
    p.add_argument("--path-score-weights", default="0.45,0.30,0.17,0.08")
    p.add_argument("--fallback-threshold", type=float, default=-0.50)
    p.add_argument("--first-token-threshold", type=float, default=-0.70)
    p.add_argument("--fallback-ar-tokens", type=int, default=4)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--e2e-prompts", type=int, default=1)
    p.add_argument("--forest-gate", choices=["overlap", "adaptive"], default="adaptive",
                   help="drafter forest schedule (see DistributedAtlasConfig.forest_gate)")
    p.add_argument("--target-stream-priority", type=int, default=-1,
                   help="CUDA priority of the target's stream (lower = higher; 0 = same as the drafter)")
    return p.parse_args()


def reference_arm(args) -> None:
    """The reference's end-to-end path needs SGLang for its drafter; report why it cannot run."""
    reason = None
    try:
        importlib.import_module("sglang")
    except Exception as exc:  # noqa: BLE001
        reason = f"reference drafter requires sglang==0.5.14 (ModelRunner + paged FlashInfer decode), not installed offline: {type(exc).__name__}"
    if reason is None:
        reason = "reference arm not wired for this image"
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def make_prompts(args, rank: int) -> list[list[int]]:
    rng = random.Random(args.seed * 1000 + rank)
    vocab = 128256
    out = []
    for _ in range(args.prompts):
        n = rng.randint(args.min_prompt, args.max_prompt)
        out.append([rng.randrange(vocab) for _ in range(n)])
    return out


class StreamTargetClient:
    """In-process target client whose calls run on the target's own CUDA stream."""

    supports_early_decision = True

    def __init__(self, backend, stream) -> None:
        rpc = _pkg("serving.rpc")
        self.inner = rpc.InProcessTargetClient(backend)
        self.stream = stream

    def health(self):
        return self.inner.health()

    def prefill(self, toks):
        import torch

        with torch.cuda.stream(self.stream):
            out = self.inner.prefill(toks)
        self.stream.synchronize()
        return out

    def verify(self, **kw):
        import torch

        with torch.cuda.stream(self.stream):
            out = self.inner.verify(**kw)
        self.stream.synchronize()
        return out


def build(args, device):
    import torch

    llama = _pkg("models.llama")
    engine = _pkg("runtime.engine")
    drafter_mod = _pkg("runtime.drafter")
    target_mod = _pkg("runtime.target")
    edge = _pkg("serving.edge")
    dtype = {"float16": torch.float16, "bfloat16": torch.bfloat16}[args.dtype]
    dcfg = llama.get_config(args.drafter)
    tcfg = llama.get_config(args.target)
    wd = llama.random_weights(dcfg, seed=args.seed + 1, dtype=dtype, device=device)
    wt = llama.random_weights(tcfg, seed=args.seed + 2, dtype=dtype, device=device)
    max_ctx = args.max_prompt + args.max_new_tokens + 4 * args.d + 64
    pages = (max_ctx // args.page_size + 8) * 4 + 256
    de = engine.LlamaEngine(wd, num_pages=pages, page_size=args.page_size, max_positions=max_ctx + 64)
    te = engine.LlamaEngine(wt, num_pages=pages, page_size=args.page_size, max_positions=max_ctx + 64)
    weights = [float(x) for x in args.path_score_weights.split(",")] if args.path_score_weights else None
    tv = target_mod.TargetVerifier(
        te,
        k=args.k,
        d=args.d,
        score_weights=weights,
        fallback_threshold=args.fallback_threshold,
        first_token_threshold=args.first_token_threshold,
        fallback_ar_tokens=args.fallback_ar_tokens,
        model_name=f"random-init {args.target}",
    )
    # The target is on the critical path of every round (verify, then fallback AR);
    # the drafter's forest only fills the wait, so the target stream gets priority.
    client = StreamTargetClient(tv, torch.cuda.Stream(device=device, priority=args.target_stream_priority))
    dr = drafter_mod.DrafterRuntime(de)
    dr.warm_graphs(args.k, args.fallback_ar_tokens)
    tv.warm_graphs()
    gen = edge.PagedDistributedAtlasGenerator(
        config=edge.DistributedAtlasConfig(
            k=args.k, d=args.d, max_new_tokens=args.max_new_tokens, fallback_ar_tokens=args.fallback_ar_tokens,
            generation_seed=args.seed, forest_gate=args.forest_gate,
        ),
        drafter=dr,
        target_client=client,
    )
    return gen, de, te


class Driver:
    """Serves prompts back to back; one step = one speculative round."""

    def __init__(self, gen, prompts) -> None:
        self.gen = gen
        self.prompts = prompts
        self.next = 0
        self.session = None
        self.rounds = 0
        self.fallback_rounds = 0
        self.prompts_started = 0
        self.breakdown: list[tuple[float, float, float, float]] = []  # round, verify, forest, handoff (s)

    def step(self) -> int:
        if self.session is None or self.session.finished:
            p = self.prompts[self.next % len(self.prompts)]
            self.next += 1
            self.prompts_started += 1
            self.session = self.gen.start(p)
        t0 = time.perf_counter()
        tr = self.session.step()
        dt = time.perf_counter() - t0
        rt = self.session.rounds_tl[-1]
        forest = sum(sp.elapsed_s for sp in rt.forest_steps)
        handoff = (rt.handoff.elapsed_s if rt.handoff is not None else 0.0) + sum(
            sp.elapsed_s for sp in rt.post_prune_tree_steps)
        self.breakdown.append((dt, rt.verify_blackbox.elapsed_s, forest, handoff))
        self.rounds += 1
        self.fallback_rounds += int(tr.decision == "fallback_ar")
        return len(tr.committed_tokens)


def main() -> int:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return 0
    import torch
    import torch.distributed as dist

    counters = _pkg("utils.counters")
    clocks = _pkg("utils.clocks")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    gen, de, te = build(args, device)
    drv = Driver(gen, make_prompts(args, rank))
    for _ in range(args.warmup):
        drv.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    c0 = counters.snapshot()
    r0, f0 = drv.rounds, drv.fallback_rounds
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    gpu_index = int(phys.split(",")[local]) if phys and phys.split(",")[local].isdigit() else local
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tokens = 0
    with clocks.ClockSampler(gpu_index) as sampler:
        start.record()
        for _ in range(args.steps):
            tokens += drv.step()
        end.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    delta = counters.delta(c0)
    clk = sampler.summary()
    de.ops.check()
    te.ops.check()
    stats = torch.tensor([float(tokens), ms, float(delta["launches"])], dtype=torch.float64, device=device)
    if world > 1:
        tok_t = stats[:1].clone()
        dist.all_reduce(tok_t, op=dist.ReduceOp.SUM)
        ms_t = stats[1:2].clone()
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        launches_t = stats[2:3].clone()
        dist.all_reduce(launches_t, op=dist.ReduceOp.SUM)
        clk_all = [None] * world
        dist.all_gather_object(clk_all, clk)
        total_tokens, ms_max, launches = float(tok_t.item()), float(ms_t.item()), int(launches_t.item())
    else:
        clk_all = [clk]
        total_tokens, ms_max, launches = float(tokens), ms, int(delta["launches"])
    value = total_tokens / (ms_max / 1000.0)

    # End-to-end through the public API: whole prompts via generate(), prompt ids
    # copied from pinned host memory, result tokens read back on the host.
    e2e_prompts = make_prompts(argparse.Namespace(**{**vars(args), "seed": args.seed + 7}), rank)[: args.e2e_prompts]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ce = counters.snapshot()
    t0 = time.perf_counter()
    e2e_tokens = 0
    e2e_rounds = 0
    for p in e2e_prompts:
        pinned = torch.tensor(p, dtype=torch.int32).pin_memory()
        dev_ids = pinned.to(device, non_blocking=True)
        counters.h2d(pinned.numel() * 4)
        res = gen.generate(dev_ids.cpu().tolist())
        out = torch.tensor(res.generated_token_ids, dtype=torch.int32, device=device).cpu()
        counters.d2h(out.numel() * 4)
        e2e_tokens += int(out.numel())
        e2e_rounds += len(res.rounds)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_delta = counters.delta(ce)
    e2e_stats = torch.tensor([float(e2e_tokens), e2e_s], dtype=torch.float64, device=device)
    if world > 1:
        t_ = e2e_stats[:1].clone()
        dist.all_reduce(t_, op=dist.ReduceOp.SUM)
        s_ = e2e_stats[1:2].clone()
        dist.all_reduce(s_, op=dist.ReduceOp.MAX)
        e2e_tokens_all, e2e_s_max = float(t_.item()), float(s_.item())
    else:
        e2e_tokens_all, e2e_s_max = float(e2e_tokens), e2e_s
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        reasons = sorted({r for c in clk_all if c for r in c.get("reasons", [])})
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(value / BASELINE_TOKENS_PER_S, 3) if world == 1 else None,
            "dtype": args.dtype.replace("float16", "fp16").replace("bfloat16", "bf16"),
            "data": "synthetic uniform-random token ids, random-init weights",
            "config": {
                "model": f"{args.drafter} drafter + {args.target} target (random init)",
                "global_batch": world,
                "seq_len": f"prompt U[{args.min_prompt},{args.max_prompt}] + {args.max_new_tokens} new",
                "parallelism": f"dp{world} (one drafter+target session per GPU)",
                "k": args.k,
                "d": args.d,
                "page_size": args.page_size,
                "path_score_weights": args.path_score_weights,
                "fallback_threshold": args.fallback_threshold,
                "first_token_threshold": args.first_token_threshold,
                "fallback_ar_tokens": args.fallback_ar_tokens,
                "forest_gate": args.forest_gate,
                "step": ("one speculative round (verify, with the forest overlapped unless the adaptive gate is closed; "
                         "handoff); next prompt's prefill inside its step"),
                "l2": "weights (~17 GB) stream every step; working set far above L2",
                "rounds_timed": drv.rounds - r0,
                "round_breakdown_ms": {
                    k: round(1e3 * sum(b[i] for b in drv.breakdown[r0:]) / max(1, drv.rounds - r0), 3)
                    for i, k in enumerate(("round_host", "target_verify_blackbox", "drafter_forest", "drafter_handoff"))
                },
                "fallback_rate_timed": round((drv.fallback_rounds - f0) / max(1, drv.rounds - r0), 3),
                "tokens_timed": int(total_tokens),
            },
            "clocks": {
                "sm_mhz": clk_all[0].get("sm_mhz") if clk_all[0] else None,
                "sm_max_mhz": clk_all[0].get("sm_max_mhz") if clk_all[0] else None,
                "reasons": reasons,
            },
            "e2e": {
                "value": round(e2e_tokens_all / e2e_s_max, 3) if e2e_s_max > 0 else None,
                "unit": "tokens/s",
                "h2d_bytes_per_step": int(delta["h2d_bytes"] / max(1, args.steps)),
                "d2h_bytes_per_step": int(delta["d2h_bytes"] / max(1, args.steps)),
                "prompts": args.e2e_prompts,
                "rounds": e2e_rounds,
                "includes": "prefill of both models + all rounds via PagedDistributedAtlasGenerator.generate",
                "e2e_h2d_bytes": int(e2e_delta["h2d_bytes"]),
                "e2e_d2h_bytes": int(e2e_delta["d2h_bytes"]),
            },
            "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
