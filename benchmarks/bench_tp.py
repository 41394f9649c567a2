#!/usr/bin/env python
"""70B-class target benchmark: tensor-parallel or fp8 target + colocated 1B drafter.

    torchrun --nproc-per-node N benchmarks/bench_tp.py --target llama-70b --mode fused|nccl [--fp8]

Rank 0 hosts the drafter, the speculative-decoding session and its shard of
the target; ranks 1..N-1 serve their target shards (``TPLlamaEngine.serve``).
With one process (N=1) the target is a single-GPU engine: bf16, or
block-scaled fp8 with ``--fp8``.  Reports, as one JSON line from rank 0:

* ``verify_ms``: device time of one masked tree-verify forward (k*d nodes,
  graph replay), CUDA events per rank, max over ranks;
* ``ar1_ms``: the same for a one-token target forward;
* ``tokens_per_s`` and ``ms_per_round``: the async tree/forest generation
  over the timed rounds (device-timed on rank 0, which drives every rank).
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def pkg(name):
    return importlib.import_module(f"0709_b200.{name}")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--target", default="llama-70b")
    p.add_argument("--drafter", default="llama-1b")
    p.add_argument("--mode", choices=["fused", "nccl"], default="fused")
    p.add_argument("--fp8", action="store_true", help="block-scaled fp8 target (single GPU)")
    p.add_argument("--dtype", default="bfloat16")
    p.add_argument("--width", dest="k", type=int, default=3)
    p.add_argument("--depth", dest="d", type=int, default=4)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--prompts", type=int, default=32)
    p.add_argument("--prompt-len", type=int, default=1024)
    p.add_argument("--max-new-tokens", type=int, default=256)
    p.add_argument("--steps", type=int, default=4, help="timed requests (each prefill + all its rounds)")
    p.add_argument("--warmup", type=int, default=4)
    p.add_argument("--micro-iters", type=int, default=30)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--profile-out", default=None, help="write a per-kernel table of 10 verify replays (rank 0)")
    return p.parse_args()


def device_time_ms(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def main() -> int:
    args = parse()
    llama = pkg("models.llama")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dtype = getattr(torch, args.dtype)
    cfg = llama.get_config(args.target)
    ctx = args.prompt_len + args.max_new_tokens + 8 * args.k * args.d + 64
    pages = 4 * math.ceil(ctx / args.page_size) + 256
    if world > 1:
        if args.fp8:
            raise SystemExit("--fp8 runs the single-GPU target (one process)")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        eng = pkg("parallel.launch").build_tp_target(cfg, mode=args.mode, seed=args.seed + 2, dtype=dtype,
                                                      num_pages=pages, page_size=args.page_size,
                                                      max_positions=ctx + 64, device=dev)
        if rank != 0:
            t0 = time.perf_counter()
            calls = eng.serve()
            torch.cuda.synchronize()
            eng.tp.check()
            stats = [calls, time.perf_counter() - t0, eng.worker_wait_s, eng.worker_handle_s]
            dist.all_gather_object([None] * world, stats)
            eng._graphs.clear()
            dist.barrier()
            eng.tp.close()
            dist.destroy_process_group()
            return 0
    elif args.fp8:
        fp8 = pkg("models.fp8")
        w = fp8.random_weights_fp8(cfg, seed=args.seed + 2, dtype=dtype, device=dev)
        eng = pkg("runtime.engine_fp8").Fp8LlamaEngine(w, num_pages=pages, page_size=args.page_size,
                                                        max_positions=ctx + 64)
    else:
        w = llama.random_weights(cfg, seed=args.seed + 2, dtype=dtype, device=dev)
        eng = pkg("runtime.engine").LlamaEngine(w, num_pages=pages, page_size=args.page_size, max_positions=ctx + 64)

    try:
        out = run_root(args, eng, dev, dtype, pages, ctx, world)
    finally:
        if world > 1:
            eng.stop_workers()
    if world > 1:
        torch.cuda.synchronize()
        eng.tp.check()
        stats: list = [None] * world
        dist.all_gather_object(stats, [eng.posted_calls, 0.0, 0.0, 0.0])
        out["worker_calls"] = [s[0] for s in stats[1:]]
        out["worker_handle_ms_per_call"] = [round(1e3 * s[3] / max(1, s[0]), 4) for s in stats[1:]]
        eng._graphs.clear()
        dist.barrier()
        eng.tp.close()
        dist.destroy_process_group()
    print(json.dumps(out), flush=True)
    return 0


def run_root(args, eng, dev, dtype, pages, ctx, world) -> dict:
    import random

    bench = importlib.import_module("bench")
    llama = pkg("models.llama")
    target = pkg("runtime.target")
    drafter = pkg("runtime.drafter")
    engine = pkg("runtime.engine")
    edge = pkg("serving.edge")
    counters = pkg("utils.counters")
    clocks = pkg("utils.clocks")
    tv = target.TargetVerifier(eng, k=args.k, d=args.d, score_weights=(0.45, 0.30, 0.17, 0.08),
                               fallback_threshold=-0.5, first_token_threshold=-0.7, fallback_ar_tokens=4,
                               model_name=f"random-init {args.target}")
    tv.warm_graphs()
    rng = random.Random(args.seed)
    prompts = [[rng.randrange(128256) for _ in range(args.prompt_len)] for _ in range(args.prompts)]
    # Microbenchmarks on the first prompt's committed prefix.
    tv.prefill(prompts[0])
    import numpy as np

    paths = [[rng.randrange(128256) for _ in range(args.d)] for _ in range(args.k)]
    tokens_, parents_, depths_, node_paths_, masks_ = tv.host.build_tree(torch.tensor(paths, dtype=torch.int64))
    n = int(tokens_.numel())
    p = len(tv.prefix_token_ids)
    scratch = tv.seq.reserve_scratch(p + n).numpy()
    tv._sync()
    row_bucket = pkg("runtime.engine").row_bucket

    def verify():
        eng.run_rows(row_bucket(n), tail_stride=1, mask_words=int(masks_.shape[1]), prefix_pages=tv.mirror.dev,
                     tokens=tokens_.numpy(), positions=depths_.numpy() + p, slots=scratch, shared_len=p,
                     n_shared_pages=len(tv.mirror.host), mask_base=p, row_full=np.full(n, p),
                     row_len=np.full(n, p + n), row_mask=masks_.numpy())

    verify_ms = device_time_ms(verify, args.micro_iters)
    if args.profile_out:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(10):
                verify()
            torch.cuda.synchronize()
        with open(args.profile_out, "w") as f:
            f.write(prof.key_averages().table(sort_by="cuda_time_total", row_limit=30, max_name_column_width=90))
    slots = tv.seq.reserve_scratch(p + 1).numpy()
    tv._sync()
    tok = torch.zeros(1, dtype=torch.int32, device=dev)

    def ar1():
        eng.run_rows(1, prefix_pages=tv.mirror.dev, tokens=tok, positions=[p], slots=slots[:1], shared_len=p,
                     n_shared_pages=len(tv.mirror.host), mask_base=p, row_full=[p + 1], row_len=[p + 1])

    ar1_ms = device_time_ms(ar1, args.micro_iters)

    dcfg = llama.get_config(args.drafter)
    dw = llama.random_weights(dcfg, seed=args.seed + 1, dtype=dtype, device=dev)
    dr = drafter.DrafterRuntime(engine.LlamaEngine(dw, num_pages=pages, page_size=args.page_size,
                                                   max_positions=ctx + 64))
    dr.warm_graphs(args.k, 4)
    client = bench.StreamTargetClient(tv, torch.cuda.Stream(device=dev))
    gen = edge.PagedDistributedAtlasGenerator(
        config=edge.DistributedAtlasConfig(k=args.k, d=args.d, max_new_tokens=args.max_new_tokens,
                                           fallback_ar_tokens=4, generation_seed=args.seed),
        drafter=dr, target_client=client)
    drv = bench.Driver(gen, prompts)
    for _ in range(args.warmup):
        drv.step()
    torch.cuda.synchronize()
    c0 = counters.snapshot()
    r0 = len(drv.rounds)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tokens = 0
    with clocks.ClockSampler(dev.index) as sampler:
        a.record()
        for _ in range(args.steps):
            tokens += drv.step()
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    delta = counters.delta(c0)
    eng.ops.check()
    gb = (eng.w.nbytes() if hasattr(eng.w, "nbytes") else 0) / 1e9
    return {
        "target": args.target, "drafter": args.drafter, "tp": world,
        "comm": None if world == 1 else args.mode, "weights": "fp8 block-scaled" if args.fp8 else args.dtype,
        "target_weight_gb_per_gpu": round(gb, 2),
        "verify_ms": round(verify_ms, 4), "verify_nodes": args.k * args.d, "ar1_ms": round(ar1_ms, 4),
        "tokens_per_s": round(tokens / (ms / 1000.0), 3), "requests": args.steps,
        "ms_per_round": round(ms / max(1, len(drv.rounds) - r0), 4), **drv.summary(r0),
        "gpu_launches_rank0": int(delta["launches"]), "clocks": sampler.summary(),
        "timing": "CUDA events on rank 0 (it drives every rank); micro: events per replay loop",
    }


if __name__ == "__main__":
    raise SystemExit(main())
