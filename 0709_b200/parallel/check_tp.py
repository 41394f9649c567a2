"""Tensor-parallel target check: ``torchrun --nproc-per-node N -m 0709_b200.parallel.check_tp``.

Every rank builds its shard of the same seeded model; the root also builds
the whole model on one device.  The root then drives both targets through
the same work -- prompt prefill, a masked tree verify, an asynchronous
tree/forest generation with a drafter -- and compares logits and committed
tokens; the other ranks serve the TP calls.  Prints one JSON line (root).

Modes: ``torch`` (CPU, gloo), ``nccl`` (GPU, NCCL collectives), ``fused``
(GPU, GEMM epilogues storing into peer memory + fused reduce/RMSNorm).
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import time

import torch
import torch.distributed as dist

from ..models.llama import get_config, random_weights
from ..runtime.drafter import DrafterRuntime
from ..runtime.engine import LlamaEngine
from ..runtime.target import TargetVerifier
from .launch import build_tp_target


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="tiny-target")
    p.add_argument("--drafter", default="tiny-drafter")
    p.add_argument("--mode", choices=["torch", "nccl", "fused"], default="torch")
    p.add_argument("--dtype", choices=["float32", "float16", "bfloat16"], default="float32")
    p.add_argument("--page-size", type=int, default=4)
    p.add_argument("--prompt-len", type=int, default=40)
    p.add_argument("--new-tokens", type=int, default=16)
    # (not --k/--d: torchrun's own parser would read "--d" as an abbreviation of its options)
    p.add_argument("--width", dest="k", type=int, default=2)
    p.add_argument("--depth", dest="d", type=int, default=3)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--fallback-threshold", type=float, default=None)
    p.add_argument("--timing-iters", type=int, default=0, help="Also time this many verify forwards (GPU).")
    p.add_argument("--json-out", default=None)
    return p.parse_args(argv)


def main(argv=None) -> int:
    args = parse_args(argv)
    backend = "gloo" if args.mode == "torch" else "nccl"
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if backend == "nccl":
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    else:
        device = torch.device("cpu")
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    dtype = getattr(torch, args.dtype)
    cfg = get_config(args.model)
    ctx = args.prompt_len + args.new_tokens + 8 * args.k * args.d + 64
    pages = 2 * math.ceil(ctx / args.page_size) + 64
    eng = build_tp_target(cfg, mode=args.mode, seed=args.seed + 1, dtype=dtype, num_pages=pages,
                          page_size=args.page_size, max_positions=ctx + 64, device=device)
    out: dict[str, object] = {}
    if eng.is_root:
        try:
            out = run_root(args, eng, cfg, device, dtype, pages, ctx)
        finally:
            eng.stop_workers()
    else:
        out = {"worker_calls": eng.serve()}
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        eng.tp.check()
    eng._graphs.clear()
    dist.barrier()
    eng.tp.close()
    dist.destroy_process_group()
    if eng.is_root:
        line = json.dumps(out, sort_keys=True)
        print(line, flush=True)
        if args.json_out:
            with open(args.json_out, "w") as f:
                f.write(line + "\n")
    return 0


def run_root(args, eng, cfg, device, dtype, pages, ctx) -> dict[str, object]:
    from ..serving.edge import DistributedAtlasConfig, PagedDistributedAtlasGenerator
    from ..serving.rpc import InProcessTargetClient

    world = eng.tp.world
    # The single-GPU reference runs the same unfused layer (separate RMSNorm and
    # RoPE kernels) as the TP engine, so the comparison isolates the parallelism.
    prev = os.environ.get("ATLAS_FUSED_NORM")
    os.environ["ATLAS_FUSED_NORM"] = "0"
    try:
        ref = LlamaEngine(random_weights(cfg, seed=args.seed + 1, dtype=dtype, device=device), num_pages=pages,
                          page_size=args.page_size, max_positions=ctx + 64)
    finally:
        if prev is None:
            os.environ.pop("ATLAS_FUSED_NORM", None)
        else:
            os.environ["ATLAS_FUSED_NORM"] = prev
    kw = dict(k=args.k, d=args.d, fallback_threshold=args.fallback_threshold)
    tv_tp, tv_ref = TargetVerifier(eng, **kw), TargetVerifier(ref, **kw)
    g = torch.Generator().manual_seed(args.seed)
    prompt = torch.randint(0, cfg.vocab_size, (args.prompt_len,), generator=g).tolist()
    a = tv_tp.prefill(prompt).next_token_logits.float().cpu()
    b = tv_ref.prefill(prompt).next_token_logits.float().cpu()
    res: dict[str, object] = {"tp": world, "mode": args.mode, "model": cfg.name, "dtype": args.dtype}
    res["prefill_logit_max_abs_diff"] = float((a - b).abs().max())
    res["prefill_argmax_equal"] = bool(int(a.argmax()) == int(b.argmax()))
    paths = [torch.randint(0, cfg.vocab_size, (args.d,), generator=g).tolist() for _ in range(args.k)]
    paths.append(paths[0][:1] + torch.randint(0, cfg.vocab_size, (args.d - 1,), generator=g).tolist())
    ta, tb = tv_tp.run_tree(paths), tv_ref.run_tree(paths)
    la, lb = ta["logits"].float().cpu(), tb["logits"].float().cpu()
    res["tree_nodes"] = int(ta["node_count"])
    res["tree_logit_max_abs_diff"] = float((la - lb).abs().max())
    res["tree_argmax_equal"] = bool(torch.equal(la.argmax(-1), lb.argmax(-1)))
    res["tree_path_logprob_max_abs_diff"] = max(
        abs(x - y) for ra, rb in zip(ta["path_logprobs"], tb["path_logprobs"]) for x, y in zip(ra, rb))
    if args.timing_iters and device.type == "cuda":
        tv_tp.warm_graphs()
        for _ in range(3):
            tv_tp.run_tree(paths)
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        for _ in range(args.timing_iters):
            tv_tp.run_tree(paths)
        torch.cuda.synchronize(device)
        res["tree_verify_ms"] = (time.perf_counter() - t0) * 1e3 / args.timing_iters

    # The drafter proposes target tokens and extends with the target's fallback tokens: one vocabulary.
    dcfg = get_config(args.drafter, vocab_size=cfg.vocab_size)
    dw = random_weights(dcfg, seed=args.seed, dtype=dtype, device=device)
    gens = []
    for tv in (TargetVerifier(eng, **kw), TargetVerifier(ref, **kw)):
        dr = DrafterRuntime(LlamaEngine(dw, num_pages=pages, page_size=args.page_size, max_positions=ctx + 64))
        conf = DistributedAtlasConfig(k=args.k, d=args.d, max_new_tokens=args.new_tokens, validate_state_alignment=True)
        if device.type == "cuda":
            # Capture every graph before the concurrent drafter/target threads start.
            tv.warm_graphs()
            dr.warm_graphs(args.k, conf.fallback_ar_tokens)
        gens.append(PagedDistributedAtlasGenerator(config=conf, drafter=dr, target_client=InProcessTargetClient(tv))
                    .generate(prompt))
    res["generated_tp"] = gens[0].generated_token_ids
    res["generated_ref"] = gens[1].generated_token_ids
    res["generation_equal"] = gens[0].generated_token_ids == gens[1].generated_token_ids
    res["decisions_tp"] = [r.decision for r in gens[0].rounds]
    res["posted_calls"] = eng.posted_calls
    return res


if __name__ == "__main__":
    raise SystemExit(main())
