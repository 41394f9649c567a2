#!/usr/bin/env python
"""Headline benchmark: asynchronous tree/forest speculative decoding throughput.

Workload (the reference's headline configuration): Llama-3.2-1B-shaped drafter + Llama-3.1-8B-shaped
target, fp16, random-init weights, k=3 d=4, page 16, path weights
0.45/0.30/0.17/0.08, fallback -0.50, first-token -0.70, 4 fallback AR tokens;
synthetic prompts of uniform-random token ids with lengths uniform in
[128, 2048], 256 new tokens each.

One step = one request served whole: both models prefill its prompt, then
speculative rounds (verify || forest, handoff) run until 256 tokens are
committed.  K steps therefore span K prompts, their prefills and every
prompt switch.

Parallelism (``--parallelism``, default ``tp``): with N GPUs the target is
sharded tensor-parallel over all N (``parallel/tp_engine.py``: fused
peer-memory GEMM->all-reduce->RMSNorm collectives, vocabulary-parallel LM head
gathered on rank 0) and the drafter runs on rank 0; the workload is the same
at every N (strong scaling), N=1 is the single-GPU engine.  ``dp`` runs one
independent session per GPU instead (weak scaling).

Timing: W untimed warm-up steps, then exactly K steps between timing marks.
A mark drains every rank's GPU and meets the other ranks (barrier) before its
CUDA event; each rank times the region with its own events and the reported
time is the max over ranks.  The weights (17 GB, or 17/N GB per GPU plus the
drafter) stream through every round, so the working set is far larger than the
126 MB L2 (no flush needed).

Extra measurements in the same line:
* ``select_path``: the same workload with both fallback thresholds disabled, so
  every round selects a drafted route (commit, compaction, stage-2 promotion
  and the forest overlap are timed; random-init weights make every round fall
  back under the config's thresholds);
* ``nccl`` (N >= 2, tp): the same requests with the collectives switched to
  NCCL ``all_reduce``/``all_gather`` (the baseline), and fused/NCCL;
* ``e2e``: whole prompts through ``PagedDistributedAtlasGenerator.generate``,
  host wall clock, with the prompt ids copied host->device from pinned memory
  and the tokens read back on the host.

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
from collections import Counter
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Reference: async GSM8K end to end, k=3 d=4, weights .45/.30/.17/.08, fallback
# -0.5/-0.7, AR4, Llama-3.2-1B + Llama-3.1-8B fp16 on 1xH800: 57.88 tok/s, with
# real weights (about 20 % of rounds fall back).
REFERENCE_PUBLISHED_TOK_S = 57.88
METRIC = "decode tokens/sec (device-timed, max over ranks) at 8B/70B; ms per spec round"


def _pkg(name: str):
    return importlib.import_module(f"0709_b200.{name}")


def parse(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8, help="timed requests")
    p.add_argument("--warmup", type=int, default=3, help="untimed requests before the timed ones")
    p.add_argument("--impl", choices=["atlas", "reference"], default="atlas")
    p.add_argument("--parallelism", choices=["tp", "dp"], default="tp",
                   help="tp: target sharded over all GPUs (strong scaling); dp: one session per GPU")
    p.add_argument("--placement", choices=["colocated", "split"], default="colocated",
                   help="split: drafter on rank 0's GPU, target on rank 1's GPU (2 ranks; config 2's placement)")
    p.add_argument("--handoff", choices=["peer", "nccl"], default="peer",
                   help="split placement: peer-memory message rings (kernels) or NCCL send/recv")
    p.add_argument("--comm", choices=["fused", "nccl", "torch"], default="fused",
                   help="TP collectives of the headline (torch: gloo collectives, CPU ranks)")
    p.add_argument("--device", choices=["cuda", "cpu"], default="cuda",
                   help="cpu runs the same control flow on CPU ranks (tiny fp32 models, gloo) for tests")
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
    p.add_argument("--e2e-prompts", type=int, default=8)
    p.add_argument("--select-steps", type=int, default=4,
                   help="timed requests with the fallback thresholds disabled (0: skip)")
    p.add_argument("--nccl-steps", type=int, default=4,
                   help="timed requests with NCCL collectives (tp, N >= 2; 0: skip)")
    p.add_argument("--forest-gate", choices=["overlap", "adaptive"], default="adaptive",
                   help="drafter forest schedule (see DistributedAtlasConfig.forest_gate)")
    p.add_argument("--target-stream-priority", type=int, default=-1,
                   help="CUDA priority of the target's stream (lower = higher; 0 = same as the drafter)")
    return p.parse_args(argv)


def reference_arm(args) -> None:
    """The reference's end-to-end path needs SGLang for its drafter; report why it cannot run."""
    reason = None
    try:
        importlib.import_module("sglang")
    except Exception as exc:  # noqa: BLE001
        reason = ("reference drafter requires sglang==0.5.14 (ModelRunner + paged FlashInfer decode), "
                  f"not installed offline: {type(exc).__name__}")
    if reason is None:
        reason = "reference arm not wired for this image"
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def make_prompts(args, rank: int, seed_offset: int = 0) -> list[list[int]]:
    rng = random.Random((args.seed + seed_offset) * 1000 + rank)
    vocab = _pkg("models.llama").get_config(args.target).vocab_size
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


def dtype_of(name: str):
    import torch

    return {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[name]


def sync(device) -> None:
    import torch

    if device.type == "cuda":
        torch.cuda.synchronize(device)


def context_sizes(args) -> tuple[int, int]:
    max_ctx = args.max_prompt + args.max_new_tokens + 4 * args.d + 64
    pages = (max_ctx // args.page_size + 8) * 4 + 256
    return max_ctx, pages


def build_target_engine(args, device, world: int, tp: bool):
    """The target engine: single-GPU, or this rank's tensor-parallel shard."""
    import torch

    llama = _pkg("models.llama")
    dtype = dtype_of(args.dtype)
    tcfg = llama.get_config(args.target)
    max_ctx, pages = context_sizes(args)
    if tp and world > 1:
        return _pkg("parallel.launch").build_tp_target(
            tcfg, mode=args.comm, seed=args.seed + 2, dtype=dtype, num_pages=pages, page_size=args.page_size,
            max_positions=max_ctx + 64, device=device)
    wt = llama.random_weights(tcfg, seed=args.seed + 2, dtype=dtype, device=device)
    return _pkg("runtime.engine").LlamaEngine(wt, num_pages=pages, page_size=args.page_size,
                                              max_positions=max_ctx + 64)


def build_session(args, device, te):
    """Drafter engine + target verifier + generator over the target engine ``te``."""
    import torch

    llama = _pkg("models.llama")
    engine = _pkg("runtime.engine")
    drafter_mod = _pkg("runtime.drafter")
    target_mod = _pkg("runtime.target")
    edge = _pkg("serving.edge")
    dtype = dtype_of(args.dtype)
    max_ctx, pages = context_sizes(args)
    wd = llama.random_weights(llama.get_config(args.drafter), seed=args.seed + 1, dtype=dtype, device=device)
    de = engine.LlamaEngine(wd, num_pages=pages, page_size=args.page_size, max_positions=max_ctx + 64)
    tv = make_verifier(args, te)
    # The target is on the critical path of every round (verify, then fallback AR);
    # the drafter's forest only fills the wait, so the target stream gets priority.
    if device.type == "cuda":
        client = StreamTargetClient(tv, torch.cuda.Stream(device=device, priority=args.target_stream_priority))
    else:
        client = _pkg("serving.rpc").InProcessTargetClient(tv)
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
    return gen, de, tv


class Driver:
    """Serves requests back to back; one step = one whole request (prefill + all its rounds)."""

    def __init__(self, gen, prompts) -> None:
        self.gen = gen
        self.prompts = prompts
        self.next = 0
        self.rounds: list[dict] = []   # per round: host ms, verify, forest, handoff, decision, mode, overlap

    def step(self) -> int:
        p = self.prompts[self.next % len(self.prompts)]
        self.next += 1
        session = self.gen.start(p)
        while not session.finished:
            t0 = time.perf_counter()
            tr = session.step()
            dt = time.perf_counter() - t0
            rt = session.rounds_tl[-1]
            self.rounds.append({
                "host_s": dt,
                "verify_s": rt.verify_blackbox.elapsed_s,
                "forest_s": sum(sp.elapsed_s for sp in rt.forest_steps),
                "handoff_s": (rt.handoff.elapsed_s if rt.handoff is not None else 0.0)
                + sum(sp.elapsed_s for sp in rt.post_prune_tree_steps),
                "overlap_s": rt.cloud_edge_overlap_s,
                "decision": tr.decision,
                "mode": tr.handoff_mode,
                "tokens": len(tr.committed_tokens),
            })
        return len(session.generated)

    def summary(self, since: int) -> dict:
        rs = self.rounds[since:]
        n = max(1, len(rs))

        def ms(key: str) -> float:
            return round(1e3 * sum(r[key] for r in rs) / n, 3)

        verify = sum(r["verify_s"] for r in rs)
        return {
            "rounds": len(rs),
            "fallback_rate": round(sum(r["decision"] == "fallback_ar" for r in rs) / n, 3),
            "tokens_per_round": round(sum(r["tokens"] for r in rs) / n, 3),
            "round_breakdown_ms": {"round_host": ms("host_s"), "target_verify_blackbox": ms("verify_s"),
                                   "drafter_forest": ms("forest_s"), "drafter_handoff": ms("handoff_s")},
            "handoff_modes": dict(Counter(r["mode"] for r in rs)),
            "cloud_hidden_ratio": round(sum(r["overlap_s"] for r in rs) / max(verify, 1e-12), 3),
        }


class LocalMarks:
    """``mark``/``elapsed_ms`` for engines without tensor parallelism (one or many independent ranks)."""

    def __init__(self, world: int, device) -> None:
        self.world = world
        self.device = device
        self.marks: dict = {}
        self.mark_launches: dict[str, int] = {}
        self.mark_hook = None

    def mark(self, tag: str, *, barrier: bool = False) -> None:
        import torch
        import torch.distributed as dist

        counters = _pkg("utils.counters")
        if barrier:
            sync(self.device)
            if self.world > 1:
                dist.barrier()
            sync(self.device)
        if self.device.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
        else:
            ev = _pkg("parallel.tp_engine").HostMark()
        self.marks[tag] = ev
        self.mark_launches[tag] = counters.snapshot()["launches"]
        if self.mark_hook is not None:
            self.mark_hook(tag)

    def elapsed_ms(self, start: str, end: str) -> float:
        sync(self.device)
        return float(self.marks[start].elapsed_time(self.marks[end]))


class RegionClocks:
    """Samples this rank's GPU clocks between ``<region>_start`` and ``<region>_end`` marks."""

    def __init__(self, gpu_index: int | None) -> None:
        self.gpu_index = gpu_index
        self.open = None
        self.summaries: dict[str, dict] = {}

    def __call__(self, tag: str) -> None:
        clocks = _pkg("utils.clocks")
        if self.gpu_index is None:
            return
        if tag.endswith("_start"):
            self.open = clocks.ClockSampler(self.gpu_index).__enter__()
        elif tag.endswith("_end") and self.open is not None:
            self.open.__exit__(None, None, None)
            self.summaries[tag[: -len("_end")]] = self.open.summary()
            self.open = None


def rank_report(marker, clocks: RegionClocks, regions) -> dict:
    out = {}
    for r in regions:
        if f"{r}_start" in marker.marks and f"{r}_end" in marker.marks:
            out[r] = {"ms": marker.elapsed_ms(f"{r}_start", f"{r}_end"),
                      "launches": marker.mark_launches[f"{r}_end"] - marker.mark_launches[f"{r}_start"],
                      "clocks": clocks.summaries.get(r)}
    return out


REGIONS = ("main", "select", "nccl")


def physical_gpu(local: int) -> int:
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = phys.split(",") if phys else []
    return int(parts[local]) if local < len(parts) and parts[local].strip().isdigit() else local


def main() -> int:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return 0
    import torch
    import torch.distributed as dist

    counters = _pkg("utils.counters")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.device == "cuda":
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    else:
        device = torch.device("cpu")
        if args.comm != "torch":
            raise SystemExit("--device cpu needs --comm torch")
    if world > 1:
        if device.type == "cuda":
            dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=180))
    if args.placement == "split":
        return split_main(args, device, world, rank, local, counters)
    tp = args.parallelism == "tp" and world > 1
    te = build_target_engine(args, device, world, tp)
    marker = te if tp else LocalMarks(world, device)
    clocks = RegionClocks(physical_gpu(local) if device.type == "cuda" else None)
    marker.mark_hook = clocks

    if tp and rank != 0:
        # Tensor-parallel worker: repeat the root's engine calls until it stops us.
        te.serve()
        sync(device)
        te.tp.check()
        te.ops.check()
        reports: list = [None] * world
        dist.all_gather_object(reports, rank_report(marker, clocks, REGIONS))
        te._graphs.clear()
        dist.barrier()
        te.tp.close()
        dist.destroy_process_group()
        return 0

    gen, de, tv = build_session(args, device, te)

    def check_errors() -> None:
        de.ops.check()
        te.ops.check()
        if tp:
            te.tp.check()

    def set_thresholds(fallback, first) -> None:
        tv.fallback_threshold, tv.first_token_threshold = fallback, first

    def to_nccl() -> None:
        te.set_comm_mode("nccl")
        tv.warm_graphs()

    try:
        line = run_root(args, device, gen, marker, counters, rank, check_errors=check_errors,
                        set_thresholds=set_thresholds,
                        to_nccl=to_nccl if tp and args.comm == "fused" else None)
    finally:
        if tp:
            te.stop_workers()
    sync(device)
    reports = [None] * world
    if world > 1:
        dist.all_gather_object(reports, rank_report(marker, clocks, REGIONS))
    else:
        reports = [rank_report(marker, clocks, REGIONS)]
    finish_line(line, reports, args, world, tp)
    tokens = float(line.pop("_tokens_rank"))
    if world > 1 and not tp:
        # Independent sessions: every rank ran its own requests.
        totals = torch.tensor([tokens], dtype=torch.float64, device=device)
        dist.all_reduce(totals, op=dist.ReduceOp.SUM)
        tokens = float(totals.item())
    line["_tokens_all"] = tokens
    if world > 1:
        if tp:
            te.tp.check()
            te._graphs.clear()
        dist.barrier()
        if tp:
            te.tp.close()
        dist.destroy_process_group()
    if rank == 0:
        emit(line, args, world)
    return 0


def make_verifier(args, te):
    weights = [float(x) for x in args.path_score_weights.split(",")] if args.path_score_weights else None
    return _pkg("runtime.target").TargetVerifier(
        te, k=args.k, d=args.d, score_weights=weights, fallback_threshold=args.fallback_threshold,
        first_token_threshold=args.first_token_threshold, fallback_ar_tokens=args.fallback_ar_tokens,
        model_name=f"random-init {args.target}")


def split_main(args, device, world, rank, local, counters) -> int:
    """Config 2's placement: the drafter and coordinator on rank 0, the target server on rank 1.

    Requests and responses travel through ``serving.peer_transport`` (peer-memory
    rings, or NCCL send/recv as the baseline).  The timing marks travel the same
    way: the target records its events when the mark request arrives.
    """
    import torch.distributed as dist

    if world != 2:
        raise SystemExit("--placement split runs on exactly 2 ranks")
    transport = _pkg("serving.peer_transport")
    kind = args.handoff if device.type == "cuda" else "nccl"  # gloo point-to-point on CPU ranks
    channel = transport.make_channel(kind, rank=rank, peer=1 - rank, device=device)
    marker = LocalMarks(1, device)
    clocks = RegionClocks(physical_gpu(local) if device.type == "cuda" else None)
    marker.mark_hook = clocks
    if rank == 1:
        te = build_target_engine(args, device, 1, False)
        tv = make_verifier(args, te)
        tv.warm_graphs()

        def mark(req):
            sync(device)
            marker.mark(str(req["tag"]))
            return {"ok": True}

        def set_thresholds(req):
            tv.fallback_threshold, tv.first_token_threshold = req["fallback"], req["first"]
            return {"ok": True}

        def report(_req):
            sync(device)
            te.ops.check()
            return {"ok": True, "report": rank_report(marker, clocks, REGIONS), "channel": dict(channel.stats)}

        transport.serve_target_channel(_pkg("serving.rpc").TargetServerApp(tv), channel,
                                       extra={"mark": mark, "set_thresholds": set_thresholds, "report": report})
        channel.close()
        dist.destroy_process_group()
        return 0

    llama = _pkg("models.llama")
    max_ctx, pages = context_sizes(args)
    wd = llama.random_weights(llama.get_config(args.drafter), seed=args.seed + 1, dtype=dtype_of(args.dtype),
                              device=device)
    de = _pkg("runtime.engine").LlamaEngine(wd, num_pages=pages, page_size=args.page_size,
                                            max_positions=max_ctx + 64)
    dr = _pkg("runtime.drafter").DrafterRuntime(de)
    dr.warm_graphs(args.k, args.fallback_ar_tokens)
    client = transport.ChannelTargetClient(channel)
    edge = _pkg("serving.edge")
    gen = edge.PagedDistributedAtlasGenerator(
        config=edge.DistributedAtlasConfig(k=args.k, d=args.d, max_new_tokens=args.max_new_tokens,
                                           fallback_ar_tokens=args.fallback_ar_tokens, generation_seed=args.seed,
                                           forest_gate=args.forest_gate),
        drafter=dr, target_client=client)

    class SplitMarks:
        """Marks on both GPUs: the target records its event when the mark request arrives."""

        def mark(self, tag: str, *, barrier: bool = False) -> None:
            sync(device)
            client.call("mark", {"tag": tag})
            marker.mark(tag)

    try:
        line = run_root(args, device, gen, SplitMarks(), counters, rank, check_errors=de.ops.check,
                        set_thresholds=lambda fb, first: client.call("set_thresholds",
                                                                     {"fallback": fb, "first": first}))
        remote = client.call("report")
    finally:
        client.stop_server()
    sync(device)
    reports = [rank_report(marker, clocks, REGIONS), remote["report"]]
    line["handoff_channel"] = {"kind": kind, "client": dict(channel.stats), "server": remote["channel"],
                               "client_wait_ms_per_call": round(1e3 * client.wait_s / max(1, client.calls), 3)}
    channel.close()
    dist.destroy_process_group()
    finish_line(line, reports, args, world, False)
    line["_tokens_all"] = float(line.pop("_tokens_rank"))
    emit(line, args, world)
    return 0


def run_root(args, device, gen, marker, counters, rank, *, check_errors, set_thresholds, to_nccl=None) -> dict:
    """The measured passes on the rank that drives the generator.

    ``check_errors()`` raises on a device error flag, ``set_thresholds(fallback,
    first_token)`` sets the target's thresholds, ``to_nccl()`` (tensor-parallel
    runs) switches the target's collectives to NCCL.
    """
    drv = Driver(gen, make_prompts(args, rank))
    line: dict = {}

    # ---- headline: config thresholds, K requests
    for _ in range(args.warmup):
        drv.step()
    r0 = len(drv.rounds)
    tokens = 0
    marker.mark("main_start", barrier=True)
    for _ in range(args.steps):
        tokens += drv.step()
    marker.mark("main_end")
    sync(device)
    check_errors()
    line["_tokens_rank"] = tokens
    line["main"] = drv.summary(r0)

    # ---- end to end through the public API: whole prompts via generate()
    e2e_prompts = make_prompts(args, rank, seed_offset=7)[: args.e2e_prompts]
    sync(device)
    ce = counters.snapshot()
    t0 = time.perf_counter()
    e2e_tokens = e2e_rounds = 0
    for p in e2e_prompts:
        res = gen.generate(p)
        e2e_tokens += len(res.generated_token_ids)
        e2e_rounds += len(res.rounds)
    sync(device)
    e2e_s = time.perf_counter() - t0
    ed = counters.delta(ce)
    check_errors()
    n_e2e = max(1, len(e2e_prompts))
    line["e2e"] = {
        "value": round(e2e_tokens / e2e_s, 3) if e2e_s > 0 else None,
        "unit": "tokens/s",
        "h2d_bytes_per_step": int(ed["h2d_bytes"] / n_e2e),
        "d2h_bytes_per_step": int(ed["d2h_bytes"] / n_e2e),
        "step": ("one request: prompt ids staged in pinned host memory and copied to both models' devices, "
                 "prefill, all rounds, generated ids returned on the host"),
        "prompts": len(e2e_prompts),
        "rounds": e2e_rounds,
        "tokens": e2e_tokens,
        "timing": "host wall clock around generate() of every prompt, rank 0",
    }

    # ---- select path: thresholds off, every round commits a drafted route
    if args.select_steps > 0:
        set_thresholds(None, None)
        gen.fallback_ema = 0.0
        drv.step()
        r1 = len(drv.rounds)
        sel_tokens = 0
        marker.mark("select_start", barrier=True)
        for _ in range(args.select_steps):
            sel_tokens += drv.step()
        marker.mark("select_end")
        sync(device)
        check_errors()
        line["select"] = {**drv.summary(r1), "tokens": sel_tokens, "requests": args.select_steps}
        set_thresholds(args.fallback_threshold, args.first_token_threshold)

    # ---- NCCL baseline: the same requests with library collectives
    if to_nccl is not None and args.nccl_steps > 0:
        to_nccl()
        gen.fallback_ema = 0.0
        drv.step()
        r2 = len(drv.rounds)
        nccl_tokens = 0
        marker.mark("nccl_start", barrier=True)
        for _ in range(args.nccl_steps):
            nccl_tokens += drv.step()
        marker.mark("nccl_end")
        sync(device)
        check_errors()
        line["nccl"] = {**drv.summary(r2), "tokens": nccl_tokens, "requests": args.nccl_steps}
    return line


def finish_line(line: dict, reports: list, args, world: int, tp: bool) -> None:
    """Fold every rank's region times (max), launches (sum) and clocks into ``line``."""
    for region in REGIONS:
        per = [r[region] for r in reports if r and region in r]
        if not per:
            continue
        line.setdefault(region, {})
        line[region]["ms_max_over_ranks"] = max(p["ms"] for p in per)
        line[region]["launches_all_ranks"] = sum(int(p["launches"]) for p in per)
        line[region]["clocks_per_rank"] = [p["clocks"] for p in per]


def _clock_summary(per_rank: list) -> dict:
    per_rank = [c for c in per_rank if c]
    reasons = sorted({r for c in per_rank for r in c.get("reasons", [])})
    sm = [c.get("sm_mhz") for c in per_rank if c.get("sm_mhz") is not None]
    mx = [c.get("sm_max_mhz") for c in per_rank if c.get("sm_max_mhz") is not None]
    return {"sm_mhz": min(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
            "ranks_sampled": len(per_rank)}


def emit(line: dict, args, world: int) -> None:
    main = line["main"]
    ms = main["ms_max_over_ranks"]
    tokens = line["_tokens_all"]
    value = tokens / (ms / 1000.0)
    tp = args.parallelism == "tp" and world > 1 and args.placement == "colocated"
    if args.placement == "split":
        parallelism = (f"split placement: drafter on GPU0, target on GPU1 ({line['handoff_channel']['kind']} "
                       "handoff through ring messages)" if line['handoff_channel']['kind'] == "peer" else
                       "split placement: drafter on GPU0, target on GPU1 (NCCL send/recv handoff)")
    elif tp:
        parallelism = f"tp{world} (target sharded over {world} GPUs, {args.comm} collectives; drafter on rank 0)"
    elif args.parallelism == "tp":
        parallelism = "tp1 (single GPU)"
    else:
        parallelism = f"dp{world} (one drafter+target session per GPU)"
    out = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong" if args.parallelism == "tp" else "weak",
        "vs_baseline": round(value / REFERENCE_PUBLISHED_TOK_S, 3) if args.parallelism == "tp" else None,
        "dtype": args.dtype.replace("float16", "fp16").replace("bfloat16", "bf16"),
        "data": "synthetic uniform-random token ids, random-init weights",
        "config": {
            "model": f"{args.drafter} drafter + {args.target} target (random init)",
            "global_batch": 1 if args.parallelism == "tp" else world,
            "seq_len": f"prompt U[{args.min_prompt},{args.max_prompt}] + {args.max_new_tokens} new",
            "parallelism": parallelism,
            "k": args.k,
            "d": args.d,
            "page_size": args.page_size,
            "path_score_weights": args.path_score_weights,
            "fallback_threshold": args.fallback_threshold,
            "first_token_threshold": args.first_token_threshold,
            "fallback_ar_tokens": args.fallback_ar_tokens,
            "forest_gate": args.forest_gate,
            "step": "one request: prefill of both models + speculative rounds until max_new_tokens are committed",
            "l2": "no flush: weights (17 GB) stream through every round; working set far above L2",
            "ms_per_round": round(ms / max(1, main["rounds"]), 4),
            "rounds_timed": main["rounds"],
            "fallback_rate_timed": main["fallback_rate"],
            "tokens_per_round": main["tokens_per_round"],
            "round_breakdown_ms": main["round_breakdown_ms"],
            "handoff_modes": main["handoff_modes"],
            "tokens_timed": int(tokens),
            "vs_baseline_basis": ("value / 57.88 tok/s, the reference's async GSM8K run on 1xH800 with real weights "
                                  "(~20 % fallback); here random-init weights make every round under the config's "
                                  "thresholds fall back, so the ratio compares the fallback-path throughput"),
        },
        "clocks": _clock_summary(main["clocks_per_rank"]),
        "e2e": line["e2e"],
        "gpu_launches": int(main["launches_all_ranks"]),
        **({"handoff_channel": line["handoff_channel"]} if "handoff_channel" in line else {}),
        "timing": "CUDA events per rank between barrier-aligned marks; max over ranks",
    }
    sel = line.get("select")
    if sel and "ms_max_over_ranks" in sel:
        sms = sel["ms_max_over_ranks"]
        out["select_path"] = {
            "value": round(sel["tokens"] / (sms / 1000.0), 3),
            "unit": "tokens/s",
            "thresholds": "fallback and first-token thresholds disabled (every round selects a route)",
            "requests": sel["requests"],
            "ms_per_round": round(sms / max(1, sel["rounds"]), 4),
            "rounds": sel["rounds"],
            "fallback_rate": sel["fallback_rate"],
            "tokens_per_round": sel["tokens_per_round"],
            "round_breakdown_ms": sel["round_breakdown_ms"],
            "handoff_modes": sel["handoff_modes"],
            "cloud_hidden_ratio": sel["cloud_hidden_ratio"],
            "clocks": _clock_summary(sel["clocks_per_rank"]),
        }
    nc = line.get("nccl")
    if nc and "ms_max_over_ranks" in nc:
        nms = nc["ms_max_over_ranks"]
        n_round = nms / max(1, nc["rounds"])
        f_round = ms / max(1, main["rounds"])
        out["nccl"] = {
            "value": round(nc["tokens"] / (nms / 1000.0), 3),
            "unit": "tokens/s",
            "requests": nc["requests"],
            "ms_per_round": round(n_round, 4),
            "rounds": nc["rounds"],
            "fallback_rate": nc["fallback_rate"],
            "fused_over_nccl_speedup_per_round": round(n_round / f_round, 3),
            "clocks": _clock_summary(nc["clocks_per_rank"]),
        }
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    raise SystemExit(main())
