#!/usr/bin/env python
"""Multi-session serving benchmark (several sessions per target, sessions over GPU pairs).

    torchrun --nproc-per-node N benchmarks/bench_sessions.py --sessions 8      (N even: GPU pairs)
    python benchmarks/bench_sessions.py --sessions 2                            (one GPU)

Independent sessions, each a Llama-3.2-1B-shaped drafter + Llama-3.1-8B-shaped
target (fp16, random init), k=4 d=5, page 16, uniform-random prompts with
lengths U[512, 8192], aggressive fallback thresholds (-0.30 path, -0.40 first
token) so rounds exercise target AR, KV compaction, pruning and page reuse.
With N GPUs, rank 2p hosts the drafters of its sessions (one thread each,
sharing one drafter engine and page pool) and rank 2p+1 serves their target
sessions (``MultiSessionTargetApp`` over the shared-memory transport); with
one GPU both sides share it.  Each session serves prompts back to back.

Reports aggregate committed tokens/s (wall time of the timed rounds, max
over drafter ranks), fallback rate, and p50 / p99 round latency (host time
of one round: verify || forest, handoff).
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import random
import sys
import threading
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
    p.add_argument("--sessions", type=int, default=8)
    p.add_argument("--drafter", default="llama-1b")
    p.add_argument("--target", default="llama-8b")
    p.add_argument("--width", dest="k", type=int, default=4)
    p.add_argument("--depth", dest="d", type=int, default=5)
    p.add_argument("--min-prompt", type=int, default=512)
    p.add_argument("--max-prompt", type=int, default=8192)
    p.add_argument("--max-new-tokens", type=int, default=256)
    p.add_argument("--fallback-threshold", type=float, default=-0.30)
    p.add_argument("--first-token-threshold", type=float, default=-0.40)
    p.add_argument("--rounds", type=int, default=16, help="timed rounds per session")
    p.add_argument("--warmup", type=int, default=3, help="untimed rounds per session")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--transport", choices=["shm", "peer"], default="shm",
                   help="drafter <-> target transport of a GPU pair: shared-memory mailbox or peer-memory rings")
    p.add_argument("--json-out", default=None)
    return p.parse_args()


def target_factory(args, engine, pool):
    target = pkg("runtime.target")

    def make(sid):
        tv = target.TargetVerifier(engine, k=args.k, d=args.d, page_pool=pool, fallback_threshold=args.fallback_threshold,
                                   first_token_threshold=args.first_token_threshold, fallback_ar_tokens=4,
                                   model_name=f"random-init {args.target}")
        tv.warm_graphs()
        return tv

    return make


def engines(args, dev, sessions_here, which):
    llama, engine_mod = pkg("models.llama"), pkg("runtime.engine")
    ctx = args.max_prompt + args.max_new_tokens + 8 * args.k * args.d + 64
    pages = sessions_here * (2 * math.ceil(ctx / 16) + 64) + 256
    name, seed = (args.drafter, 1) if which == "drafter" else (args.target, 2)
    w = llama.random_weights(llama.get_config(name), seed=args.seed + seed, dtype=torch.float16, device=dev)
    e = engine_mod.LlamaEngine(w, num_pages=pages, page_size=16, max_positions=ctx + 64)
    return e, pkg("ops._native").host().PagePool(e.num_pages - 1, 16)


def run_sessions(args, dev, sids, clients, rank) -> dict:
    drafter_mod, edge = pkg("runtime.drafter"), pkg("serving.edge")
    de, dpool = engines(args, dev, len(sids), "drafter")
    gens = []
    for sid, client in zip(sids, clients):
        dr = drafter_mod.DrafterRuntime(de, page_pool=dpool)
        dr.warm_graphs(args.k, 4)
        cfg = edge.DistributedAtlasConfig(k=args.k, d=args.d, max_new_tokens=args.max_new_tokens,
                                          fallback_ar_tokens=4, generation_seed=args.seed)
        gens.append(edge.PagedDistributedAtlasGenerator(config=cfg, drafter=dr, target_client=client))
    lat: list[float] = []
    stats = {"tokens": 0, "rounds": 0, "fallback": 0, "prompts": 0}
    lock = threading.Lock()
    start = threading.Barrier(len(sids) + 1)
    errors: list[BaseException] = []

    def worker(i):
        rng = random.Random(args.seed * 7919 + rank * 131 + i)
        try:
            sess = None
            start.wait()
            for r in range(args.warmup + args.rounds):
                if sess is None or sess.finished:
                    n = rng.randint(args.min_prompt, args.max_prompt)
                    sess = gens[i].start([rng.randrange(128256) for _ in range(n)])
                    with lock:
                        stats["prompts"] += 1
                t0 = time.perf_counter()
                tr = sess.step()
                dt = time.perf_counter() - t0
                if r >= args.warmup:
                    with lock:
                        lat.append(dt)
                        stats["tokens"] += len(tr.committed_tokens)
                        stats["rounds"] += 1
                        stats["fallback"] += int(tr.decision == "fallback_ar")
        except BaseException as exc:  # noqa: BLE001
            errors.append(exc)
            try:
                start.abort()
            except threading.BrokenBarrierError:
                pass

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(sids))]
    for t in threads:
        t.start()
    start.wait()
    t0 = time.perf_counter()
    for t in threads:
        t.join()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    if errors:
        raise errors[0]
    de.ops.check()
    return {**stats, "latencies": lat, "wall_s": wall}


def pct(xs, q):
    xs = sorted(xs)
    if not xs:
        return None
    return xs[min(len(xs) - 1, max(0, int(math.ceil(q / 100.0 * len(xs))) - 1))]


def main() -> int:
    args = parse()
    sessions_mod = pkg("serving.sessions")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        if world % 2:
            raise SystemExit("use an even number of GPUs (drafter, target) pairs, or one GPU")
        dist.init_process_group("gloo", timeout=timedelta(seconds=1800))
    pairs = max(1, world // 2)
    pair = rank // 2 if world > 1 else 0
    transport = pkg("serving.peer_transport")
    use_peer = args.transport == "peer" and world > 1
    # One process group per drafter/target pair (every rank creates all of them, in order).
    pair_group = [dist.new_group([2 * q, 2 * q + 1]) for q in range(pairs)][pair] if use_peer else None
    sids = [f"s{i}" for i in range(args.sessions) if i % pairs == pair]
    shm = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
    base = os.path.join(shm, f"atlas_sess_{os.environ.get('MASTER_PORT', os.getpid())}_{pair}")
    result = None
    if world == 1:
        te, tpool = engines(args, dev, len(sids), "target")
        app = sessions_mod.MultiSessionTargetApp(target_factory(args, te, tpool))
        for sid in sids:
            app._app(sid)  # capture every session's graphs before the threads start
        th = threading.Thread(target=lambda: sessions_mod.serve_target_shm(
            app, sessions_mod.ShmChannel(base, server=True)), daemon=True)
        th.start()
        ch = sessions_mod.ShmChannel(base, server=False)
        lock = threading.Lock()
        clients = [sessions_mod.ShmTargetClient(ch, session_id=s, lock=lock) for s in sids]
        result = run_sessions(args, dev, sids, clients, rank)
        clients[0].stop_server()
        results = [result]
    elif rank % 2 == 1:
        te, tpool = engines(args, dev, len(sids), "target")
        app = sessions_mod.MultiSessionTargetApp(target_factory(args, te, tpool))
        for sid in sids:
            app._app(sid)
        dist.barrier()
        if use_peer:
            ch = transport.PeerChannel(rank=rank, peer=rank - 1, device=dev, group=pair_group)
            transport.serve_target_channel(app, ch)
            ch.close()
        else:
            ch = sessions_mod.ShmChannel(base, server=True)
            sessions_mod.serve_target_shm(app, ch)
        torch.cuda.synchronize(dev)
        te.ops.check()
        results = [None] * world
        dist.all_gather_object(results, None)
    else:
        dist.barrier()
        lock = threading.Lock()
        if use_peer:
            ch = transport.PeerChannel(rank=rank, peer=rank + 1, device=dev, group=pair_group)
            clients = [transport.ChannelTargetClient(ch, session_id=s, lock=lock) for s in sids]
        else:
            ch = sessions_mod.ShmChannel(base, server=False)
            clients = [sessions_mod.ShmTargetClient(ch, session_id=s, lock=lock) for s in sids]
        result = run_sessions(args, dev, sids, clients, rank)
        clients[0].stop_server()
        if use_peer:
            ch.close()
        results = [None] * world
        dist.all_gather_object(results, result)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        rs = [r for r in results if r]
        lat = [x for r in rs for x in r["latencies"]]
        tokens = sum(r["tokens"] for r in rs)
        rounds = sum(r["rounds"] for r in rs)
        wall = max(r["wall_s"] for r in rs)
        line = {
            "benchmark": "multi-session serving (config 5)", "n_gpus": world, "sessions": args.sessions,
            "model": f"{args.drafter} drafter + {args.target} target (random init, fp16)", "k": args.k, "d": args.d,
            "tokens_per_s": round(tokens / wall, 3), "rounds": rounds, "tokens": tokens,
            "fallback_rate": round(sum(r["fallback"] for r in rs) / max(1, rounds), 3),
            "round_latency_ms": {"p50": round(1e3 * pct(lat, 50), 3), "p99": round(1e3 * pct(lat, 99), 3),
                                 "mean": round(1e3 * sum(lat) / len(lat), 3)},
            "prompts_started": sum(r["prompts"] for r in rs), "wall_s": round(wall, 3),
            "layout": "one GPU (both sides)" if world == 1 else f"{pairs} drafter/target GPU pairs",
            "transport": "shared-memory mailbox" if not use_peer else "peer-memory rings",
            "thresholds": {"fallback": args.fallback_threshold, "first_token": args.first_token_threshold},
        }
        print(json.dumps(line), flush=True)
        if args.json_out:
            with open(args.json_out, "w") as f:
                f.write(json.dumps(line) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
