#!/usr/bin/env python
"""Isolated component benchmark: tree / forest vs matched batch AR, target AR1 and tree verify.

    python benchmarks/bench_isolated_components.py --prefix 8192 --pairs 6

Drafter side (decode-ready, d depths each):
* ``tree``: k stage-1 routes, global top-k per depth;
* ``batch_ar_k``: the same k first tokens extended by per-route top-1 (the
  matched batch-AR baseline: same rows, same depths, no cross-route selection);
* ``forest`` (k^2 routes, per-root top-k) and ``batch_ar_k2``.
Tree and batch AR are measured as interleaved ABBA pairs so clock or
thermal drift cancels.  Target side: one-token AR forward and the masked
tree verify of k synthetic routes of depth d sharing their first two tokens
(scoring, selection and KV commit included).  Every number is CUDA-event
device time of the whole operation, which includes the per-depth host
synchronisation the frontier needs; host wall time is reported beside it.

Parity: reference benchmarks/bench_atlas_0709_isolated_components.py:1042-1233
(paired ABBA protocol, synthetic verify paths with shared leading tokens); like it, an
odd iteration count is rejected and the per-block ratios are summarized by their geometric
mean (:1034, :1132-1153).
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

# Reference (1x H800, P=8192, k=3 d=4, eager): HANDOFF numbers quoted in the survey.
REFERENCE_H800_MS = {"batch_ar_k": 25.096, "tree": 28.978, "batch_ar_k2": 26.806, "forest": 31.686,
                     "target_verify": 24.224, "target_ar1": 18.402, "target_ar2": 34.734,
                     "target_linear_verify": 28.484}


def pkg(name):
    return importlib.import_module(f"0709_b200.{name}")


class PerRouteTop1Selection:
    """Matched batch AR: every route keeps only its own best child."""

    def __init__(self) -> None:
        self.phase = pkg("types").DecodePhase.STAGE1

    def select_indices(self, candidates, *, k, active_routes):
        n = len(active_routes)
        return torch.arange(n, device=candidates.pending_token_ids.device) * candidates.candidates_per_parent

    def select(self, candidates, *, k, active_routes):
        return [c for c in candidates if c.rank_in_parent == 0]


def abba_order(i: int) -> tuple[str, str]:
    """Arm order of iteration ``i``: A B, then B A, so each block of two iterations is A B B A."""
    return ("a", "b") if i % 2 == 0 else ("b", "a")


def check_pairs(n: int) -> int:
    """Iteration counts must fill whole ABBA blocks (an odd count leaves one arm's drift unmatched)."""
    if int(n) < 2 or int(n) % 2:
        raise ValueError(f"--pairs must be a positive even number (whole A B B A blocks), got {n}")
    return int(n)


def block_ratios(a_ms, b_ms) -> dict[str, float]:
    """B/A per ABBA block (sums over the block's two iterations of each arm) and their
    geometric mean, minimum and maximum."""
    if len(a_ms) != len(b_ms) or len(a_ms) % 2:
        raise ValueError("block_ratios needs two equally long lists of whole ABBA blocks")
    ratios = [(b_ms[j] + b_ms[j + 1]) / (a_ms[j] + a_ms[j + 1]) for j in range(0, len(a_ms), 2)]
    return {"geometric_mean": round(math.exp(statistics.fmean(math.log(r) for r in ratios)), 4),
            "min": round(min(ratios), 4), "max": round(max(ratios), 4), "blocks": len(ratios)}


def timed(fn):
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b), (time.perf_counter() - t0) * 1e3


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--drafter", default="llama-1b")
    ap.add_argument("--target", default="llama-8b")
    ap.add_argument("--prefix", type=int, default=8192)
    ap.add_argument("--width", dest="k", type=int, default=3)
    ap.add_argument("--depth", dest="d", type=int, default=4)
    ap.add_argument("--pairs", type=int, default=6, help="timed iterations per arm (even: whole ABBA blocks)")
    ap.add_argument("--dtype", default="float16")
    ap.add_argument("--skip-target", action="store_true")
    ap.add_argument("--json-out", default=None)
    args = ap.parse_args()
    check_pairs(args.pairs)
    llama, engine_mod = pkg("models.llama"), pkg("runtime.engine")
    drafter_mod, store_mod, builders = pkg("runtime.drafter"), pkg("runtime.store"), pkg("runtime.builders")
    frontier = pkg("runtime.frontier")
    dt = getattr(torch, args.dtype)
    dev = torch.device("cuda")
    k, d, P = args.k, args.d, args.prefix
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 128256, (P,), generator=g).tolist()
    pages = 2 * (P // 16) + 512
    out: dict[str, object] = {"prefix": P, "k": k, "d": d, "pairs": args.pairs, "dtype": args.dtype,
                              "reference_h800_ms": REFERENCE_H800_MS}

    dw = llama.random_weights(llama.get_config(args.drafter), seed=1, dtype=dt, device=dev)
    dr = drafter_mod.DrafterRuntime(engine_mod.LlamaEngine(dw, num_pages=pages, page_size=16,
                                                           max_positions=P + 256))
    dr.warm_graphs(k, 4)
    store = store_mod.KVTreeStore()
    dr.bind_store(store)
    dr.prefill(prompt)

    def tree():
        routes = builders.initialize_stage1_routes(dr.prefix_state(), k=k, route_store=store)
        res = builders.build_tree_depths(routes, depth=d, k=k, route_store=store, model_backend=dr)
        return routes, res

    def batch_ar(width):
        routes = builders.initialize_stage1_routes(dr.prefix_state(), k=width, route_store=store)
        for _ in range(d):
            routes = frontier.advance_frontier_one_token(routes, k=1, route_store=store, model_backend=dr,
                                                         selection_policy=PerRouteTop1Selection()).next_routes

    def forest_after_tree():
        # The stage-1 tree is built untimed; the timed part is forest init + d forest depths.
        _, res = tree()
        return lambda: builders.build_forest_depths(
            builders.initialize_forest_routes(res.completed_routes, res.last_logits, k=k, route_store=store),
            depth=d, k=k, route_store=store, model_backend=dr)

    def run(name, fn):
        if name == "forest":
            fn = fn()
        dev_ms, host_ms = timed(fn)
        dr.drop_speculative()
        return dev_ms, host_ms

    for name, fn in (("tree", tree), ("batch_ar_k", lambda: batch_ar(k)), ("forest", forest_after_tree),
                     ("batch_ar_k2", lambda: batch_ar(k * k))):  # warm-up
        run(name, fn)
    results: dict[str, list[tuple[float, float]]] = {n: [] for n in ("tree", "batch_ar_k", "forest", "batch_ar_k2")}
    # Arm A is the matched batch AR, arm B the tree (forest); the order alternates A B / B A.
    arms = {"a": ("batch_ar_k", lambda: batch_ar(k)), "b": ("tree", tree)}
    arms2 = {"a": ("batch_ar_k2", lambda: batch_ar(k * k)), "b": ("forest", forest_after_tree)}
    orders = []
    for i in range(args.pairs):
        order = abba_order(i)
        orders.append("".join(order).upper())
        for name, fn in [arms[x] for x in order] + [arms2[x] for x in order]:
            results[name].append(run(name, fn))
    out["orders"] = orders
    out["tree_over_batch_ar_blocks"] = block_ratios([v[0] for v in results["batch_ar_k"]],
                                                    [v[0] for v in results["tree"]])
    out["forest_over_batch_ar_blocks"] = block_ratios([v[0] for v in results["batch_ar_k2"]],
                                                      [v[0] for v in results["forest"]])
    for name, vals in results.items():
        out[f"{name}_ms"] = round(statistics.mean(v[0] for v in vals), 3)
        out[f"{name}_host_ms"] = round(statistics.mean(v[1] for v in vals), 3)
    out["tree_over_batch_ar"] = round(out["tree_ms"] / out["batch_ar_k_ms"], 4)
    out["forest_over_batch_ar"] = round(out["forest_ms"] / out["batch_ar_k2_ms"], 4)
    dr.engine.ops.check()
    del dr, dw
    torch.cuda.empty_cache()

    if not args.skip_target:
        target_mod = pkg("runtime.target")
        types = pkg("types")
        tw = llama.random_weights(llama.get_config(args.target), seed=2, dtype=dt, device=dev)
        te = engine_mod.LlamaEngine(tw, num_pages=pages, page_size=16, max_positions=P + 1024)
        tv = target_mod.TargetVerifier(te, k=k, d=d)
        tv.warm_graphs()
        tv.prefill(prompt)

        def synthetic_routes():
            shared = torch.randint(0, 128256, (2,), generator=g).tolist()
            return [types.VerifyRoutePayload(route_id=r, token_ids=tuple(
                shared + torch.randint(0, 128256, (d - 2,), generator=g).tolist()), draft_logprob=-1.0,
                draft_token_logprobs=tuple([-0.25] * d)) for r in range(k)]

        ver, ar = [], []
        for i in range(args.pairs + 2):
            routes = synthetic_routes()
            ver.append(timed(lambda: tv.verify_payloads(prefix_token_ids=tv.prefix_token_ids, routes=routes)))
            p = len(tv.prefix_token_ids)
            slots = tv.seq.reserve_scratch(p + 1).numpy()
            tv._sync()
            tok = torch.zeros(1, dtype=torch.int32, device=dev)
            ar.append(timed(lambda: te.run_rows(1, prefix_pages=tv.mirror.dev, tokens=tok, positions=[p],
                                                slots=slots[:1], shared_len=p, n_shared_pages=len(tv.mirror.host),
                                                mask_base=p, row_full=[p + 1], row_len=[p + 1])))
        ver, ar = ver[2:], ar[2:]
        # Two dependent one-token forwards (the second token fed on the device) and the
        # linear (non-deduplicated) verify of the same kind of routes, without commit.
        ar2, lin, tree_fwd = [], [], []
        for i in range(args.pairs + 2):
            p = len(tv.prefix_token_ids)
            slots = tv.seq.reserve_scratch(p + 2).numpy()
            tv._sync()
            tok = torch.zeros(2, dtype=torch.int32, device=dev)

            def two():
                for j in range(2):
                    te.run_rows(1, prefix_pages=tv.mirror.dev, tokens=tok[j:j + 1], positions=[p + j],
                                slots=slots[j:j + 1], shared_len=p + j, n_shared_pages=len(tv.mirror.host),
                                mask_base=p + j, row_full=[p + j + 1], row_len=[p + j + 1])

            ar2.append(timed(two))
            paths = [list(r.token_ids) for r in synthetic_routes()]
            lin.append(timed(lambda: tv.run_tree(paths, deduplicate=False)))
            tree_fwd.append(timed(lambda: tv.run_tree(paths)))
        out["target_ar2_ms"] = round(statistics.mean(v[0] for v in ar2[2:]), 3)
        out["target_linear_verify_ms"] = round(statistics.mean(v[0] for v in lin[2:]), 3)
        out["target_tree_forward_ms"] = round(statistics.mean(v[0] for v in tree_fwd[2:]), 3)
        out["target_verify_ms"] = round(statistics.mean(v[0] for v in ver), 3)
        out["target_verify_host_ms"] = round(statistics.mean(v[1] for v in ver), 3)
        out["target_ar1_ms"] = round(statistics.mean(v[0] for v in ar), 3)
        te.ops.check()
    out["speedup_vs_reference_h800"] = {
        name: round(REFERENCE_H800_MS[name] / out[f"{name}_ms"], 2)
        for name in REFERENCE_H800_MS if f"{name}_ms" in out}
    line = json.dumps(out)
    print(line, flush=True)
    if args.json_out:
        with open(args.json_out, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
