#!/usr/bin/env python
"""Isolated component benchmark: tree / forest vs matched batch AR, target AR1 and tree verify.

    python benchmarks/bench_isolated_components.py --prefix 8192 --pairs 6
    python benchmarks/bench_isolated_components.py --drafter-model llama-1b --target-model llama-8b \
        --prefix-len 8192 --k 3 --d 4 --iters 6 --warmup 1 --pair-order-seed 0   # the reference's flags

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


class DrafterArms:
    """The drafter workloads on one prefilled drafter (``dr`` bound to ``store``): the stage-1
    tree, the matched batch AR of any width, and the forest grown after an untimed tree."""

    def __init__(self, dr, store, k: int, d: int) -> None:
        self.dr, self.store, self.k, self.d = dr, store, int(k), int(d)
        self.builders, self.frontier = pkg("runtime.builders"), pkg("runtime.frontier")

    def tree(self):
        b = self.builders
        routes = b.initialize_stage1_routes(self.dr.prefix_state(), k=self.k, route_store=self.store)
        return routes, b.build_tree_depths(routes, depth=self.d, k=self.k, route_store=self.store,
                                           model_backend=self.dr)

    def batch_ar(self, width: int) -> None:
        routes = self.builders.initialize_stage1_routes(self.dr.prefix_state(), k=width, route_store=self.store)
        for _ in range(self.d):
            routes = self.frontier.advance_frontier_one_token(
                routes, k=1, route_store=self.store, model_backend=self.dr,
                selection_policy=PerRouteTop1Selection()).next_routes

    def forest_after_tree(self):
        """Build the tree (untimed) and return the timed part: forest init + d forest depths."""
        b = self.builders
        _, res = self.tree()
        return lambda: b.build_forest_depths(
            b.initialize_forest_routes(res.completed_routes, res.last_logits, k=self.k, route_store=self.store),
            depth=self.d, k=self.k, route_store=self.store, model_backend=self.dr)


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


def timed(fn, cuda: bool = True):
    """(device ms, host ms) of ``fn``: CUDA events on the current stream with a synchronize on
    both sides (wall time twice on CPU)."""
    if not cuda:
        t0 = time.perf_counter()
        fn()
        ms = (time.perf_counter() - t0) * 1e3
        return ms, ms
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b), (time.perf_counter() - t0) * 1e3


# Settings of the reference's SGLang runtime with no counterpart here (accepted, ignored).
_INERT = (("--mem-fraction-static", float), ("--max-running-requests", int), ("--max-total-tokens", int),
          ("--nccl-port", int), ("--prefill-chunk-size", int), ("--workspace-mb", int))


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="Tree / forest vs matched batch AR (paired ABBA), target AR1, AR2, "
                                             "linear and masked verify.  The reference's flag names are accepted.")
    ap.add_argument("--drafter", "--drafter-model", dest="drafter", default="llama-1b")
    ap.add_argument("--target", "--target-model", dest="target", default="llama-8b")
    ap.add_argument("--prefix", "--prefix-len", dest="prefix", type=int, default=8192)
    ap.add_argument("--width", "--k", dest="k", type=int, default=3)
    ap.add_argument("--depth", "--d", dest="d", type=int, default=4)
    ap.add_argument("--pairs", "--iters", dest="pairs", type=int, default=6,
                    help="timed iterations per arm (even: whole A B B A blocks)")
    ap.add_argument("--warmup", type=int, default=1, help="untimed iterations of every arm before the timed ones")
    ap.add_argument("--pair-order-seed", type=int, default=0, help="odd: the first block runs B A A B")
    ap.add_argument("--page-size", type=int, default=16)
    ap.add_argument("--context-length", type=int, default=None, help="engine positions (default prefix + 1024)")
    ap.add_argument("--repeat-token-id", type=int, default=None,
                    help="prefix = this token repeated (default: seeded random ids)")
    ap.add_argument("--shared-path-tokens", type=int, default=2,
                    help="leading tokens the synthetic verify routes share")
    ap.add_argument("--skip-tree", action="store_true")
    ap.add_argument("--skip-forest", action="store_true")
    ap.add_argument("--skip-native-batch-ar", action="store_true")
    ap.add_argument("--skip-verify", "--skip-target", dest="skip_target", action="store_true")
    ap.add_argument("--dtype", default="float16")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--gpu-id", type=int, default=None, help="CUDA device index")
    for flag, typ in _INERT:
        ap.add_argument(flag, type=typ, default=None, help="No-op (a setting of the reference's SGLang runtime).")
    for flag in ("--legacy-token-attention-metadata", "--skip-page-layout-validation", "--trust-remote-code"):
        ap.add_argument(flag, action="store_true", help="No-op (the reference's SGLang page-table switches).")
    ap.add_argument("--json-out", default=None)
    return ap


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    check_pairs(args.pairs)
    llama, engine_mod = pkg("models.llama"), pkg("runtime.engine")
    drafter_mod, store_mod = pkg("runtime.drafter"), pkg("runtime.store")
    dt = getattr(torch, args.dtype)
    dev = torch.device(args.device if args.gpu_id is None else f"cuda:{args.gpu_id}")
    if dev.type == "cuda" and dev.index is not None:
        torch.cuda.set_device(dev)
    cuda = dev.type == "cuda"
    k, d, P, ps = args.k, args.d, args.prefix, int(args.page_size)
    dcfg, tcfg = llama.get_config(args.drafter), llama.get_config(args.target)
    vocab = min(dcfg.vocab_size, tcfg.vocab_size)
    g = torch.Generator().manual_seed(0)
    if args.repeat_token_id is not None:
        prompt = [int(args.repeat_token_id) % vocab] * P
    else:
        prompt = torch.randint(0, vocab, (P,), generator=g).tolist()
    ctx = int(args.context_length or P + 1024)
    if ctx < P + 2 * k * k * d + 64:
        raise SystemExit(f"--context-length {ctx} leaves no room for {k * k} routes of depth {d} after {P} tokens")
    pages = 2 * (ctx // ps) + 512
    run_tree, run_forest, run_ar = not args.skip_tree, not args.skip_forest, not args.skip_native_batch_ar
    out: dict[str, object] = {"prefix": P, "k": k, "d": d, "pairs": args.pairs, "warmup": args.warmup,
                              "pair_order_seed": args.pair_order_seed, "dtype": args.dtype, "device": str(dev),
                              "reference_h800_ms": REFERENCE_H800_MS}

    dw = llama.random_weights(dcfg, seed=1, dtype=dt, device=dev)
    dr = drafter_mod.DrafterRuntime(engine_mod.LlamaEngine(dw, num_pages=pages, page_size=ps, max_positions=ctx))
    if cuda:
        dr.warm_graphs(k, 4)
    store = store_mod.KVTreeStore()
    dr.bind_store(store)
    dr.prefill(prompt)

    arms_ = DrafterArms(dr, store, k, d)
    tree, batch_ar, forest_after_tree = arms_.tree, arms_.batch_ar, arms_.forest_after_tree

    counters = pkg("utils.counters")
    hot: dict[str, list[dict[str, int]]] = {}

    def run(name, fn):
        if name == "forest":
            fn = fn()  # the untimed tree: before the counter snapshot too
        before = counters.snapshot()
        dev_ms, host_ms = timed(fn, cuda)
        hot.setdefault(name, []).append(counters.delta(before))
        dr.drop_speculative()
        return dev_ms, host_ms

    # Arm A is the matched batch AR, arm B the tree (forest); each block of two iterations is
    # A B B A (B A A B with an odd --pair-order-seed).
    pairs = [({"a": ("batch_ar_k", lambda: batch_ar(k)), "b": ("tree", tree)}, run_ar, run_tree),
             ({"a": ("batch_ar_k2", lambda: batch_ar(k * k)), "b": ("forest", forest_after_tree)}, run_ar,
              run_forest)]
    enabled = {"a": None, "b": None}
    results: dict[str, list[tuple[float, float]]] = {}
    orders = []
    for i in range(-int(args.warmup), args.pairs):
        order = abba_order(i + int(args.pair_order_seed))
        if i >= 0:
            orders.append("".join(order).upper())
        for arms, a_on, b_on in pairs:
            enabled["a"], enabled["b"] = a_on, b_on
            for x in order:
                if not enabled[x]:
                    continue
                name, fn = arms[x]
                r = run(name, fn)
                if i >= 0:
                    results.setdefault(name, []).append(r)
    out["orders"] = orders
    # Hot-path counters per timed iteration (kernel launches of this package, host<->device bytes),
    # averaged over the arm's timed and warm-up runs; set-up work is outside the snapshots.
    out["hot_path_counters"] = {name: {key: round(statistics.mean(d[key] for d in ds), 1) for key in ds[0]}
                                for name, ds in hot.items()}
    for name, vals in results.items():
        out[f"{name}_ms"] = round(statistics.mean(v[0] for v in vals), 3)
        out[f"{name}_host_ms"] = round(statistics.mean(v[1] for v in vals), 3)
    for b_name, a_name, key in (("tree", "batch_ar_k", "tree_over_batch_ar"),
                                ("forest", "batch_ar_k2", "forest_over_batch_ar")):
        if b_name in results and a_name in results:
            out[key] = round(out[f"{b_name}_ms"] / out[f"{a_name}_ms"], 4)
            out[f"{key}_blocks"] = block_ratios([v[0] for v in results[a_name]], [v[0] for v in results[b_name]])
    dr.engine.ops.check()
    del dr, dw
    if cuda:
        torch.cuda.empty_cache()

    if not args.skip_target:
        target_mod = pkg("runtime.target")
        types = pkg("types")
        tw = llama.random_weights(tcfg, seed=2, dtype=dt, device=dev)
        te = engine_mod.LlamaEngine(tw, num_pages=pages, page_size=ps, max_positions=ctx)
        tv = target_mod.TargetVerifier(te, k=k, d=d)
        if cuda:
            tv.warm_graphs()
        tv.prefill(prompt)
        shared_n = max(0, min(int(args.shared_path_tokens), d))

        def synthetic_routes():
            shared = torch.randint(0, vocab, (shared_n,), generator=g).tolist()
            return [types.VerifyRoutePayload(route_id=r, token_ids=tuple(
                shared + torch.randint(0, vocab, (d - shared_n,), generator=g).tolist()), draft_logprob=-1.0,
                draft_token_logprobs=tuple([-0.25] * d)) for r in range(k)]

        def one_row(n):
            p = len(tv.prefix_token_ids)
            slots = tv.seq.reserve_scratch(p + n).numpy()
            tv._sync()
            tok = torch.zeros(n, dtype=torch.int32, device=dev)

            def fwd():
                for j in range(n):
                    te.run_rows(1, prefix_pages=tv.mirror.dev, tokens=tok[j:j + 1], positions=[p + j],
                                slots=slots[j:j + 1], shared_len=p + j, n_shared_pages=len(tv.mirror.host),
                                mask_base=p + j, row_full=[p + j + 1], row_len=[p + j + 1])
            return fwd

        warm = max(1, int(args.warmup))
        ver, ar, ar2, lin, tree_fwd = [], [], [], [], []
        for i in range(args.pairs + warm):
            routes = synthetic_routes()
            ver.append(timed(lambda: tv.verify_payloads(prefix_token_ids=tv.prefix_token_ids, routes=routes), cuda))
            ar.append(timed(one_row(1), cuda))
            # Two dependent one-token forwards and the linear (non-deduplicated) verify of the same
            # kind of routes, without commit.
            ar2.append(timed(one_row(2), cuda))
            paths = [list(r.token_ids) for r in synthetic_routes()]
            lin.append(timed(lambda: tv.run_tree(paths, deduplicate=False), cuda))
            tree_fwd.append(timed(lambda: tv.run_tree(paths), cuda))
        for name, vals in (("target_verify", ver), ("target_ar1", ar), ("target_ar2", ar2),
                           ("target_linear_verify", lin), ("target_tree_forward", tree_fwd)):
            out[f"{name}_ms"] = round(statistics.mean(v[0] for v in vals[warm:]), 3)
        out["target_verify_host_ms"] = round(statistics.mean(v[1] for v in ver[warm:]), 3)
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
