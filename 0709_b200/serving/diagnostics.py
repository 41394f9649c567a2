"""Correctness diagnostics for a real checkpoint (or a preset): KV reuse against recompute.

    python -m 0709_b200.serving.diagnostics target-commit --model llama-8b --rounds 16 --json-out t.json
    python -m 0709_b200.serving.diagnostics drafter-alignment --model llama-1b --k 3 --d 4 --json-out a.json

``target-commit``: a persistent target verifies ``--rounds`` rounds of three synthetic routes
(sharing their first token) and commits the first route each round, so the committed prefix is
built from compacted tree KV; a fresh target then prefills the same tokens.  Per round the
persistent target's next-token logits and, at the end, the committed prefix's K/V pages are
compared with the fresh ones (max abs diff within ``--max-logit-diff`` / ``--max-kv-diff``,
top-1 equal).

``drafter-alignment``: the drafter builds a depth-d tree, a forest over it (unless
``--skip-forest``), commits a stage-1 route and decodes one step more; every decoded row's
logits are compared with an fp32 recompute of the row's whole token sequence with no cache
(``|diff| <= atol + rtol * |ref|`` elementwise, top-1 equal).

Both exit 1 when a check fails.  Parity: reference tools/smoke_target_incremental_commit.py
(:56-170) and tools/smoke_flashinfer_paged_tree_forest.py (:154-211, 302-385); there the
reference is Hugging Face recompute, here this package's fp32 oracle (``models.llama``).
"""

from __future__ import annotations

import argparse
import json
import math
import sys

import torch

_INERT = (("--mem-fraction-static", float), ("--max-running-requests", int), ("--max-total-tokens", int),
          ("--nccl-port", int), ("--workspace-mb", int))


def _common(p) -> None:
    p.add_argument("--model", required=True, help="preset (seeded random init) or checkpoint directory")
    p.add_argument("--prompt", default="ATLAS staged decode smoke test.")
    p.add_argument("--prompt-token-ids", default=None, help="comma-separated ids (overrides --prompt)")
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--d", "--depth", dest="d", type=int, default=4)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--context-length", type=int, default=8192)
    p.add_argument("--dtype", default="float16", choices=["float16", "bfloat16", "float32"])
    p.add_argument("--device", default=None)
    p.add_argument("--gpu-id", type=int, default=None)
    p.add_argument("--seed", type=int, default=0)
    for flag, typ in _INERT:
        p.add_argument(flag, type=typ, default=None, help="No-op (a setting of the reference's runtimes).")
    p.add_argument("--trust-remote-code", action="store_true", help="No-op (checkpoints are read as safetensors).")
    p.add_argument("--json-out", default=None)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="KV-reuse correctness diagnostics.", allow_abbrev=False)
    sub = p.add_subparsers(dest="cmd", required=True)
    t = sub.add_parser("target-commit", allow_abbrev=False)
    _common(t)
    t.add_argument("--rounds", type=int, default=4)
    t.add_argument("--route-selection-policy", choices=["target_best", "first_route"], default="first_route")
    t.add_argument("--max-logit-diff", type=float, default=1.0)
    t.add_argument("--max-kv-diff", type=float, default=1.0)
    a = sub.add_parser("drafter-alignment", allow_abbrev=False)
    _common(a)
    a.add_argument("--k", type=int, default=3)
    a.add_argument("--skip-forest", action="store_true")
    a.add_argument("--alignment-atol", type=float, default=1.0)
    a.add_argument("--alignment-rtol", type=float, default=0.05)
    a.add_argument("--check-hf-logits", action="store_true",
                   help="accepted for the reference's command line: the recompute check always runs")
    a.add_argument("--logits-tensor-out", default=None,
                   help="torch.save every checked row's logits and its recompute reference to this file")
    for flag in ("--legacy-token-attention-metadata", "--skip-page-layout-validation"):
        a.add_argument(flag, action="store_true", help="No-op (the reference's SGLang page-table switches).")
    return p


def _device(args) -> torch.device:
    if args.device:
        return torch.device(args.device)
    if args.gpu_id is not None:
        return torch.device("cuda", args.gpu_id)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def _prompt(args, vocab: int) -> list[int]:
    if args.prompt_token_ids:
        ids = [int(x) for x in args.prompt_token_ids.split(",") if x.strip()]
    else:
        from .prompts import encode, load_tokenizer

        ids = encode(load_tokenizer(args.tokenizer), args.prompt)
    ids = [t % vocab for t in ids]
    if not ids:
        raise SystemExit("the prompt is empty")
    return ids


def _engine(w, args):
    from ..runtime.engine import LlamaEngine

    ctx = int(args.context_length)
    return LlamaEngine(w, num_pages=2 * math.ceil(ctx / args.page_size) + 64, page_size=args.page_size,
                       max_positions=ctx)


def prefix_kv(engine, pages: list[int], n: int) -> torch.Tensor:
    """K/V of the first ``n`` positions through the page table ``pages``: [layers, 2, n, heads, dim]."""
    ps = engine.page_size
    pos = torch.arange(n, device=engine.kv.device)
    page = torch.tensor(pages, device=engine.kv.device, dtype=torch.long)[pos // ps]
    # kv: [layers, pages, 2, kv_heads, page_size, head_dim]; the two index tensors are not adjacent,
    # so their (position) dimension comes first: [n, layers, 2, kv_heads, head_dim].
    return engine.kv[:, page, :, :, pos % ps, :].permute(1, 2, 0, 3, 4)


def target_commit(args) -> dict:
    from ..models.loader import resolve_model
    from ..runtime.target import TargetVerifier
    from ..types import VerifyRoutePayload

    if args.rounds <= 0:
        raise SystemExit("--rounds must be positive")
    dev = _device(args)
    w = resolve_model(args.model, dtype=args.dtype, device=dev, seed=args.seed)
    vocab = w.config.vocab_size
    prompt = _prompt(args, vocab)
    if len(prompt) + args.rounds * args.d + 64 > args.context_length:
        raise SystemExit("--context-length is too short for the prompt and the committed rounds")
    tv = TargetVerifier(_engine(w, args), k=3, d=args.d, route_selection_policy=args.route_selection_policy)
    tv.prefill(prompt)
    g = torch.Generator().manual_seed(args.seed)
    rounds = []
    ok = True
    for rnd in range(int(args.rounds)):
        first = int(torch.randint(0, vocab, (1,), generator=g))
        routes = [VerifyRoutePayload(route_id=10 * rnd + j, draft_logprob=-1.0,
                                     token_ids=(first, *torch.randint(0, vocab, (args.d - 1,), generator=g).tolist()))
                  for j in range(3)]
        res = tv.verify_payloads(prefix_token_ids=list(tv.prefix_token_ids), routes=routes)
        persistent = tv.prefix_logits.float().reshape(-1)
        fresh_tv = TargetVerifier(_engine(w, args), k=3, d=args.d)
        fresh = fresh_tv.prefill(list(tv.prefix_token_ids)).next_token_logits.float().reshape(-1)
        diff = float((persistent - fresh).abs().max())
        top1 = int(persistent.argmax()) == int(fresh.argmax())
        r = {"round": rnd, "decision": res.decision, "selected_route_id": res.selected_route_id,
             "prefix_len": len(tv.prefix_token_ids), "max_logit_diff": diff, "top1_equal": top1}
        if rnd == int(args.rounds) - 1:
            n = len(tv.prefix_token_ids)
            a = prefix_kv(tv.engine, list(tv.mirror.host), n).float()
            b = prefix_kv(fresh_tv.engine, list(fresh_tv.mirror.host), n).float()
            r["max_kv_diff"] = float((a - b).abs().max())
            r["mean_kv_diff"] = float((a - b).abs().mean())
            ok = ok and r["max_kv_diff"] <= args.max_kv_diff
        ok = ok and res.decision == "select" and diff <= args.max_logit_diff and top1
        rounds.append(r)
        del fresh_tv
    tv.engine.ops.check()
    return {"check": "target_incremental_commit", "passed": ok, "model": args.model, "prompt_len": len(prompt),
            "rounds": rounds, "max_logit_diff_allowed": args.max_logit_diff, "max_kv_diff_allowed": args.max_kv_diff}


def drafter_alignment(args) -> dict:
    from ..models import llama
    from ..models.loader import resolve_model
    from ..runtime import builders
    from ..runtime.drafter import DrafterRuntime
    from ..runtime.store import KVTreeStore

    dev = _device(args)
    w = resolve_model(args.model, dtype=args.dtype, device=dev, seed=args.seed)
    w_ref = llama.weights_to(w, dtype=torch.float32)
    prompt = _prompt(args, w.config.vocab_size)
    k, d = int(args.k), int(args.d)
    dr = DrafterRuntime(_engine(w, args))
    store = KVTreeStore()
    dr.bind_store(store)
    dr.prefill(prompt)
    steps = []
    trace: list[dict] = []

    def check(stage: str, depth: int, step, prefix) -> None:
        logits = step.decode_output.next_token_logits.float()
        rows = []
        for i, r in enumerate(step.decoded_routes):
            toks = list(prefix) + list(store.materialized_token_path(r))
            ref = llama.reference_forward(w_ref, toks)[-1]
            got = logits[i].to(ref.device)
            if args.logits_tensor_out:
                trace.append({"stage": stage, "depth": depth, "tokens": toks, "logits": got.cpu(),
                              "reference": ref.cpu()})
            gap = (got - ref).abs()
            rows.append({"max_abs_diff": float(gap.max()),
                         "within": bool((gap <= args.alignment_atol + args.alignment_rtol * ref.abs()).all()),
                         "top1_equal": int(got.argmax()) == int(ref.argmax())})
        steps.append({"stage": stage, "depth": depth, "rows": len(rows),
                      "max_abs_diff": max(r["max_abs_diff"] for r in rows),
                      "passed": all(r["within"] and r["top1_equal"] for r in rows)})

    tree = builders.build_tree_depths(builders.initialize_stage1_routes(dr.prefix_state(), k=k, route_store=store),
                                      depth=d, k=k, route_store=store, model_backend=dr)
    for i, st in enumerate(tree.steps):
        check("tree", i + 1, st, prompt)
    if not args.skip_forest:
        seeds = builders.initialize_forest_routes(tree.completed_routes, tree.last_logits, k=k, route_store=store)
        half = max(1, d // 2)
        forest = builders.build_forest_depths(seeds, depth=half, k=k, route_store=store, model_backend=dr)
        for i, st in enumerate(forest.steps):
            check("forest", i + 1, st, prompt)
        chosen = tree.completed_routes[0]
        committed = list(prompt) + list(store.materialized_token_path(chosen))
        retained = builders.select_routes_by_stage1_root(forest.next_frontier_routes, int(chosen.route_id))
        promoted, _ = dr.commit_stage1_and_promote(committed_route=chosen, retained_routes=retained)
        check("post_commit_forest", half + 1,
              builders.build_tree_one_depth(promoted, k=k, route_store=store, model_backend=dr), committed)
    dr.engine.ops.check()
    if args.logits_tensor_out:
        torch.save(trace, args.logits_tensor_out)
    return {"check": "drafter_route_kv_alignment", "passed": all(s["passed"] for s in steps), "model": args.model,
            "k": k, "d": d, "prompt_len": len(prompt), "atol": args.alignment_atol, "rtol": args.alignment_rtol,
            "steps": steps}


def main(argv=None) -> int:
    args = build_parser().parse_args(sys.argv[1:] if argv is None else argv)
    report = target_commit(args) if args.cmd == "target-commit" else drafter_alignment(args)
    text = json.dumps(report, indent=2)
    print(json.dumps({"check": report["check"], "passed": report["passed"]}))
    if args.json_out:
        with open(args.json_out, "w") as f:
            f.write(text + "\n")
    return 0 if report["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
