#!/usr/bin/env python
"""Verify-attention microbenchmark (the reference's masked-verify configuration): ancestor-masked paged tree attention.

    python benchmarks/bench_verify_attention.py [--prefixes 1024,4096,16384] [--flashinfer]

Llama-3.1-8B head geometry (32 q / 8 kv heads, head_dim 128, fp16), a committed
prefix in 16-token pages, and the routes of one ATLAS round: k=3 stage-1
routes plus k^2=9 forest routes of depth 4 sharing prefixes (48 raw tokens),
deduplicated into a trie whose ancestor mask drives the attention.  Reports
the attention time of one layer (CUDA events, L2 flushed before every launch)
and its fraction of the measured HBM roofline (K and V of prefix + nodes read
once).  With ``--flashinfer`` the same problem also runs through FlashInfer's
BatchPrefillWithPagedKVCacheWrapper with a custom mask, the reference's
library path, on the same GPU.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def pkg(name):
    return importlib.import_module(f"0709_b200.{name}")


def round_routes(k: int, d: int, g: torch.Generator) -> list[list[int]]:
    """k tree routes (the first two share their first token) + k*k forest routes reusing 2 tree tokens."""
    rnd = lambda n: torch.randint(0, 128256, (n,), generator=g).tolist()  # noqa: E731
    tree = [rnd(d) for _ in range(k)]
    tree[1][0] = tree[0][0]
    forest = [tree[i][:2] + rnd(d - 2) for i in range(k) for _ in range(k)]
    return tree + forest


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--prefixes", default="1024,4096,16384")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--flashinfer", action="store_true")
    ap.add_argument("--merge", default="two",
                    help="comma list of split-merge paths: two (separate merge kernel), fused8, fused16 "
                         "(merge inside the kernel, clusters of at most 8 / 16 CTAs)")
    ap.add_argument("--rows", default="tree", help="tree (the deduplicated round), or a row count (decode rows)")
    ap.add_argument("--json-out", default=None)
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    from bench_kernels import peaks, timeit

    host = pkg("ops._native").host()
    attn_desc = pkg("ops.attn_desc")
    ops = pkg("ops.cuda_ops").CudaOps(device=torch.device("cuda"))
    hbm, _, src = peaks()
    hq, hkv, ps, hd = 32, 8, 16, 128
    g = torch.Generator().manual_seed(0)
    routes = round_routes(3, 4, g)
    tokens, parents, depths, node_paths, masks = host.build_tree(torch.tensor(routes, dtype=torch.int64))
    n = int(tokens.numel())
    if args.rows != "tree":  # decode rows: each row sees the prefix and itself
        n = int(args.rows)
        masks = torch.tensor([[1 << i] for i in range(n)], dtype=torch.int64)
    rows = []
    for P in (int(x) for x in args.prefixes.split(",")):
        npages = (P + n + ps - 1) // ps + 1
        kv = torch.randn(1, npages, 2, hkv, ps, hd, device="cuda").half()
        ops.engine = type("E", (), {"kv": kv})()
        pages = torch.arange(npages, dtype=torch.int32, device="cuda")
        desc = attn_desc.single_sequence_desc(
            pages, torch.full((n,), P + n, dtype=torch.int32, device="cuda"), shared_len=P, mask_base=P,
            masks=masks.to("cuda"), full=torch.full((n,), P, dtype=torch.int32, device="cuda"))
        q = torch.randn(n, hq, hd, device="cuda").half()
        ops.reserve_attention_workspace(64, hq, hkv, P + 64, ps)
        splits = ops.attention_splits(n, hq, hkv, P, ps)
        nbytes = 2 * (P + n) * hkv * hd * 2
        row = {"prefix": P, "raw_nodes": len(routes) * 4, "dedup_nodes": n, "rows": n, "splits": splits}
        for mode in args.merge.split(","):
            ops.fused_merge = mode.startswith("fused")
            ops.cluster_cap = int(mode[5:]) if ops.fused_merge else ops.cluster_cap
            us = timeit(lambda: ops.attention(q, kv[0], desc, splits=splits), args.iters)
            tag = "" if mode == "two" else f"_{mode}"
            row.update({f"us{tag}": round(us, 2), f"GB/s{tag}": round(nbytes / us / 1e3, 1),
                        f"hbm_frac_of_{src}{tag}": round(nbytes / us / 1e3 / hbm, 3)})
        ops.fused_merge = False
        if args.flashinfer:
            row.update(flashinfer_case(kv, q, P, n, masks, ps, args.iters, timeit, nbytes, hbm, src))
        rows.append(row)
        print(json.dumps(row), flush=True)
        del kv
    if args.json_out:
        with open(args.json_out, "w") as f:
            json.dump(rows, f, indent=1)
    return 0


def flashinfer_case(kv, q, P, n, masks, ps, iters, timeit, nbytes, hbm, src) -> dict:
    try:
        import flashinfer

        hq, hkv, hd = q.shape[1], kv.shape[3], q.shape[2]
        ws = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
        w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "HND")
        npages = (P + n + ps - 1) // ps
        # Dense [n, P + n] mask: prefix fully visible, node region from the ancestor bits.
        bits = masks[:, 0].to(torch.int64)
        node_vis = ((bits[:, None] >> torch.arange(n)[None, :]) & 1).bool()
        mask = torch.cat((torch.ones(n, P, dtype=torch.bool), node_vis), dim=1).reshape(-1).to("cuda")
        w.plan(torch.tensor([0, n], dtype=torch.int32, device="cuda"),
               torch.tensor([0, npages], dtype=torch.int32, device="cuda"),
               torch.arange(npages, dtype=torch.int32, device="cuda"),
               torch.tensor([(P + n - 1) % ps + 1], dtype=torch.int32, device="cuda"),
               hq, hkv, hd, ps, custom_mask=mask, causal=False, q_data_type=torch.float16)
        us = timeit(lambda: w.run(q, kv[0]), iters)
        return {"flashinfer_us": round(us, 2), f"flashinfer_hbm_frac_of_{src}": round(nbytes / us / 1e3 / hbm, 3)}
    except Exception as exc:  # noqa: BLE001 - report why the library path did not run
        return {"flashinfer": f"unavailable: {type(exc).__name__}: {str(exc)[:160]}"}


if __name__ == "__main__":
    raise SystemExit(main())
