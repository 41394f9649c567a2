#!/usr/bin/env python
"""Run the paged attention of one layer a few times (8B head geometry) for ncu captures.

    python benchmarks/profile_attention.py --prefix 1024 --rows 12 --splits 0 --reps 3

``--splits 0`` uses the engine's graph choice for a context of ``--max-context``.
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--prefix", type=int, default=1024)
    ap.add_argument("--rows", type=int, default=12)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--max-context", type=int, default=2400)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    attn_desc = importlib.import_module("0709_b200.ops.attn_desc")
    ops = importlib.import_module("0709_b200.ops.cuda_ops").CudaOps(device=torch.device("cuda"))
    hq, hkv, ps, rows, prefix = 32, 8, 16, args.rows, args.prefix
    npages = (prefix + rows + ps - 1) // ps + 1
    kv = torch.randn(1, npages, 2, hkv, ps, 128, device="cuda").half()
    ops.engine = type("E", (), {"kv": kv})()
    pages = torch.arange(npages, dtype=torch.int32, device="cuda")
    masks = torch.full((rows, 1), -1, dtype=torch.int64, device="cuda")
    lens = torch.full((rows,), prefix + rows, dtype=torch.int32, device="cuda")
    full = torch.full((rows,), prefix, dtype=torch.int32, device="cuda")
    desc = attn_desc.single_sequence_desc(pages, lens, shared_len=prefix, mask_base=prefix, masks=masks, full=full)
    q = torch.randn(rows, hq, 128, device="cuda").half()
    sp = args.splits or ops.attention_splits(rows, hq, hkv, args.max_context, ps)
    ops.reserve_attention_workspace(64, hq, hkv, args.max_context, ps)
    for _ in range(args.reps):
        ops.attention(q, kv[0], desc, splits=sp)
    torch.cuda.synchronize()
    ops.check()
    print(f"splits={sp} ok", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
