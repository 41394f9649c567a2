#!/usr/bin/env python
"""Replay one graphed forward (default: Llama-3.1-8B shape, 12 rows, P=2048) a few times.

Used under ``ncu --metrics gpu__time_duration.sum`` to list every kernel of
a decode/verify forward with its device time:

    python benchmarks/profile_forward.py --model llama-8b --rows 12 --replays 3
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-8b")
    ap.add_argument("--rows", type=int, default=12)
    ap.add_argument("--prefix", type=int, default=2048)
    ap.add_argument("--replays", type=int, default=3)
    args = ap.parse_args()
    llama = importlib.import_module("0709_b200.models.llama")
    engine_mod = importlib.import_module("0709_b200.runtime.engine")
    cfg = llama.get_config(args.model)
    w = llama.random_weights(cfg, seed=1, dtype=torch.float16, device="cuda")
    pages_needed = (args.prefix + args.rows) // 16 + 4
    eng = engine_mod.LlamaEngine(w, num_pages=pages_needed + 8, page_size=16, max_positions=args.prefix + 4096)
    pages = torch.arange(pages_needed, dtype=torch.int32, device="cuda")
    r, p = args.rows, args.prefix
    fields = dict(tokens=np.arange(r), positions=np.arange(p, p + r), slots=np.arange(p, p + r), shared_len=p,
                  n_shared_pages=pages_needed, mask_base=p, row_full=np.full(r, p), row_len=np.full(r, p + r))
    b = engine_mod.row_bucket(r)
    eng.warm_graph(b, prefix_pages=pages)
    torch.cuda.synchronize()
    print("PROFILE_START", flush=True)
    for _ in range(args.replays):
        eng.run_rows(b, prefix_pages=pages, **fields)
    torch.cuda.synchronize()
    eng.ops.check()
    print("done", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
