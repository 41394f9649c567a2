#!/usr/bin/env python
"""Kernel timeline of graphed forwards (CUPTI activity records through torch.profiler).

    python benchmarks/trace_forward.py --model llama-1b --rows 9 --prefix 2048

Replays one forward's CUDA graph a few times under ``torch.profiler`` (kernel
activity records only, no replay or serialization), then reports for the
last replay: the span from the first kernel start to the last kernel end,
the summed kernel durations, the summed gaps between consecutive kernels
(launch / dependency latency not hidden by programmatic dependent launch)
and the overlap, plus per-kernel averages.  Timestamps come from CUPTI;
the numbers are for attribution, the headline timings use CUDA events.
"""

from __future__ import annotations

import argparse
import collections
import importlib
import json
import os
import re
import sys

import numpy as np
import torch
from torch.profiler import ProfilerActivity, profile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-1b")
    ap.add_argument("--rows", type=int, default=9)
    ap.add_argument("--prefix", type=int, default=2048)
    ap.add_argument("--replays", type=int, default=3)
    ap.add_argument("--json-out", default=None)
    ap.add_argument("--fp8", action="store_true", help="block-scaled fp8 weights (Fp8LlamaEngine)")
    ap.add_argument("--window", type=int, nargs=2, default=None, metavar=("FIRST", "COUNT"),
                    help="also list kernels FIRST..FIRST+COUNT-1 of the last forward with start/end offsets (us)")
    args = ap.parse_args()
    llama = importlib.import_module("0709_b200.models.llama")
    engine_mod = importlib.import_module("0709_b200.runtime.engine")
    cfg = llama.get_config(args.model)
    npages = (args.prefix + args.rows) // 16 + 4
    if args.fp8:
        fp8 = importlib.import_module("0709_b200.models.fp8")
        w = fp8.random_weights_fp8(cfg, seed=1, dtype=torch.bfloat16, device="cuda")
        eng = importlib.import_module("0709_b200.runtime.engine_fp8").Fp8LlamaEngine(
            w, num_pages=npages + 8, page_size=16, max_positions=args.prefix + 4096)
    else:
        w = llama.random_weights(cfg, seed=1, dtype=torch.float16, device="cuda")
        eng = engine_mod.LlamaEngine(w, num_pages=npages + 8, page_size=16, max_positions=args.prefix + 4096)
    pages = torch.arange(npages, dtype=torch.int32, device="cuda")
    r, p = args.rows, args.prefix
    fields = dict(tokens=np.arange(r), positions=np.arange(p, p + r), slots=np.arange(p, p + r), shared_len=p,
                  n_shared_pages=npages, mask_base=p, row_full=np.full(r, p), row_len=np.full(r, p + r))
    b = engine_mod.row_bucket(r)
    eng.warm_graph(b, prefix_pages=pages)
    for _ in range(3):
        eng.run_rows(b, prefix_pages=pages, **fields)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.replays):
            eng.run_rows(b, prefix_pages=pages, **fields)
        torch.cuda.synchronize()
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA and "Memcpy" not in e.name
           and "Memset" not in e.name]
    evs.sort(key=lambda e: e.time_range.start)
    per = len(evs) // args.replays
    last = evs[-per:]
    t0 = last[0].time_range.start
    span = last[-1].time_range.end - t0
    busy = sum(e.time_range.end - e.time_range.start for e in last)
    gaps, overlap = 0.0, 0.0
    end = last[0].time_range.end
    for e in last[1:]:
        if e.time_range.start > end:
            gaps += e.time_range.start - end
        else:
            overlap += min(end, e.time_range.end) - e.time_range.start
        end = max(end, e.time_range.end)
    kinds = collections.defaultdict(list)
    for e in last:
        kinds[re.sub(r"\(.*", "", e.name)[:70]].append(e.time_range.end - e.time_range.start)
    out = {"model": args.model, "rows": r, "prefix": p, "kernels": len(last), "span_us": round(span, 1),
           "kernel_sum_us": round(busy, 1), "gap_sum_us": round(gaps, 1), "overlap_us": round(overlap, 1),
           "per_kernel": {k: {"n": len(v), "avg_us": round(sum(v) / len(v), 2), "sum_us": round(sum(v), 1)}
                          for k, v in sorted(kinds.items(), key=lambda kv: -sum(kv[1]))}}
    if args.window:
        a, n = args.window
        w0 = last[a].time_range.start
        out["window"] = [[re.sub(r"\(.*", "", e.name)[:60], round(e.time_range.start - w0, 2),
                          round(e.time_range.end - w0, 2)] for e in last[a: a + n]]
    print(json.dumps(out, indent=1))
    if args.json_out:
        with open(args.json_out, "w") as f:
            json.dump(out, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
