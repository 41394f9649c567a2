#!/usr/bin/env python
"""Where the tensor-core attention kernel's time goes inside a graphed forward.

    python benchmarks/attention_phases.py --model llama-8b --rows 1 --prefix 2048

Switches on the kernel's phase stamps (SM clock at each pipeline step of every
CTA, see ``attn_shared_tc``), captures and replays one forward's CUDA graph,
and reports for the last layer's launch the median and maximum over the CTAs
that own keys of: set-up, the wait for the previous kernel, Q staging, the
first S and P of the pipeline, the final O, the partial stores and the exit --
each as cycles after the CTA's PDL wait returned, and as microseconds at the
clock given.  Profiling only: the stamps cost a few instructions per step.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

NAMES = {0: "entry", 1: "set_up", 2: "pdl_wait_done", 3: "q_staged", 4: "s0_ready", 5: "p0_published",
         6: "s1_ready", 7: "p1_published", 8: "o_final", 9: "partials_stored", 10: "exit",
         11: "mma_first_stage", 12: "mma_done", 13: "producer_first_load", 14: "producer_last_load",
         16: "q_stored", 17: "q_fenced", 18: "q_reduced", 19: "q_atomic"}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-8b")
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--prefix", type=int, default=2048)
    ap.add_argument("--mhz", type=float, default=1965.0, help="SM clock for the cycle -> us conversion")
    args = ap.parse_args()
    llama = importlib.import_module("0709_b200.models.llama")
    engine_mod = importlib.import_module("0709_b200.runtime.engine")
    ext = importlib.import_module("0709_b200.ops._native").cuda()
    cfg = llama.get_config(args.model)
    npages = (args.prefix + args.rows) // 16 + 4
    buf = torch.zeros(8192 * 20, dtype=torch.int64, device="cuda")
    ext.set_attention_phase_buffer(buf)
    try:
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
        buf.zero_()
        eng.run_rows(b, prefix_pages=pages, **fields)
        torch.cuda.synchronize()
    finally:
        ext.set_attention_phase_buffer(torch.empty(0, dtype=torch.int64, device="cuda"))
    st = buf.view(-1, 20).cpu().numpy().astype(np.int64)
    ctas = st[(st[:, 0] != 0) & (st[:, 8] != 0)]
    with_keys = ctas[ctas[:, 11] != 0] if (ctas[:, 11] != 0).any() else ctas
    base = with_keys[:, 2:3]
    rel = {NAMES[k]: with_keys[:, k] - base[:, 0] for k in NAMES if (with_keys[:, k] != 0).any()}
    to_us = 1.0 / args.mhz
    out = {
        "model": args.model, "rows": args.rows, "prefix": args.prefix, "ctas_stamped": int(len(ctas)),
        "ctas_with_keys": int(len(with_keys)),
        "entry_spread_us": round(float(np.ptp(with_keys[:, 15])) / 1e3, 2),
        "cycles_after_pdl_wait": {k: {"median": int(np.median(v)), "max": int(v.max())} for k, v in rel.items()},
        "us_after_pdl_wait_median": {k: round(float(np.median(v)) * to_us, 2) for k, v in rel.items()},
    }
    print(json.dumps(out, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
