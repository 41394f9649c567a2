#!/usr/bin/env python
"""GPU busy/idle timeline of headline decode rounds (CUPTI records through torch.profiler).

    python benchmarks/trace_round.py --rounds 6 [bench.py flags]

Builds the drafter + target of ``bench.py`` (same flags and defaults), warms
up, then profiles a few rounds of one request (rounds only: no prefill).  For each round it reports the host wall time,
the time at least one kernel was running on the GPU (union over streams), the
idle remainder, and the largest idle gaps with the kernels on either side --
the places where host work (selection, scoring, thread handoffs, syncs)
leaves the GPU waiting.  Kernel names are grouped by template.  Timestamps
come from CUPTI; headline timings use CUDA events (``bench.py``).
"""

from __future__ import annotations

import argparse
import collections
import json
import os
import re
import sys
import time

import torch
from torch.profiler import ProfilerActivity, profile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def short(name: str) -> str:
    return re.sub(r"\(.*", "", name).replace("void ", "")[:60]


def analyze_rounds(events, bounds, walls, *, top_gaps: int = 12) -> dict:
    """Busy/idle accounting of GPU activity records.

    ``events``: (start_us, end_us, name) of every kernel / copy, any order;
    ``bounds``: (start_us, end_us) of each round; ``walls``: host seconds per round.
    Busy time is the union of the intervals that start inside the round; each
    idle gap is attributed to the pair of activities on either side of it.
    """
    events = sorted(events)
    out_rounds = []
    gap_kinds: dict[str, list[float]] = collections.defaultdict(list)
    for ri, (lo, hi) in enumerate(bounds[: len(walls)]):
        ks = [e for e in events if lo <= e[0] < hi]
        busy = 0.0
        gaps = []
        end = lo
        prev = "(round start)"
        for s, t, name in ks:
            if s > end:
                gaps.append((s - end, prev, short(name)))
            busy += max(0.0, t - max(s, end))
            if t > end:
                end = t
                prev = short(name)
        if hi > end:
            gaps.append((hi - end, prev, "(round end)"))
        gaps.sort(reverse=True)
        for g, a, b in gaps:
            gap_kinds[f"{a}  ->  {b}"].append(g)
        per = collections.Counter(short(e[2]) for e in ks)
        out_rounds.append({
            "round": ri,
            "wall_us": round(walls[ri] * 1e6, 1),
            "span_us": round(hi - lo, 1),
            "gpu_busy_us": round(busy, 1),
            "gpu_idle_us": round(hi - lo - busy, 1),
            "gpu_events": len(ks),
            "largest_gaps_us": [[round(g, 1), a, b] for g, a, b in gaps[:top_gaps]],
            "top_kernels": per.most_common(8),
        })
    n = max(1, len(out_rounds))
    return {
        "rounds": len(out_rounds),
        "mean_wall_us": round(1e6 * sum(walls) / max(1, len(walls)), 1),
        "mean_span_us": round(sum(r["span_us"] for r in out_rounds) / n, 1),
        "mean_gpu_busy_us": round(sum(r["gpu_busy_us"] for r in out_rounds) / n, 1),
        "mean_gpu_idle_us": round(sum(r["gpu_idle_us"] for r in out_rounds) / n, 1),
        "idle_by_boundary_us_per_round": {
            k: round(sum(v) / n, 1) for k, v in sorted(gap_kinds.items(), key=lambda kv: -sum(kv[1]))[:20]
        },
        "per_round": out_rounds,
    }


def main() -> int:
    ap = argparse.ArgumentParser(add_help=False)
    ap.add_argument("--rounds", type=int, default=6)
    ap.add_argument("--trace-warmup", type=int, default=8)
    ap.add_argument("--json-out", default=None)
    ap.add_argument("--top-gaps", type=int, default=12)
    own, rest = ap.parse_known_args()
    import bench

    sys.argv = [sys.argv[0], *rest]
    args = bench.parse()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    te = bench.build_target_engine(args, device, 1, False)
    gen, _, _ = bench.build_session(args, device, te)
    prompts = iter(bench.make_prompts(args, 0) * 1000)
    session = gen.start(next(prompts))

    def one_round():
        nonlocal session
        if session.finished:
            session = gen.start(next(prompts))  # prefill outside the profiled round
        session.step()

    for _ in range(own.trace_warmup):
        one_round()
    if session.finished:
        session = gen.start(next(prompts))
    torch.cuda.synchronize()
    walls = []
    # Round boundaries: torch's tiny spin kernel on the default stream between
    # full synchronizes (CUDA activity only, so the host is not slowed by CPU tracing).
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(own.rounds):
            torch.cuda.synchronize()
            torch.cuda._sleep(100)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if session.finished:
                break
            session.step()
            torch.cuda.synchronize()
            walls.append(time.perf_counter() - t0)
        torch.cuda._sleep(100)
        torch.cuda.synchronize()
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    evs.sort(key=lambda e: e.time_range.start)
    marks = [i for i, e in enumerate(evs) if "spin_kernel" in e.name]
    gpu = [e for e in evs if "spin_kernel" not in e.name]
    bounds = [(evs[a].time_range.end, evs[b].time_range.start) for a, b in zip(marks, marks[1:])]
    if len(bounds) < len(walls):
        print(f"warning: found {len(marks)} round markers for {len(walls)} rounds", file=sys.stderr)
    summary = analyze_rounds([(e.time_range.start, e.time_range.end, e.name) for e in gpu], bounds, walls,
                             top_gaps=own.top_gaps)
    print(json.dumps({k: v for k, v in summary.items() if k != "per_round"}, indent=1))
    if own.json_out:
        with open(own.json_out, "w") as f:
            json.dump(summary, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
