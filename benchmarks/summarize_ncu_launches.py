#!/usr/bin/env python
"""Summarize an ncu launch list (``--metrics gpu__time_duration.sum --csv``) per kernel.

    python benchmarks/summarize_ncu_launches.py launches.csv N

Takes the last N launches (one forward) and prints total, share, count and
mean device time per kernel.
"""
import csv, sys, re, collections
def load(path, per_fwd=None):
    rows = []
    with open(path) as f:
        lines = [l for l in f if l.startswith('"')]
    rd = csv.DictReader(lines)
    for r in rd:
        if r.get("Metric Name") == "gpu__time_duration.sum":
            rows.append((r["Kernel Name"], float(r["Metric Value"]), r["Metric Unit"]))
    return rows
path, n = sys.argv[1], int(sys.argv[2])
rows = load(path, n)
last = rows[-n:]
tot = collections.defaultdict(float); cnt = collections.Counter()
for name, v, unit in last:
    us = v / 1000.0 if unit in ("ns", "nsecond") else (v if unit in ("us", "usecond") else v * 1000.0)
    key = re.sub(r"\(.*", "", name)[:60]
    tot[key] += us; cnt[key] += 1
s = sum(tot.values())
print(f"{path}: {len(rows)} launches captured, last {n}: total {s:.1f} us")
for k, v in sorted(tot.items(), key=lambda x: -x[1]):
    print(f"  {v:9.1f} us {100*v/s:5.1f}%  n={cnt[k]:4d}  avg={v/cnt[k]:7.2f}  {k}")
