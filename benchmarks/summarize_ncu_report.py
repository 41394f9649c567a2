#!/usr/bin/env python
"""Print the metrics the profile summaries quote from an ncu report (``--set full`` capture).

    python benchmarks/summarize_ncu_report.py report.ncu-rep
"""
import csv, subprocess, sys
rep = sys.argv[1]
out = subprocess.run(["ncu", "-i", rep, "--page", "raw", "--csv"], capture_output=True, text=True).stdout
r = list(csv.reader(out.splitlines()))
hdr, units = r[0], r[1]
want = ["gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum",
        "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "sm__throughput.avg.pct_of_peak_sustained_elapsed",
        "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed", "sm__warps_active.avg.pct_of_peak_sustained_active",
        "launch__grid_size", "launch__cluster_size", "launch__block_size", "launch__registers_per_thread",
        "launch__shared_mem_per_block_dynamic", "lts__t_bytes.sum"]
for row in r[2:]:
    name = row[hdr.index("Kernel Name")]
    print(f"### {name[:110]}")
    for w in want:
        if w in hdr:
            i = hdr.index(w)
            print(f"| {w} | {row[i]} {units[i]} |")
    items = [(h, v) for h, v in zip(hdr, row) if h.startswith("smsp__pcsamp_warps_issue_stalled") and not h.endswith("not_issued")]
    items = sorted([(h, float(v)) for h, v in items if v.replace('.', '', 1).isdigit()], key=lambda x: -x[1])
    tot = sum(v for _, v in items) or 1
    print("| top stall reasons (pc samples) | " + ", ".join(f"{h.replace('smsp__pcsamp_warps_issue_stalled_', '')} {100*v/tot:.0f}%" for h, v in items[:5]) + " |")
    print()
