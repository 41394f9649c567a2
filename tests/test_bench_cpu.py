"""``bench.py`` control flow on CPU ranks: tensor-parallel target over 2 gloo ranks and one process.

The tiny fp32 models run the same code as the GPU headline (requests as steps,
barrier-aligned timing marks on every rank, the all-select pass, end to end
through ``generate``); the JSON line must carry the keys the driver reads.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import REPO
from test_tp_cpu import free_port, last_json

ARGS = ["--device", "cpu", "--comm", "torch", "--drafter", "tiny-drafter", "--target", "tiny-target",
        "--dtype", "float32", "--steps", "2", "--warmup", "1", "--max-new-tokens", "16", "--min-prompt", "40",
        "--max-prompt", "80", "--e2e-prompts", "2", "--select-steps", "1"]


def _check(d: dict, n: int) -> None:
    assert d["n_gpus"] == n and d["steps"] == 2 and d["warmup"] == 1
    assert d["scaling"] == "strong" and d["config"]["parallelism"].startswith(f"tp{n}")
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["tokens_timed"] == 2 * 16
    assert d["config"]["fallback_rate_timed"] == 1.0  # random weights under the config's thresholds
    sel = d["select_path"]
    assert sel["fallback_rate"] == 0.0 and sel["rounds"] >= 4
    assert "partial_forest_pruned_then_build_tree" in sel["handoff_modes"] or \
        "completed_forest_reused" in sel["handoff_modes"]
    e2e = d["e2e"]
    assert e2e["prompts"] == 2 and e2e["tokens"] == 32 and e2e["h2d_bytes_per_step"] >= 0
    json.dumps(d)


def test_bench_tp_two_gloo_ranks():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), "bench.py", "--gpus", "2", *ARGS]
    r = subprocess.run(cmd, cwd=REPO, env=dict(os.environ, OMP_NUM_THREADS="1"), capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    _check(last_json(r.stdout), 2)


def test_bench_single_process():
    r = subprocess.run([sys.executable, "bench.py", *ARGS], cwd=REPO, env=dict(os.environ, OMP_NUM_THREADS="1"),
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    _check(last_json(r.stdout), 1)


def test_bench_split_placement_two_gloo_ranks():
    """Config 2's placement: drafter + coordinator on rank 0, target server on rank 1 (gloo send/recv here)."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), "bench.py", "--gpus", "2",
           "--placement", "split", *ARGS]
    r = subprocess.run(cmd, cwd=REPO, env=dict(os.environ, OMP_NUM_THREADS="1"), capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    d = last_json(r.stdout)
    assert d["config"]["parallelism"].startswith("split placement")
    assert d["config"]["tokens_timed"] == 32 and d["select_path"]["fallback_rate"] == 0.0
    ch = d["handoff_channel"]
    assert ch["client"]["messages_sent"] == ch["server"]["messages_received"] + 1  # the stop message
