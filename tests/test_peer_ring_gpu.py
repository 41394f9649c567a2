"""Peer-memory message rings between two GPUs (the drafter <-> target handoff), in child processes."""

from __future__ import annotations

import os
import subprocess
import sys

import pytest
import torch

from conftest import REPO
from test_tp_cpu import free_port, last_json

pytestmark = pytest.mark.gpu


def test_peer_ring_round_trips_and_silent_peer_timeout():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (the two ranks must not share a GPU)")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(REPO, "tests", "peer_ring_job.py")]
    r = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=360,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stderr[-4000:]
    d = last_json(r.stdout)
    assert d["peer"]["intact"] and d["nccl"]["intact"]
    t = d["peer"]["silent_peer_timeout"]
    assert t["lost"] and 0.4 < t["waited_s"] < 5.0 and t["recovered"]
