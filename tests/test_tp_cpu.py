"""Tensor parallelism on CPU ranks (gloo): sharding, worker protocol, host-side failure detection."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
import time

import pytest
import torch

from conftest import REPO, mod


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def torchrun(nproc: int, module: str, *args: str, timeout: int = 240) -> subprocess.CompletedProcess:
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(nproc),
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), "-m", module, *args]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    return subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=timeout)


def last_json(out: str) -> dict:
    for line in reversed(out.strip().splitlines()):
        if line.startswith("{"):
            return json.loads(line)
    raise AssertionError("no JSON line in output:\n" + out[-3000:])


def test_random_weights_tp_matches_sharded_full_model():
    llama = mod("models.llama")
    shard = mod("parallel.shard")
    cfg = llama.get_config("tiny-target")
    full = llama.random_weights(cfg, seed=5, dtype=torch.float32)
    for rank in range(2):
        a = shard.random_weights_tp(cfg, rank=rank, tp=2, seed=5, dtype=torch.float32)
        b = shard.shard_weights(full, rank, 2)
        assert a.config == b.config and a.config.num_heads == 2 and a.config.num_kv_heads == 1
        for x, y in zip(a.tensors(), b.tensors()):
            assert torch.equal(x, y)


def test_tp_partial_sums_equal_full_layer():
    # sum over ranks of the row-parallel outputs == the full projection.
    llama = mod("models.llama")
    shard = mod("parallel.shard")
    cfg = llama.get_config("tiny-target")
    full = llama.random_weights(cfg, seed=2, dtype=torch.float32)
    x = torch.randn(3, cfg.hidden_size)
    lw = full.layers[0]
    parts = [shard.shard_weights(full, r, 2).layers[0] for r in range(2)]
    qkv = x @ lw.wqkv.t()
    q = qkv[:, :cfg.q_size]
    o_full = q @ lw.wo.t()
    o_tp = sum((x @ p.wqkv.t())[:, :cfg.q_size // 2] @ p.wo.t() for p in parts)
    torch.testing.assert_close(o_tp, o_full, rtol=1e-5, atol=1e-5)


def test_check_tp_two_gloo_ranks():
    r = torchrun(2, "0709_b200.parallel.check_tp", "--mode", "torch", "--fallback-threshold", "-3")
    assert r.returncode == 0, r.stderr[-3000:]
    d = last_json(r.stdout)
    assert d["tp"] == 2 and d["generation_equal"]
    assert d["tree_argmax_equal"] and d["prefill_argmax_equal"]
    assert d["tree_logit_max_abs_diff"] < 1e-4
    assert "fallback_ar" in d["decisions_tp"]


def test_mailbox_round_trip_and_lost_root(tmp_path):
    mb_mod = mod("parallel.mailbox")
    path = str(tmp_path / "mb")
    root = mb_mod.Mailbox(path, rank=0, world=2, create=True, ack_timeout_s=5)
    worker = mb_mod.Mailbox(path, rank=1, world=2, create=False, idle_timeout_s=3)
    root.post(mb_mod.OP_CALL, ("x", {"a": 1}))
    assert worker.receive() == (mb_mod.OP_CALL, ("x", {"a": 1}))
    root.post(mb_mod.OP_CALL, ("y", {}))
    assert worker.receive()[1] == ("y", {})
    # The root stops posting: the worker gives up after its idle limit instead of spinning forever.
    t0 = time.monotonic()
    with pytest.raises(mb_mod.PeerLost):
        worker.receive()
    assert time.monotonic() - t0 < 30
    worker.close()
    root.close()


def test_mailbox_root_detects_missing_worker(tmp_path):
    mb_mod = mod("parallel.mailbox")
    root = mb_mod.Mailbox(str(tmp_path / "mb"), rank=0, world=3, create=True, ack_timeout_s=0.5)
    w1 = mb_mod.Mailbox(str(tmp_path / "mb"), rank=1, world=3, create=False)
    root.post(mb_mod.OP_CALL, 1)
    w1.receive()  # rank 2 never reads
    with pytest.raises(mb_mod.PeerLost, match=r"\[2\]"):
        root.post(mb_mod.OP_CALL, 2)
    w1.close()
    root.close()


def test_worker_detects_dead_root(tmp_path):
    # A root process that exits without posting stop: the worker notices within seconds.
    mb_mod = mod("parallel.mailbox")
    path = str(tmp_path / "mb")
    code = (
        "import importlib, sys, time; sys.path.insert(0, %r);"
        "m = importlib.import_module('0709_b200.parallel.mailbox');"
        "r = m.Mailbox(%r, rank=0, world=2, create=True); r.owner = False; time.sleep(3); r.post(m.OP_CALL, 'hello')"
    ) % (str(REPO), path)
    proc = subprocess.Popen([sys.executable, "-c", code])
    t0 = time.monotonic()
    while not os.path.exists(path) or os.path.getsize(path) == 0:
        assert time.monotonic() - t0 < 60
        time.sleep(0.05)
    w = mb_mod.Mailbox(path, rank=1, world=2, create=False)
    assert w.receive() == (mb_mod.OP_CALL, "hello")
    assert proc.wait(timeout=60) == 0
    t0 = time.monotonic()
    with pytest.raises(mb_mod.PeerLost, match="root rank exited"):
        w.receive()
    assert time.monotonic() - t0 < 30
    w.close()
    os.unlink(path)


def test_root_detects_a_worker_that_left():
    # The worker exits (between calls) after its first few commands; the root's next
    # command is never acknowledged and it raises PeerLost instead of hanging.
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), os.path.join(REPO, "tests", "tp_fault_job.py")]
    env = dict(os.environ, OMP_NUM_THREADS="1", ATLAS_TP_FAULT_EXIT_AFTER="4", ATLAS_TP_ACK_TIMEOUT="3")
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=240)
    d = last_json(r.stdout)
    assert d["peer_lost"], r.stdout[-2000:] + r.stderr[-2000:]
    assert d["kind"] in ("PeerLost", "RuntimeError")
    assert "did not acknowledge" in d["message"] or "Connection" in d["message"] or "closed" in d["message"]
