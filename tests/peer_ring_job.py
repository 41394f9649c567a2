"""Two-rank job for the peer-memory message rings (run by tests/test_peer_ring_gpu.py under torchrun).

Each rank owns one GPU.  Checks, printed as one JSON line by rank 0:
* round trips of messages from 1 byte to 1 MB arrive intact over the peer ring
  and over NCCL send/recv, with their mean round-trip times;
* a receive whose peer is alive but silent gives up after its limit with
  ``PeerLost`` (bounded waits, no hang), and the ring works again afterwards.
"""

from __future__ import annotations

import importlib
import json
import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
transport = importlib.import_module("0709_b200.serving.peer_transport")
mailbox = importlib.import_module("0709_b200.parallel.mailbox")


def round_trips(ch, rank: int, sizes, reps: int) -> tuple[bool, float]:
    ok = True
    t0 = time.perf_counter()
    for i in range(reps):
        for n in sizes:
            msg = {"i": i, "blob": bytes((j * 7 + i) % 251 for j in range(n))}
            if rank == 0:
                ch.send(msg)
                back = ch.recv()
                ok &= back == {"echo": msg}
            else:
                got = ch.recv()
                ch.send({"echo": got})
    return ok, (time.perf_counter() - t0) * 1e3 / (reps * len(sizes))


def main() -> int:
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    out: dict = {}
    sizes = [1, 100, 4096, 65536, 1 << 20]
    for kind in ("peer", "nccl"):
        ch = transport.make_channel(kind, rank=rank, peer=1 - rank, device=dev, poll_ms=50)
        round_trips(ch, rank, [16], 5)  # warm-up
        ok, ms = round_trips(ch, rank, sizes, 4)
        small_ok, small_ms = round_trips(ch, rank, [64], 50)
        out[kind] = {"intact": ok and small_ok, "mean_round_trip_ms_mixed": round(ms, 3),
                     "mean_round_trip_ms_64B": round(small_ms, 4)}
        if kind == "peer":
            # Rank 1 waits for a message that rank 0 does not send yet: bounded, reported, recoverable.
            if rank == 1:
                t0 = time.perf_counter()
                try:
                    ch.recv(timeout_s=0.5)
                    lost = False
                except mailbox.PeerLost:
                    lost = True
                waited = time.perf_counter() - t0
                ch.send({"lost": lost, "waited_s": waited})
                ch.send(ch.recv())  # echo the next message: the ring still works
            else:
                timeout_report = ch.recv()
                ch.send({"after": "timeout"})
                out["peer"]["silent_peer_timeout"] = {**timeout_report, "recovered": ch.recv() == {"after": "timeout"}}
        ch.close() if kind == "peer" else None
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
