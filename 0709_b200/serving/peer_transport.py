"""Drafter <-> target transport between two GPUs: message rings in peer memory (NCCL p2p as baseline).

Split placement of the 1B + 8B configuration: the drafter (and the coordinator) on one GPU,
the target on another, one process per GPU.  ``PeerChannel`` moves each
request and response through a ring in the RECEIVER's GPU memory, mapped into
the sender by CUDA IPC (``csrc/cuda/peer_ring.cu``): the sender's kernel stores
the message over NVLink and publishes a sequence number with a system-scope
release.  The receiving host watches that flag with 4-byte copies (the copy
engine: no SM is held while it waits, so a GPU serving other sessions keeps all
of its SMs) and then launches the receive kernel, which re-checks the flag with
bounded acquire polls, copies the message out and reports a timeout in the
ring's own error flag instead of hanging.  Between checks the host also makes
sure that the peer process is alive, so a lost peer ends in ``PeerLost`` after
``timeout_s``, not in a hang.

``NcclChannel`` is the library baseline: the same messages as uint8 tensors
through ``torch.distributed`` point-to-point ``send``/``recv``.

Messages are pickled dicts (``TargetServerApp`` requests and responses; the
client sends the committed prefix as its length plus its last tokens).  The
reference's transport between these two processes is HTTP JSON
(src/atlas_0709/rpc.py:245-303, driven from src/atlas_0709/distributed_system.py:282-336).
"""

from __future__ import annotations

import os
import pickle
import struct
import threading
import time
from typing import Any, Sequence

import numpy as np
import torch
import torch.distributed as dist

from ..parallel.mailbox import PeerLost, _pid_alive

HEADER = 16            # {payload bytes, sequence number, 0, 0}
RING_SLOT_OFFSET = 256
PEER_TIMEOUT = 4       # kErrPeerTimeout
STOP = "__stop__"


def _align16(n: int) -> int:
    return (n + 15) // 16 * 16


class PeerChannel:
    """Two one-message rings between this rank and ``peer`` (one in each GPU's memory).

    Every rank of the pair constructs it with the same ``group``; the ring
    handles and process ids are exchanged with ``all_gather_object``.
    """

    def __init__(self, *, rank: int, peer: int, device: torch.device, capacity: int = 4 << 20, group=None,
                 timeout_s: float = 600.0, poll_ms: float = 200.0, idle_sleep_us: float = 20.0) -> None:
        from ..ops import _native

        self.ext = _native.cuda()
        self.rank, self.peer = int(rank), int(peer)
        self.device = torch.device(device)
        self.dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.capacity = int(capacity)
        self.timeout_s = float(timeout_s)
        self.poll_ns = int(poll_ms * 1e6)
        self.stream = torch.cuda.Stream(device=self.device)
        nbytes = RING_SLOT_OFFSET + HEADER + self.capacity
        self.ring = self.ext.ipc_malloc(nbytes, self.dev_index)   # where the peer writes to us
        world = dist.get_world_size(group)
        infos: list = [None] * world
        dist.all_gather_object(infos, (self.rank, os.getpid(), self.ext.ipc_handle(self.ring, self.dev_index)),
                               group=group)
        peer_info = next(i for i in infos if i[0] == self.peer)
        self.peer_pid = int(peer_info[1])
        self.peer_ring = self.ext.ipc_open(peer_info[2], self.dev_index)  # where we write to the peer
        cap = HEADER + self.capacity
        self.stage_host = torch.empty(cap, dtype=torch.uint8).pin_memory()
        self.stage_dev = torch.empty(cap, dtype=torch.uint8, device=self.device)
        self.recv_dev = torch.empty(cap, dtype=torch.uint8, device=self.device)
        self.recv_host = torch.empty(cap, dtype=torch.uint8).pin_memory()
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)  # payload bytes, error
        # The receive ring's sequence flag, read by a 4-byte copy (the copy engine, no SM) while a
        # message is awaited; the bounded pop kernel is launched only once it has arrived, so a
        # waiting receiver holds no SM of a GPU that serves other sessions meanwhile.
        self.flag_dev = self.ext.wrap_ptr(self.ring, [1], torch.int32, self.dev_index)
        self.flag_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.idle_sleep_s = float(idle_sleep_us) * 1e-6
        self.group = group
        self.sent = 0
        self.received = 0
        self.stats = {"messages_sent": 0, "messages_received": 0, "bytes_sent": 0, "bytes_received": 0,
                      "idle_polls": 0}
        dist.barrier(group=group)

    # ------------------------------------------------------------------ send
    def send(self, obj: Any) -> None:
        data = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)
        if len(data) > self.capacity:
            raise ValueError(f"message of {len(data)} bytes exceeds the ring capacity {self.capacity}")
        self.sent += 1
        total = _align16(HEADER + len(data))
        view = self.stage_host.numpy()
        view[:HEADER] = np.frombuffer(struct.pack("<IIII", len(data), self.sent & 0xFFFFFFFF, 0, 0), dtype=np.uint8)
        view[HEADER:HEADER + len(data)] = np.frombuffer(data, dtype=np.uint8)
        with torch.cuda.stream(self.stream):
            self.stage_dev[:total].copy_(self.stage_host[:total], non_blocking=True)
            self.ext.ring_push(self.stage_dev.data_ptr(), total, self.peer_ring, self.sent & 0xFFFFFFFF,
                               self.dev_index)
        self.stream.synchronize()  # the staging buffers are reused by the next message
        self.stats["messages_sent"] += 1
        self.stats["bytes_sent"] += len(data)

    # --------------------------------------------------------------- receive
    def _arrived(self, seq: int) -> bool:
        """Whether the ring's flag shows message ``seq`` (a hint; the pop kernel re-checks it)."""
        with torch.cuda.stream(self.stream):
            self.flag_host.copy_(self.flag_dev, non_blocking=True)
        self.stream.synchronize()
        return ((int(self.flag_host[0]) & 0xFFFFFFFF) - seq) & 0xFFFFFFFF < 0x80000000

    def recv(self, timeout_s: float | None = None) -> Any:
        limit = self.timeout_s if timeout_s is None else float(timeout_s)
        seq = (self.received + 1) & 0xFFFFFFFF
        t0 = time.monotonic()
        polls = 0
        while not self._arrived(seq):
            polls += 1
            if polls % 256 == 0:
                if not _pid_alive(self.peer_pid):
                    raise PeerLost(f"peer process {self.peer_pid} (rank {self.peer}) is gone")
                if time.monotonic() - t0 > limit:
                    raise PeerLost(f"no message from rank {self.peer} within {limit:.0f} s")
            time.sleep(self.idle_sleep_s)
        self.stats["idle_polls"] += polls
        while True:
            with torch.cuda.stream(self.stream):
                self.ext.ring_pop(self.ring, seq, self.recv_dev.data_ptr(), self.recv_dev.numel(),
                                  self.status[0:1], self.status[1:2], self.poll_ns)
                stat = self.status.cpu()
            n, err = int(stat[0]), int(stat[1])
            if err == 0 and n >= 0:
                break
            if err != PEER_TIMEOUT:
                self.status.zero_()
                raise RuntimeError(f"peer ring reported error {err} (message {seq}, {n} bytes)")
            self.status.zero_()
            self.stats["idle_polls"] += 1
            if not _pid_alive(self.peer_pid):
                raise PeerLost(f"peer process {self.peer_pid} (rank {self.peer}) is gone")
            if time.monotonic() - t0 > limit:
                raise PeerLost(f"no message from rank {self.peer} within {limit:.0f} s")
        total = _align16(HEADER + n)
        with torch.cuda.stream(self.stream):
            self.recv_host[:total].copy_(self.recv_dev[:total], non_blocking=True)
        self.stream.synchronize()
        self.received += 1
        self.stats["messages_received"] += 1
        self.stats["bytes_received"] += n
        return pickle.loads(self.recv_host.numpy()[HEADER:HEADER + n].tobytes())

    def close(self) -> None:
        """Unmap the peer's ring, wait until the peer has unmapped ours, then free ours (every rank calls it)."""
        if self.peer_ring:
            torch.cuda.synchronize(self.device)
            self.ext.ipc_close(self.peer_ring, self.dev_index)
            self.peer_ring = 0
        dist.barrier(group=self.group)
        if self.ring:
            self.ext.ipc_free(self.ring, self.dev_index)
            self.ring = 0


class NcclChannel:
    """The same messages through NCCL (or gloo) point-to-point send/recv: size first, then the bytes."""

    def __init__(self, *, rank: int, peer: int, device: torch.device, group=None, **_: Any) -> None:
        self.rank, self.peer = int(rank), int(peer)
        self.device = torch.device(device)
        self.group = group
        self.stats = {"messages_sent": 0, "messages_received": 0, "bytes_sent": 0, "bytes_received": 0}

    def send(self, obj: Any) -> None:
        data = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)
        size = torch.tensor([len(data)], dtype=torch.int64, device=self.device)
        payload = torch.frombuffer(bytearray(data), dtype=torch.uint8).to(self.device)
        dist.send(size, self.peer, group=self.group)
        dist.send(payload, self.peer, group=self.group)
        self.stats["messages_sent"] += 1
        self.stats["bytes_sent"] += len(data)

    def recv(self, timeout_s: float | None = None) -> Any:
        size = torch.zeros(1, dtype=torch.int64, device=self.device)
        dist.recv(size, self.peer, group=self.group)
        n = int(size.item())
        payload = torch.empty(n, dtype=torch.uint8, device=self.device)
        dist.recv(payload, self.peer, group=self.group)
        self.stats["messages_received"] += 1
        self.stats["bytes_received"] += n
        return pickle.loads(payload.cpu().numpy().tobytes())

    def close(self) -> None:
        pass


def make_channel(kind: str, **kw):
    if kind == "peer":
        return PeerChannel(**kw)
    if kind == "nccl":
        return NcclChannel(**kw)
    raise ValueError(f"unknown channel kind {kind!r} (peer or nccl)")


class ChannelTargetClient:
    """Target client (generator interface) over a channel to a ``serve_target_channel`` loop."""

    supports_early_decision = False

    def __init__(self, channel, *, tail: int = 8, session_id: str | None = None, lock=None) -> None:
        """``session_id`` addresses one session of a multi-session server; clients of one channel
        in several threads share ``lock`` (one request in flight per channel)."""
        self.ch = channel
        self.tail = int(tail)
        self.session_id = session_id
        self.lock = lock if lock is not None else threading.Lock()
        self.calls = 0
        self.wait_s = 0.0

    def _call(self, name: str, request: dict[str, Any]) -> dict[str, Any]:
        if self.session_id is not None:
            request = {**request, "session_id": self.session_id}
        with self.lock:
            t0 = time.perf_counter()
            self.ch.send((name, request))
            out = self.ch.recv()
            self.wait_s += time.perf_counter() - t0
        self.calls += 1
        if not out.get("ok"):
            raise RuntimeError(f"target {name} failed: {out.get('error', out)}")
        return out

    def health(self) -> dict[str, Any]:
        return {**self._call("health", {}), "transport": type(self.ch).__name__}

    def prefill(self, prompt_token_ids: Sequence[int]) -> dict[str, Any]:
        return self._call("prefill", {"prompt_token_ids": [int(t) for t in prompt_token_ids]})

    def verify(self, *, prefix_token_ids, routes, fallback_max_tokens=None, selected_path_max_tokens=None,
               eos_token_id=None, route_sampling_seed=None, route_sampling_round=None, **_: Any) -> dict[str, Any]:
        prefix = list(prefix_token_ids)
        req: dict[str, Any] = {"prefix_len": len(prefix), "prefix_tail_token_ids": prefix[-self.tail:],
                               "routes": [dict(r) for r in routes]}
        for key, val in (("fallback_max_tokens", fallback_max_tokens),
                         ("selected_path_max_tokens", selected_path_max_tokens), ("eos_token_id", eos_token_id),
                         ("route_sampling_seed", route_sampling_seed),
                         ("route_sampling_round", route_sampling_round)):
            if val is not None:
                req[key] = int(val)
        return self._call("verify", req)

    def call(self, name: str, request: dict[str, Any] | None = None) -> dict[str, Any]:
        """Any other server operation (``serve_target_channel``'s ``extra`` handlers)."""
        return self._call(name, dict(request or {}))

    def stop_server(self) -> None:
        with self.lock:
            self.ch.send((STOP, {}))
            self.ch.recv()


def serve_target_channel(app, channel, *, extra: dict | None = None) -> int:
    """Serve ``app`` (a ``TargetServerApp``) over ``channel`` until the client stops it.

    ``extra`` maps further operation names to handlers ``fn(request) -> dict``.
    Errors travel back to the client as ``{"ok": False, "error": ...}``.
    """
    handlers = dict(extra or {})
    served = 0
    while True:
        name, request = channel.recv()
        if name == STOP:
            channel.send({"ok": True, "served": served})
            return served
        try:
            fn = handlers.get(name) or getattr(app, name)
            out = fn(request) if name != "health" else fn()
        except Exception as exc:  # noqa: BLE001 - reported to the client
            out = {"ok": False, "error": repr(exc)}
        channel.send(out)
        served += 1
