"""Host command channel from the root rank to tensor-parallel worker ranks.

The root rank runs the serving logic (routes, trie, selection); every model
call it makes on the sharded target must be repeated, in the same order, by
every worker rank on its own shard.  The root posts each call here: a
memory-mapped file in ``/dev/shm`` holding a header (sequence number, opcode,
payload length, root pid, heartbeat time), one acknowledgement word per rank
and a pickled payload.  Workers poll the sequence number (a few hundred
nanoseconds per poll), copy the payload, acknowledge, and run the call; the
root waits for every acknowledgement before it overwrites the payload.

Failure detection on the host: a worker that sees no new command checks every
second whether the root process is still alive and gives up with
``PeerLost`` when it is not (or after ``idle_timeout_s``); the root gives up
waiting for acknowledgements after ``ack_timeout_s``.  The payload ordering
relies on x86-64 total store order (payload written before the sequence word).
"""

from __future__ import annotations

import mmap
import os
import pickle
import time

import numpy as np

HEADER_WORDS = 8   # seq, op, nbytes, root_pid, heartbeat_ns, pad...
ACK_WORDS = 64
PAYLOAD_OFF = (HEADER_WORDS + ACK_WORDS) * 8

OP_STOP = 0
OP_CALL = 1


class PeerLost(RuntimeError):
    pass


def _pid_alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    return True


class Mailbox:
    def __init__(self, path: str, *, rank: int, world: int, create: bool, size: int = 8 << 20,
                 ack_timeout_s: float = 120.0, idle_timeout_s: float | None = None) -> None:
        self.path = path
        self.rank = int(rank)
        self.world = int(world)
        if world > ACK_WORDS:
            raise ValueError(f"at most {ACK_WORDS} ranks")
        self.ack_timeout_s = float(ack_timeout_s)
        self.idle_timeout_s = idle_timeout_s
        if create:
            fd = os.open(path, os.O_CREAT | os.O_RDWR | os.O_TRUNC, 0o600)
            os.ftruncate(fd, size)
        else:
            fd = os.open(path, os.O_RDWR)
            size = os.fstat(fd).st_size
        self.size = size
        self.mm = mmap.mmap(fd, size)
        os.close(fd)
        self.words = np.frombuffer(self.mm, dtype=np.int64, count=HEADER_WORDS + ACK_WORDS)
        self.owner = create
        if create:
            self.words[:] = 0
            self.words[3] = os.getpid()
        # Readers start from zero: a message posted before they attached is
        # still theirs (the writer waits for every reader's acknowledgement
        # before it overwrites the payload).
        self.seq = int(self.words[0]) if create else 0
        self.posted = 0

    # ------------------------------------------------------------- root
    def _wait_acks(self) -> None:
        if self.posted == 0:
            return
        acks = self.words[HEADER_WORDS: HEADER_WORDS + self.world]
        t0 = time.monotonic()
        spins = 0
        while True:
            if all(int(acks[r]) >= self.seq for r in range(1, self.world)):
                return
            spins += 1
            if spins % 1024 == 0:
                if time.monotonic() - t0 > self.ack_timeout_s:
                    missing = [r for r in range(1, self.world) if int(acks[r]) < self.seq]
                    raise PeerLost(f"tensor-parallel ranks {missing} did not acknowledge command {self.seq}")
                time.sleep(0)

    def post(self, op: int, payload: object = None) -> None:
        data = pickle.dumps(payload, protocol=pickle.HIGHEST_PROTOCOL)
        if PAYLOAD_OFF + len(data) > self.size:
            raise ValueError(f"command payload of {len(data)} bytes exceeds the mailbox")
        self._wait_acks()
        self.mm[PAYLOAD_OFF: PAYLOAD_OFF + len(data)] = data
        self.words[1] = op
        self.words[2] = len(data)
        self.words[4] = time.monotonic_ns()
        self.seq += 1
        self.words[0] = self.seq
        self.posted += 1

    def drain(self) -> None:
        """Wait until every worker has taken the last command."""
        self._wait_acks()

    # ----------------------------------------------------------- worker
    def receive(self) -> tuple[int, object]:
        t0 = time.monotonic()
        last_check = t0
        spins = 0
        while int(self.words[0]) == self.seq:
            spins += 1
            if spins % 4096 == 0:
                now = time.monotonic()
                if now - last_check > 1.0:
                    last_check = now
                    if not _pid_alive(int(self.words[3])):
                        raise PeerLost("the root rank exited without a stop command")
                    if self.idle_timeout_s is not None and now - t0 > self.idle_timeout_s:
                        raise PeerLost(f"no command from the root rank for {self.idle_timeout_s:.0f} s")
                time.sleep(0)
        self.seq = int(self.words[0])
        op = int(self.words[1])
        n = int(self.words[2])
        payload = pickle.loads(bytes(self.mm[PAYLOAD_OFF: PAYLOAD_OFF + n]))
        self.words[HEADER_WORDS + self.rank] = self.seq
        return op, payload

    @classmethod
    def attach(cls, path: str, *, rank: int, world: int, timeout_s: float = 120.0, **kw) -> "Mailbox":
        """Wait for the writer to create ``path``, then attach as reader ``rank``."""
        t0 = time.monotonic()
        while not (os.path.exists(path) and os.path.getsize(path) > PAYLOAD_OFF):
            if time.monotonic() - t0 > timeout_s:
                raise PeerLost(f"mailbox {path} was not created within {timeout_s:.0f} s")
            time.sleep(0.01)
        return cls(path, rank=rank, world=world, create=False, **kw)

    def close(self) -> None:
        try:
            self.words = None  # type: ignore[assignment]
            self.mm.close()
        except (BufferError, ValueError):
            pass
        if self.owner:
            try:
                os.unlink(self.path)
            except FileNotFoundError:
                pass
