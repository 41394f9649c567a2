"""Multi-session serving: many independent ATLAS sessions on shared engines.

``MultiSessionTargetApp`` hosts one ``TargetVerifier`` per session over one
target engine and one page pool (pages return to the pool when a session is
released), behind the same ``prefill`` / ``verify`` / ``health`` calls as
the single-session server plus a ``session_id`` field and ``release``.
Requests are served one at a time (the GPU is shared).

``ShmChannel`` is a same-node transport for it: a request mailbox and a
response mailbox in ``/dev/shm`` (pickled dicts, a sequence word per
direction, bounded waits and peer-liveness checks; see
``parallel.mailbox``).  ``ShmTargetClient`` sends the committed prefix as
(length, last tokens) instead of the whole prefix every round.

The reference serves one session per target server (a global lock around
one backend, src/atlas_0709/rpc.py:66-128); this module is this framework's
data-parallel serving layer (several sessions per target engine, sessions spread over GPU pairs).
"""

from __future__ import annotations

import threading
import time
from typing import Any, Callable, Mapping, Sequence

from ..parallel.mailbox import OP_CALL, OP_STOP, Mailbox, PeerLost
from .rpc import TargetServerApp


class MultiSessionTargetApp:
    def __init__(self, factory: Callable[[str], Any], *, max_sessions: int = 64) -> None:
        self.factory = factory
        self.max_sessions = int(max_sessions)
        self.sessions: dict[str, TargetServerApp] = {}
        self.lock = threading.Lock()
        self.served = {"prefill": 0, "verify": 0, "release": 0}

    def _app(self, sid: str) -> TargetServerApp:
        app = self.sessions.get(sid)
        if app is None:
            if len(self.sessions) >= self.max_sessions:
                raise RuntimeError(f"session limit {self.max_sessions} reached")
            app = TargetServerApp(self.factory(sid))
            self.sessions[sid] = app
        return app

    @staticmethod
    def _sid(request: Mapping[str, Any] | None) -> str:
        return str((request or {}).get("session_id", "default"))

    def health(self, request: Mapping[str, Any] | None = None) -> dict[str, object]:
        from .rpc import CAPABILITIES

        return {"ok": True, "service": "atlas_0709_target_multi_session", "capabilities": list(CAPABILITIES),
                "sessions": sorted(self.sessions), "served": dict(self.served)}

    def prefill(self, request: Mapping[str, Any]) -> dict[str, object]:
        with self.lock:
            self.served["prefill"] += 1
            return {**self._app(self._sid(request)).prefill(request), "session_id": self._sid(request)}

    def verify(self, request: Mapping[str, Any]) -> dict[str, object]:
        with self.lock:
            self.served["verify"] += 1
            return {**self._app(self._sid(request)).verify(request), "session_id": self._sid(request)}

    def release(self, request: Mapping[str, Any]) -> dict[str, object]:
        sid = self._sid(request)
        with self.lock:
            app = self.sessions.pop(sid, None)
            if app is not None and hasattr(app.backend, "release"):
                app.backend.release()
            self.served["release"] += 1
        return {"ok": True, "session_id": sid, "released": app is not None}


class ShmChannel:
    """Request/response mailboxes between one client process and one server process.

    Each side creates the mailbox it writes and attaches to the one it reads
    (waiting for the peer to create it), so either side may start first.
    """

    def __init__(self, base_path: str, *, server: bool, timeout_s: float = 600.0) -> None:
        mine, theirs = (".resp", ".req") if server else (".req", ".resp")
        self.out = Mailbox(base_path + mine, rank=0, world=2, create=True, ack_timeout_s=timeout_s)
        self.inp = Mailbox.attach(base_path + theirs, rank=1, world=2, timeout_s=timeout_s)
        self.req, self.resp = (self.inp, self.out) if server else (self.out, self.inp)

    def close(self) -> None:
        self.out.close()
        self.inp.close()


def serve_target_shm(app, channel: ShmChannel) -> int:
    """Serve requests until the client posts stop; errors go back as ``{"ok": False, "error": ...}``."""
    n = 0
    while True:
        op, payload = channel.req.receive()
        if op == OP_STOP:
            channel.resp.post(OP_STOP, None)
            return n
        name, request = payload
        try:
            out = getattr(app, name)(request)
        except Exception as exc:  # noqa: BLE001 - the error travels to the client
            out = {"ok": False, "error": repr(exc)}
        channel.resp.post(OP_CALL, out)
        n += 1


class ShmTargetClient:
    """Target client over ``ShmChannel`` with the generator interface; one session id per client."""

    def __init__(self, channel: ShmChannel, *, session_id: str = "default", tail: int = 8,
                 lock: threading.Lock | None = None) -> None:
        self.ch = channel
        self.session_id = str(session_id)
        self.tail = int(tail)
        # Clients of one channel in several threads share one lock (one request in flight).
        self.lock = lock or threading.Lock()
        self.calls = 0
        self.wait_s = 0.0

    def _call(self, name: str, request: dict[str, object]) -> dict[str, object]:
        request = {**request, "session_id": self.session_id}
        with self.lock:
            t0 = time.perf_counter()
            self.ch.req.post(OP_CALL, (name, request))
            op, out = self.ch.resp.receive()
            self.wait_s += time.perf_counter() - t0
        self.calls += 1
        if op == OP_STOP:
            raise PeerLost("target server stopped")
        if not out.get("ok"):
            raise RuntimeError(f"target {name} failed: {out.get('error', out)}")
        return out

    def health(self) -> dict[str, object]:
        return self._call("health", {})

    def prefill(self, prompt_token_ids: Sequence[int]) -> dict[str, object]:
        return self._call("prefill", {"prompt_token_ids": [int(t) for t in prompt_token_ids]})

    def verify(self, *, prefix_token_ids, routes, fallback_max_tokens=None, selected_path_max_tokens=None,
               eos_token_id=None, route_sampling_seed=None, route_sampling_round=None) -> dict[str, object]:
        prefix = list(prefix_token_ids)
        req: dict[str, object] = {"prefix_len": len(prefix), "prefix_tail_token_ids": prefix[-self.tail:],
                                  "routes": [dict(r) for r in routes]}
        for key, val in (("fallback_max_tokens", fallback_max_tokens),
                         ("selected_path_max_tokens", selected_path_max_tokens), ("eos_token_id", eos_token_id),
                         ("route_sampling_seed", route_sampling_seed),
                         ("route_sampling_round", route_sampling_round)):
            if val is not None:
                req[key] = int(val)
        return self._call("verify", req)

    def release(self) -> dict[str, object]:
        return self._call("release", {})

    def stop_server(self) -> None:
        with self.lock:
            self.ch.req.post(OP_STOP, None)
            self.ch.resp.receive()
