"""Target transport: JSON wire format, HTTP server/client, in-process client.

Endpoints (wire-compatible with the reference's Target service):
``GET /health``, ``POST /prefill`` ``{"prompt_token_ids": [...]}``,
``POST /verify`` ``{"prefix_token_ids", "routes", "fallback_max_tokens",
"selected_path_max_tokens", "eos_token_id", "route_sampling_seed",
"route_sampling_round"}``.  Errors come back as HTTP 500 with ``repr(exc)``.

Beyond the reference, ``/verify`` accepts ``prefix_len`` plus
``prefix_tail_token_ids`` instead of the full prefix (the server checks the
length and the tail), so a long prefix is not re-sent every round.

Parity: reference src/atlas_0709/rpc.py:15-309.
"""

from __future__ import annotations

import json
import threading
import urllib.error
import urllib.request
from dataclasses import dataclass
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any, Mapping, Sequence

from ..types import TargetRouteScore, TargetVerifyResult, verify_payload_from_mapping


def target_score_to_dict(score: TargetRouteScore) -> dict[str, object]:
    return {
        "route_id": int(score.route_id),
        "token_ids": [int(t) for t in score.token_ids],
        "target_logprob": float(score.target_logprob),
        "draft_logprob": float(score.draft_path_logprob),
        "draft_path_logprob": float(score.draft_path_logprob),
        "legacy_cumulative_draft_logprob": float(score.draft_logprob),
        "token_logprobs": [float(v) for v in score.token_logprobs],
        "first_token_logprob": None if score.first_token_logprob is None else float(score.first_token_logprob),
        "selection_score": None if score.selection_score is None else float(score.selection_score),
        "score_weights": [float(v) for v in score.score_weights],
        "draft_token_logprobs": [float(v) for v in score.draft_token_logprobs],
        "draft_first_token_logprob": score.draft_first_token_logprob,
    }


def target_verify_result_to_dict(result: TargetVerifyResult) -> dict[str, object]:
    out: dict[str, object] = {
        "decision": str(result.decision),
        "scores": [target_score_to_dict(s) for s in result.scores],
        "metadata": dict(result.metadata),
    }
    if result.decision == "fallback_ar":
        out.update(
            {
                "selected_route_id": None,
                "fallback_token_ids": [int(t) for t in result.fallback_token_ids],
                "fallback_reason": result.fallback_reason,
            }
        )
    else:
        out.update(
            {
                "selected_route_id": int(result.selected_route_id),
                "selected_score": target_score_to_dict(result.selected_score),
            }
        )
    return out


def selected_route_id_from_response(response: Mapping[str, object]) -> int:
    if str(response.get("decision", "select")) != "select":
        raise ValueError(f"no route was selected (decision {response.get('decision')!r})")
    return int(response["selected_route_id"])


# What this server understands beyond the reference's wire format (reported by /health, so a
# client sends the compact forms only to a server that announced them).
CAPABILITIES = ("prefix_tail_token_ids",)


def _opt_int(v) -> int | None:
    return None if v is None else int(v)


def _resolve_prefix(backend, request: Mapping[str, Any]) -> list[int]:
    prefix = request.get("prefix_token_ids")
    if isinstance(prefix, list):
        return [int(t) for t in prefix]
    n = request.get("prefix_len")
    tail = request.get("prefix_tail_token_ids", [])
    if n is None or not isinstance(tail, list):
        raise ValueError("a verify request names its committed prefix: prefix_token_ids, or prefix_len with prefix_tail_token_ids")
    have = list(backend.prefix_token_ids)
    if int(n) != len(have) or (tail and have[-len(tail):] != [int(t) for t in tail]):
        raise RuntimeError(
            "the request's committed prefix differs from the one whose KV the target holds (it never re-prefills silently): "
            f"request_len={int(n)}, target_len={len(have)}"
        )
    return have


@dataclass
class TargetServerApp:
    backend: Any

    def __post_init__(self) -> None:
        self.lock = threading.Lock()

    def health(self) -> dict[str, object]:
        return {"ok": True, "service": "atlas_0709_target", "capabilities": list(CAPABILITIES),
                "metadata": self.backend.runtime_metadata()}

    def prefill(self, request: Mapping[str, Any]) -> dict[str, object]:
        toks = request.get("prompt_token_ids")
        if not isinstance(toks, list):
            raise ValueError("a prefill request carries prompt_token_ids as a list of ints")
        with self.lock:
            st = self.backend.prefill([int(t) for t in toks])
        return {"ok": True, "prompt_len": int(st.committed_length), "metadata": dict(st.metadata)}

    def verify(self, request: Mapping[str, Any]) -> dict[str, object]:
        routes = request.get("routes")
        if not isinstance(routes, list):
            raise ValueError("a verify request carries routes as a list of objects")
        payloads = [verify_payload_from_mapping(dict(r)) for r in routes]
        with self.lock:
            prefix = _resolve_prefix(self.backend, request)
            result = self.backend.verify_payloads(
                prefix_token_ids=prefix,
                routes=payloads,
                fallback_max_tokens=_opt_int(request.get("fallback_max_tokens")),
                selected_path_max_tokens=_opt_int(request.get("selected_path_max_tokens")),
                eos_token_id=_opt_int(request.get("eos_token_id")),
                route_sampling_seed=_opt_int(request.get("route_sampling_seed")),
                route_sampling_round=_opt_int(request.get("route_sampling_round")),
            )
        return {"ok": True, **target_verify_result_to_dict(result)}


@dataclass
class InProcessTargetClient:
    """Target client with the generator interface, without HTTP or JSON encoding.

    It reports the verify decision early (``on_decision``), before the target
    runs its fallback AR, so the generator can stop speculative forest work
    that a fallback round discards anyway.
    """

    backend: Any
    supports_early_decision = True

    def health(self) -> dict[str, object]:
        return {
            "ok": True,
            "service": "atlas_0709_target_in_process",
            "transport": "in_process",
            "metadata": self.backend.runtime_metadata(),
        }

    def prefill(self, prompt_token_ids: Sequence[int]) -> dict[str, object]:
        st = self.backend.prefill(prompt_token_ids)
        return {"ok": True, "prompt_len": int(st.committed_length), "metadata": dict(st.metadata)}

    def verify(self, *, prefix_token_ids, routes, fallback_max_tokens=None, selected_path_max_tokens=None,
               eos_token_id=None, route_sampling_seed=None, route_sampling_round=None,
               on_decision=None) -> dict[str, object]:
        result = self.backend.verify_payloads(
            prefix_token_ids=prefix_token_ids,
            routes=[verify_payload_from_mapping(dict(r)) for r in routes],
            fallback_max_tokens=fallback_max_tokens,
            selected_path_max_tokens=selected_path_max_tokens,
            eos_token_id=eos_token_id,
            route_sampling_seed=route_sampling_seed,
            route_sampling_round=route_sampling_round,
            on_decision=on_decision,
        )
        return {"ok": True, **target_verify_result_to_dict(result)}


def make_target_handler(app: TargetServerApp) -> type[BaseHTTPRequestHandler]:
    class Handler(BaseHTTPRequestHandler):
        server_version = "AtlasB200TargetRPC/1.0"

        def do_GET(self) -> None:  # noqa: N802
            if self.path == "/health":
                self._write(200, app.health())
            else:
                self._write(404, {"ok": False, "error": f"unknown endpoint: {self.path}"})

        def do_POST(self) -> None:  # noqa: N802
            try:
                body = self._read()
                if self.path == "/prefill":
                    resp = app.prefill(body)
                elif self.path == "/verify":
                    resp = app.verify(body)
                elif self.path == "/release" and hasattr(app, "release"):
                    resp = app.release(body)  # multi-session servers: end a session, free its pages
                else:
                    self._write(404, {"ok": False, "error": f"unknown endpoint: {self.path}"})
                    return
                self._write(200, resp)
            except Exception as exc:  # noqa: BLE001 - the wire contract reports any failure
                self._write(500, {"ok": False, "error": repr(exc)})

        def log_message(self, fmt: str, *args: object) -> None:
            if getattr(app, "verbose", False):
                print(f"[target-rpc] {self.address_string()} - {fmt % args}", flush=True)

        def _read(self) -> dict[str, Any]:
            n = int(self.headers.get("content-length", "0"))
            return json.loads(self.rfile.read(n).decode("utf-8")) if n > 0 else {}

        def _write(self, status: int, payload: Mapping[str, Any]) -> None:
            data = json.dumps(payload, ensure_ascii=False).encode("utf-8")
            self.send_response(status)
            self.send_header("content-type", "application/json; charset=utf-8")
            self.send_header("content-length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

    return Handler


def make_server(app: TargetServerApp, *, host: str, port: int) -> ThreadingHTTPServer:
    return ThreadingHTTPServer((host, int(port)), make_target_handler(app))


def serve_target(app: TargetServerApp, *, host: str, port: int) -> None:
    server = make_server(app, host=host, port=port)
    meta = app.backend.runtime_metadata() if hasattr(app, "backend") else app.health()
    print(json.dumps({"service": "atlas_0709_target", "host": host, "port": int(server.server_address[1]),
                      "metadata": meta}, indent=2, sort_keys=True), flush=True)
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        server.server_close()


class RemoteTargetClient:
    """HTTP client; ``session_id`` (optional) addresses one session of a multi-session server.

    ``prefix_tail`` (default 8): when the server's ``/health`` announces ``prefix_tail_token_ids``,
    a verify request carries the prefix length and its last ``prefix_tail`` tokens instead of the
    whole committed prefix (the server checks both against the prefix whose KV it holds), so a
    round's request no longer grows with the context.  ``None`` always sends the full prefix (the
    reference's wire format, which every server accepts).
    """

    def __init__(self, base_url: str, *, timeout: float = 600.0, session_id: str | None = None,
                 prefix_tail: int | None = 8) -> None:
        self.base_url = base_url.rstrip("/")
        self.timeout = float(timeout)
        self.session_id = session_id
        self.prefix_tail = None if prefix_tail is None else max(1, int(prefix_tail))
        self._compact: bool | None = None  # learned from /health on the first verify

    def health(self) -> dict[str, object]:
        with urllib.request.urlopen(f"{self.base_url}/health", timeout=self.timeout) as r:
            return json.loads(r.read().decode("utf-8"))

    def prefill(self, prompt_token_ids: Sequence[int]) -> dict[str, object]:
        return self._post("/prefill", {"prompt_token_ids": [int(t) for t in prompt_token_ids]})

    def verify(self, *, prefix_token_ids, routes, fallback_max_tokens=None, selected_path_max_tokens=None,
               eos_token_id=None, route_sampling_seed=None, route_sampling_round=None) -> dict[str, object]:
        prefix = [int(t) for t in prefix_token_ids]
        if self._compact is None:
            self._compact = self.prefix_tail is not None and "prefix_tail_token_ids" in (
                self.health().get("capabilities") or [])
        if self._compact:
            payload: dict[str, object] = {"prefix_len": len(prefix),
                                          "prefix_tail_token_ids": prefix[-self.prefix_tail:]}
        else:
            payload = {"prefix_token_ids": prefix}
        payload["routes"] = [dict(r) for r in routes]
        for key, val in (
            ("fallback_max_tokens", fallback_max_tokens),
            ("selected_path_max_tokens", selected_path_max_tokens),
            ("eos_token_id", eos_token_id),
            ("route_sampling_seed", route_sampling_seed),
            ("route_sampling_round", route_sampling_round),
        ):
            if val is not None:
                payload[key] = int(val)
        return self._post("/verify", payload)

    def release(self) -> dict[str, object]:
        return self._post("/release", {})

    def _post(self, path: str, payload: Mapping[str, object]) -> dict[str, object]:
        if self.session_id is not None:
            payload = {**payload, "session_id": self.session_id}
        req = urllib.request.Request(
            f"{self.base_url}{path}",
            data=json.dumps(payload).encode("utf-8"),
            headers={"content-type": "application/json; charset=utf-8"},
            method="POST",
        )
        try:
            with urllib.request.urlopen(req, timeout=self.timeout) as r:
                out = json.loads(r.read().decode("utf-8"))
        except urllib.error.HTTPError as exc:
            body = exc.read().decode("utf-8", errors="replace")
            raise RuntimeError(f"target RPC {path} failed with HTTP {exc.code}: {body}") from exc
        if not out.get("ok"):
            raise RuntimeError(f"target RPC {path} failed: {out}")
        return out
