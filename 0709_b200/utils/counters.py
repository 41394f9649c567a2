"""Process-wide counters: host<->device bytes on the hot path and kernel launches.

The runtimes call ``h2d``/``d2h`` where a round's inputs go to the device and
its results come back; ``CudaOps`` counts every launch of this package's
kernels.  Benchmarks read deltas around their timed region.

The reference keeps per-route-pool counters of the same kind (attention metadata builds,
copy-on-write pages, host transfer batches and elements:
src/atlas_0709/flashinfer_paged/sglang_runtime.py:110-126, 1094-1117); the drafter's
``hot_path_counters()`` reports those names, these counters add the byte totals.
"""

from __future__ import annotations

import threading

_LOCK = threading.Lock()
_C = {"h2d_bytes": 0, "d2h_bytes": 0, "launches": 0}


def h2d(nbytes: int) -> None:
    with _LOCK:
        _C["h2d_bytes"] += int(nbytes)


def d2h(nbytes: int) -> None:
    with _LOCK:
        _C["d2h_bytes"] += int(nbytes)


def launches(n: int = 1) -> None:
    with _LOCK:
        _C["launches"] += int(n)


def snapshot() -> dict[str, int]:
    with _LOCK:
        return dict(_C)


def delta(before: dict[str, int]) -> dict[str, int]:
    now = snapshot()
    return {k: now[k] - before.get(k, 0) for k in now}
