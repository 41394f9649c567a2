"""Host -> device copies of token ids for the serving path.

A prompt (or a fallback suffix) arrives as host integers; it is staged in
pinned (page-locked) host memory and copied asynchronously on the current
stream, so the copy overlaps whatever the host does next.  PyTorch's caching
host allocator keeps the pinned block alive until the copy has completed.
Every copy is counted in ``utils.counters`` (the benchmarks report bytes per
request).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from . import counters


def ids_to_device(ids: Sequence[int] | torch.Tensor, device: torch.device) -> torch.Tensor:
    """``ids`` as an int32 tensor on ``device`` (pinned staging + async copy on CUDA)."""
    host = ids.to(torch.int32) if isinstance(ids, torch.Tensor) else torch.tensor(list(ids), dtype=torch.int32)
    if torch.device(device).type != "cuda":
        return host
    if host.device.type != "cpu":
        return host.to(device)
    staged = host.pin_memory()
    counters.h2d(staged.numel() * staged.element_size())
    return staged.to(device, non_blocking=True)


ERROR_NAMES = {
    1: "bounded wait timed out (mbarrier or peer flag)",
    2: "index out of range",
    3: "unsupported configuration",
    4: "peer rank did not deliver its partial in time",
}


class KernelError(RuntimeError):
    """A kernel recorded an error in its device flag (it never traps; it reports and returns)."""

    def __init__(self, code: int, where: str = "") -> None:
        self.code = int(code)
        name = ERROR_NAMES.get(self.code, "unknown")
        super().__init__(f"device kernel reported error {self.code}: {name}" + (f" ({where})" if where else ""))


def _as_words(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().reshape(-1)
    if t.dtype == torch.float32 or t.dtype == torch.int32:
        return t.contiguous().view(torch.int32)
    if t.dtype == torch.int64:
        return t.to(torch.int32)  # token ids and small indices
    raise TypeError(f"read_back packs int32, int64 and float32 tensors, got {t.dtype}")


def read_back(parts: Sequence[torch.Tensor], status: torch.Tensor | None = None, *,
              where: str = "") -> list[np.ndarray]:
    """One device->host copy of small result tensors, with the device error flag riding along.

    ``parts`` (int32, int64 holding values below 2^31, or float32) are packed into
    one int32 buffer together with ``status`` (the int32 error flag the kernels
    write instead of trapping), copied with a single wait, and unpacked as numpy
    arrays of each part's shape (int64 parts come back as int64).  A nonzero flag
    is cleared and raised as ``KernelError`` before the caller can act on the
    values, so no token computed after a device fault is committed.  The reference
    packs a depth's candidates the same way, float64 bits in int64 words
    (src/atlas_0709/flashinfer_paged/frontier.py:192-307,
    src/atlas_0709/flashinfer_paged/utils.py:135-151), without a status word.
    """
    words = [_as_words(p) for p in parts]
    if status is not None:
        words.append(status.reshape(-1)[:1].to(torch.int32))
    packed = torch.cat(words) if len(words) > 1 else words[0]
    if packed.device.type != "cpu":
        counters.d2h(packed.numel() * 4)
    host = packed.cpu().numpy()
    if status is not None:
        code = int(host[-1])
        if code:
            status.zero_()
            raise KernelError(code, where)
    out: list[np.ndarray] = []
    off = 0
    for p in parts:
        n = p.numel()
        chunk = host[off: off + n]
        off += n
        if p.dtype == torch.float32:
            arr = chunk.view(np.float32)
        elif p.dtype == torch.int64:
            arr = chunk.astype(np.int64)
        else:
            arr = chunk.copy()
        out.append(arr.reshape(tuple(p.shape)))
    return out
