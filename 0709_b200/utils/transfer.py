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
