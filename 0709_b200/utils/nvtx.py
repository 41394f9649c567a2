"""Optional NVTX ranges (``ATLAS_NVTX=1``) around serving phases, for Nsight timelines.

Zero cost when disabled: the context manager does nothing.  The reference has no NVTX
ranges; its timing is host ``perf_counter`` spans (src/atlas_0709/edge_timeline.py:11-126),
which ``utils/timeline.py`` keeps.
"""

from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("ATLAS_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx_range(name: str):
    if ENABLED and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
