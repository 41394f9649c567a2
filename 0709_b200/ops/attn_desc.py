"""Attention descriptor shared by every paged-attention kernel.

A batch of ``M`` query rows reads one paged KV cache.  Position ``x`` of
row ``r`` lives in ``prefix_pages[x // page]`` when ``x < shared_len`` or
``x // page < n_shared_pages``, and in ``tail_pages[r, x // page - n_shared_pages]``
otherwise (a route's private copy of the prefix's partial page holds the same
committed slots, so both views agree below ``shared_len``).  Key position ``x`` is
visible to row ``r`` when ``x < row_full[r]``, or when
``row_full[r] <= x < row_len[r]`` and bit ``x - mask_base`` of ``row_mask[r]``
is set (``row_mask`` is [M, W] int64 words, bit ``b`` of word ``b // 64``).  Positions ``[0, shared_len)`` are fully visible to every row and read
through ``prefix_pages`` -- the kernels process that range once for all rows
(split-KV on tensor cores) and the remaining per-row range separately.

- drafter decode: ``shared_len`` = committed prefix, ``row_full = row_len`` = route length;
- target tree verify: ``shared_len = row_full = mask_base`` = prefix, ``row_len`` =
  prefix + nodes, ``row_mask`` = ancestor masks;
- target AR / single sequence: ``row_full = row_len`` = position + 1.

This one descriptor replaces two reference structures: FlashInfer's paged-KV metadata
(``kv_indptr / kv_page_indices / kv_last_page_len``, built per batch from token-slot paths in
src/atlas_0709/flashinfer_paged/paged_metadata.py:32-120) and the verify tree's dense
``[N, prefix + N]`` custom mask (src/atlas_0709/flashinfer_full_verify.py:704-741).  The mask
here covers the node region only, one bit per key.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class AttnDesc:
    prefix_pages: torch.Tensor  # int32 [P_pages]
    n_shared_pages: int
    shared_len: int
    mask_base: int
    row_full: torch.Tensor  # int32 [M]
    row_len: torch.Tensor  # int32 [M]
    row_mask: torch.Tensor  # int64 [M, W]
    tail_pages: torch.Tensor  # int32 [M, T] (T >= 1)

    @property
    def rows(self) -> int:
        return int(self.row_len.numel())

    def max_len(self) -> int:
        return int(self.row_len.max().item()) if self.rows else 0


def single_sequence_desc(
    pages: torch.Tensor, lens: torch.Tensor, shared_len: int, *, mask_base: int = 0, masks: torch.Tensor | None = None,
    full: torch.Tensor | None = None,
) -> AttnDesc:
    """All rows read one page list (target verify, AR decode, prefill)."""
    m = int(lens.numel())
    dev = lens.device
    return AttnDesc(
        prefix_pages=pages,
        n_shared_pages=int(pages.numel()),
        shared_len=int(shared_len),
        mask_base=int(mask_base),
        row_full=lens.to(torch.int32) if full is None else full.to(torch.int32),
        row_len=lens.to(torch.int32),
        row_mask=(torch.full((m, 1), -1, dtype=torch.int64, device=dev) if masks is None else masks.to(torch.int64)),
        tail_pages=torch.zeros((m, 1), dtype=torch.int32, device=dev),
    )
