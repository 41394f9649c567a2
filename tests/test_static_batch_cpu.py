"""The static batch's one input copy: fields, padding, auxiliary words and copy-on-write pages.

``StaticBatch.load`` packs every per-forward input (metadata, tokens,
positions, slots, row limits, tail pages, row masks and free-form auxiliary
words) into one host buffer and one host->device copy; ``run_rows(cow=...)``
sends the drafter's copy-on-write page list in those auxiliary words and
copies the pages before the forward.  CPU engine (torch ops), tiny model.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import mod


@pytest.fixture(scope="module")
def engine():
    llama = mod("models.llama")
    w = llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32, device=torch.device("cpu"))
    return mod("runtime.engine").LlamaEngine(w, num_pages=64, page_size=16, max_positions=1024)


def test_load_packs_fields_padding_and_aux(engine):
    sb = engine.static_batch(4, 3, 1)
    n = sb.load(tokens=[5, 6], positions=[10, 11], slots=[40, 41], shared_len=10, n_shared_pages=1, mask_base=10,
                row_full=[11, 12], row_len=[11, 12], tail_pages=np.array([[7, 8, 9], [1, 2, 3]]),
                row_mask=np.array([[1], [3]]), aux=np.array([9, 8, 7]))
    assert n == 2
    assert sb.tokens.tolist() == [5, 6, 0, 0]
    assert sb.slots.tolist() == [40, 41, engine.trash_slot, engine.trash_slot]
    assert sb.tail_pages.tolist() == [[7, 8, 9], [1, 2, 3], [0, 0, 0], [0, 0, 0]]
    assert sb.row_mask[:, 0].tolist() == [1, 3, -1, -1]
    assert sb.aux[:3].tolist() == [9, 8, 7]
    assert sb.dparams.tolist()[:3] == [10, 1, 10]
    # A second load with fewer rows re-pads the rows the first one used.
    sb.load(tokens=[4], positions=[12], slots=[42], shared_len=12, n_shared_pages=1, mask_base=12, row_full=[13],
            row_len=[13])
    assert sb.tokens.tolist() == [4, 0, 0, 0]
    assert sb.tail_pages.tolist() == [[0, 0, 0]] * 4
    assert sb.row_mask[:, 0].tolist() == [-1] * 4
    with pytest.raises(ValueError):
        sb.load(tokens=[1], positions=[1], slots=[1], shared_len=1, n_shared_pages=1, mask_base=1, row_full=[1],
                row_len=[1], aux=np.zeros(sb.aux.numel() + 1, dtype=np.int32))


def test_run_rows_applies_copy_on_write_pages_first(engine):
    kv = engine.kv
    g = torch.Generator().manual_seed(0)
    kv[:, 3].copy_(torch.randn(kv[:, 3].shape, generator=g))
    kv[:, 9].zero_()
    engine.run_rows(1, prefix_pages=torch.arange(8, dtype=torch.int32), tokens=[1], positions=[5], slots=[9 * 16 + 5],
                    shared_len=5, n_shared_pages=1, mask_base=5, row_full=[6], row_len=[6], cow=np.array([[3, 9, 5]]))
    # Tokens 0..4 of page 3 were copied to page 9 in every layer before the forward wrote token 5.
    assert torch.equal(kv[:, 9, :, :, :5], kv[:, 3, :, :, :5])
