"""The allocation-free top-k entry point, called through its exported C symbol.

Callers that cannot allocate device memory while serving (a fixed device-memory
budget accounted at start-up, a foreign runtime that owns the allocator, plain
C/C++ hosts without PyTorch's allocator) use ``atlas_topk_logprobs_noalloc``,
whose scratch is a fixed device array inside the library.  This file is named
to be collected last, so a run that stops at the first failure has already run
every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import mod

pytestmark = pytest.mark.gpu

OK, EINVAL, ETOOLARGE = 0, -1, -2


@pytest.fixture(scope="module")
def entry():
    ext = mod("ops._native").cuda()  # loads the library (and its PyTorch dependencies) first
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.atlas_topk_logprobs_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_float,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def call(fn, logits, k, keys=None, inv_temp=1.0):
    rows, vocab = logits.shape
    lp = torch.empty(rows, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(rows, k, dtype=torch.int64, device=logits.device)
    rc = fn(logits.data_ptr(), rows, vocab, k, None if keys is None else keys.data_ptr(), inv_temp, lp.data_ptr(),
            ids.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return rc, lp, ids


@pytest.mark.parametrize("rows,vocab,k,sampled", [(12, 128256, 4, False), (1, 128256, 1, False), (9, 50000, 3, True)])
def test_matches_existing_entry_point_twice(entry, rows, vocab, k, sampled):
    ops = mod("ops.cuda_ops").CudaOps(device=torch.device("cuda"))
    g = torch.Generator(device="cuda").manual_seed(rows * 31 + vocab)
    logits = torch.randn(rows, vocab, device="cuda", generator=g) * 3
    keys = torch.arange(rows, dtype=torch.int64, device="cuda") * 7919 + 11 if sampled else None
    ref_lp, ref_ids = ops.topk_logprobs(logits, k, keys, 0.8 if sampled else 1.0)
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        rc, lp, ids = call(entry, logits, k, keys, 1.0 / 0.8 if sampled else 1.0)
        torch.cuda.synchronize()
        assert rc == OK
        assert torch.equal(ids, ref_ids)
        assert torch.allclose(lp, ref_lp, atol=1e-4)


def test_rejects_sizes_beyond_the_fixed_scratch(entry):
    logits = torch.zeros(5000, 1024, device="cuda")  # one chunk per row: 5000 records > 4096
    rc, _, _ = call(entry, logits, 2)
    assert rc == ETOOLARGE
    rc, _, _ = call(entry, logits[:4], 9)
    assert rc == EINVAL
