"""Cross-GPU waits give up after their run-time limit and report, on one GPU.

The fused tensor-parallel kernels wait for peers' flags (``tp_wait``) or for
peers' partial tiles to overwrite sentinel words (``tp_reduce_rmsnorm``).
Here nothing ever writes them -- a peer that never delivers -- and the limit is
set to 50 ms: each kernel must return on its own, record ``kErrPeerTimeout``
(4) in the error flag, and leave the context usable.  No GPU fault is made:
the waits are plain bounded polls of this GPU's own memory.
"""

from __future__ import annotations

import time

import pytest
import torch

from conftest import mod

pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000  # 50 ms


@pytest.fixture()
def ext():
    e = mod("ops._native").cuda()
    old = e.peer_wait_ns(0)
    e.set_peer_wait_ns(LIMIT_NS, 0)
    assert e.peer_wait_ns(0) == LIMIT_NS
    yield e
    e.set_peer_wait_ns(old, 0)


def _timed(fn) -> float:
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    return time.perf_counter() - t0


def test_flag_wait_times_out_with_peer_timeout(ext):
    dev = torch.device("cuda", 0)
    flags = torch.zeros(4, dtype=torch.int32, device=dev)   # no peer ever raises them
    seq = torch.ones(1, dtype=torch.int32, device=dev)       # the sequence number they should reach
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    dt = _timed(lambda: ext.tp_wait(flags.data_ptr(), seq.data_ptr(), 4, err))
    assert int(err.item()) == 4
    assert 0.04 < dt < 2.0
    # The flag being set, a second wait gives up at once instead of costing another timeout.
    dt2 = _timed(lambda: ext.tp_wait(flags.data_ptr(), seq.data_ptr(), 4, err))
    assert dt2 < 0.04 and int(err.item()) == 4
    # The context still works, and a wait whose flags are raised passes.
    err.zero_()
    flags.fill_(1)
    ext.tp_wait(flags.data_ptr(), seq.data_ptr(), 4, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def test_sentinel_reduce_times_out_with_peer_timeout(ext):
    dev = torch.device("cuda", 0)
    m, h, nsrc = 2, 1024, 2
    recv = torch.full((nsrc, m, h), -1, dtype=torch.int32, device=dev)  # sentinel words: nothing arrived
    hres = torch.zeros((m, h), dtype=torch.float32, device=dev)
    gamma = torch.ones(h, dtype=torch.bfloat16, device=dev)
    x = torch.empty((m, h), dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    dt = _timed(lambda: ext.tp_reduce_rmsnorm(recv.data_ptr(), m * h, 0, 0, nsrc, hres, gamma, x, 1e-5, err, True))
    assert int(err.item()) == 4
    assert dt < 2.0  # one timeout in total, not one per polled float4
    # The slots are back at the sentinel for their next use.
    assert bool((recv == -1).all())
    # Slots that do arrive are summed in rank order with the residual.
    err.zero_()
    hres.zero_()  # the timed-out call added sentinel NaNs to the residual
    vals = torch.randn((nsrc, m, h), device=dev)
    recv.view(torch.float32).copy_(vals)
    ext.tp_reduce_rmsnorm(recv.data_ptr(), m * h, 0, 0, nsrc, hres, gamma, x, 1e-5, err, True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    torch.testing.assert_close(hres, vals[0] + vals[1])
    ref = hres * torch.rsqrt(hres.pow(2).mean(-1, keepdim=True) + 1e-5)
    torch.testing.assert_close(x.float(), ref, rtol=2e-2, atol=2e-2)
