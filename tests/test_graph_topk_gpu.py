"""Top-k candidates selected inside the drafter forward's CUDA graph (greedy drafting).

``LlamaEngine.run_rows_topk`` captures the top-k kernel, the packing of
[ids | log-probs | error flag] and the copy to pinned host memory into the
forward's graph.  Its read-out must equal the eager path (the same graph's
logits through ``topk_logprobs`` and ``read_back``) for every row of the
bucket, including padded buckets, and must report a device error flag.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import mod

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine():
    llama = mod("models.llama")
    w = llama.random_weights(llama.get_config("small-drafter"), seed=3, dtype=torch.float16,
                             device=torch.device("cuda", 0))
    return mod("runtime.engine").LlamaEngine(w, num_pages=256, page_size=16, max_positions=4096)


def _fields(rows: int, p: int = 300):
    return dict(tokens=np.arange(7, 7 + rows), positions=np.arange(p, p + rows), slots=np.arange(p, p + rows),
                shared_len=p, n_shared_pages=(p + 15) // 16, mask_base=p, row_full=np.full(rows, p),
                row_len=np.full(rows, p + rows))


@pytest.mark.parametrize("rows,k", [(1, 1), (3, 3), (9, 3), (5, 8)])
def test_graph_topk_matches_eager(engine, rows, k):
    transfer = mod("utils.transfer")
    pages = torch.arange(64, dtype=torch.int32, device="cuda")
    b = mod("runtime.engine").row_bucket(rows)
    logits, readout = engine.run_rows_topk(b, k, prefix_pages=pages, **_fields(rows))
    ids, lps = readout.get()
    lp_ref, id_ref = engine.ops.topk_logprobs(logits, k)
    id_h, lp_h = transfer.read_back([id_ref, lp_ref], engine.ops.err)
    assert ids.shape == (rows, k)
    np.testing.assert_array_equal(ids, id_h)
    np.testing.assert_allclose(lps, lp_h, rtol=0, atol=1e-6)
    # The plain forward of the same inputs gives the same logits.
    again = engine.run_rows(b, prefix_pages=pages, **_fields(rows))
    torch.cuda.synchronize()
    assert torch.equal(again, logits)


def test_graph_topk_reports_device_error(engine):
    transfer = mod("utils.transfer")
    pages = torch.arange(64, dtype=torch.int32, device="cuda")
    b = mod("runtime.engine").row_bucket(2)
    engine.run_rows_topk(b, 2, prefix_pages=pages, **_fields(2))[1].get()  # captured and clean
    engine.ops.err.fill_(2)  # as a kernel would record an out-of-range index
    _, readout = engine.run_rows_topk(b, 2, prefix_pages=pages, **_fields(2))
    with pytest.raises(transfer.KernelError):
        readout.get()
    assert int(engine.ops.err.item()) == 0  # cleared when raised


def test_extend_selects_prefix_children_in_graph():
    """After an extend, the prefix's children come from the extend graph and equal top-k of its logits."""
    llama = mod("models.llama")
    transfer = mod("utils.transfer")
    w = llama.random_weights(llama.get_config("small-drafter"), seed=4, dtype=torch.float16,
                             device=torch.device("cuda", 0))
    eng = mod("runtime.engine").LlamaEngine(w, num_pages=256, page_size=16, max_positions=4096)
    dr = mod("runtime.drafter").DrafterRuntime(eng)
    dr.warm_graphs(3, 4)
    dr.prefill(list(range(100, 400)))
    assert dr.prefix_state().candidates is None  # a prefill selects nothing in-graph
    dr.append_known_tokens_as_prefix([5, 6, 7, 8])
    st = dr.prefix_state()
    ids, lps = st.candidates.get()
    lp_ref, id_ref = eng.ops.topk_logprobs(st.next_token_logits, 3)
    id_h, lp_h = transfer.read_back([id_ref, lp_ref], eng.ops.err)
    np.testing.assert_array_equal(ids, id_h)
    np.testing.assert_allclose(lps, lp_h, rtol=0, atol=1e-6)


def test_copy_on_write_inside_the_graph():
    """A drafter engine's graphs copy the tail pages named in the static batch before the forward."""
    llama = mod("models.llama")
    w = llama.random_weights(llama.get_config("small-drafter"), seed=5, dtype=torch.float16,
                             device=torch.device("cuda", 0))
    eng = mod("runtime.engine").LlamaEngine(w, num_pages=256, page_size=16, max_positions=4096)
    eng.cow_in_graph = True
    pages = torch.arange(64, dtype=torch.int32, device="cuda")
    kv = eng.kv
    g = torch.Generator(device="cuda").manual_seed(1)
    for call in range(3):  # the first call captures (and copies eagerly), the others replay
        kv[:, 40].copy_(torch.randn(kv[:, 40].shape, generator=g, device="cuda").half())
        kv[:, 41].zero_()
        eng.run_rows(1, prefix_pages=pages, tokens=[3], positions=[300], slots=[41 * 16 + 9], shared_len=300,
                     n_shared_pages=19, mask_base=300, row_full=[301], row_len=[301], cow=np.array([[40, 41, 9]]))
        torch.cuda.synchronize()
        assert torch.equal(kv[:, 41, :, :, :9], kv[:, 40, :, :, :9]), f"call {call}"
    key = next(k for k in eng._graphs)
    assert eng._graphs[key].cow
    eng.ops.check()
