"""The serving path reads the device error flag with the results it copies back, and stops.

Kernels record faults (bad index, bounded wait that ran out, peer timeout) in
an int32 flag instead of trapping.  The target's verify and fallback AR, and
every drafter depth, copy that flag back together with their small results;
a set flag raises ``KernelError`` before any route is selected, committed,
grown or promoted.  Here the op table is the CPU one wrapped with a flag that
the test sets, as a kernel would.
"""

from __future__ import annotations

import pytest
import torch

from conftest import mod


class FlaggedOps:
    """CPU op table plus an error flag (what ``CudaOps`` exposes as ``err``)."""

    def __init__(self) -> None:
        self.base = mod("ops.torch_ops")
        self.err = torch.zeros(1, dtype=torch.int32)

    def __getattr__(self, name):
        return getattr(self.base, name)


@pytest.fixture(scope="module")
def weights():
    llama = mod("models.llama")
    return (llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32),
            llama.random_weights(llama.get_config("tiny-target"), seed=2, dtype=torch.float32))


def _engine(w):
    e = mod("runtime.engine").LlamaEngine(w, num_pages=256, page_size=4, max_positions=512)
    e.ops = FlaggedOps()
    return e


def _payload(rid, toks):
    return mod("types").VerifyRoutePayload(route_id=rid, token_ids=tuple(toks), draft_logprob=-1.0,
                                           draft_token_logprobs=tuple([-1.0 / len(toks)] * len(toks)))


def _target_state(tv):
    return (tv.prefix_token_ids, int(tv.seq.prefix_len), int(tv.page_pool.used_pages), tv._pending_token)


ROUTES = [(1, [5, 6, 7]), (2, [5, 8, 9]), (3, [4, 4, 4])]


@pytest.mark.parametrize("threshold", [None, 1e9])  # select path, fallback AR path
def test_target_round_raises_and_leaves_state_unchanged(weights, threshold):
    kerr = mod("utils.transfer").KernelError
    tv = mod("runtime.target").TargetVerifier(_engine(weights[1]), k=3, d=3, fallback_threshold=threshold)
    prompt = list(range(30, 47))
    tv.prefill(prompt)
    routes = [_payload(r, t) for r, t in ROUTES]
    before = _target_state(tv)
    tv.engine.ops.err[0] = 2  # a kernel found an index out of range
    with pytest.raises(kerr, match="index out of range"):
        tv.verify_payloads(prefix_token_ids=prompt, routes=routes)
    assert _target_state(tv) == before
    assert int(tv.engine.ops.err[0]) == 0  # read, reported and cleared
    res = tv.verify_payloads(prefix_token_ids=prompt, routes=routes)
    assert res.decision == ("fallback_ar" if threshold else "select")


def test_fallback_ar_error_after_decision_commits_nothing(weights):
    kerr = mod("utils.transfer").KernelError
    tv = mod("runtime.target").TargetVerifier(_engine(weights[1]), k=3, d=3, fallback_threshold=1e9)
    prompt = list(range(30, 47))
    tv.prefill(prompt)
    before = _target_state(tv)

    def fault(decision):  # the AR steps that follow the decision hit a fault
        assert decision == "fallback_ar"
        tv.engine.ops.err[0] = 1

    with pytest.raises(kerr, match="timed out"):
        tv.verify_payloads(prefix_token_ids=prompt, routes=[_payload(r, t) for r, t in ROUTES], on_decision=fault)
    assert _target_state(tv) == before


def test_drafter_depth_raises_before_routes_grow(weights):
    kerr = mod("utils.transfer").KernelError
    dr = mod("runtime.drafter").DrafterRuntime(_engine(weights[0]))
    store = mod("runtime.store").KVTreeStore()
    dr.bind_store(store)
    builders = mod("runtime.builders")
    dr.prefill(list(range(10, 30)))
    routes = builders.initialize_stage1_routes(dr.prefix_state(), k=3, route_store=store, model_backend=dr)
    snapshot = [(r.route_id, r.stage1_depth, r.kv_view.node_ids, r.pending_token_id) for r in routes]
    n_routes = len(store.routes)
    dr.engine.ops.err[0] = 4  # a peer's partial never arrived
    with pytest.raises(kerr, match="peer"):
        builders.build_tree_one_depth(routes, k=3, route_store=store, model_backend=dr)
    assert [(r.route_id, r.stage1_depth, r.kv_view.node_ids, r.pending_token_id) for r in routes] == snapshot
    assert len(store.routes) == n_routes  # no child spawned
    assert dr.prefix_token_ids == tuple(range(10, 30))
    # The session drops its speculative state and starts a fresh tree from the committed prefix.
    dr.drop_speculative()
    routes = builders.initialize_stage1_routes(dr.prefix_state(), k=3, route_store=store, model_backend=dr)
    step = builders.build_tree_one_depth(routes, k=3, route_store=store, model_backend=dr)
    assert len(step.next_routes) == 3


def test_seed_reads_the_flag(weights):
    kerr = mod("utils.transfer").KernelError
    dr = mod("runtime.drafter").DrafterRuntime(_engine(weights[0]))
    store = mod("runtime.store").KVTreeStore()
    dr.bind_store(store)
    dr.prefill(list(range(10, 30)))
    dr.engine.ops.err[0] = 3
    with pytest.raises(kerr, match="unsupported"):
        mod("runtime.builders").initialize_stage1_routes(dr.prefix_state(), k=3, route_store=store,
                                                         model_backend=dr)
    assert not store.routes


def test_read_back_round_trips_dtypes():
    t = mod("utils.transfer")
    ids = torch.tensor([[1, 2], [3, 2 ** 31 - 1]], dtype=torch.int64)
    lp = torch.tensor([[-0.5, -1.25], [-3.0, float("-inf")]], dtype=torch.float32)
    i32 = torch.tensor([7, -7], dtype=torch.int32)
    flag = torch.zeros(1, dtype=torch.int32)
    a, b, c = t.read_back([ids, lp, i32], flag)
    assert a.dtype.name == "int64" and a.tolist() == ids.tolist()
    assert b.dtype.name == "float32" and b.tolist() == lp.tolist()
    assert c.tolist() == [7, -7]


def test_arena_ids_never_repeat_and_shrink_on_commit(weights):
    dr = mod("runtime.drafter").DrafterRuntime(mod("runtime.engine").LlamaEngine(
        weights[0], num_pages=256, page_size=4, max_positions=512))
    store = mod("runtime.store").KVTreeStore()
    dr.bind_store(store)
    builders = mod("runtime.builders")
    dr.prefill(list(range(10, 30)))
    seen: set[int] = set()
    for _ in range(4):
        routes = builders.initialize_stage1_routes(dr.prefix_state(), k=2, route_store=store, model_backend=dr)
        tree = builders.build_tree_depths(routes, depth=2, k=2, route_store=store, model_backend=dr)
        forest = builders.initialize_forest_routes(tree.completed_routes, tree.last_logits, k=2, route_store=store,
                                                   model_backend=dr)
        fr = builders.build_forest_one_depth(forest, k=2, route_store=store, model_backend=dr)
        ids = {n for r in fr.decoded_routes for n in r.kv_view.node_ids}
        sel = tree.completed_routes[0]
        keep = builders.select_routes_by_stage1_root(fr.decoded_routes, sel.route_id)
        new = {n for s in [fr, *tree.steps] for n in s.decode_output.new_node_ids_cpu}
        assert not (new & seen)
        seen |= new
        promoted, _ = dr.commit_stage1_and_promote(committed_route=sel, retained_routes=keep)
        assert all(r.stage1_depth == 1 and r.stage2_depth == 0 and r.stage1_root_id == r.route_id for r in promoted)
        assert store.arena_size <= 2 * 2  # only the last forest depth's block is left
        dr.drop_speculative()
        store.reset_speculative()
        dr.prefix_next_token_logits = tree.last_logits[:1]
