"""Drafter route KV vs full recompute, depth by depth.

Every route the drafter decodes reads its context from paged KV that was written by
earlier steps: the prefill, the tree depths, the forest depths, and -- after a
stage-1 route is committed and its forest children promoted -- the committed prefix
rebuilt from route pages.  Each decoded row's next-token logits must equal an fp32
recompute of the route's whole token sequence (committed prefix + route path) with
no cache at all.  This is the reference's drafter alignment check
(tools/smoke_flashinfer_paged_tree_forest.py:154-211, 302-385: every tree depth,
every forest depth and one post-commit forest step against Hugging Face full
recompute, logits within tolerance and top-1 equal).
"""

from __future__ import annotations

import pytest
import torch

from conftest import mod

K, D, FOREST_DEPTH = 3, 4, 2


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float().to(a.device)
    return float((a - b).norm() / b.norm().clamp_min(1e-6))


def _check_step(step, store, prefix, w_ref, tol, seen):
    llama = mod("models.llama")
    logits = step.decode_output.next_token_logits
    assert logits.shape[0] == len(step.decoded_routes)
    for i, r in enumerate(step.decoded_routes):
        toks = list(prefix) + list(store.materialized_token_path(r))  # decoded token included
        ref = llama.reference_forward(w_ref, toks)[-1]
        got = logits[i].float()
        assert rel_err(got, ref) < tol, (len(toks), rel_err(got, ref))
        # Top-1 must agree unless the oracle's top two are closer than twice the largest
        # logit error (only then can rounding reorder them).
        top2 = torch.topk(ref, 2).values
        if float(top2[0] - top2[1]) > 2 * float((got - ref.to(got.device)).abs().max()):
            assert int(got.argmax()) == int(ref.argmax())
        seen.append(len(toks))


def run_alignment(w, w_ref, prompt, tol):
    """Tree of depth D, forest of depth FOREST_DEPTH, commit, one post-commit step."""
    engine, drafter = mod("runtime.engine"), mod("runtime.drafter")
    store_mod, builders = mod("runtime.store"), mod("runtime.builders")
    dr = drafter.DrafterRuntime(engine.LlamaEngine(w, num_pages=512, page_size=16, max_positions=2048))
    store = store_mod.KVTreeStore()
    dr.bind_store(store)
    dr.prefill(prompt)
    seen: list[int] = []

    stage1 = builders.initialize_stage1_routes(dr.prefix_state(), k=K, route_store=store)
    tree = builders.build_tree_depths(stage1, depth=D, k=K, route_store=store, model_backend=dr)
    assert len(tree.steps) == D
    for st in tree.steps:
        _check_step(st, store, prompt, w_ref, tol, seen)

    seeds = builders.initialize_forest_routes(tree.completed_routes, tree.last_logits, k=K, route_store=store)
    forest = builders.build_forest_depths(seeds, depth=FOREST_DEPTH, k=K, route_store=store, model_backend=dr)
    assert len(forest.steps) == FOREST_DEPTH
    for st in forest.steps:
        _check_step(st, store, prompt, w_ref, tol, seen)

    # The target selects the second stage-1 route: commit it, keep its forest children.
    chosen = tree.completed_routes[1]
    committed = list(prompt) + list(store.materialized_token_path(chosen))
    retained = builders.select_routes_by_stage1_root(forest.next_frontier_routes, int(chosen.route_id))
    assert len(retained) == K
    promoted, stats = dr.commit_stage1_and_promote(committed_route=chosen, retained_routes=retained)
    assert tuple(dr.prefix_token_ids) == tuple(committed)
    assert stats["retained_routes"] == K
    step = builders.build_tree_one_depth(promoted, k=K, route_store=store, model_backend=dr)
    _check_step(step, store, committed, w_ref, tol, seen)
    dr.engine.ops.check()
    return seen


def test_drafter_alignment_cpu():
    llama = mod("models.llama")
    w = llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32)
    prompt = torch.randint(0, 1024, (37,), generator=torch.Generator().manual_seed(5)).tolist()
    seen = run_alignment(w, w, prompt, 1e-4)
    # K rows per tree depth, K*K per forest depth, K after the commit.
    assert len(seen) == D * K + FOREST_DEPTH * K * K + K


@pytest.mark.gpu
@pytest.mark.parametrize("prompt_len", [40, 150])
def test_drafter_alignment_cuda(prompt_len):
    """The CUDA engine (fp16, hd-128, 16-token pages): prompts ending inside and across pages."""
    llama = mod("models.llama")
    w32 = llama.random_weights(llama.get_config("small-drafter"), seed=1, dtype=torch.float32, device="cuda")
    w = llama.weights_to(w32, dtype=torch.float16)
    prompt = torch.randint(0, 4096, (prompt_len,), generator=torch.Generator().manual_seed(6)).tolist()
    run_alignment(w, llama.weights_to(w, dtype=torch.float32), prompt, 3e-2)
