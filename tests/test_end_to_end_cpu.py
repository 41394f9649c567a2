"""End-to-end CPU plumbing: tiny random-init Llama drafter and target.

Checks against the fp32 oracle:
- fallback on every round (threshold above any log-prob) == target greedy AR;
- k=1 with the first-route policy == drafter greedy AR (the reference's own
  equivalence contract, tools/check_async_greedy_equivalence.py:220-227);
- the masked tree forward's logits == the oracle with an explicit ancestor mask;
- the serial generator and the async generator agree token for token.
"""

from __future__ import annotations

import torch
import pytest

from conftest import mod

K, D, PAGE = 2, 3, 4


@pytest.fixture(scope="module")
def models():
    llama = mod("models.llama")
    dw = llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32)
    tw = llama.random_weights(llama.get_config("tiny-target"), seed=2, dtype=torch.float32)
    return dw, tw


def prompts(n=8, length=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, 1024, (length,), generator=g).tolist() for _ in range(n)]


def greedy(w, prompt, n):
    llama = mod("models.llama")
    toks = list(prompt)
    for _ in range(n):
        toks.append(int(llama.reference_forward(w, toks)[-1].argmax()))
    return toks[len(prompt):]


def make_generator(dw, tw, *, k=K, d=D, serial=False, cfg_kw=None, **target_kw):
    engine = mod("runtime.engine")
    drafter = mod("runtime.drafter")
    target = mod("runtime.target")
    edge = mod("serving.edge")
    rpc = mod("serving.rpc")
    de = engine.LlamaEngine(dw, num_pages=512, page_size=PAGE, max_positions=512)
    te = engine.LlamaEngine(tw, num_pages=512, page_size=PAGE, max_positions=512)
    tv = target.TargetVerifier(te, k=k, d=d, **target_kw)
    cls = mod("serving.serial").SerialAtlasGenerator if serial else edge.PagedDistributedAtlasGenerator
    kw = dict(k=k, d=d, max_new_tokens=16, validate_state_alignment=True, fixed_forest_depth=None if serial else 2)
    kw.update(cfg_kw or {})
    cfg = edge.DistributedAtlasConfig(**kw)
    return cls(config=cfg, drafter=drafter.DrafterRuntime(de), target_client=rpc.InProcessTargetClient(tv))


def test_fallback_every_round_equals_target_greedy(models):
    dw, tw = models
    p = prompts(2)[1]
    res = make_generator(dw, tw, fallback_threshold=1e9).generate(p)
    assert all(r.decision == "fallback_ar" for r in res.rounds)
    assert {r.fallback_reason for r in res.rounds} == {"path_score_below_threshold"}
    assert res.generated_token_ids == greedy(tw, p, 16)


def test_k1_first_route_equals_drafter_greedy(models):
    dw, tw = models
    p = prompts(1, seed=3)[0]
    res = make_generator(dw, tw, k=1, route_selection_policy="first_route").generate(p)
    assert res.generated_token_ids == greedy(dw, p, 16)


def test_tree_forward_matches_oracle(models):
    _, tw = models
    llama = mod("models.llama")
    engine = mod("runtime.engine")
    target = mod("runtime.target")
    te = engine.LlamaEngine(tw, num_pages=512, page_size=PAGE, max_positions=512)
    tv = target.TargetVerifier(te, k=3, d=3)
    prompt = prompts(1, length=30)[0]
    tv.prefill(prompt)
    out = tv.run_tree([(5, 6, 7), (5, 6, 8), (9, 6, 7)])
    toks, parents, depth = [5, 6, 7, 8, 9, 6, 7], [-1, 0, 1, 1, -1, 4, 5], [0, 1, 2, 2, 0, 1, 2]
    p = len(prompt)
    vis = torch.zeros(p + 7, p + 7, dtype=torch.bool)
    vis[:p, :p] = torch.tril(torch.ones(p, p, dtype=torch.bool))
    for i in range(7):
        vis[p + i, :p] = True
        a = i
        while a >= 0:
            vis[p + i, p + a] = True
            a = parents[a]
    ref = llama.reference_forward(tw, prompt + toks, positions=list(range(p)) + [p + x for x in depth], visible=vis)
    assert torch.allclose(out["logits"], ref[p:], atol=1e-4, rtol=1e-4)
    assert out["node_count"] == 7


def test_config1_async_generation_schema(models):
    """Config 1: 8 prompts x 64 tokens, k=2 d=3, page 4, greedy; result JSON per the reference schema."""
    dw, tw = models
    gen = make_generator(dw, tw)
    for p in prompts(8):
        res = gen.generate(p)
        assert len(res.generated_token_ids) == 16
        d = res.to_dict()
        assert set(d) == {"prompt_token_ids", "generated_token_ids", "token_ids", "text", "rounds", "metadata"}
        r0 = d["rounds"][0]
        for key in ("decision", "fallback_reason", "handoff_mode", "target_scores", "target_unique_tree_nodes",
                    "forest_depth", "committed_tokens", "released_kv_pages"):
            assert key in r0
        assert r0["handoff_mode"] in {"completed_forest_reused", "partial_forest_pruned_then_build_tree", "stopped"}
        assert d["metadata"]["edge_blackbox_timeline"]["rounds"] == len(d["rounds"])


def test_serial_equals_async_when_target_selects(models):
    """With no fallback and greedy drafting both schedules commit the same tokens."""
    dw, tw = models
    p = prompts(1, seed=5)[0]
    a = make_generator(dw, tw).generate(p)
    s = make_generator(dw, tw, serial=True).generate(p)
    assert a.generated_token_ids == s.generated_token_ids
    assert all(r.handoff_mode.startswith("serial_") for r in s.rounds)


def test_adaptive_forest_gate_keeps_tokens(models):
    """Gated rounds (after repeated fallbacks) build no tree or forest; the tokens do not change."""
    dw, tw = models
    p = prompts(3)[2]
    out = {}
    for gate in ("overlap", "adaptive"):
        cfg = dict(fixed_forest_depth=None, forest_gate=gate, max_new_tokens=32)
        res = make_generator(dw, tw, cfg_kw=cfg, fallback_threshold=1e9).generate(p)
        assert all(r.decision == "fallback_ar" for r in res.rounds)
        out[gate] = res
    assert out["adaptive"].generated_token_ids == out["overlap"].generated_token_ids == greedy(tw, p, 32)
    assert out["overlap"].metadata["forest_gated_rounds"] == 0
    gated = out["adaptive"].metadata["forest_gated_rounds"]
    assert gated >= 3
    # Gated fallback rounds grew no forest.
    assert sum(r.forest_depth == 0 for r in out["adaptive"].rounds) >= gated


def test_forest_gate_stays_open_when_routes_are_selected(models):
    dw, tw = models
    p = prompts(4)[3]
    cfg = dict(fixed_forest_depth=None, forest_gate="adaptive", max_new_tokens=16)
    res = make_generator(dw, tw, k=1, cfg_kw=cfg, route_selection_policy="first_route").generate(p)
    assert all(r.decision == "select" for r in res.rounds)
    assert res.metadata["forest_gated_rounds"] == 0


@pytest.mark.parametrize("forest_depth", [0, 1, 2, 3])
def test_every_handoff_depth_keeps_greedy_equivalence(models, forest_depth):
    """k=1 first-route selection with the forest stopped at each depth (completed at d):
    every handoff -- including a deferred last tree depth of zero to d-1 prebuilt steps --
    commits the drafter's greedy tokens and passes the state-alignment checks."""
    dw, tw = models
    p = prompts(1, seed=7)[0]
    cfg = dict(fixed_forest_depth=forest_depth, max_new_tokens=14)
    res = make_generator(dw, tw, k=1, cfg_kw=cfg, route_selection_policy="first_route").generate(p)
    assert res.generated_token_ids == greedy(dw, p, 14)
    modes = {r.handoff_mode for r in res.rounds[:-1]}
    want = "completed_forest_reused" if forest_depth == D else "partial_forest_pruned_then_build_tree"
    assert modes == {want}


def test_equivalence_checker_cli(tmp_path):
    """The user-facing k=1 first-route checker: greedy and keyed sampling both match AR."""
    import json

    chk = mod("serving.check_equivalence")
    base = ["--drafter-model", "tiny-drafter", "--target-model", "tiny-target", "--device", "cpu", "--dtype",
            "float32", "--page-size", "4", "--prompt-token-ids", "5,6,7,8,9,10", "--forest-depths", "live,0,3",
            "--repeats", "1", "--max-new-tokens", "10", "--context-length", "256", "--d", "3"]
    for extra in ([], ["--drafter-do-sample", "--drafter-temperature", "0.7", "--seed", "3"]):
        out = tmp_path / f"eq{len(extra)}.json"
        assert chk.main(base + extra + ["--json-out", str(out)]) == 0
        rep = json.loads(out.read_text())
        assert rep["passed"] and rep["checked"] == 3
    with pytest.raises(SystemExit):
        chk.check_target_policy({"route_selection_policy": "target_best"})
    with pytest.raises(SystemExit):
        chk.check_target_policy({"route_selection_policy": "first_route", "fallback_threshold": -0.5})


def test_kv_reuse_diagnostics_cli(tmp_path):
    import json

    diag = mod("serving.diagnostics")
    base = ["--device", "cpu", "--dtype", "float32", "--page-size", "4", "--prompt-token-ids", "5,6,7,8,9,10,11",
            "--context-length", "256"]
    out = tmp_path / "tc.json"
    assert diag.main(["target-commit", "--model", "tiny-target", "--d", "3", "--rounds", "3", "--max-logit-diff",
                      "1e-3", "--max-kv-diff", "1e-4", "--json-out", str(out), *base]) == 0
    rep = json.loads(out.read_text())
    assert rep["passed"] and rep["rounds"][-1]["prefix_len"] == 16 and "max_kv_diff" in rep["rounds"][-1]
    out = tmp_path / "da.json"
    assert diag.main(["drafter-alignment", "--model", "tiny-drafter", "--k", "2", "--d", "2", "--alignment-atol",
                      "1e-4", "--alignment-rtol", "1e-4", "--json-out", str(out), *base]) == 0
    stages = [s["stage"] for s in json.loads(out.read_text())["steps"]]
    assert stages == ["tree", "tree", "forest", "post_commit_forest"]
    trace = tmp_path / "trace.pt"
    assert diag.main(["drafter-alignment", "--model", "tiny-drafter", "--k", "2", "--d", "2", "--skip-forest",
                      "--check-hf-logits", "--logits-tensor-out", str(trace), *base]) == 0
    rows = torch.load(trace)
    assert len(rows) == 4 and torch.allclose(rows[0]["logits"], rows[0]["reference"], atol=1e-3)
    assert diag.main(["target-commit", "--model", "tiny-target", "--d", "2", "--rounds", "2",
                      "--route-selection-policy", "target_best", *base]) == 0


def test_prefix_kv_reads_positions_through_the_page_table():
    diag, engine_mod, llama = mod("serving.diagnostics"), mod("runtime.engine"), mod("models.llama")
    w = llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32)
    eng = engine_mod.LlamaEngine(w, num_pages=16, page_size=4, max_positions=64)
    eng.kv.copy_(torch.randn_like(eng.kv))
    pages = [7, 3, 11]
    kv = diag.prefix_kv(eng, pages, 10)
    L = eng.kv.shape[0]
    assert tuple(kv.shape) == (L, 2, 10, eng.kv.shape[3], eng.kv.shape[5])
    for pos in (0, 5, 9):
        assert torch.equal(kv[1, 0, pos], eng.kv[1, pages[pos // 4], 0, :, pos % 4, :])


def test_equivalence_checker_against_a_target_server(tmp_path):
    """The checker's usual set-up: a running target server (first route, fallback off) over HTTP."""
    import json
    import threading

    chk, rpc = mod("serving.check_equivalence"), mod("serving.rpc")
    engine, target, llama = mod("runtime.engine"), mod("runtime.target"), mod("models.llama")
    tw = llama.random_weights(llama.get_config("tiny-target"), seed=1, dtype=torch.float32)
    tv = target.TargetVerifier(engine.LlamaEngine(tw, num_pages=256, page_size=4, max_positions=512), k=1, d=3,
                               route_selection_policy="first_route")
    server = rpc.make_server(rpc.TargetServerApp(tv), host="127.0.0.1", port=0)
    threading.Thread(target=server.serve_forever, daemon=True).start()
    try:
        out = tmp_path / "eq.json"
        url = f"http://127.0.0.1:{server.server_address[1]}"
        assert chk.main(["--drafter-model", "tiny-drafter", "--target-url", url, "--device", "cpu", "--dtype",
                         "float32", "--page-size", "4", "--prompt-token-ids", "3,4,5,6,7", "--forest-depths",
                         "live,1", "--repeats", "1", "--max-new-tokens", "8", "--context-length", "256", "--d", "3",
                         "--json-out", str(out)]) == 0
        rep = json.loads(out.read_text())
        assert rep["passed"] and rep["checked"] == 2 and rep["target_transport"] == "http"
    finally:
        server.shutdown()
        server.server_close()
