"""Benchmark helpers and the edge timeline on CPU."""

from __future__ import annotations

import importlib.util
import json
import os

import torch

from conftest import REPO, mod


def _load(name):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REPO, "benchmarks", f"{name}.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_matched_batch_ar_keeps_each_routes_greedy_child():
    bench = _load("bench_isolated_components")
    llama, engine, drafter = mod("models.llama"), mod("runtime.engine"), mod("runtime.drafter")
    store_mod, builders, frontier = mod("runtime.store"), mod("runtime.builders"), mod("runtime.frontier")
    w = llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32)
    dr = drafter.DrafterRuntime(engine.LlamaEngine(w, num_pages=256, page_size=4, max_positions=256))
    store = store_mod.KVTreeStore()
    dr.bind_store(store)
    prompt = list(range(30, 45))
    dr.prefill(prompt)
    routes = builders.initialize_stage1_routes(dr.prefix_state(), k=3, route_store=store)
    firsts = [r.pending_token_id for r in routes]
    for _ in range(3):
        routes = frontier.advance_frontier_one_token(routes, k=1, route_store=store, model_backend=dr,
                                                     selection_policy=bench.PerRouteTop1Selection()).next_routes
    assert len(routes) == 3
    for r, f in zip(routes, firsts):
        path = list(store.materialized_token_path(r)) + [r.pending_token_id]
        toks = prompt + [f]
        for _ in range(3):
            toks.append(int(llama.reference_forward(w, toks)[-1].argmax()))
        assert path == toks[len(prompt):]


def test_timeline_overlap_exposed_wait_json_and_svg(tmp_path):
    tl = mod("utils.timeline")
    S = tl.EdgeSpan
    r = tl.EdgeRoundTimeline(
        round_index=0, verify_blackbox=S("verify", 0.0, 0.030),
        forest_steps=[S("forest_1", 0.001, 0.008), S("forest_2", 0.008, 0.020)],
        post_prune_tree_steps=[], handoff=S("handoff", 0.030, 0.032), forest_depth=2, accepted_tokens=4,
        generated_tokens=4, handoff_mode="completed_forest_reused", verify_returned_before_forest_done=False)
    assert abs(r.cloud_edge_overlap_s - 0.019) < 1e-12 and abs(r.exposed_cloud_wait_s - 0.010) < 1e-12
    t = tl.EdgeBlackboxTimeline(edge_prefill=S("p", 0, 0.01), cloud_prefill_blackbox=S("c", 0, 0.02),
                                initial_tree=S("t", 0.02, 0.03), rounds=[r], elapsed_s=0.1, generated_tokens=4)
    s = t.summary()
    assert s["rounds"] == 1 and abs(s["cloud_hidden_ratio"] - 0.019 / 0.030) < 1e-9
    tl.write_timeline_json(tmp_path / "t.json", t)
    tl.write_timeline_svg(tmp_path / "t.svg", t, width=800)
    assert json.loads((tmp_path / "t.json").read_text())["summary"]["rounds"] == 1
    assert (tmp_path / "t.svg").read_text().startswith("<svg")


def test_round_trace_accounting():
    tr = _load("trace_round")
    # Round 0 spans [0, 100): kernels A [10, 40), B [30, 60) overlap; copy C [80, 90).
    events = [(30.0, 60.0, "void B<float>(int)"), (10.0, 40.0, "A"), (80.0, 90.0, "Memcpy HtoD"),
              (120.0, 150.0, "A")]
    out = tr.analyze_rounds(events, [(0.0, 100.0), (100.0, 200.0)], [1e-4, 1e-4])
    r0, r1 = out["per_round"]
    assert r0["gpu_busy_us"] == 60.0 and r0["gpu_idle_us"] == 40.0
    assert r0["largest_gaps_us"][0] == [20.0, "B<float>", "Memcpy HtoD"]
    assert {tuple(g) for g in r0["largest_gaps_us"]} == {(20.0, "B<float>", "Memcpy HtoD"),
                                                         (10.0, "(round start)", "A"),
                                                         (10.0, "Memcpy HtoD", "(round end)")}
    assert r1["gpu_busy_us"] == 30.0 and r1["gpu_idle_us"] == 70.0
    assert out["mean_gpu_idle_us"] == 55.0


def test_abba_protocol_helpers():
    import pytest

    bench = _load("bench_isolated_components")
    assert [bench.abba_order(i) for i in range(4)] == [("a", "b"), ("b", "a"), ("a", "b"), ("b", "a")]
    for bad in (0, 1, 3, 7):
        with pytest.raises(ValueError):
            bench.check_pairs(bad)
    assert bench.check_pairs(6) == 6
    # Block ratios: (b0 + b1) / (a0 + a1) per block; geometric mean of 2 and 0.5 is 1.
    r = bench.block_ratios([1.0, 1.0, 2.0, 2.0], [2.0, 2.0, 1.0, 1.0])
    assert r["blocks"] == 2 and r["min"] == 0.5 and r["max"] == 2.0
    assert abs(r["geometric_mean"] - 1.0) < 1e-9
    with pytest.raises(ValueError):
        bench.block_ratios([1.0, 2.0, 3.0], [1.0, 2.0, 3.0])


def test_full_verify_benchmark_aligns_on_cpu(capsys):
    bench = _load("bench_full_verify")
    assert bench.main(["--model", "tiny-target", "--device", "cpu", "--dtype", "float32", "--prefix-len", "32",
                       "--page-size", "4", "--k", "3", "--d", "3", "--warmup", "0", "--iters", "1",
                       "--alignment-atol", "1e-4", "--alignment-rtol", "1e-4", "--fail-on-logit-mismatch",
                       "--use-packed-custom-mask", "--flashinfer-backend", "auto"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["logits_aligned"] and out["masked_verify"]["nodes"] == 7 and out["linear_verify"]["nodes"] == 9
    assert out["logit_alignment"]["masked_tree"]["top1_match_rate"] == 1.0
    assert bench.prefix_tokens(bench.build_parser().parse_args(
        ["--model", "m", "--prefix-len", "5", "--prompt-token-ids", "1,2"])) == [1, 2, 1, 2, 1]


def test_isolated_benchmark_reference_flags_on_cpu(capsys):
    bench = _load("bench_isolated_components")
    base = ["--drafter-model", "tiny-drafter", "--target-model", "tiny-target", "--device", "cpu", "--dtype",
            "float32", "--prefix-len", "48", "--page-size", "4", "--k", "2", "--d", "2", "--iters", "2",
            "--warmup", "0", "--mem-fraction-static", "0.7", "--legacy-token-attention-metadata"]
    assert bench.main(base + ["--pair-order-seed", "1", "--skip-verify"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["orders"] == ["BA", "AB"] and out["tree_over_batch_ar_blocks"]["blocks"] == 1
    assert set(out["hot_path_counters"]) == {"tree", "batch_ar_k", "forest", "batch_ar_k2"}
    assert {"launches", "h2d_bytes", "d2h_bytes"} <= set(out["hot_path_counters"]["forest"])
    assert "target_verify_ms" not in out and "forest_ms" in out
    assert bench.main(base + ["--skip-forest", "--skip-native-batch-ar", "--shared-path-tokens", "1",
                              "--repeat-token-id", "9"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert "tree_ms" in out and "forest_ms" not in out and "batch_ar_k_ms" not in out
    assert "tree_over_batch_ar" not in out and out["target_verify_ms"] > 0


def test_tree_forest_sweep_on_cpu(capsys):
    bench = _load("bench_tree_forest_sweep")
    assert bench.main(["--model", "tiny-drafter", "--target-model", "tiny-target", "--device", "cpu", "--dtype",
                       "float32", "--prefix-len", "40", "--page-size", "4", "--pairs", "2", "2", "--pairs", "3", "1",
                       "--warmup", "0", "--iters", "1", "--context-length", "64", "--nccl-port", "1",
                       "--alignment-atol", "1e-4", "--alignment-rtol", "1e-4", "--fail-on-logit-mismatch"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert [(p["k"], p["d"]) for p in out["pairs"]] == [(2, 2), (3, 1)]
    p = out["pairs"][1]
    assert {"batch1_ar_1_tokens", "batch3_ar_1_tokens", "atlas_tree_k3_d1", "batch9_ar_1_tokens",
            "atlas_forest_k3_d1"} <= set(p)
    assert p["target"]["logits_aligned"] and out["metadata"]["effective_context_length"] >= 40 + 2 + 64


def test_hf_kv_baseline_arms_match_the_oracle(capsys):
    """The transformers baseline runs the same model as this package's oracle, and its tree step
    (global top-k, cache reordered to the parents) decodes the routes it selected."""
    bench = _load("bench_hf_kv_baseline")
    llama = mod("models.llama")
    assert bench.main(["--drafter-model", "tiny-drafter", "--device", "cpu", "--dtype", "float32",
                       "--prefix-len", "24", "--k", "2", "--d", "2", "--warmup", "0", "--iters", "1"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert {"batch1_ar_2_tokens", "build_tree_stage1_k2_d2", "build_forest_stage2_k2_4_d2"} <= set(out["drafter"])
    assert "target_verify_k2_paths_d2" in out["target"]

    w = llama.random_weights(llama.get_config("tiny-drafter"), seed=0, dtype=torch.float32)
    model = bench.load_hf("tiny-drafter", dtype=torch.float32, device=torch.device("cpu"), seed=0, trust=False)
    prompt = [(7 * i + 3) % 1000 for i in range(24)]
    arms = bench.HFArms(model, prompt, torch.device("cpu"))
    k = 3
    state = arms.tree_state(k)
    ref = torch.log_softmax(llama.reference_forward(w, prompt)[-1], -1)
    lp0, t0 = torch.topk(ref, k)
    assert torch.equal(state[1], t0)
    past, ids, scores = arms.tree(state, k, 1)
    # Expected depth-1 selection from the oracle: the k best of the k x k children.
    cands = []
    for r in range(k):
        lp = torch.log_softmax(llama.reference_forward(w, prompt + [int(t0[r])])[-1], -1)
        v, t = torch.topk(lp, k)
        cands += [(float(lp0[r] + v[j]), r, int(t[j])) for j in range(k)]
    best = sorted(cands, key=lambda c: -c[0])[:k]
    assert [c[2] for c in best] == ids.tolist()
    assert torch.allclose(scores, torch.tensor([c[0] for c in best]), atol=1e-4)
    got = arms.step(past, ids)
    for i, (_, r, tok) in enumerate(best):
        want = llama.reference_forward(w, prompt + [int(t0[r]), tok])[-1]
        assert float((got[i] - want).abs().max()) < 1e-3
