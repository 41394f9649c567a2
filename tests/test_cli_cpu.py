"""CPU tests for the command lines, the checkpoint loader, the AR baseline and the HTTP transport."""

from __future__ import annotations

import json
import threading

import pytest
import torch

from conftest import mod


@pytest.fixture(scope="module")
def tiny():
    llama = mod("models.llama")
    return (llama.random_weights(llama.get_config("tiny-drafter"), seed=1, dtype=torch.float32),
            llama.random_weights(llama.get_config("tiny-target"), seed=2, dtype=torch.float32))


def greedy(w, prompt, n):
    llama = mod("models.llama")
    toks = list(prompt)
    for _ in range(n):
        toks.append(int(llama.reference_forward(w, toks)[-1].argmax()))
    return toks[len(prompt):]


def test_checkpoint_round_trip(tmp_path, tiny):
    loader = mod("models.loader")
    llama = mod("models.llama")
    dw, _ = tiny
    loader.save_hf_checkpoint(dw, tmp_path / "ckpt")
    back = loader.resolve_model(str(tmp_path / "ckpt"), dtype="float32")
    assert back.config.num_layers == dw.config.num_layers
    assert back.config.rope_scaling == dw.config.rope_scaling
    toks = list(range(5, 25))
    torch.testing.assert_close(llama.reference_forward(back, toks), llama.reference_forward(dw, toks))
    cfg = json.loads((tmp_path / "ckpt" / "config.json").read_text())
    assert cfg["num_key_value_heads"] == dw.config.num_kv_heads


def test_paged_ar_equals_oracle_greedy(tiny):
    engine = mod("runtime.engine")
    drafter = mod("runtime.drafter")
    ar = mod("serving.ar")
    dw, _ = tiny
    gen = ar.PagedGreedyARGenerator(drafter=drafter.DrafterRuntime(
        engine.LlamaEngine(dw, num_pages=256, page_size=4, max_positions=256)))
    prompt = list(range(100, 123))
    res = gen.generate(prompt, max_new_tokens=12)
    assert res.generated_token_ids == greedy(dw, prompt, 12)
    assert res.finish_reason == "length"
    # Reusable: a second generation on the same runtime gives the same tokens.
    assert gen.generate(prompt, max_new_tokens=12).generated_token_ids == res.generated_token_ids
    eos = res.generated_token_ids[3]
    assert gen.generate(prompt, max_new_tokens=12, eos_token_id=eos).finish_reason == "eos"


def test_clean_cli_mock(capsys):
    cli = mod("serving.cli")
    assert cli.main(["--backend", "mock", "--max-new-tokens", "10", "--k", "2", "--d", "3"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert len(out["result"]["generated_token_ids"]) == 10
    assert out["config"]["forest_decode"] == "ordinary_batch_4"


def test_clean_cli_prompt_text(capsys):
    import pytest

    cli = mod("serving.cli")
    assert cli.main(["--backend", "recompute", "--max-new-tokens", "3", "--k", "2", "--d", "2", "--prompt", "hi!",
                     "--trust-remote-code"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["result"]["prompt_token_ids"] == list(b"hi!") and len(out["result"]["generated_token_ids"]) == 3
    with pytest.raises(SystemExit):
        cli.main(["--backend", "mock", "--prompt", "hi"])


def test_clean_cli_recompute_matches_paged_greedy_contract(capsys):
    # k=1: the clean controller's single route is drafter greedy; with the
    # recompute backends the committed tokens are the target's choice among one
    # route, i.e. the drafter's greedy path.
    cli = mod("serving.cli")
    llama = mod("models.llama")
    assert cli.main(["--backend", "recompute", "--max-new-tokens", "6", "--k", "1", "--d", "2",
                     "--prompt-token-ids", "5,6,7,8,9"]) == 0
    out = json.loads(capsys.readouterr().out)
    dw = llama.random_weights(llama.get_config("tiny-drafter"), seed=0, dtype=torch.float32)
    assert out["result"]["generated_token_ids"] == greedy(dw, [5, 6, 7, 8, 9], 6)


def test_http_target_round_trip(tiny):
    engine = mod("runtime.engine")
    drafter = mod("runtime.drafter")
    target = mod("runtime.target")
    edge = mod("serving.edge")
    rpc = mod("serving.rpc")
    dw, tw = tiny
    tv = target.TargetVerifier(engine.LlamaEngine(tw, num_pages=256, page_size=4, max_positions=256), k=2, d=2)
    server = rpc.make_server(rpc.TargetServerApp(tv), host="127.0.0.1", port=0)
    th = threading.Thread(target=server.serve_forever, daemon=True)
    th.start()
    try:
        url = f"http://127.0.0.1:{server.server_address[1]}"
        cfg = edge.DistributedAtlasConfig(k=2, d=2, max_new_tokens=10, validate_state_alignment=True)
        results = {}
        # The compact prefix this server announces, then the reference's full prefix; the server keeps
        # one session, so the second generation starts from its own /prefill.
        for tail in (8, None):
            client = rpc.RemoteTargetClient(url, timeout=60, prefix_tail=tail)
            assert client.health()["ok"] is True
            sent = []
            post = client._post
            client._post = lambda path, payload, post=post: (sent.append(dict(payload)), post(path, payload))[1]
            dr = drafter.DrafterRuntime(engine.LlamaEngine(dw, num_pages=256, page_size=4, max_positions=256))
            results[tail] = edge.PagedDistributedAtlasGenerator(config=cfg, drafter=dr,
                                                                target_client=client).generate(list(range(40, 60)))
            verifies = [p for p in sent if "routes" in p]
            assert verifies
            if tail:
                assert all("prefix_token_ids" not in p and len(p["prefix_tail_token_ids"]) <= tail for p in verifies)
            else:
                assert all(len(p["prefix_token_ids"]) >= 20 for p in verifies)
    finally:
        server.shutdown()
        server.server_close()
    tv2 = target.TargetVerifier(engine.LlamaEngine(tw, num_pages=256, page_size=4, max_positions=256), k=2, d=2)
    dr2 = drafter.DrafterRuntime(engine.LlamaEngine(dw, num_pages=256, page_size=4, max_positions=256))
    local = edge.PagedDistributedAtlasGenerator(config=cfg, drafter=dr2,
                                                target_client=rpc.InProcessTargetClient(tv2)).generate(
        list(range(40, 60)))
    for remote in results.values():
        assert remote.generated_token_ids == local.generated_token_ids
        assert [r.decision for r in remote.rounds] == [r.decision for r in local.rounds]


def test_client_sends_full_prefix_to_a_server_without_the_capability():
    rpc = mod("serving.rpc")
    client = rpc.RemoteTargetClient("http://127.0.0.1:9", prefix_tail=8)
    sent = []
    client.health = lambda: {"ok": True, "service": "atlas_0709_target"}  # e.g. the reference's server
    client._post = lambda path, payload: sent.append(dict(payload)) or {}
    client.verify(prefix_token_ids=list(range(30)), routes=[])
    assert sent[0]["prefix_token_ids"] == list(range(30)) and "prefix_len" not in sent[0]


def test_edge_cli_in_process_target(tmp_path, capsys):
    ds = mod("serving.distributed_system")
    out = tmp_path / "res.json"
    svg = tmp_path / "t.svg"
    rc = ds.main(["--drafter-model", "tiny-drafter", "--target-model", "tiny-target", "--dtype", "float32",
                  "--prompt-token-ids", ",".join(str(i) for i in range(30, 50)), "--k", "2", "--d", "2",
                  "--max-new-tokens", "8", "--page-size", "4", "--warmup-runs", "1", "--max-total-tokens", "2048",
                  "--json-out", str(out), "--timeline-svg", str(svg), "--validate-state-alignment"])
    assert rc == 0
    res = json.loads(out.read_text())
    assert len(res["generated_token_ids"]) == 8
    assert res["metadata"]["warmup_runs"] == 1
    assert svg.read_text().startswith("<svg")


def test_target_server_parser_defaults():
    ts = mod("serving.target_server")
    args = ts.build_parser().parse_args(["--model", "tiny-target", "--port", "0", "--path-score-weights",
                                          "0.45,0.30,0.17,0.08"])
    assert ts.parse_score_weights(args.path_score_weights) == (0.45, 0.30, 0.17, 0.08)
    assert args.route_selection_policy == "target_best"


def test_prompt_helpers():
    prompts = mod("serving.prompts")
    assert prompts.parse_token_ids("1, 2,3", tokenizer=None, prompt="x") == [1, 2, 3]
    assert prompts.parse_token_ids(None, tokenizer=None, prompt="x", prefix_len=5, repeat_token_id=7) == [7] * 5
    ids = prompts.parse_token_ids(None, tokenizer=None, prompt="hé")
    assert prompts.decode(None, ids) == "hé"


def test_forest_gate_flags_and_validation(tmp_path):
    ds = mod("serving.distributed_system")
    edge = mod("serving.edge")
    out = tmp_path / "res.json"
    rc = ds.main(["--drafter-model", "tiny-drafter", "--target-model", "tiny-target", "--dtype", "float32",
                  "--prompt-token-ids", ",".join(str(i) for i in range(40, 60)), "--k", "2", "--d", "2",
                  "--max-new-tokens", "6", "--page-size", "4", "--max-total-tokens", "2048",
                  "--forest-gate", "overlap", "--json-out", str(out)])
    assert rc == 0
    meta = json.loads(out.read_text())["metadata"]
    assert meta["forest_gate"] == "overlap" and meta["forest_gated_rounds"] == 0
    with pytest.raises(ValueError):
        edge.DistributedAtlasConfig(forest_gate="sometimes").validate()
    with pytest.raises(ValueError):
        edge.DistributedAtlasConfig(forest_gate_threshold=0.0).validate()


def test_console_scripts_resolve():
    """Every console script of pyproject.toml names a function of the entry module whose command
    module exists and has a ``main``."""
    import importlib
    import os
    import tomllib

    from conftest import REPO

    with open(os.path.join(REPO, "pyproject.toml"), "rb") as f:
        scripts = tomllib.load(f)["project"]["scripts"]
    assert "atlas-0709-run" in scripts and "atlas-target-server" in scripts
    entry = importlib.import_module("atlas_b200_entry")
    for name, ref in scripts.items():
        module, func = ref.split(":")
        assert module == "atlas_b200_entry" and callable(getattr(entry, func)), name
    for module in ("serving.cli", "serving.target_server", "serving.distributed_system", "serving.check_equivalence",
                   "serving.diagnostics", "eval.gsm8k", "eval.mtbench", "eval.sweep", "eval.compare_interventions"):
        assert callable(mod(module).main)
