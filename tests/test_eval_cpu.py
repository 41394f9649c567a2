"""Evaluation drivers on CPU with tiny random-init models (plumbing; the answers are noise)."""

from __future__ import annotations

import json
import threading
from http.server import BaseHTTPRequestHandler, HTTPServer

from conftest import mod


def _flags(tmp_path, backend):
    return ["--backend", backend, "--model", "tiny-drafter", "--target-model", "tiny-target", "--dtype", "float32",
            "--page-size", "4", "--max-new-tokens", "6", "--k", "2", "--d", "2", "--path-score-weights", "",
            "--device", "cpu", "--context-length", "512"]


def test_answer_extraction():
    g = mod("eval.gsm8k")
    assert g.gold_answer({"answer": "blah\n#### 1,234"}) == "1234"
    assert g.extract("... so 3 + 4 = 7. The final answer is $7.") == "7"
    assert g.extract("numbers 3 and 12.50") == "12.5"
    assert g.extract("no marker 5", strict=True) is None


def test_gsm8k_driver_atlas_and_resume(tmp_path):
    g = mod("eval.gsm8k")
    data = tmp_path / "test.jsonl"
    data.write_text("\n".join(json.dumps({"question": f"What is {i}+1?", "answer": f"x\n#### {i + 1}"})
                              for i in range(3)) + "\n")
    out = tmp_path / "out"
    assert g.main(_flags(tmp_path, "atlas") + ["--data-file", str(data), "--output-dir", str(out),
                                                 "--max-examples", "2"]) == 0
    rows = [json.loads(l) for l in (out / "predictions.jsonl").read_text().splitlines()]
    assert [r["index"] for r in rows] == [0, 1] and all("target_intervention" in r for r in rows)
    assert g.main(_flags(tmp_path, "atlas") + ["--data-file", str(data), "--output-dir", str(out), "--resume"]) == 0
    rows = [json.loads(l) for l in (out / "predictions.jsonl").read_text().splitlines()]
    assert [r["index"] for r in rows] == [0, 1, 2]
    summary = json.loads((out / "summary.json").read_text())
    assert summary["samples"] == 3 and summary["target_intervention"]["samples_with_statistics"] == 3


def test_mtbench_generate_and_judge_against_local_endpoint(tmp_path):
    mt = mod("eval.mtbench")
    q = tmp_path / "q.jsonl"
    q.write_text(json.dumps({"question_id": 1, "category": "math", "turns": ["hi", "and then?"]}) + "\n")
    out = tmp_path / "mt"
    assert mt.main(["generate", *_flags(tmp_path, "atlas"), "--questions", str(q), "--output-dir", str(out)]) == 0
    ans = json.loads((out / "answers.jsonl").read_text().splitlines()[0])
    assert len(ans["turns"]) == 2 and "rounds_detail" in ans["turns"][0]

    class H(BaseHTTPRequestHandler):
        def do_POST(self):  # noqa: N802
            self.rfile.read(int(self.headers["content-length"]))
            body = json.dumps({"choices": [{"message": {"content": "fine. Rating: [[7]]"}}]}).encode()
            self.send_response(200)
            self.send_header("content-type", "application/json")
            self.send_header("content-length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def log_message(self, *a):
            pass

    srv = HTTPServer(("127.0.0.1", 0), H)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        url = f"http://127.0.0.1:{srv.server_address[1]}/v1/chat/completions"
        assert mt.main(["judge", "--answers", str(out / "answers.jsonl"), "--questions", str(q), "--judge-url", url,
                        "--api-key-env", ""]) == 0
    finally:
        srv.shutdown()
    j = [json.loads(l) for l in (out / "judgments.jsonl").read_text().splitlines()]
    assert [x["rating"] for x in j] == [7.0, 7.0]


class _Judge:
    """A local chat-completions endpoint: answers ``[[7]]``, first failing ``fail_first`` calls with 503."""

    def __init__(self, fail_first: int = 0) -> None:
        self.bodies: list[dict] = []
        self.fail_first = fail_first
        owner = self

        class H(BaseHTTPRequestHandler):
            def do_POST(self):  # noqa: N802
                owner.bodies.append(json.loads(self.rfile.read(int(self.headers["content-length"]))))
                if owner.fail_first > 0:
                    owner.fail_first -= 1
                    self.send_response(503)
                    self.send_header("content-length", "0")
                    self.end_headers()
                    return
                body = json.dumps({"choices": [{"message": {"content": "ok. Rating: [[7]]"}}]}).encode()
                self.send_response(200)
                self.send_header("content-type", "application/json")
                self.send_header("content-length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def log_message(self, *a):
                pass

        self.srv = HTTPServer(("127.0.0.1", 0), H)
        self.base = f"http://127.0.0.1:{self.srv.server_address[1]}/v1"
        threading.Thread(target=self.srv.serve_forever, daemon=True).start()

    def close(self) -> None:
        self.srv.shutdown()


def test_generation_flag_helpers():
    c = mod("eval.common")
    w = c.exponential_path_weights(4, 0.5)
    assert abs(sum(w) - 1.0) < 1e-12 and all(a > b for a, b in zip(w, w[1:]))
    assert c.exponential_path_weights(3, 0.0) == (1 / 3, 1 / 3, 1 / 3)
    mt = mod("eval.mtbench")
    assert mt.chat_completions_url("https://x/v1/") == "https://x/v1/chat/completions"
    assert mt.chat_completions_url("https://x/v1/chat/completions") == "https://x/v1/chat/completions"
    assert mt.parse_rating("Rating: [[8.5]]") == 8.5
    assert mt.parse_rating('```json\n{"score": 6, "reason": "r"}\n```') == 6.0
    assert mt.parse_rating("no score") is None


def test_gsm8k_reference_flags(tmp_path):
    import pytest

    g = mod("eval.gsm8k")
    data = tmp_path / "test.jsonl"
    data.write_text(json.dumps({"question": "What is 1+1?", "answer": "x\n#### 2"}) + "\n")
    out = tmp_path / "out"
    ref_flags = ["--path-weight-alpha", "0.3", "--fixed-forest-depth", "1", "--validate-state-alignment",
                 "--drafter-do-sample", "--drafter-temperature", "0.8", "--mem-fraction-static", "0.75",
                 "--max-running-requests", "32", "--nccl-port", "29500", "--warmup-runs", "0",
                 "--system-prompt", "Be brief.", "--protocol", "zero-shot", "--use-packed-custom-mask"]
    assert g.main(_flags(tmp_path, "atlas") + ["--data-file", str(data), "--output-dir", str(out)] + ref_flags) == 0
    assert json.loads((out / "summary.json").read_text())["samples"] == 1
    with pytest.raises(SystemExit):
        g.main(_flags(tmp_path, "atlas") + ["--data-file", str(data), "--output-dir", str(out),
                                              "--protocol", "llama-8shot"])


def test_mtbench_reference_one_command_form(tmp_path, monkeypatch):
    mt = mod("eval.mtbench")
    q = tmp_path / "q.jsonl"
    q.write_text("\n".join(json.dumps({"question_id": i, "category": "c", "turns": ["hi", "more?"]})
                           for i in range(3)) + "\n")
    out = tmp_path / "mt"
    judge = _Judge(fail_first=1)
    monkeypatch.setenv("TEST_JUDGE_KEY", "k")
    flags = ["--drafter-model", "tiny-drafter", "--target-model", "tiny-target", "--dtype", "float32",
             "--page-size", "4", "--max-new-tokens", "4", "--k", "2", "--d", "2", "--path-score-weights", "",
             "--device", "cpu", "--context-length", "256", "--questions-file", str(q), "--output-dir", str(out),
             "--max-questions", "2", "--turn-mode", "first", "--execution-mode", "serial", "--warmup-runs", "0",
             "--judge-base-url", judge.base, "--deepseek-api-key-env", "TEST_JUDGE_KEY", "--judge-retry-delay", "0",
             "--judge-thinking", "enabled", "--judge-reasoning-effort", "high", "--judge-repeats", "2"]
    try:
        assert mt.main(flags) == 0
        answers = [json.loads(l) for l in (out / "answers.jsonl").read_text().splitlines()]
        assert [a["question_id"] for a in answers] == [0, 1] and all(len(a["turns"]) == 1 for a in answers)
        assert answers[0]["backend"] == "atlas_serial"
        js = [json.loads(l) for l in (out / "judgments.jsonl").read_text().splitlines()]
        assert len(js) == 4 and {x["rating"] for x in js} == {7.0} and {x["repeat"] for x in js} == {0, 1}
        # One 503 retried; the DeepSeek fields and the token limit ride in every request.
        assert len(judge.bodies) == 5
        assert judge.bodies[-1]["thinking"] == {"type": "enabled"} and judge.bodies[-1]["reasoning_effort"] == "high"
        assert judge.bodies[-1]["max_tokens"] == 4096
        # Resume: nothing generated or judged again; AR answers are graded beside them.
        ar = tmp_path / "ar.jsonl"
        ar.write_text(json.dumps({"question_id": 0, "model": "ar_1b", "run_id": "r1",
                                  "turns": [{"turn": 0, "answer": "x"}]}) + "\n")
        n = len(judge.bodies)
        assert mt.main(flags + ["--skip-generate", "--resume-judge", "--ar-generations", str(ar),
                                "--ar-run-id", "r1"]) == 0
        assert len(judge.bodies) == n + 2
        js = [json.loads(l) for l in (out / "judgments.jsonl").read_text().splitlines()]
        assert sorted({x["source"] for x in js}) == ["answers", "ar:ar_1b"]
    finally:
        judge.close()


def test_gsm8k_sweeps(tmp_path):
    sw = mod("eval.sweep")
    data = tmp_path / "test.jsonl"
    data.write_text("\n".join(json.dumps({"question": f"What is {i}+1?", "answer": f"x\n#### {i + 1}"})
                              for i in range(2)) + "\n")
    gen = ["--data-file", str(data), "--dtype", "float32", "--page-size", "4", "--max-new-tokens", "4", "--k", "2",
           "--d", "2", "--device", "cpu", "--context-length", "512", "--warmup-runs", "0"]
    out = tmp_path / "fb"
    assert sw.main(["fallback", "--drafter-model", "tiny-drafter", "--target-model", "tiny-target", "--output-dir",
                    str(out), "--thresholds", "none", "1e9", *gen]) == 0
    rows = json.loads((out / "results.json").read_text())
    assert [r["fallback_threshold"] for r in rows] == [None, 1e9]
    assert rows[0]["fallback_rounds"] == 0 and rows[1]["fallback_rate"] == 1.0 and rows[1]["count"] == 2
    assert rows[0]["fallback_enabled"] is False and rows[1]["serial_overall_tokens_per_second"] > 0
    exp = json.loads((out / "experiment.json").read_text())
    assert exp["changed_variable"] == "fallback_threshold" and len(exp["fixed_path_score_weights"]) == 2
    assert (out / "threshold_none" / "summary.json").exists() and (out / "results.csv").exists()
    pw = tmp_path / "pw"
    assert sw.main(["path-weights", "--drafter-model", "tiny-drafter", "--target-model", "tiny-target",
                    "--output-dir", str(pw), "--alphas", "0", "0.5", "--dry-run", *gen]) == 0
    exp = json.loads((pw / "experiment.json").read_text())
    assert [r["output_dir"].rsplit("/", 1)[-1] for r in exp["runs"]] == ["alpha_0", "alpha_0p5"]
    assert exp["weights_by_alpha"]["0"] == [0.5, 0.5] and not (pw / "results.json").exists()


def test_gsm8k_launcher_script(tmp_path):
    import os
    import subprocess

    from conftest import REPO

    data = tmp_path / "test.jsonl"
    data.write_text(json.dumps({"question": "What is 1+1?", "answer": "x\n#### 2"}) + "\n")
    env = dict(os.environ, DRAFTER_MODEL="tiny-drafter", TARGET_MODEL="tiny-target", GSM8K_FILE=str(data),
               OUTPUT_DIR=str(tmp_path / "out"), K="2", D="2", MAX_NEW_TOKENS="4", CONTEXT_LENGTH="512",
               WARMUP_RUNS="0")
    script = os.path.join(REPO, "0709_b200", "eval", "run_gsm8k.sh")
    r = subprocess.run(["bash", script, "atlas-serial", "--device", "cpu", "--dtype", "float32", "--page-size", "4",
                        "--path-score-weights", ""], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    summary = json.loads((tmp_path / "out" / "summary.json").read_text())
    assert summary["backend"] == "atlas_serial" and summary["count"] == 1 and summary["settings"]["k"] == 2
    assert summary["serial_speed"]["rounds"] > 0 and summary["serial_speed"]["overall_tokens_per_second"] > 0
    bad = subprocess.run(["bash", script, "nope"], env=env, capture_output=True, text=True, timeout=60)
    assert bad.returncode == 2


def test_gsm8k_records_failed_samples_and_goes_on(tmp_path, monkeypatch):
    g = mod("eval.gsm8k")
    data = tmp_path / "test.jsonl"
    data.write_text("\n".join(json.dumps({"question": f"q{i}", "answer": f"#### {i}"}) for i in range(3)) + "\n")
    calls = []

    def fake_make_generate(args):
        def run(ids, seed=None):
            calls.append(len(ids))
            if len(calls) == 2:
                raise RuntimeError("boom")
            return [ord(c) for c in "The final answer is 2."], {}, []
        return run

    monkeypatch.setattr(g, "make_generate", fake_make_generate)
    out = tmp_path / "out"
    assert g.main(["--backend", "ar", "--model", "m", "--data-file", str(data), "--output-dir", str(out),
                   "--warmup-runs", "0"]) == 0
    summary = json.loads((out / "summary.json").read_text())
    assert summary["count"] == 2 and summary["failures"] == 1 and summary["correct"] == 1
    assert json.loads((out / "failures.jsonl").read_text())["index"] == 1


def test_gsm8k_request_seeds_and_sampled_ar(tmp_path):
    """Each GSM8K request gets seed = generation seed + index; the AR backend samples with it."""
    g = mod("eval.gsm8k")
    data = tmp_path / "test.jsonl"
    data.write_text("\n".join(json.dumps({"question": f"What is {i}+1?", "answer": f"#### {i + 1}"})
                              for i in range(2)) + "\n")
    rows = {}
    for name, extra in (("greedy", []), ("sampled", ["--drafter-do-sample", "--drafter-temperature", "1.5"])):
        out = tmp_path / name
        assert g.main(["--backend", "ar", "--model", "tiny-drafter", "--dtype", "float32", "--page-size", "4",
                       "--max-new-tokens", "8", "--device", "cpu", "--context-length", "256", "--warmup-runs", "0",
                       "--generation-seed", "10", "--data-file", str(data), "--output-dir", str(out), *extra]) == 0
        rows[name] = [json.loads(l) for l in (out / "predictions.jsonl").read_text().splitlines()]
        assert json.loads((out / "summary.json").read_text())["settings"]["request_seed_rule"] == \
            "generation_seed_plus_gsm8k_index"
    assert [r["generation_seed"] for r in rows["sampled"]] == [10, 11]
    assert [r["response"] for r in rows["greedy"]] != [r["response"] for r in rows["sampled"]]


def test_compare_interventions_pairs_runs(tmp_path):
    import pytest

    g, cmp_ = mod("eval.gsm8k"), mod("eval.compare_interventions")
    data = tmp_path / "test.jsonl"
    data.write_text("\n".join(json.dumps({"question": f"What is {i}+1?", "answer": f"x\n#### {i + 1}"})
                              for i in range(2)) + "\n")
    runs = {}
    for policy in ("target_best", "first_route"):
        out = tmp_path / policy
        extra = ["--fallback-threshold", "none", "--first-token-threshold", "none"] if policy == "first_route" else []
        assert g.main(_flags(tmp_path, "atlas_serial") + ["--data-file", str(data), "--output-dir", str(out),
                                                        "--route-selection-policy", policy, "--warmup-runs", "0",
                                                        *extra]) == 0
        runs[policy] = out
    rep = cmp_.compare(runs["target_best"], runs["first_route"])
    assert rep["alignment"]["samples"] == 2 and rep["alignment"]["prompt_hash_checked"] == 2
    assert rep["policies"] == {"target_best": "target_best", "first_route": "first_route",
                               "policy_metadata_missing": False}
    assert rep["paired_quality"]["pair_count"] == 2
    with pytest.raises(ValueError):
        cmp_.compare(runs["first_route"], runs["target_best"])  # the policies do not match their flags
    out = tmp_path / "cmp.json"
    assert cmp_.main(["--target-best", str(runs["target_best"] / "predictions.jsonl"), "--first-route",
                      str(runs["first_route"]), "--json-out", str(out)]) == 0
    assert json.loads(out.read_text())["comparison"] == "paired_target_best_vs_first_route"


def test_mtbench_ar_baselines_feed_the_atlas_run(tmp_path, monkeypatch):
    mt = mod("eval.mtbench")
    q = tmp_path / "q.jsonl"
    q.write_text("\n".join(json.dumps({"question_id": i, "category": "c", "turns": ["hi"]}) for i in range(2)) + "\n")
    judge = _Judge()
    monkeypatch.setenv("TEST_JUDGE_KEY", "k")
    common = ["--dtype", "float32", "--page-size", "4", "--max-new-tokens", "3", "--device", "cpu",
              "--context-length", "128", "--questions-file", str(q), "--warmup-runs", "0",
              "--judge-base-url", judge.base, "--deepseek-api-key-env", "TEST_JUDGE_KEY", "--judge-retry-delay", "0"]
    try:
        ar_out = tmp_path / "ar"
        assert mt.main(["--model-1b", "tiny-drafter", "--model-8b", "tiny-target", "--output-dir", str(ar_out),
                        *common]) == 0
        gens = [json.loads(l) for l in (ar_out / "generations.jsonl").read_text().splitlines()]
        assert sorted((g["model"], g["question_id"]) for g in gens) == [("ar_1b", 0), ("ar_1b", 1), ("ar_8b", 0),
                                                                      ("ar_8b", 1)]
        rid = gens[0]["run_id"]
        assert {g["run_id"] for g in gens} == {rid}
        js = [json.loads(l) for l in (ar_out / "judgments.jsonl").read_text().splitlines()]
        assert sorted({x["source"] for x in js}) == ["ar:ar_1b", "ar:ar_8b"] and len(js) == 4
        # The ATLAS run grades its own answers and the AR run's, named by its run id.
        out = tmp_path / "atlas"
        assert mt.main(["--drafter-model", "tiny-drafter", "--target-model", "tiny-target", "--k", "2", "--d", "2",
                        "--path-score-weights", "", "--output-dir", str(out), "--ar-generations",
                        str(ar_out / "generations.jsonl"), "--ar-run-id", rid, *common]) == 0
        js = [json.loads(l) for l in (out / "judgments.jsonl").read_text().splitlines()]
        assert sorted({x["source"] for x in js}) == ["answers", "ar:ar_1b", "ar:ar_8b"]
    finally:
        judge.close()


def _chat_tokenizer(path):
    """A small word-level tokenizer with a chat template and an end-of-turn token."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    words = ["<unk>", "<|eot_id|>", "<s>", "user:", "assistant:", "system:"] + [str(i) for i in range(10)] + \
        ["What", "is", "The", "final", "answer", "Question:", "Solve", "the", "problem", "step", "by"]
    t = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="<unk>"))
    t.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok = PreTrainedTokenizerFast(tokenizer_object=t, unk_token="<unk>", eos_token="<s>")
    tok.chat_template = ("{% for m in messages %}{{ m['role'] }}: {{ m['content'] }} <|eot_id|> {% endfor %}"
                         "{% if add_generation_prompt %}assistant: {% endif %}")
    tok.save_pretrained(path)
    return tok


def test_gsm8k_chat_template_prompts(tmp_path):
    g, prompts = mod("eval.gsm8k"), mod("serving.prompts")
    tok_dir = tmp_path / "tok"
    _chat_tokenizer(str(tok_dir))
    chat = prompts.load_chat_tokenizer(str(tok_dir))
    assert chat is not None and prompts.chat_stop_token(chat) == 1
    assert prompts.load_chat_tokenizer(str(tmp_path)) is None  # no template there
    data = tmp_path / "test.jsonl"
    data.write_text(json.dumps({"question": "What is 1 1", "answer": "#### 2"}) + "\n")
    out = tmp_path / "out"
    assert g.main(_flags(tmp_path, "atlas") + ["--data-file", str(data), "--output-dir", str(out), "--tokenizer",
                                                 str(tok_dir), "--warmup-runs", "0", "--system-prompt", "by"]) == 0
    row = json.loads((out / "predictions.jsonl").read_text())
    want = prompts.chat_ids(chat, g.build_messages("What is 1 1", [], "by"))
    assert row["prompt_tokens"] == len(want) and want[-1] == chat.convert_tokens_to_ids("assistant:")
    summary = json.loads((out / "summary.json").read_text())
    assert summary["settings"]["eos_token_id"] == 1 and summary["settings"]["chat_template"] == "auto"


def test_mtbench_chat_template_conversation(tmp_path):
    mt, prompts = mod("eval.mtbench"), mod("serving.prompts")
    tok_dir = tmp_path / "tok"
    chat = _chat_tokenizer(str(tok_dir))
    q = tmp_path / "q.jsonl"
    q.write_text(json.dumps({"question_id": 1, "category": "math", "turns": ["What is 1", "The 2"]}) + "\n")
    out = tmp_path / "mt"
    assert mt.main(["generate", *_flags(tmp_path, "atlas"), "--questions", str(q), "--output-dir", str(out),
                    "--tokenizer", str(tok_dir), "--warmup-runs", "0"]) == 0
    ans = json.loads((out / "answers.jsonl").read_text())
    assert len(ans["turns"]) == 2
    # The second prompt is the whole conversation rendered by the template (no tokens lost between turns).
    first = prompts.chat_ids(chat, [{"role": "user", "content": "What is 1"}])
    second = prompts.chat_ids(chat, [{"role": "user", "content": "What is 1"},
                                     {"role": "assistant", "content": ans["turns"][0]["answer"]},
                                     {"role": "user", "content": "The 2"}])
    assert [t["prompt_tokens"] for t in ans["turns"]] == [len(first), len(second)]
