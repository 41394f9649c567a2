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
