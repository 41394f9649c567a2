"""MT-Bench style evaluation: multi-turn generation and single-answer LLM grading.

    python -m 0709_b200.eval.mtbench generate --backend atlas --questions q.jsonl --output-dir out ...
    python -m 0709_b200.eval.mtbench judge --answers out/answers.jsonl --judge-url https://.../v1/chat/completions

``generate`` reads local question records (``question_id``, ``category``,
``turns``: list of user turns), runs each conversation turn by turn (the
next prompt is the previous prompt + the model's answer + the new turn), and
writes one answer record per question with a compact per-round detail of the
ATLAS rounds (decision, fallback reason, best selection score, first-token
log-prob) and the target-intervention summary.  ``judge`` sends each answer
to an OpenAI-compatible chat-completions endpoint (API key from
``--api-key-env``), parses the ``[[rating]]`` the grading prompt asks for,
and writes judgments plus a per-category average.  This machine has no
network, so ``judge`` only runs where the endpoint is reachable.

Parity: reference scripts/mtbench_deepseek_eval.py (generate_answers,
rounds_detail, judge client).
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import urllib.request
from pathlib import Path

from ..serving.prompts import decode, encode, load_tokenizer
from ..utils.interventions import summarize_generation_interventions
from .common import add_generation_flags, append_jsonl, make_generate, read_jsonl, timed

RATING_RE = re.compile(r"\[\[(\d+(?:\.\d+)?)\]\]")
JUDGE_PROMPT = (
    "Please act as an impartial judge and evaluate the quality of the response provided by an AI assistant to "
    "the user question displayed below. Consider helpfulness, relevance, accuracy, depth and level of detail. "
    "Begin with a short explanation, then rate the response on a scale of 1 to 10 strictly in this format: "
    "\"[[rating]]\", for example \"Rating: [[5]]\".\n\n[Question]\n{question}\n\n[The Start of Assistant's Answer]\n"
    "{answer}\n[The End of Assistant's Answer]"
)


def compact_rounds(rounds) -> list[dict]:
    out = []
    for r in rounds:
        md = dict(getattr(r, "target_decision_metadata", {}) or {})
        out.append({"round_index": r.round_index, "decision": r.decision, "fallback_reason": r.fallback_reason,
                    "committed_tokens": len(r.committed_tokens), "handoff_mode": r.handoff_mode,
                    "best_selection_score": md.get("best_selection_score"),
                    "best_first_token_logprob": md.get("best_first_token_logprob")})
    return out


def cmd_generate(args) -> int:
    tok = load_tokenizer(args.tokenizer)
    qs = read_jsonl(args.questions)
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    path = out / "answers.jsonl"
    done = {r["question_id"] for r in read_jsonl(path)} if (args.resume and path.exists()) else set()
    if not args.resume and path.exists():
        path.unlink()
    generate = make_generate(args)
    for q in qs:
        if q["question_id"] in done:
            continue
        history: list[int] = []
        turns = []
        for t, user in enumerate(q["turns"]):
            ids = history + encode(tok, f"User: {user}\nAssistant:")
            (gen, meta, rounds), secs = timed(generate, ids)
            text = decode(tok, gen) or ""
            turn = {"turn": t, "answer": text, "generated_tokens": len(gen), "elapsed_s": secs}
            if rounds:
                turn["rounds_detail"] = compact_rounds(rounds)
                turn["target_intervention"] = {k: v for k, v in summarize_generation_interventions(
                    [r.to_dict() for r in rounds]).items() if k != "rounds"}
            turns.append(turn)
            history = ids + list(gen) + encode(tok, "\n")
        append_jsonl(path, {"question_id": q["question_id"], "category": q.get("category"), "model": args.model,
                            "backend": args.backend, "turns": turns})
    print(json.dumps({"answers": str(path), "questions": len(qs)}))
    return 0


def judge_one(url: str, model: str, key: str | None, question: str, answer: str, timeout: float) -> tuple[float | None, str]:
    body = {"model": model, "temperature": 0.0,
            "messages": [{"role": "user", "content": JUDGE_PROMPT.format(question=question, answer=answer)}]}
    req = urllib.request.Request(url, data=json.dumps(body).encode(), method="POST",
                                 headers={"content-type": "application/json",
                                          **({"authorization": f"Bearer {key}"} if key else {})})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        content = json.loads(r.read().decode())["choices"][0]["message"]["content"]
    m = RATING_RE.search(content)
    return (float(m.group(1)) if m else None), content


def cmd_judge(args) -> int:
    answers = read_jsonl(args.answers)
    qs = {q["question_id"]: q for q in read_jsonl(args.questions)}
    key = os.environ.get(args.api_key_env) if args.api_key_env else None
    out = Path(args.output or (Path(args.answers).parent / "judgments.jsonl"))
    scores: dict[str, list[float]] = {}
    failures = 0
    for a in answers:
        q = qs[a["question_id"]]
        for t in a["turns"]:
            try:
                rating, raw = judge_one(args.judge_url, args.judge_model, key, q["turns"][t["turn"]], t["answer"],
                                        args.timeout)
            except Exception as exc:  # noqa: BLE001 - recorded, the run continues
                rating, raw = None, f"error: {exc!r}"
                failures += 1
            append_jsonl(out, {"question_id": a["question_id"], "turn": t["turn"], "rating": rating, "judgment": raw})
            if rating is not None:
                scores.setdefault(str(a.get("category")), []).append(rating)
    allv = [v for vs in scores.values() for v in vs]
    print(json.dumps({"mean": statistics.fmean(allv) if allv else None, "judged": len(allv), "failures": failures,
                      "by_category": {c: statistics.fmean(v) for c, v in sorted(scores.items())}}))
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="MT-Bench generation and judging")
    sub = p.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("generate")
    add_generation_flags(g)
    g.add_argument("--questions", required=True)
    g.add_argument("--output-dir", required=True)
    j = sub.add_parser("judge")
    j.add_argument("--answers", required=True)
    j.add_argument("--questions", required=True)
    j.add_argument("--judge-url", required=True)
    j.add_argument("--judge-model", default="deepseek-chat")
    j.add_argument("--api-key-env", default="JUDGE_API_KEY")
    j.add_argument("--timeout", type=float, default=120.0)
    j.add_argument("--output", default=None)
    args = p.parse_args(argv)
    return cmd_generate(args) if args.cmd == "generate" else cmd_judge(args)


if __name__ == "__main__":
    raise SystemExit(main())
