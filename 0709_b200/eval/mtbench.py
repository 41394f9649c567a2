"""MT-Bench style evaluation: multi-turn generation and single-answer LLM grading.

    python -m 0709_b200.eval.mtbench generate --backend atlas --questions q.jsonl --output-dir out ...
    python -m 0709_b200.eval.mtbench judge --answers out/answers.jsonl --judge-url https://.../v1/chat/completions
    python -m 0709_b200.eval.mtbench --drafter-model ... --target-url ... --questions-file q.jsonl --output-dir out
    python -m 0709_b200.eval.mtbench --model-1b ... --model-8b ... --questions-file q.jsonl --output-dir ar_out

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

The fourth form writes the AR baselines: greedy answers of a 1B and an 8B model into one
``generations.jsonl`` under a run id that an ATLAS run names with ``--ar-generations`` /
``--ar-run-id``, then grades them.  The third form is the reference's one command (generate, then judge; ``--skip-*`` and
``--resume-*`` per phase; ``--ar-generations`` grades AR answers in the same run).  The judge
retries HTTP 429 / 5xx and connection errors, can grade each answer ``--judge-repeats`` times,
and sends the DeepSeek ``thinking`` / ``reasoning_effort`` fields when they are given.

Parity: reference scripts/mtbench_deepseek_eval.py (generate_answers :314-542,
rounds_detail :164-207, judge client :545-662, flags :1299-1383).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
import statistics
import sys
import time
import urllib.error
import urllib.request
from dataclasses import dataclass
from pathlib import Path

from ..serving.prompts import chat_ids, chat_stop_token, decode, encode, load_chat_tokenizer, load_tokenizer
from ..utils.interventions import summarize_generation_interventions
from .common import add_atlas_flags, add_generation_flags, add_runtime_compat_flags, append_jsonl, make_generate, \
    read_jsonl, timed, warm_up

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


def select_questions(qs: list[dict], args) -> list[dict]:
    """``--question-start`` / ``--question-end`` slice, then at most ``--max-questions``."""
    qs = qs[int(getattr(args, "question_start", 0) or 0): getattr(args, "question_end", None)]
    n = getattr(args, "max_questions", None)
    return qs[: int(n)] if n is not None else qs


def cmd_generate(args, *, path: Path | None = None, extra: dict | None = None, keep_file: bool = False) -> int:
    """Answer every selected question into ``path`` (default ``<output-dir>/answers.jsonl``).
    ``extra`` fields go into every record (an AR run's label and run id); with ``--resume`` the
    questions already answered under the same ``extra`` are skipped; ``keep_file`` keeps records
    of other runs in a shared file."""
    tok = load_tokenizer(args.tokenizer)
    qs = select_questions(read_jsonl(args.questions), args)
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    path = path or out / "answers.jsonl"
    extra = dict(extra or {})

    def mine(r) -> bool:
        return all(r.get(key) == val for key, val in extra.items())

    done = {r["question_id"] for r in read_jsonl(path) if mine(r)} if (args.resume and path.exists()) else set()
    if not args.resume and path.exists() and not keep_file:
        path.unlink()
    chat = load_chat_tokenizer(args.tokenizer) if getattr(args, "chat_template", "auto") == "auto" else None
    if chat is not None and args.eos_token_id is None:
        args.eos_token_id = chat_stop_token(chat)
    generate = make_generate(args)
    sys_prompt = getattr(args, "system_prompt", "") or ""
    system = f"System: {sys_prompt}\n" if sys_prompt else ""
    pending = [q for q in qs if q["question_id"] not in done]
    if pending:
        first = pending[0]["turns"][0]
        warm_up(generate, chat_ids(chat, [{"role": "user", "content": first}]) if chat is not None
                else encode(tok, f"{system}User: {first}\nAssistant:"), args.warmup_runs)
    for q in pending:
        history: list[int] = encode(tok, system) if system and chat is None else []
        messages = [{"role": "system", "content": sys_prompt}] if sys_prompt else []
        turns = []
        user_turns = q["turns"][:1] if getattr(args, "turn_mode", "conversation") == "first" else q["turns"]
        for t, user in enumerate(user_turns):
            if chat is not None:
                # The conversation so far, rendered by the checkpoint's own chat template.
                messages.append({"role": "user", "content": user})
                ids = chat_ids(chat, messages)
            else:
                ids = history + encode(tok, f"User: {user}\nAssistant:")
            (gen, meta, rounds), secs = timed(generate, ids)
            text = (chat.decode(gen, skip_special_tokens=True) if chat is not None else decode(tok, gen)) or ""
            if chat is not None:
                messages.append({"role": "assistant", "content": text})
            turn = {"turn": t, "answer": text, "prompt_tokens": len(ids), "generated_tokens": len(gen),
                    "elapsed_s": secs}
            if rounds:
                turn["rounds_detail"] = compact_rounds(rounds)
                turn["target_intervention"] = {k: v for k, v in summarize_generation_interventions(
                    [r.to_dict() for r in rounds]).items() if k != "rounds"}
            turns.append(turn)
            history = ids + list(gen) + encode(tok, "\n")
        append_jsonl(path, {"question_id": q["question_id"], "category": q.get("category"), "model": args.model,
                            "backend": args.backend, "turns": turns, **extra})
    print(json.dumps({"answers": str(path), "questions": len(qs)}))
    return 0


@dataclass(frozen=True)
class JudgeSettings:
    """One chat-completions endpoint and how to call it.  ``thinking`` / ``reasoning_effort`` are
    DeepSeek request fields (sent only when set); HTTP 429 / 5xx and connection errors are
    retried ``retries`` times with exponentially growing delays."""

    url: str
    model: str
    key: str | None = None
    timeout: float = 120.0
    retries: int = 0
    retry_delay: float = 2.0
    max_tokens: int | None = None
    thinking: str | None = None
    reasoning_effort: str | None = None


def chat_completions_url(base: str) -> str:
    base = base.rstrip("/")
    return base if base.endswith("/chat/completions") else f"{base}/chat/completions"


def parse_rating(content: str) -> float | None:
    """``[[r]]`` as the grading prompt asks, else the ``score`` of a JSON object answer."""
    m = RATING_RE.search(content or "")
    if m:
        return float(m.group(1))
    text = (content or "").strip().strip("`")
    text = text[4:] if text.startswith("json") else text
    try:
        obj = json.loads(text)
    except ValueError:
        return None
    score = obj.get("score") if isinstance(obj, dict) else None
    return float(score) if isinstance(score, (int, float)) and not isinstance(score, bool) else None


def judge_one(s: JudgeSettings, question: str, answer: str) -> tuple[float | None, str]:
    body: dict = {"model": s.model, "temperature": 0.0, "stream": False,
                  "messages": [{"role": "user", "content": JUDGE_PROMPT.format(question=question, answer=answer)}]}
    if s.max_tokens:
        body["max_tokens"] = int(s.max_tokens)
    if s.thinking:
        body["thinking"] = {"type": s.thinking}
        if s.thinking == "enabled" and s.reasoning_effort:
            body["reasoning_effort"] = s.reasoning_effort
    data = json.dumps(body, ensure_ascii=False).encode("utf-8")
    headers = {"content-type": "application/json; charset=utf-8", **({"authorization": f"Bearer {s.key}"} if s.key else {})}
    last: Exception | None = None
    for attempt in range(int(s.retries) + 1):
        try:
            req = urllib.request.Request(s.url, data=data, method="POST", headers=headers)
            with urllib.request.urlopen(req, timeout=s.timeout) as r:
                content = json.loads(r.read().decode("utf-8"))["choices"][0]["message"]["content"]
            if not content:
                raise ValueError("empty judge content")
            return parse_rating(content), content
        except urllib.error.HTTPError as exc:
            last = exc
            if exc.code != 429 and not 500 <= exc.code < 600:
                raise
        except (urllib.error.URLError, TimeoutError, KeyError, IndexError, ValueError) as exc:
            last = exc
        if attempt < int(s.retries):
            time.sleep(float(s.retry_delay) * 2 ** attempt)
    raise RuntimeError(f"judge failed after {int(s.retries) + 1} attempts: {last!r}")


def _answer_sets(args) -> list[tuple[str, list[dict]]]:
    """(label, answer records) of every answer file to grade: ``--answers`` and, with
    ``--ar-generations``, the AR answers (records of ``generate --backend ar``; ``--ar-run-id``
    keeps the records whose ``run_id`` matches).  Each answer is graded on its own, so the
    judge never sees which system wrote it."""
    sets = [("answers", read_jsonl(args.answers))] if getattr(args, "answers", None) else []
    extra = getattr(args, "ar_generations", None)
    if extra:
        recs = read_jsonl(extra)
        run = getattr(args, "ar_run_id", None)
        if run is not None:
            recs = [r for r in recs if str(r.get("run_id")) == str(run)]
            if not recs:
                raise SystemExit(f"--ar-run-id {run}: no record of {extra} carries that run_id")
        groups: dict[str, list[dict]] = {}
        for r in recs:
            groups.setdefault(f"ar:{r.get('model', 'unknown')}", []).append(r)
        sets += sorted(groups.items())
    return sets


def cmd_judge(args) -> int:
    qs = {q["question_id"]: q for q in read_jsonl(args.questions)}
    settings = JudgeSettings(
        url=args.judge_url or chat_completions_url(args.judge_base_url), model=args.judge_model,
        key=os.environ.get(args.api_key_env) if args.api_key_env else None, timeout=args.timeout,
        retries=args.judge_retries, retry_delay=args.judge_retry_delay, max_tokens=args.judge_max_tokens,
        thinking=args.judge_thinking, reasoning_effort=args.judge_reasoning_effort)
    out = Path(args.output or (Path(args.answers or args.ar_generations).parent / "judgments.jsonl"))
    done: set[tuple] = set()
    if out.exists():
        if getattr(args, "resume", False):
            done = {(str(r.get("source", "answers")), r["question_id"], r["turn"], r.get("repeat", 0))
                    for r in read_jsonl(out) if r.get("rating") is not None}
        else:
            out.unlink()
    scores: dict[str, dict[str, list[float]]] = {}
    failures = 0
    for label, answers in _answer_sets(args):
        for a in answers:
            q = qs[a["question_id"]]
            for t in a["turns"]:
                for rep in range(max(1, int(args.judge_repeats))):
                    key = (label, a["question_id"], t["turn"], rep)
                    if key in done:
                        continue
                    try:
                        rating, raw = judge_one(settings, q["turns"][t["turn"]], t["answer"])
                    except Exception as exc:  # noqa: BLE001 - recorded, the run continues
                        rating, raw = None, f"error: {exc!r}"
                        failures += 1
                    append_jsonl(out, {"source": label, "question_id": a["question_id"], "turn": t["turn"],
                                       "repeat": rep, "rating": rating, "judgment": raw})
    for r in read_jsonl(out) if out.exists() else []:
        if r.get("rating") is not None:
            cat = str(qs.get(r["question_id"], {}).get("category"))
            scores.setdefault(str(r.get("source", "answers")), {}).setdefault(cat, []).append(float(r["rating"]))
    summary = {}
    for label, cats in scores.items():
        allv = [v for vs in cats.values() for v in vs]
        summary[label] = {"mean": statistics.fmean(allv), "judged": len(allv),
                          "by_category": {c: statistics.fmean(v) for c, v in sorted(cats.items())}}
    main_set = summary.get("answers", {})
    print(json.dumps({"mean": main_set.get("mean"), "judged": main_set.get("judged", 0), "failures": failures,
                      "by_category": main_set.get("by_category", {}), "sources": summary}))
    return 0


def add_judge_flags(j, *, flat: bool) -> None:
    if not flat:
        j.add_argument("--judge-url", default=None, help="full chat-completions URL (or --judge-base-url)")
        j.add_argument("--api-key-env", default="JUDGE_API_KEY")
        j.add_argument("--timeout", type=float, default=120.0)
        j.add_argument("--output", default=None)
        j.add_argument("--resume", action="store_true", help="keep judgments already made (with a rating)")
        j.add_argument("--ar-generations", default=None, help="AR answers to grade in the same run")
        j.add_argument("--ar-run-id", default=None)
    j.add_argument("--judge-base-url", default="https://api.deepseek.com")
    j.add_argument("--judge-model", default="deepseek-chat")
    j.add_argument("--judge-thinking", choices=["enabled", "disabled"], default=None)
    j.add_argument("--judge-reasoning-effort", choices=["high", "max"], default=None)
    j.add_argument("--judge-max-tokens", type=int, default=None)
    j.add_argument("--judge-retries", type=int, default=0)
    j.add_argument("--judge-retry-delay", type=float, default=2.0)
    j.add_argument("--judge-repeats", type=int, default=1)


def flat_parser() -> argparse.ArgumentParser:
    """The reference's one-command form (scripts/mtbench_deepseek_eval.py:1299-1383): generate,
    then judge, each skippable and resumable."""
    p = argparse.ArgumentParser(description="MT-Bench generation + judging in one command")
    p.add_argument("--drafter-model", required=True, help="ATLAS drafter (preset or checkpoint dir)")
    add_atlas_flags(p)
    p.add_argument("--execution-mode", choices=["async", "serial"], default="async")
    p.add_argument("--questions-file", required=True, help="local MT-Bench question JSONL")
    p.add_argument("--questions-url", default=None, help="not fetched: there is no network here")
    p.add_argument("--download-timeout", type=float, default=60.0, help="No-op (nothing is downloaded).")
    p.add_argument("--output-dir", required=True)
    add_question_flags(p)
    p.add_argument("--skip-generate", action="store_true")
    p.add_argument("--resume-generate", action="store_true")
    p.add_argument("--skip-judge", action="store_true")
    p.add_argument("--resume-judge", action="store_true")
    p.add_argument("--ar-generations", default=None)
    p.add_argument("--ar-run-id", default=None)
    p.add_argument("--deepseek-api-key-env", default="DEEPSEEK_API_KEY")
    p.add_argument("--judge-timeout", type=float, default=180.0)
    add_judge_flags(p, flat=True)
    # The reference's defaults for this form: longer answers and context, a patient judge.
    p.set_defaults(max_new_tokens=1024, context_length=16384, judge_max_tokens=4096, judge_retries=4)
    return p


def add_question_flags(p) -> None:
    p.add_argument("--question-start", type=int, default=0)
    p.add_argument("--question-end", type=int, default=None)
    p.add_argument("--max-questions", type=int, default=None)
    p.add_argument("--turn-mode", choices=["first", "conversation"], default="conversation")
    p.add_argument("--system-prompt", default="")
    p.add_argument("--chat-template", choices=["auto", "off"], default="auto",
                   help="auto: turns rendered by the tokenizer's chat template (its end-of-turn token as EOS) "
                        "when --tokenizer is a directory that has one")


def run_flat(argv) -> int:
    a = flat_parser().parse_args(argv)
    if not Path(a.questions_file).exists():
        raise SystemExit(f"{a.questions_file}: not found (questions are not downloaded; there is no network here)")
    out = Path(a.output_dir)
    if not a.skip_generate:
        g = argparse.Namespace(**vars(a))
        g.backend = "atlas_serial" if a.execution_mode == "serial" else "atlas"
        g.model, g.questions, g.resume = a.drafter_model, a.questions_file, a.resume_generate
        rc = cmd_generate(g)
        if rc:
            return rc
    if a.skip_judge:
        return 0
    j = argparse.Namespace(**vars(a))
    j.answers, j.questions, j.output = str(out / "answers.jsonl"), a.questions_file, None
    j.judge_url, j.api_key_env, j.timeout, j.resume = None, a.deepseek_api_key_env, a.judge_timeout, a.resume_judge
    return cmd_judge(j)


def ar_parser() -> argparse.ArgumentParser:
    """The reference's AR-baseline command (scripts/mtbench_ar_deepseek_eval.py): greedy AR answers
    of a 1B and an 8B model under one run id, then (optionally) their judging."""
    p = argparse.ArgumentParser(description="MT-Bench AR baselines (1B and 8B greedy), then judging",
                                allow_abbrev=False)
    p.add_argument("--model-1b", default=None, help="preset or checkpoint directory")
    p.add_argument("--model-8b", default=None, help="preset or checkpoint directory")
    p.add_argument("--candidate", choices=["1b", "8b", "both"], default="both",
                   help="generate one AR candidate or both, one after the other")
    p.add_argument("--questions-file", required=True)
    p.add_argument("--questions-url", default=None, help="not fetched: there is no network here")
    p.add_argument("--download-timeout", type=float, default=60.0, help="No-op (nothing is downloaded).")
    p.add_argument("--output-dir", required=True)
    add_question_flags(p)
    p.add_argument("--max-new-tokens", type=int, default=1024)
    p.add_argument("--eos-token-id", type=int, default=None)
    p.add_argument("--dtype", choices=["float16", "bfloat16", "float32"], default="float16")
    p.add_argument("--context-length", type=int, default=16384)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--device", default=None)
    p.add_argument("--seed", type=int, default=0, help="seed of random-init presets")
    add_runtime_compat_flags(p)
    p.add_argument("--skip-generate", action="store_true")
    p.add_argument("--resume-generate", action="store_true")
    p.add_argument("--skip-judge", action="store_true")
    p.add_argument("--resume-judge", action="store_true")
    p.add_argument("--deepseek-api-key-env", default="DEEPSEEK_API_KEY")
    p.add_argument("--judge-timeout", type=float, default=180.0)
    add_judge_flags(p, flat=True)
    p.set_defaults(judge_max_tokens=4096, judge_retries=4)
    return p


def ar_run_id(a) -> str:
    """A stable id of the generation settings, so a later ATLAS run can name this AR run."""
    keys = ("model_1b", "model_8b", "candidate", "questions_file", "question_start", "question_end", "max_questions",
            "turn_mode", "system_prompt", "max_new_tokens", "eos_token_id", "dtype", "page_size", "seed")
    blob = json.dumps({key: getattr(a, key) for key in keys}, sort_keys=True, default=str)
    return hashlib.sha256(blob.encode()).hexdigest()[:12]


def run_ar(argv) -> int:
    a = ar_parser().parse_args(argv)
    if not Path(a.questions_file).exists():
        raise SystemExit(f"{a.questions_file}: not found (questions are not downloaded; there is no network here)")
    out = Path(a.output_dir)
    gens = out / "generations.jsonl"
    rid = ar_run_id(a)
    if not a.skip_generate:
        chosen = [(label, model) for label, model, key in (("ar_1b", a.model_1b, "1b"), ("ar_8b", a.model_8b, "8b"))
                  if a.candidate in (key, "both")]
        if gens.exists() and not a.resume_generate:
            # Start these candidates over; other runs' and other candidates' answers stay.
            labels = {label for label, _ in chosen}
            keep = [r for r in read_jsonl(gens) if not (r.get("run_id") == rid and r.get("model") in labels)]
            gens.write_text("".join(json.dumps(r) + "\n" for r in keep))
        for label, model in chosen:
            if model is None:
                raise SystemExit(f"--candidate {a.candidate} needs --model-{label[3:]}")
            g = argparse.Namespace(**vars(a), backend="ar", model=model, questions=a.questions_file,
                                   resume=a.resume_generate, k=1, d=1, generation_seed=0, drafter_do_sample=False,
                                   drafter_temperature=1.0, fallback_ar_tokens=1)
            rc = cmd_generate(g, path=gens, extra={"model": label, "checkpoint": str(model), "run_id": rid},
                              keep_file=True)
            if rc:
                return rc
    print(json.dumps({"generation_run_id": rid, "generations": str(gens)}))
    if a.skip_judge:
        return 0
    j = argparse.Namespace(**vars(a))
    j.answers, j.questions, j.output = None, a.questions_file, str(out / "judgments.jsonl")
    j.ar_generations, j.ar_run_id = str(gens), rid
    j.judge_url, j.api_key_env, j.timeout, j.resume = None, a.deepseek_api_key_env, a.judge_timeout, a.resume_judge
    return cmd_judge(j)


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--model-1b" in argv or "--model-8b" in argv:
        return run_ar(argv)
    if not argv or argv[0] not in ("generate", "judge", "-h", "--help"):
        return run_flat(argv)
    p = argparse.ArgumentParser(description="MT-Bench generation and judging (or the reference's one-command "
                                            "form: --drafter-model ... --questions-file ... --output-dir ...)")
    sub = p.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("generate")
    add_generation_flags(g)
    g.add_argument("--questions", required=True)
    g.add_argument("--output-dir", required=True)
    add_question_flags(g)
    j = sub.add_parser("judge")
    j.add_argument("--answers", required=True)
    j.add_argument("--questions", required=True)
    add_judge_flags(j, flat=False)
    args = p.parse_args(argv)
    if args.cmd == "judge" and not (args.judge_url or args.judge_base_url):
        p.error("judge needs --judge-url or --judge-base-url")
    return cmd_generate(args) if args.cmd == "generate" else cmd_judge(args)


if __name__ == "__main__":
    raise SystemExit(main())
