"""GSM8K exact-match evaluation: ``python -m 0709_b200.eval.gsm8k --backend atlas ...``.

Reads a local GSM8K-format JSONL (``question``, ``answer`` with ``#### N``),
generates with the chosen backend (drafter AR, asynchronous ATLAS, or serial
ATLAS), extracts the final number, and appends one row per sample to
``predictions.jsonl`` (``--resume`` skips done indices).  ATLAS rows carry the
per-sample target-intervention summary (``utils.interventions``) and the
prompt's token hash so paired runs can be aligned; ``summary.json`` holds
accuracy, throughput and the aggregated intervention statistics.

Prompts: zero-shot with an answer-format instruction, or few-shot from
``--fewshot-file`` (JSONL of question/answer pairs; ``--protocol llama-8shot``
insists on eight), optionally after ``--system-prompt``.  There is no network
here, so the dataset must be a local file.  Parity: reference
scripts/gsm8k_eval.py (backends, resume, interventions, summary; its flags,
:318-422, are accepted -- the SGLang memory and scheduler settings as no-ops).
"""

from __future__ import annotations

import argparse
import json
import re
import statistics
import sys
from pathlib import Path

from ..serving.prompts import chat_ids, chat_stop_token, decode, encode, load_chat_tokenizer, load_tokenizer
from ..utils.interventions import aggregate_prediction_interventions, summarize_generation_interventions
from .common import add_generation_flags, append_jsonl, done_indices, make_generate, read_jsonl, rows_summary, \
    timed, token_ids_sha256, warm_up

GOLD_RE = re.compile(r"####\s*([^\n\r]+)")
FINAL_RE = re.compile(r"final answer is\s*\$?\s*(-?[\d,]*\.?\d+)", re.IGNORECASE)
NUM_RE = re.compile(r"-?\d[\d,]*\.?\d*")
INSTRUCTION = "Solve the problem step by step. End with the sentence: The final answer is <number>."


def normalize(x: str | None) -> str | None:
    if x is None:
        return None
    s = x.strip().replace(",", "").replace("$", "").rstrip(".")
    try:
        v = float(s)
    except ValueError:
        return None
    return str(int(v)) if v == int(v) else repr(v)


def gold_answer(row: dict) -> str | None:
    m = GOLD_RE.search(str(row.get("answer", "")))
    return normalize(m.group(1)) if m else None


def extract(text: str, *, strict: bool = False) -> str | None:
    m = FINAL_RE.search(text or "")
    if m:
        return normalize(m.group(1))
    if strict:
        return None
    nums = NUM_RE.findall(text or "")
    return normalize(nums[-1]) if nums else None


def build_prompt(question: str, fewshot: list[dict], system_prompt: str = "") -> str:
    parts = ([system_prompt, ""] if system_prompt else []) + [INSTRUCTION, ""]
    for ex in fewshot:
        parts += [f"Question: {ex['question']}", f"Answer: {ex['answer']}", ""]
    parts += [f"Question: {question}", "Answer:"]
    return "\n".join(parts)


# Per-sample timing of the serial generator kept in each prediction row, summed by ``serial_speed``.
SERIAL_KEYS = ("generated_tokens", "rounds", "fallback_rounds", "drafter_elapsed_s", "target_elapsed_s",
               "total_elapsed_s", "fallback_appended_tokens", "fallback_append_elapsed_s")


def serial_speed(preds: list[dict]) -> dict:
    """Drafter / target / overall committed-token rates of the serial generator over all samples
    (target prompt prefill excluded, as in its per-sample metadata)."""
    tot = {key: sum(float((r.get("serial") or {}).get(key) or 0) for r in preds) for key in SERIAL_KEYS}
    n = tot["generated_tokens"]

    def rate(t: float) -> float | None:
        return n / t if t else None

    return {**tot, "fallback_rate": tot["fallback_rounds"] / tot["rounds"] if tot["rounds"] else None,
            "drafter_tokens_per_second": rate(tot["drafter_elapsed_s"]),
            "target_tokens_per_second": rate(tot["target_elapsed_s"]),
            "overall_tokens_per_second": rate(tot["total_elapsed_s"]),
            "fallback_append_tokens_per_second": (tot["fallback_appended_tokens"] / tot["fallback_append_elapsed_s"]
                                                  if tot["fallback_append_elapsed_s"] else None),
            "token_definition": "committed_generated_tokens", "excludes_target_prompt_prefill": True}


def settings(args, num_fewshot: int) -> dict:
    """The generation settings of the run, recorded beside its results."""
    atlas = args.backend.startswith("atlas")
    keep = ("protocol", "chat_template", "max_new_tokens", "strict_marker", "system_prompt", "context_length", "dtype",
            "page_size", "eos_token_id", "generation_seed", "drafter_do_sample", "drafter_temperature")
    out = {key: getattr(args, key) for key in keep}
    out["num_fewshot"] = num_fewshot
    out["request_seed_rule"] = "generation_seed_plus_gsm8k_index"
    out["target_model"] = (args.target_model or args.target_url) if atlas else None
    for key in ("k", "d", "fixed_forest_depth", "path_score_weights", "path_weight_alpha", "fallback_threshold",
                "first_token_threshold", "fallback_ar_tokens", "route_selection_policy",
                "route_sampling_temperature"):
        out[key] = getattr(args, key) if atlas else None
    return out


def build_messages(question: str, fewshot: list[dict], system_prompt: str = "") -> list[dict]:
    """The same prompt as chat turns: the system prompt, each exemplar as a user/assistant pair,
    then the question."""
    msgs = [{"role": "system", "content": system_prompt}] if system_prompt else []
    for ex in fewshot:
        msgs += [{"role": "user", "content": f"{INSTRUCTION}\n\nQuestion: {ex['question']}"},
                 {"role": "assistant", "content": str(ex["answer"])}]
    msgs.append({"role": "user", "content": f"{INSTRUCTION}\n\nQuestion: {question}"})
    return msgs


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="GSM8K exact match")
    add_generation_flags(p)
    p.add_argument("--data-file", required=True)
    p.add_argument("--fewshot-file", default=None)
    p.add_argument("--output-dir", required=True)
    p.add_argument("--start", type=int, default=0)
    p.add_argument("--end", type=int, default=None)
    p.add_argument("--max-examples", type=int, default=None)
    p.add_argument("--strict-marker", action="store_true", help="require 'The final answer is'")
    p.add_argument("--protocol", choices=["auto", "llama-8shot", "zero-shot"], default="auto",
                   help="llama-8shot: the eight chain-of-thought exemplars of --fewshot-file; zero-shot: none; "
                        "auto: few-shot exactly when --fewshot-file is given")
    p.add_argument("--system-prompt", default="", help="text placed before the instruction")
    p.add_argument("--chat-template", choices=["auto", "off"], default="auto",
                   help="auto: prompts as chat turns rendered by the tokenizer's chat template (and its "
                        "end-of-turn token as EOS) when --tokenizer is a directory that has one")
    return p


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    pred_path = out / "predictions.jsonl"
    rows = read_jsonl(args.data_file)[args.start:args.end]
    if args.max_examples is not None:
        rows = rows[: args.max_examples]
    fewshot = read_jsonl(args.fewshot_file) if args.fewshot_file and args.protocol != "zero-shot" else []
    if args.protocol == "llama-8shot" and len(fewshot) != 8:
        raise SystemExit("--protocol llama-8shot needs the eight exemplars as JSONL in --fewshot-file "
                         f"(got {len(fewshot)}); there is no network here to fetch them")
    tok = load_tokenizer(args.tokenizer)
    chat = load_chat_tokenizer(args.tokenizer) if args.chat_template == "auto" else None
    if chat is not None and args.eos_token_id is None:
        args.eos_token_id = chat_stop_token(chat)

    def prompt_ids(question: str) -> list[int]:
        if chat is not None:
            return chat_ids(chat, build_messages(question, fewshot, args.system_prompt))
        return encode(tok, build_prompt(question, fewshot, args.system_prompt))

    def text_of(ids) -> str:
        return (chat.decode(ids, skip_special_tokens=True) if chat is not None else decode(tok, ids)) or ""

    done = done_indices(pred_path) if args.resume else set()
    if not args.resume and pred_path.exists():
        pred_path.unlink()
    generate = make_generate(args)
    pending = [(i, row) for i, row in enumerate(rows, start=args.start) if i not in done]
    if pending:
        warm_up(generate, prompt_ids(str(pending[0][1]["question"])), args.warmup_runs)
    failures_path = out / "failures.jsonl"
    for i, row in pending:
        ids = prompt_ids(str(row["question"]))
        seed = int(args.generation_seed) + int(i)  # one request seed per GSM8K index
        try:
            (gen_ids, meta, rounds), secs = timed(generate, ids, seed)
        except Exception as exc:  # noqa: BLE001 - recorded per sample; the run goes on (resume retries it)
            print(f"sample {i} failed: {exc!r}", file=sys.stderr, flush=True)
            append_jsonl(failures_path, {"index": i, "error": repr(exc)})
            continue
        text = text_of(gen_ids)
        pred, gold = extract(text, strict=args.strict_marker), gold_answer(row)
        rec = {"index": i, "question": row["question"], "gold": gold, "prediction": pred,
               "correct": pred is not None and pred == gold, "response": text, "model": args.model,
               "backend": args.backend, "prompt_tokens": len(ids), "prompt_token_ids_sha256": token_ids_sha256(ids),
               "generated_tokens": len(gen_ids), "elapsed_s": secs, "generation_seed": seed}
        if rounds:
            rec["target_intervention"] = {k: v for k, v in summarize_generation_interventions(
                [r.to_dict() if hasattr(r, "to_dict") else r for r in rounds]).items() if k != "rounds"}
            rec["rounds"] = len(rounds)
            rec["fallback_rounds"] = sum(getattr(r, "decision", "") == "fallback_ar" for r in rounds)
        if args.backend == "atlas_serial":
            rec["serial"] = {key: meta.get(key) for key in SERIAL_KEYS}
        append_jsonl(pred_path, rec)
    preds = read_jsonl(pred_path) if pred_path.exists() else []
    acc = sum(bool(r["correct"]) for r in preds) / len(preds) if preds else None
    speeds = [r["generated_tokens"] / r["elapsed_s"] for r in preds if r.get("elapsed_s")]
    base = rows_summary(preds)
    summary = {"accuracy": acc, "correct": sum(bool(r["correct"]) for r in preds), **base, "count": len(preds),
               "mean_tokens_per_second": statistics.fmean(speeds) if speeds else None,
               "end_to_end_tokens_per_second": base["tokens_per_s"],
               "extraction_failures": sum(r["prediction"] is None for r in preds),
               "failures": len(read_jsonl(failures_path)) if failures_path.exists() else 0,
               "backend": args.backend, "model": args.model, "target": args.target_model or args.target_url,
               "target_intervention": aggregate_prediction_interventions(preds),
               "serial_speed": serial_speed(preds) if args.backend == "atlas_serial" else None,
               "settings": settings(args, len(fewshot))}
    (out / "summary.json").write_text(json.dumps(summary, indent=2, sort_keys=True) + "\n")
    print(json.dumps({k: summary[k] for k in ("accuracy", "samples", "tokens_per_s")}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
