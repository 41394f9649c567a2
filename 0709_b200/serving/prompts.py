"""Prompt token handling shared by the command-line tools.

Parity: reference src/atlas_0709/distributed_system.py:906-932 (parse_token_ids,
required_context_length).  Without a tokenizer, text prompts are mapped to
their UTF-8 bytes (ids 0..255), which every vocabulary here contains.
"""

from __future__ import annotations

from typing import Sequence


def load_tokenizer(path: str | None):
    if not path:
        return None
    from tokenizers import Tokenizer
    import os

    f = os.path.join(path, "tokenizer.json") if os.path.isdir(path) else path
    return Tokenizer.from_file(f)


def encode(tokenizer, text: str) -> list[int]:
    if tokenizer is None:
        return list(text.encode("utf-8"))
    return list(tokenizer.encode(text, add_special_tokens=False).ids)


def decode(tokenizer, ids: Sequence[int]) -> str | None:
    if tokenizer is None:
        # Byte fallback (the inverse of encode without a tokenizer); ids outside
        # 0..255 come from a real vocabulary and have no text without it.
        if all(0 <= int(t) < 256 for t in ids):
            return bytes(int(t) for t in ids).decode("utf-8", errors="replace")
        return None
    return tokenizer.decode([int(t) for t in ids], skip_special_tokens=False)


def load_chat_tokenizer(path: str | None):
    """transformers' tokenizer of a checkpoint or tokenizer directory that carries a chat template
    (``chat_template.jinja``, or ``chat_template`` in ``tokenizer_config.json``); else None."""
    import json
    import os

    if not path or not os.path.isdir(path):
        return None
    cfg = os.path.join(path, "tokenizer_config.json")
    has = os.path.exists(os.path.join(path, "chat_template.jinja"))
    if not has and os.path.exists(cfg):
        with open(cfg, encoding="utf-8") as f:
            has = bool(json.load(f).get("chat_template"))
    if not has:
        return None
    from transformers import AutoTokenizer

    return AutoTokenizer.from_pretrained(path)


def chat_ids(tokenizer, messages: Sequence[dict]) -> list[int]:
    """Token ids of ``messages`` rendered by the tokenizer's chat template, ending with the
    assistant's generation prompt."""
    enc = tokenizer.apply_chat_template(list(messages), tokenize=True, add_generation_prompt=True)
    if isinstance(enc, dict) or hasattr(enc, "keys"):
        enc = enc["input_ids"]
    if hasattr(enc, "tolist"):
        enc = enc.tolist()
    if enc and isinstance(enc[0], list):
        enc = enc[0]
    return [int(t) for t in enc]


def chat_stop_token(tokenizer) -> int | None:
    """The end-of-turn token of a chat tokenizer (``<|eot_id|>`` where the vocabulary has it),
    else its end-of-sequence token."""
    tid = tokenizer.convert_tokens_to_ids("<|eot_id|>")
    if isinstance(tid, int) and tid >= 0 and tid != getattr(tokenizer, "unk_token_id", None):
        return tid
    return getattr(tokenizer, "eos_token_id", None)


def parse_token_ids(raw: str | None, *, tokenizer, prompt: str, prefix_len: int | None = None,
                    repeat_token_id: int | None = None) -> list[int]:
    if repeat_token_id is not None:
        if prefix_len is None or prefix_len <= 0:
            raise ValueError("--repeat-token-id builds a prompt of --prefix-len tokens, so give a positive --prefix-len")
        return [int(repeat_token_id)] * int(prefix_len)
    toks = [int(p.strip()) for p in raw.split(",") if p.strip()] if raw else encode(tokenizer, prompt)
    if not toks:
        raise ValueError("the prompt has no tokens")
    if prefix_len is None:
        return toks
    return (toks * ((int(prefix_len) + len(toks) - 1) // len(toks)))[: int(prefix_len)]


def required_context_length(prompt_len: int, *, max_new_tokens: int, depth: int) -> int:
    return int(prompt_len) + int(max_new_tokens) + 2 * int(depth)
