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
