"""Clean-controller runner: ``python -m 0709_b200.serving.cli --backend mock``.

Runs the tree/forest/verify race without physical KV, with the deterministic
mock backends or the no-KV recompute backends (``--backend recompute``; the
alias ``hf`` is accepted).  Parity: reference src/atlas_0709/cli.py:12-120.
"""

from __future__ import annotations

import argparse
import json

from ..runtime.clean import AtlasCleanConfig, AtlasCleanGenerator, DeterministicMockBackend


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Run the clean staged decode controller.")
    p.add_argument("--backend", choices=["mock", "recompute", "hf"], default="mock")
    p.add_argument("--k", type=int, default=3)
    p.add_argument("--d", type=int, default=4)
    p.add_argument("--max-new-tokens", type=int, default=32)
    p.add_argument("--eos-token-id", type=int, default=None)
    p.add_argument("--prompt-token-ids", default="1,2,3,4")
    p.add_argument("--prompt", default=None,
                   help="prompt text (model backends): encoded with --tokenizer, or as UTF-8 bytes without one")
    p.add_argument("--tokenizer", default=None, help="tokenizer.json or its directory")
    p.add_argument("--trust-remote-code", action="store_true", help="No-op: checkpoints are read as safetensors.")
    p.add_argument("--drafter-model", default="tiny-drafter")
    p.add_argument("--target-model", default="tiny-target")
    p.add_argument("--dtype", choices=["float16", "bfloat16", "float32"], default="float32")
    p.add_argument("--device", default="cpu")
    p.add_argument("--mock-vocab-size", type=int, default=128)
    p.add_argument("--seed", type=int, default=0)
    return p


def parse_ids(raw: str) -> list[int]:
    ids = [int(x.strip()) for x in raw.split(",") if x.strip()]
    if not ids:
        raise ValueError("--prompt-token-ids parsed to an empty list")
    return ids


def make_backends(args):
    if args.backend == "mock":
        return (DeterministicMockBackend(name="drafter", vocab_size=args.mock_vocab_size, salt=3),
                DeterministicMockBackend(name="target", vocab_size=args.mock_vocab_size, salt=19))
    from ..models.loader import resolve_model
    from ..runtime.recompute import RecomputeBatchBackend

    dw = resolve_model(args.drafter_model, dtype=args.dtype, device=args.device, seed=args.seed)
    tw = resolve_model(args.target_model, dtype=args.dtype, device=args.device, seed=args.seed + 1)
    return RecomputeBatchBackend(dw, name="drafter"), RecomputeBatchBackend(tw, name="target")


def result_to_jsonable(res) -> dict[str, object]:
    return {
        "prompt_token_ids": list(res.prompt_token_ids),
        "generated_token_ids": list(res.generated_token_ids),
        "token_ids": res.token_ids,
        "rounds": [
            {
                "round_index": t.round_index,
                "selected_route_id": t.selected_route_id,
                "committed_tokens": list(t.committed_tokens),
                "forest_depth": t.forest_depth,
                "verify_returned_before_forest_done": t.verify_returned_before_forest_done,
                "target_scores": [{"route_id": r, "target_logprob": s} for r, s in t.target_scores],
            }
            for t in res.rounds
        ],
    }


def prompt_ids(args) -> list[int]:
    if args.prompt is None:
        return parse_ids(args.prompt_token_ids)
    if args.backend == "mock":
        raise SystemExit("--prompt needs a model backend (recompute/hf); the mock backends take --prompt-token-ids")
    from .prompts import encode, load_tokenizer

    ids = encode(load_tokenizer(args.tokenizer), args.prompt)
    if not ids:
        raise SystemExit("--prompt encoded to no tokens")
    return ids


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    ids = prompt_ids(args)
    drafter, target = make_backends(args)
    cfg = AtlasCleanConfig(k=args.k, d=args.d, max_new_tokens=args.max_new_tokens, eos_token_id=args.eos_token_id)
    res = AtlasCleanGenerator(config=cfg, drafter=drafter, target=target).generate(ids)
    print(json.dumps({
        "config": {"k": cfg.k, "d": cfg.d, "max_new_tokens": cfg.max_new_tokens, "eos_token_id": cfg.eos_token_id,
                   "tree_decode": f"ordinary_batch_{cfg.k}", "forest_decode": f"ordinary_batch_{cfg.k * cfg.k}",
                   "target_verify": "ordinary_batch_stage1_paths"},
        "result": result_to_jsonable(res),
    }, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
