"""Two-rank gloo job for the TP failure-detection test: the worker leaves between calls."""

import datetime
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import importlib  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> int:
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    pkg = lambda n: importlib.import_module(f"0709_b200.{n}")  # noqa: E731
    cfg = pkg("models.llama").get_config("tiny-target")
    eng = pkg("parallel.launch").build_tp_target(cfg, mode="torch", seed=1, dtype=torch.float32, num_pages=128,
                                                 page_size=4, max_positions=256, device=torch.device("cpu"))
    if not eng.is_root:
        eng.serve()
        return 0
    tv = pkg("runtime.target").TargetVerifier(eng, k=2, d=2)
    lost, kind = None, None
    try:
        tv.prefill(list(range(10, 30)))
        for r in range(50):
            tv.run_tree([[1 + r, 2], [3, 4 + r]])
    except (pkg("parallel.mailbox").PeerLost, RuntimeError) as exc:
        # Either the command is never acknowledged (mailbox) or the collective
        # reports the closed connection (gloo) -- both end the call with an error.
        lost, kind = str(exc), type(exc).__name__
    print(json.dumps({"peer_lost": lost is not None, "kind": kind, "message": lost}), flush=True)
    os._exit(0)


if __name__ == "__main__":
    raise SystemExit(main())
