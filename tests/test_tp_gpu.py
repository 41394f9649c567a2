"""Tensor-parallel target on 2+ GPUs: NCCL baseline and fused peer-memory collectives vs one GPU."""

from __future__ import annotations

import pytest
import torch

from test_tp_cpu import last_json, torchrun

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("mode", ["nccl", "fused"])
def test_tp_target_matches_single_gpu(mode):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    r = torchrun(2, "0709_b200.parallel.check_tp", "--mode", mode, "--model", "small-tp-target", "--drafter",
                 "small-drafter", "--dtype", "bfloat16", "--page-size", "16", "--prompt-len", "100",
                 "--new-tokens", "24", "--timing-iters", "20", timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    d = last_json(r.stdout)
    assert d["tp"] == 2 and d["mode"] == mode
    # bf16 activations: different summation order across ranks, so compare with a tolerance.
    assert d["prefill_logit_max_abs_diff"] < 5e-2
    assert d["tree_logit_max_abs_diff"] < 5e-2
    assert d["tree_path_logprob_max_abs_diff"] < 5e-2
