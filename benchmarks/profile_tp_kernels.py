#!/usr/bin/env python
"""One-GPU harness for the fused tensor-parallel kernels (for timing and ncu captures).

    python benchmarks/profile_tp_kernels.py --tp 8 --rows 12 --reps 5

Emulates rank 0 of a TP group on one GPU: the row-parallel GEMM with the peer
epilogue stores its fp32 tile into ``tp`` receive slots (here all in this
GPU's memory instead of the peers' IPC mappings) and raises their flags;
``tp_reduce_rmsnorm`` then finds every flag set, sums the slots in rank
order, adds the residual and applies RMSNorm.  Shapes default to the 70B
o_proj at the given TP degree (H = 8192, K = 8192 / tp).  Prints CUDA-event
times of both kernels and of the unfused pair (GEMM to a local fp32 buffer,
then the same reduce with one source).
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--rows", type=int, default=12)
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--k", type=int, default=0, help="reduction length (default hidden / tp)")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    from bench_kernels import timeit

    ops = importlib.import_module("0709_b200.ops.cuda_ops").CudaOps(device=torch.device("cuda"))
    ext = ops.ext
    H, tp, m = args.hidden, args.tp, args.rows
    K = args.k or H // tp
    w = (torch.randn(H, K, device="cuda") * 0.02).to(torch.bfloat16)
    a = torch.randn(m, K, device="cuda").to(torch.bfloat16)
    gamma = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    recv = torch.zeros(tp, 64, H, device="cuda")
    ctrl = torch.zeros(1024, dtype=torch.int32, device="cuda")  # flags [0, 64), ticket 512, seq 513
    base = ctrl.data_ptr()
    h = torch.zeros(m, H, device="cuda")
    x = torch.empty(m, H, device="cuda", dtype=torch.bfloat16)
    slot = 64 * H
    dst = [recv.data_ptr() + r * slot * 4 for r in range(tp)]
    flags = [base + 4 * r for r in range(tp)]

    recv.view(torch.int32).fill_(-1)  # sentinel: every slot unwritten

    def fused_gemm():
        ext.gemm_peer(w, a, dst, H, [], 0, 0, ops.ws, ops.counters, ops.err, True)

    def fused_reduce():
        ext.tp_reduce_rmsnorm(recv.data_ptr(), slot, 0, 0, tp, h, gamma, x, 1e-5, ops.err, True)

    def flag_gemm():
        ext.gemm_peer(w, a, dst, H, flags, base + 4 * 512, base + 4 * 513, ops.ws, ops.counters, ops.err, False)

    def flag_reduce():
        ext.tp_reduce_rmsnorm(recv.data_ptr(), slot, base, base + 4 * 513, tp, h, gamma, x, 1e-5, ops.err, False)

    part = torch.empty(m, H, device="cuda")

    def plain_gemm():
        ops._gemm(a, w, part, ext.EPI_F32)

    def plain_reduce():
        ext.tp_reduce_rmsnorm(part.data_ptr(), 0, 0, 0, 1, h, gamma, x, 1e-5, ops.err, False)

    ref = a.float() @ w.float().t()
    fused_gemm()
    torch.cuda.synchronize()
    got = recv[:, :m].sum(0) / tp
    err = float((got - ref).abs().max())
    fused_reduce()
    torch.cuda.synchronize()
    assert bool((recv.view(torch.int32) == -1).all()), "reduce must restore the sentinel"
    for _ in range(args.reps):
        fused_gemm()
        fused_reduce()
    torch.cuda.synchronize()
    ops.check()
    out = {"tp": tp, "rows": m, "H": H, "K": K, "max_abs_err_vs_fp32": err,
           "sentinel_gemm_peer_plus_reduce_us": round(timeit(lambda: (fused_gemm(), fused_reduce()), 20), 2),
           "gemm_peer_flags_plus_reduce_us": round(timeit(lambda: (flag_gemm(), flag_reduce()), 20), 2),
           "gemm_f32_plus_reduce_1src_us": round(timeit(lambda: (plain_gemm(), plain_reduce()), 20), 2),
           "weight_bytes": H * K * 2, "push_bytes_per_rank": (tp - 1) * m * H * 4}
    print(json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
