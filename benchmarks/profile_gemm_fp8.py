#!/usr/bin/env python
"""One block-scaled fp8 GEMM at a Llama-3.1-70B shape, for timing and ncu captures (one GPU).

    python benchmarks/profile_gemm_fp8.py --shape gate_up --rows 12 --reps 3

e4m3 weights with 128x128 block scales, activations quantized per token per 128
columns (``quant_fp8``), ``tcgen05.mma.kind::f8f6f4`` with the scale promotion
of ``csrc/cuda/gemm_fp8.cu``.  Shapes: qkv (10240 x 8192), o (8192 x 8192),
gate_up (57344 x 8192, 470 MB of fp8 weights: larger than L2), down
(8192 x 28672).  Prints CUDA-event time per launch (L2 flushed), the fraction of
the measured HBM bandwidth for the bytes moved, and the max error against the
fp32 product of the dequantized operands.
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
SHAPES = {"qkv": (10240, 8192), "o": (8192, 8192), "gate_up": (57344, 8192), "down": (8192, 28672)}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", choices=sorted(SHAPES), default="gate_up")
    ap.add_argument("--rows", type=int, default=12)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(ROOT, "benchmarks"))
    from bench_kernels import peaks, timeit

    fp8 = importlib.import_module("0709_b200.models.fp8")
    ops = importlib.import_module("0709_b200.ops.cuda_ops").CudaOps(device=torch.device("cuda"))
    n_out, k = SHAPES[args.shape]
    g = torch.Generator(device="cuda").manual_seed(0)
    w = fp8.quantize_blockwise((torch.randn(n_out, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16))
    x = torch.randn(args.rows, k, device="cuda", generator=g).to(torch.bfloat16)
    xq, sa = ops.quant_fp8(x)
    out = torch.empty(args.rows, n_out, device="cuda", dtype=torch.bfloat16)
    ops.gemm_fp8(xq, sa, w, out, ops.ext.EPI_STORE)
    ref = fp8.dequantize_activations(xq, sa)[: args.rows].float() @ w.dequantize().t()
    torch.cuda.synchronize()
    err = float((out.float() - ref).abs().max() / ref.abs().max())
    for _ in range(args.reps):
        ops.gemm_fp8(xq, sa, w, out, ops.ext.EPI_STORE)
    torch.cuda.synchronize()
    ops.check()
    us = timeit(lambda: ops.gemm_fp8(xq, sa, w, out, ops.ext.EPI_STORE), args.iters)
    hbm, _, src = peaks()
    nbytes = w.nbytes + xq.numel() + out.numel() * 2
    print(json.dumps({"shape": args.shape, "n_out": n_out, "k": k, "rows": args.rows, "us": round(us, 2),
                      "GB/s": round(nbytes / us / 1e3, 1), f"hbm_frac_of_{src}": round(nbytes / us / 1e3 / hbm, 3),
                      "max_rel_err_vs_fp32_dequant": err, "config": ops.last_gemm_config}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
