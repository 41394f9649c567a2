#!/usr/bin/env python
"""Per-kernel microbenchmark at Llama-3.1-8B / Llama-3.2-1B decode and verify shapes.

Each kernel is timed with CUDA events on the launching stream after warm-up,
with L2 flushed (a 512 MB write) before every timed launch; results are
reported against the measured HBM copy bandwidth (MEASURED_PEAKS.json,
``hbm_gbs``) and cuBLAS bf16 peak (``bf16_tflops``).

    python benchmarks/bench_kernels.py [--only gemm|attn|misc] [--iters 20]
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


def pkg(name):
    return importlib.import_module(f"0709_b200.{name}")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


FLUSH = None


def flush():
    global FLUSH
    if FLUSH is None:
        FLUSH = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    FLUSH.fill_(1.0)


def timeit(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) * 1000.0)
    ts.sort()
    return ts[len(ts) // 2]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--dtype", default="float16")
    ap.add_argument("--json-out", default=None, help="also write every row to this JSON file")
    args = ap.parse_args()
    dt = {"float16": torch.float16, "bfloat16": torch.bfloat16}[args.dtype]
    hbm, tflops, src = peaks()
    ops = pkg("ops.cuda_ops").CudaOps(device=torch.device("cuda"))
    out = []

    def report(name, us, nbytes, flops=0.0, **extra):
        gbs = nbytes / (us * 1e-6) / 1e9
        row = {"kernel": name, "us": round(us, 2), "GB/s": round(gbs, 1),
               f"hbm_frac_of_{src}": round(gbs / hbm, 3), **extra}
        if flops:
            row["TFLOP/s"] = round(flops / (us * 1e-6) / 1e12, 1)
        out.append(row)
        print(json.dumps(row), flush=True)

    if args.only in ("all", "gemm"):
        shapes = [("8b.qkv", 6144, 4096), ("8b.o", 4096, 4096), ("8b.gate_up", 28672, 4096), ("8b.down", 4096, 14336),
                  ("8b.lm_head", 128256, 4096), ("1b.qkv", 6144, 2048), ("1b.gate_up", 16384, 2048),
                  ("1b.down", 2048, 8192)]
        for n in (1, 12):
            for name, m, k in shapes:
                w = (torch.randn(m, k, device="cuda") * 0.02).to(dt)
                x = torch.randn(n, k, device="cuda").to(dt)
                o = torch.empty(n, m, device="cuda", dtype=dt)
                fn = lambda: ops._gemm(x, w, o, ops.ext.EPI_STORE)  # noqa: E731
                us = timeit(fn, args.iters)
                report(f"gemm {name}", us, m * k * 2 + n * k * 2 + n * m * 2, 2.0 * m * k * n, rows=n,
                       config=ops.last_gemm_config)
                del w
        for name, m, k, n in (("prefill.qkv", 6144, 4096, 2048), ("prefill.gate_up", 28672, 4096, 2048)):
            w = (torch.randn(m, k, device="cuda") * 0.02).to(dt)
            x = torch.randn(n, k, device="cuda").to(dt)
            o = torch.empty(n, m, device="cuda", dtype=dt)
            us = timeit(lambda: ops._gemm(x, w, o, ops.ext.EPI_STORE), args.iters)
            report(f"gemm {name}", us, m * k * 2 + n * k * 2 + n * m * 2, 2.0 * m * k * n, rows=n,
                   config=ops.last_gemm_config, tflops_frac=round(2.0 * m * k * n / (us * 1e-6) / 1e12 / tflops, 3))
    if args.only in ("all", "attn"):
        attn_desc = pkg("ops.attn_desc")
        hq, hkv, ps = 32, 8, 16
        for prefix in (2048, 8192, 16384):
            for nodes in (1, 12, 48):
                npages = (prefix + nodes + ps - 1) // ps + 1
                kv = torch.randn(1, npages, 2, hkv, ps, 128, device="cuda").to(dt)
                ops.engine = type("E", (), {"kv": kv})()
                pages = torch.arange(npages, dtype=torch.int32, device="cuda")
                masks = torch.full((nodes, 1), -1, dtype=torch.int64, device="cuda")
                lens = torch.full((nodes,), prefix + nodes, dtype=torch.int32, device="cuda")
                full = torch.full((nodes,), prefix, dtype=torch.int32, device="cuda")
                desc = attn_desc.single_sequence_desc(pages, lens, shared_len=prefix, mask_base=prefix, masks=masks,
                                                      full=full)
                q = torch.randn(nodes, hq, 128, device="cuda").to(dt)
                us = timeit(lambda: ops.attention(q, kv[0], desc), args.iters)
                kv_bytes = 2 * (prefix + nodes) * hkv * 128 * 2
                report(f"attn prefix={prefix} rows={nodes}", us, kv_bytes, 4.0 * nodes * hq * 128 * prefix,
                       splits=ops.attention_splits(nodes, hq, hkv, prefix, ps))
                us = timeit(lambda: ops.attention(q, kv[0], desc, stages=(True, False)), args.iters)
                report(f"  tensor-core part only", us, kv_bytes)
                us = timeit(lambda: ops.attention(q, kv[0], desc, stages=(False, True)), args.iters)
                report(f"  combine+tail part only", us, kv_bytes)
                del kv
    if args.only in ("all", "misc"):
        logits = torch.randn(12, 128256, device="cuda")
        us = timeit(lambda: ops.topk_logprobs(logits, 4), args.iters)
        report("topk k=4 rows=12 V=128256", us, logits.numel() * 4)
        x = torch.randn(12, 4096, device="cuda")
        w = torch.ones(4096, device="cuda", dtype=dt)
        us = timeit(lambda: ops.rmsnorm(x, w, 1e-5, dt), args.iters)
        report("rmsnorm rows=12 H=4096", us, x.numel() * 6)
    if args.only in ("all", "chain"):
        # GEMMs only: 32 layers of (qkv, o + residual, gate/up + SiLU, down + residual) at 8B shapes,
        # captured in one CUDA graph with PDL -- the weight-streaming ceiling of a forward.
        llama = pkg("models.llama")
        cfg = llama.get_config("llama-8b")
        w = llama.random_weights(cfg, seed=1, dtype=dt, device="cuda")
        for rows in (1, 12):
            x = torch.randn(rows, cfg.hidden_size, device="cuda").to(dt)
            h = torch.zeros(rows, cfg.hidden_size, device="cuda")
            a = torch.randn(rows, cfg.q_size, device="cuda").to(dt)

            def chain():
                for lw in w.layers:
                    ops.linear(x, lw.wqkv)
                    ops.linear_residual(a, lw.wo, h)
                    act = ops.gate_up_silu(x, lw.wgu)
                    ops.linear_residual(act, lw.wd, h)

            chain()
            g = torch.cuda.CUDAGraph()
            s_ = torch.cuda.Stream()
            s_.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s_):
                chain()
                g.capture_begin()
                chain()
                g.capture_end()
            torch.cuda.current_stream().wait_stream(s_)
            us = timeit(g.replay, max(5, args.iters // 2))
            nbytes = sum(t.numel() * t.element_size() for lw in w.layers for t in (lw.wqkv, lw.wo, lw.wgu, lw.wd))
            report(f"gemm chain 8b x32 layers rows={rows}", us, nbytes)
        del w
        torch.cuda.empty_cache()
    if args.only in ("all", "forward"):
        import numpy as np

        llama = pkg("models.llama")
        engine_mod = pkg("runtime.engine")
        for name, rows in (("llama-8b", 12), ("llama-8b", 1), ("llama-1b", 9), ("llama-1b", 4), ("llama-1b", 3)):
            cfg = llama.get_config(name)
            w = llama.random_weights(cfg, seed=1, dtype=dt, device="cuda")
            eng = engine_mod.LlamaEngine(w, num_pages=512, page_size=16, max_positions=8192)
            pages = torch.arange(300, dtype=torch.int32, device="cuda")
            fields = dict(tokens=np.arange(rows), positions=np.arange(2048, 2048 + rows),
                          slots=np.arange(2048, 2048 + rows), shared_len=2048, n_shared_pages=300, mask_base=2048,
                          row_full=np.full(rows, 2048), row_len=np.full(rows, 2048 + rows))
            b = engine_mod.row_bucket(rows)
            for graphs in (True, False):
                eng.use_graphs = graphs
                us = timeit(lambda: eng.run_rows(b, prefix_pages=pages, **fields), max(5, args.iters // 2))
                report(f"forward {name} rows={rows} P=2048 {'graph+pdl' if graphs else 'eager'}", us,
                       w.nbytes() + 2 * 2048 * cfg.num_layers * cfg.kv_size * 2)
            del eng, w
            torch.cuda.empty_cache()
    if args.json_out:
        with open(args.json_out, "w") as f:
            json.dump(out, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
