#!/usr/bin/env python
"""Per-collective latency of the tensor-parallel layer boundary, on N GPUs (one process each).

    torchrun --nproc-per-node N benchmarks/bench_tp_collective.py --hidden 4096 --rows 1 13

One "collective" is the row-parallel GEMM of a layer (o_proj or down_proj
shard, K = hidden / N) followed by the sum over ranks, the residual add and
the next RMSNorm -- ``TPGroup.allreduce_norm``:

* ``fused``: the GEMM's epilogue stores its fp32 tile into every rank's
  receive slot over NVLink (peer stores, sentinel slots), and
  ``tp_reduce_rmsnorm`` polls, sums in rank order and normalizes;
* ``nccl``: the GEMM into a local fp32 buffer, NCCL ``all_reduce``, then the
  same reduce + RMSNorm kernel with one source;
* ``local``: the GEMM and the one-source reduce with no communication (the
  floor: what the layer boundary costs without tensor parallelism).

Each variant runs ``--chain`` boundaries back to back captured in one CUDA
graph (as in a forward), replayed ``--iters`` times; time per boundary =
graph time / chain, CUDA events on every rank, max over ranks.  Also reported:
the bytes each rank pushes per fused boundary and the time those bytes take
at the measured 770 GB/s peer bandwidth, for the roofline fraction (the
slower of weight streaming at the measured HBM bandwidth and the push over
NVLink, over the measured fused time).
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

PEER_GBS = 770.0   # measured peer copy bandwidth per direction (this pool)
HBM_GBS = 6540.2   # measured copy bandwidth (MEASURED_PEAKS.json)


def pkg(name):
    return importlib.import_module(f"0709_b200.{name}")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--rows", type=int, nargs="+", default=[1, 13])
    ap.add_argument("--chain", type=int, default=64, help="boundaries per graph (a forward has 2 per layer)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--dtype", default="bfloat16")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    comm = pkg("parallel.comm")
    ops = pkg("ops.cuda_ops").CudaOps(device=dev)
    dtype = getattr(torch, args.dtype)
    H = args.hidden
    K = H // world
    groups = {"fused": comm.TPGroup(rank=rank, world=world, device=dev, mode="fused", hidden=H, vocab=world * 128),
              "nccl": comm.TPGroup(rank=rank, world=world, device=dev, mode="nccl", hidden=H, vocab=world * 128)}
    t = torch.zeros(1, device=dev)
    dist.all_reduce(t)
    torch.cuda.synchronize()
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    w = (torch.randn(H, K, device=dev, generator=g) * 0.02).to(dtype)
    gamma = torch.ones(H, device=dev, dtype=dtype)
    result: dict = {"world": world, "hidden": H, "k_per_rank": K, "chain": args.chain, "dtype": args.dtype}
    for m in args.rows:
        a = torch.randn(m, K, device=dev, generator=g).to(dtype)
        h = torch.zeros(m, H, device=dev)
        per: dict = {}
        for name in ("local", "fused", "nccl"):
            if name == "local":
                part = torch.empty(m, H, device=dev)

                def boundary():
                    ops._gemm(a, w, part, ops.ext.EPI_F32)
                    x = torch.empty(m, H, device=dev, dtype=dtype)
                    ops.ext.tp_reduce_rmsnorm(part.data_ptr(), 0, 0, 0, 1, h, gamma, x, 1e-5, ops.err, False)
            else:
                grp = groups[name]

                def boundary(grp=grp):
                    grp.allreduce_norm(ops, a, w, h, gamma, 1e-5, comm.SITE_O)
            for _ in range(3):
                boundary()
            torch.cuda.synchronize()
            dist.barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(args.chain):
                    boundary()
            graph.replay()
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iters):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us = torch.tensor([e0.elapsed_time(e1) * 1e3 / (args.iters * args.chain)], device=dev)
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            per[f"{name}_us"] = round(float(us.item()), 2)
            del graph
            dist.barrier()
        push = (world - 1) * m * H * 4
        floor_us = max(H * K * 2 / (HBM_GBS * 1e3), push / (PEER_GBS * 1e3))
        per.update({
            "push_bytes_per_rank": push,
            "roofline_us": round(floor_us, 2),
            "fused_fraction_of_roofline": round(floor_us / per["fused_us"], 3),
            "fused_over_nccl_speedup": round(per["nccl_us"] / per["fused_us"], 3),
            "fused_collective_overhead_us": round(per["fused_us"] - per["local_us"], 2),
        })
        result[f"rows{m}"] = per
    for grp in groups.values():
        grp.check()
    ops.check()
    torch.cuda.synchronize()
    dist.barrier()
    for grp in groups.values():
        grp.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
