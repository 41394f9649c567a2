"""Set up a tensor-parallel target group inside a ``torch.distributed`` job.

``build_tp_target`` is called by every rank of the TP group (one process per
GPU; the root is rank 0).  It creates the process group's TP communicator,
the host mailbox and this rank's ``TPLlamaEngine`` over its weight shard.
The root then wraps the engine in a ``TargetVerifier`` and serves; the other
ranks call ``engine.serve()``.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..models.llama import LlamaConfig
from .comm import TPGroup
from .mailbox import Mailbox
from .shard import random_weights_tp
from .tp_engine import TPLlamaEngine


def mailbox_path(tag: str = "") -> str:
    port = os.environ.get("MASTER_PORT", "0")
    root = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
    return os.path.join(root, f"atlas_tp_{port}{tag}")


def build_tp_target(cfg: LlamaConfig, *, mode: str, seed: int, dtype: torch.dtype, num_pages: int, page_size: int,
                    max_positions: int, device: torch.device, group=None, tag: str = "") -> TPLlamaEngine:
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    path = mailbox_path(tag)
    mb = None
    ack_timeout = float(os.environ.get("ATLAS_TP_ACK_TIMEOUT", "120"))
    if world > 1 and rank == 0:
        mb = Mailbox(path, rank=0, world=world, create=True, ack_timeout_s=ack_timeout)
    dist.barrier(group=group)
    if world > 1 and rank != 0:
        mb = Mailbox(path, rank=rank, world=world, create=False)
    w = random_weights_tp(cfg, rank=rank, tp=world, seed=seed, dtype=dtype, device=device)
    tpg = TPGroup(rank=rank, world=world, device=device, mode=mode, hidden=cfg.hidden_size, vocab=cfg.vocab_size,
                  group=group)
    if device.type == "cuda" and world > 1:
        # Bring up the NCCL communicator outside any graph capture.
        t = torch.zeros(1, device=device)
        dist.all_reduce(t, group=group)
        torch.cuda.synchronize(device)
    eng = TPLlamaEngine(w, group=tpg, model_config=cfg, mailbox=mb, num_pages=num_pages, page_size=page_size,
                        max_positions=max_positions)
    dist.barrier(group=group)
    return eng
