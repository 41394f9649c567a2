"""Tensor-parallel communication for the target model.

Three interchangeable implementations of the two collectives a TP Llama
layer needs -- "row-parallel GEMM, sum over ranks, residual add, RMSNorm"
(twice per layer) and "vocabulary-parallel LM head, gather logits on the
root" (once per forward):

``fused`` (CUDA, the product)
    One symmetric buffer per rank (plain ``cudaMalloc``, mapped into every
    peer by CUDA IPC; no NVLink multicast objects).  The row-parallel GEMM's
    epilogue stores its fp32 partial tile straight into slot ``rank`` of every
    rank's receive buffer over NVLink.  Receive slots hold a sentinel NaN
    pattern until written, so each value is its own arrival flag and the
    producer needs no fence: the next kernel (``tp_reduce_rmsnorm``) polls
    every float4 of every slot (bounded wait), restores the sentinel, sums the
    slots in rank order -- bit-identical on every rank -- adds the residual
    and applies the following RMSNorm.  The LM head's epilogue stores each
    rank's vocabulary slice into the root's logits buffer and raises a
    sequence flag per rank (release/acquire at system scope); the root waits
    on the flags.  Receive buffers alternate between two sets (o_proj,
    down_proj): a rank writes a set again only after every peer has consumed
    the other set, which follows their consumption (and sentinel reset) of
    the set's previous use.
    Rows beyond ``max_rows`` (prefill chunks) take the NCCL path.
``nccl`` (CUDA, the baseline)
    GEMM into a local fp32 buffer, ``all_reduce`` / ``all_gather`` on the
    NCCL process group, then the same reduce+RMSNorm kernel with one source.
``torch`` (CPU ``gloo`` ranks, for tests)
    PyTorch matmuls and ``gloo`` collectives.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

FLAG_OFF = 0            # u32 [3 sites][64 sources]
TICKET_OFF = 1024       # u32 [3 sites]
SEQ_OFF = 1280          # u32 [3 sites]
RECV_OFF = 4096
SITE_O, SITE_DOWN, SITE_LOGITS = 0, 1, 2
MODES = ("fused", "nccl", "torch")


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


@dataclass
class TPGroup:
    rank: int
    world: int
    device: torch.device
    mode: str
    hidden: int
    vocab: int
    group: object = None
    max_rows: int = 64
    # Wall-time limit of every cross-GPU wait in the fused kernels; a peer that
    # misses it makes the kernel record kErrPeerTimeout and return.
    peer_wait_ms: float | None = None

    def __post_init__(self) -> None:
        if self.mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        if self.vocab % self.world:
            raise ValueError("vocabulary must split evenly over the TP ranks")
        self.root = 0
        self.is_root = self.rank == self.root
        self.local_vocab = self.vocab // self.world
        self.base = 0
        self.peers: list[int] = []
        self.ext = None
        self.err = None
        if self.mode != "torch" and self.device.type != "cuda":
            raise ValueError(f"TP mode {self.mode!r} needs CUDA devices")
        if self.mode in ("fused", "nccl"):
            from ..ops import _native

            from ..ops.cuda_ops import device_error_flag

            self.ext = _native.cuda()
            self.err = device_error_flag(self.device)
            wait_ms = self.peer_wait_ms if self.peer_wait_ms is not None else float(
                os.environ.get("ATLAS_PEER_WAIT_MS", "5000"))
            self.ext.set_peer_wait_ns(int(wait_ms * 1e6), self.device.index if self.device.index is not None
                                      else torch.cuda.current_device())
        if self.mode == "fused":
            self._setup_symmetric()

    # ------------------------------------------------------------ setup
    def _setup_symmetric(self) -> None:
        r, w, H = self.rank, self.world, self.hidden
        self.recv_bytes = 2 * w * self.max_rows * H * 4
        self.logits_off = _align(RECV_OFF + self.recv_bytes)
        self.nbytes = _align(self.logits_off + self.max_rows * self.vocab * 4)
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.dev_index = dev
        for p in range(w):
            if p != r and p < torch.cuda.device_count() and not self.ext.can_access_peer(dev, p):
                raise RuntimeError(f"GPU {dev} cannot access peer GPU {p} (no NVLink/P2P path)")
        self.base = self.ext.ipc_malloc(self.nbytes, dev)
        handle = self.ext.ipc_handle(self.base, dev)
        handles: list = [None] * w
        dist.all_gather_object(handles, handle, group=self.group)
        self.peers = []
        self._opened: list[int] = []
        for p in range(w):
            if p == r:
                self.peers.append(self.base)
            else:
                ptr = self.ext.ipc_open(handles[p], dev)
                self._opened.append(ptr)
                self.peers.append(ptr)
        dist.barrier(group=self.group)
        self.logits_buf = self.ext.wrap_ptr(self.base + self.logits_off, [self.max_rows, self.vocab], torch.float32,
                                            dev)
        # Receive slots start as the sentinel (all-ones words); readers restore it after each use.
        recv = self.ext.wrap_ptr(self.base + RECV_OFF, [self.recv_bytes // 4], torch.int32, dev)
        recv.fill_(-1)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers, wait until every peer has unmapped ours, then free ours (all ranks call it)."""
        if self.base:
            torch.cuda.synchronize(self.device)
            for ptr in self._opened:
                self.ext.ipc_close(ptr, self.dev_index)
            self._opened = []
            if self.world > 1:
                dist.barrier(group=self.group)
            self.ext.ipc_free(self.base, self.dev_index)
            self.base = 0

    # ------------------------------------------------------- addresses
    def _recv(self, base: int, site: int, slot: int) -> int:
        return base + RECV_OFF + ((site * self.world + slot) * self.max_rows * self.hidden) * 4

    def _flag(self, base: int, site: int, src: int) -> int:
        return base + FLAG_OFF + (site * 64 + src) * 4

    def check(self) -> None:
        if self.err is not None:
            code = int(self.err.item())
            if code:
                self.err.zero_()
                raise RuntimeError(f"tensor-parallel kernel reported error {code} on rank {self.rank}")

    # ------------------------------------------------------ collectives
    def allreduce_norm(self, ops, a: torch.Tensor, w: torch.Tensor, h: torch.Tensor, gamma: torch.Tensor,
                       eps: float, site: int) -> torch.Tensor:
        """h += sum_ranks(a @ w^T);  returns RMSNorm(h) * gamma in the activation dtype."""
        m, hid = a.shape[0], h.shape[1]
        if self.mode == "torch":
            part = a.float() @ w.float().t()
            if self.world > 1:
                dist.all_reduce(part, group=self.group)
            h += part
            hf = h
            return (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()).to(a.dtype)
        x = torch.empty((m, hid), dtype=a.dtype, device=a.device)
        if self.mode == "fused" and m <= self.max_rows:
            dst = [self._recv(self.peers[p], site, self.rank) for p in range(self.world)]
            self.ext.gemm_peer(w, a, dst, hid, [], 0, 0, ops.ws, ops.counters, self.err, True)
            self.ext.tp_reduce_rmsnorm(self._recv(self.base, site, 0), self.max_rows * hid, 0, 0, self.world, h,
                                       gamma, x, float(eps), self.err, True)
            _count(2)
            return x
        part = torch.empty((m, hid), dtype=torch.float32, device=a.device)
        ops._gemm(a, w, part, self.ext.EPI_F32)
        if self.world > 1:
            dist.all_reduce(part, group=self.group)
        self.ext.tp_reduce_rmsnorm(part.data_ptr(), 0, 0, 0, 1, h, gamma, x, float(eps), self.err, False)
        _count(1)
        return x

    def lm_head(self, ops, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor | None:
        """Vocabulary-parallel LM head; the root gets fp32 logits [M, V], other ranks None."""
        m = x.shape[0]
        v = self.local_vocab
        if self.mode == "torch":
            local = x.float() @ w.float().t()
            if self.world == 1:
                return local
            parts = [torch.empty_like(local) for _ in range(self.world)]
            dist.all_gather(parts, local, group=self.group)
            return torch.cat(parts, dim=1) if self.is_root else None
        if self.mode == "fused" and m <= self.max_rows:
            root = self.peers[self.root]
            self.ext.gemm_peer(w, x, [root + self.logits_off + self.rank * v * 4], self.vocab,
                               [self._flag(root, SITE_LOGITS, self.rank)], self.base + TICKET_OFF + 4 * SITE_LOGITS,
                               self.base + SEQ_OFF + 4 * SITE_LOGITS, ops.ws, ops.counters, self.err, False)
            _count(1)
            if not self.is_root:
                return None
            self.ext.tp_wait(self._flag(self.base, SITE_LOGITS, 0), self.base + SEQ_OFF + 4 * SITE_LOGITS,
                             self.world, self.err)
            _count(1)
            out = self.logits_buf[:m]
            return out if torch.cuda.is_current_stream_capturing() else out.clone()
        local = torch.empty((m, v), dtype=torch.float32, device=x.device)
        ops._gemm(x, w, local, self.ext.EPI_F32)
        if self.world == 1:
            return local
        gathered = torch.empty((self.world, m, v), dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        return gathered.permute(1, 0, 2).reshape(m, self.vocab) if self.is_root else None


def _count(n: int) -> None:
    from ..utils import counters

    counters.launches(n)
