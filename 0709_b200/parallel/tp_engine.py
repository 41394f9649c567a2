"""Tensor-parallel target engine.

``TPLlamaEngine`` is a ``LlamaEngine`` over one rank's shard (``heads/tp``
query and KV heads, ``ffn/tp`` MLP rows, ``vocab/tp`` LM-head rows) whose
forward replaces the single-GPU residual epilogues by the TP collectives of
``TPGroup``:

    h = embed(tokens);  x = RMSNorm(h)
    per layer:  qkv = x Wqkv_r;  rope + KV append (local KV heads);  attention
                x = RMSNorm(h += sum_r  attn_r Wo_r)       (fused collective)
                x = RMSNorm'(h += sum_r  silu·mul(x Wgu_r) Wd_r)
    logits = gather_r(x Wlm_r)  on the root

The root rank (rank 0) runs the serving logic and calls the engine like a
single-GPU one; every call (graph replay, prefill, KV moves, page-table
updates, graph capture) is first posted to the worker ranks through the host
mailbox, and the workers repeat it on their shards in the same order, so the
device-side collectives pair up.  Workers run ``serve()`` until the root
posts stop.

The reference has no tensor parallelism; this is the 70B-target
configuration's TP=2/4/8 target.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch

from ..models.llama import LlamaConfig, LlamaWeights
from ..runtime.engine import LlamaEngine
from .comm import SITE_DOWN, SITE_O, TPGroup
from .mailbox import OP_CALL, OP_STOP, Mailbox


class HostMark:
    """A host timestamp with the ``elapsed_time`` of a CUDA event (CPU ranks)."""

    def __init__(self) -> None:
        self.t = time.perf_counter()

    def elapsed_time(self, other: "HostMark") -> float:
        return (other.t - self.t) * 1e3


class TPLlamaEngine(LlamaEngine):
    def __init__(self, weights: LlamaWeights, *, group: TPGroup, model_config: LlamaConfig, mailbox: Mailbox | None,
                 num_pages: int, page_size: int = 16, max_positions: int = 32768) -> None:
        super().__init__(weights, num_pages=num_pages, page_size=page_size, max_positions=max_positions)
        self.tp = group
        self.model_cfg = model_config
        self.mailbox = mailbox
        self.is_root = group.is_root
        self._mirrors: dict[int, torch.Tensor] = {}   # worker: root mirror id -> local page table
        self._root_mirrors: dict[int, object] = {}    # root: id -> mirror
        self.posted_calls = 0
        # Timing marks: CUDA events recorded by every rank at the same point of the
        # call stream (``mark``); ``mark_hook(tag)`` runs on each rank right after.
        self.marks: dict[str, torch.cuda.Event] = {}
        self.mark_launches: dict[str, int] = {}
        self.mark_hook = None

    # ---------------------------------------------------------- forward
    @torch.inference_mode()
    def forward(self, tokens, positions, slots, desc, *, logits_rows=None, causal_start=None):
        o = self.ops
        c = self.cfg
        tp = self.tp
        self.stats.calls += 1
        self.stats.rows += int(tokens.numel())
        layers = self.w.layers
        h = o.embed(tokens, self.w.embed)
        x = o.rmsnorm(h, layers[0].attn_norm, c.rms_eps, self.dtype)
        fuse_rope = hasattr(o, "qkv_rope") and c.head_dim == 128
        for li, lw in enumerate(layers):
            if fuse_rope:
                # RoPE + KV append in the QKV GEMM epilogue (x is already normalized: no rstd scaling).
                q = o.qkv_rope(x, lw.wqkv, None, 0.0, self.rope, positions, slots, self.kv[li], c.num_heads,
                               c.num_kv_heads)
            else:
                qkv = o.linear(x, lw.wqkv)
                q = o.rope_qkv_append(qkv, self.rope, positions, slots, self.kv[li], c.num_heads, c.num_kv_heads)
            if causal_start is not None and hasattr(o, "attention_causal"):
                a = o.attention_causal(q, self.kv[li], desc, causal_start, self.scale)
            else:
                a = o.attention(q, self.kv[li], desc, self.scale)
            x = tp.allreduce_norm(o, a, lw.wo, h, lw.mlp_norm, c.rms_eps, SITE_O)
            act = o.gate_up_silu(x, lw.wgu)
            gamma = layers[li + 1].attn_norm if li + 1 < len(layers) else self.w.final_norm
            x = tp.allreduce_norm(o, act, lw.wd, h, gamma, c.rms_eps, SITE_DOWN)
        if logits_rows is not None:
            x = x.index_select(0, logits_rows.long())
        return tp.lm_head(o, x, self.w.lm_head)

    # ------------------------------------------------------ root -> all
    def _post(self, name: str, **kw) -> None:
        if self.is_root and self.mailbox is not None and self.tp.world > 1:
            self.mailbox.post(OP_CALL, (name, kw))
            self.posted_calls += 1

    def register_mirror(self, mirror) -> None:
        """Forward a page-table mirror's updates (root) to the workers' copies."""
        mid = int(mirror.dev.data_ptr())
        self._root_mirrors[mid] = mirror
        self._post("mirror_new", mid=mid, capacity=int(mirror.dev.numel()))

        def hook(start: int, values: list[int], _mid=mid) -> None:
            self._post("mirror_update", mid=_mid, start=int(start), values=np.asarray(values, dtype=np.int32))

        mirror.on_update = hook

    def _pages(self, t: torch.Tensor) -> tuple[int, int]:
        """(mirror id, length) of a root page-table tensor (a view of a registered mirror)."""
        for mid, m in self._root_mirrors.items():
            base = m.dev.data_ptr()
            off = t.data_ptr() - base
            if 0 <= off < m.dev.numel() * 4 and off % 4 == 0:
                if off:
                    raise ValueError("page tables must start at the mirror's first entry")
                return mid, int(t.numel())
        raise ValueError("page table is not a registered mirror; call register_mirror first")

    def _local_pages(self, mid: int, n: int | None = None) -> torch.Tensor:
        t = self._mirrors[mid]
        return t if n is None else t[:n]

    @torch.inference_mode()
    def run_rows(self, rows: int, *, tail_stride: int = 1, mask_words: int = 1, prefix_pages: torch.Tensor, **fields):
        if self.is_root and self.tp.world > 1:
            toks = fields.get("tokens")
            if isinstance(toks, torch.Tensor):
                # Device-fed token (target fallback AR): the workers need its value.
                fields = dict(fields, tokens=toks.cpu().numpy().astype(np.int32))
            mid, _ = self._pages(prefix_pages)
            self._post("run_rows", rows=int(rows), tail_stride=int(tail_stride), mask_words=int(mask_words), mid=mid,
                       fields={k: (np.asarray(v) if not np.isscalar(v) else v) for k, v in fields.items()})
        return self._run_rows_local(rows, tail_stride=tail_stride, mask_words=mask_words, prefix_pages=prefix_pages,
                                    **fields)

    @torch.inference_mode()
    def _run_rows_local(self, rows: int, *, tail_stride: int, mask_words: int, prefix_pages: torch.Tensor, **fields):
        sb = self.static_batch(rows, tail_stride, mask_words)
        n = sb.load(**fields)
        desc = sb.desc(prefix_pages)
        if self.device.type != "cuda" or not self.use_graphs:
            logits = self.forward(sb.tokens, sb.positions, sb.slots, desc)
            return None if logits is None else logits[sb.real_slice(n)].clone()
        key = (sb.key, prefix_pages.data_ptr(), None)  # same key as ``warm_graph`` (no graph top-k)
        graph = self._graphs.get(key)
        if graph is None:
            graph = self._capture(sb, desc)
            self._graphs[key] = graph
        for g in graph.graphs:
            g.replay()
        if graph.launches:
            from ..utils import counters

            counters.launches(graph.launches)
        self.stats.calls += 1
        self.stats.rows += n
        return None if graph.out is None else graph.out[sb.real_slice(n)].clone()

    @torch.inference_mode()
    def warm_graph(self, rows: int, *, tail_stride: int = 1, mask_words: int = 1, prefix_pages: torch.Tensor) -> None:
        if self.device.type != "cuda" or not self.use_graphs:
            return
        if self.is_root:
            mid, _ = self._pages(prefix_pages)
            self._post("warm_graph", rows=int(rows), tail_stride=int(tail_stride), mask_words=int(mask_words), mid=mid)
        super().warm_graph(rows, tail_stride=tail_stride, mask_words=mask_words, prefix_pages=prefix_pages)

    def prefill_sequence(self, tokens, *, start_pos, slots, pages, chunk_size=8192):
        if self.is_root:
            mid, n = self._pages(pages)
            self._post("prefill", tokens=tokens.cpu().numpy(), start_pos=int(start_pos), slots=slots.cpu().numpy(),
                       mid=mid, n_pages=n, chunk_size=int(chunk_size))
        return super().prefill_sequence(tokens, start_pos=start_pos, slots=slots, pages=pages, chunk_size=chunk_size)

    def copy_pages(self, copies: torch.Tensor) -> None:
        if copies.numel():
            self._post("copy_pages", copies=copies.cpu().numpy())
        super().copy_pages(copies)

    def move_slots(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        if src.numel():
            self._post("move_slots", src=src.cpu().numpy(), dst=dst.cpu().numpy())
        super().move_slots(src, dst)

    def mark(self, tag: str, *, barrier: bool = False) -> None:
        """Record a CUDA event named ``tag`` on every rank at this point of the call stream.

        With ``barrier`` each rank first drains its GPU work and meets the others, so
        the events open a region that every rank starts together; without it the
        event follows the rank's previously issued work (the end of a region).
        ``elapsed_ms(a, b)`` then gives each rank's device time between two marks.
        """
        self._post("mark", tag=str(tag), barrier=bool(barrier))
        self._w_mark(str(tag), bool(barrier))

    def elapsed_ms(self, start: str, end: str) -> float:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        return float(self.marks[start].elapsed_time(self.marks[end]))

    def set_comm_mode(self, mode: str) -> None:
        """Switch every rank's collectives (``fused`` or ``nccl``); captured graphs are dropped."""
        self._post("set_comm_mode", mode=str(mode))
        self._w_set_comm_mode(str(mode))

    def stop_workers(self) -> None:
        if self.is_root and self.mailbox is not None and self.tp.world > 1:
            self.mailbox.post(OP_STOP, None)
            self.mailbox.drain()

    # ------------------------------------------------------------ worker
    @torch.inference_mode()
    def serve(self) -> int:
        """Worker loop: repeat the root's calls until it posts stop; returns the number of calls."""
        assert not self.is_root and self.mailbox is not None
        calls = 0
        self.worker_wait_s = 0.0
        self.worker_handle_s = 0.0
        # Host-side fault injection for tests: leave between two calls, as a crashed
        # rank would (never inside a kernel or collective).
        exit_after = int(os.environ.get("ATLAS_TP_FAULT_EXIT_AFTER", "-1"))
        while True:
            if 0 <= exit_after <= calls:
                os._exit(0)
            t0 = time.perf_counter()
            op, payload = self.mailbox.receive()
            t1 = time.perf_counter()
            self.worker_wait_s += t1 - t0
            if op == OP_STOP:
                return calls
            name, kw = payload
            getattr(self, "_w_" + name)(**kw)
            self.worker_handle_s += time.perf_counter() - t1
            calls += 1

    def _w_mark(self, tag: str, barrier: bool) -> None:
        from ..utils import counters

        cuda = self.device.type == "cuda"
        if barrier:
            if cuda:
                torch.cuda.synchronize(self.device)
            if self.tp.world > 1:
                import torch.distributed as dist

                dist.barrier(group=self.tp.group)
                if cuda:
                    torch.cuda.synchronize(self.device)
        if cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
        else:
            ev = HostMark()
        self.marks[tag] = ev
        self.mark_launches[tag] = counters.snapshot()["launches"]
        if self.mark_hook is not None:
            self.mark_hook(tag)

    def _w_set_comm_mode(self, mode: str) -> None:
        from .comm import MODES

        if mode not in MODES:
            raise ValueError(f"comm mode must be one of {MODES}")
        if mode == "fused" and not self.tp.base:
            raise ValueError("fused collectives need the peer buffers mapped at start-up (build in fused mode)")
        self.drop_graphs()
        self.tp.mode = mode

    def _w_mirror_new(self, mid: int, capacity: int) -> None:
        self._mirrors[mid] = torch.zeros(capacity, dtype=torch.int32, device=self.device)

    def _w_mirror_update(self, mid: int, start: int, values: np.ndarray) -> None:
        t = self._mirrors[mid]
        t[start:start + len(values)].copy_(torch.from_numpy(values).to(self.device, non_blocking=False))

    def _w_run_rows(self, rows: int, tail_stride: int, mask_words: int, mid: int, fields: dict) -> None:
        self._run_rows_local(rows, tail_stride=tail_stride, mask_words=mask_words, prefix_pages=self._mirrors[mid],
                             **fields)

    def _w_warm_graph(self, rows: int, tail_stride: int, mask_words: int, mid: int) -> None:
        LlamaEngine.warm_graph(self, rows, tail_stride=tail_stride, mask_words=mask_words,
                               prefix_pages=self._mirrors[mid])

    def _w_prefill(self, tokens, start_pos, slots, mid, n_pages, chunk_size) -> None:
        dev = self.device
        LlamaEngine.prefill_sequence(self, torch.from_numpy(tokens).to(dev), start_pos=start_pos,
                                     slots=torch.from_numpy(slots).to(dev), pages=self._local_pages(mid, n_pages),
                                     chunk_size=chunk_size)

    def _w_copy_pages(self, copies) -> None:
        LlamaEngine.copy_pages(self, torch.from_numpy(copies))

    def _w_move_slots(self, src, dst) -> None:
        LlamaEngine.move_slots(self, torch.from_numpy(src), torch.from_numpy(dst))
