"""Llama forward executor over a paged KV cache.

One engine owns a model's weights, its KV cache
``[layers, pages, 2, kv_heads, page_size, head_dim]`` and a rotary table.
``forward`` runs any batch of rows (drafter routes, target tree nodes, an AR
token, a prefill chunk): each row has a token, a position, the KV slot it
writes, and an attention descriptor row.  On CUDA devices every op is an
sm_100a kernel from the ``atlas_cuda`` extension (the forward raises if the
extension is missing); on CPU the PyTorch ops in ``ops.torch_ops`` run.

Parity: reference src/atlas_0709/flashinfer_full_verify.py:1065-1231 (manual
Llama layer loop with RoPE, suffix KV write and paged attention) and the
SGLang decode forward the drafter uses (fp/flashinfer_backends.py:89-132).
"""

from __future__ import annotations

import math
import os
import threading
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np
import torch

from ..models.llama import LlamaWeights, rope_table
from ..ops import torch_ops
from ..ops.attn_desc import AttnDesc, single_sequence_desc


def kv_bytes_per_token(cfg) -> int:
    return cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2


@dataclass
class ForwardStats:
    calls: int = 0
    rows: int = 0
    prefill_tokens: int = 0


class LlamaEngine:
    def __init__(
        self,
        weights: LlamaWeights,
        *,
        num_pages: int,
        page_size: int = 16,
        max_positions: int = 32768,
        ops=None,
    ) -> None:
        self.w = weights
        self.cfg = weights.config
        self.device = weights.device
        self.dtype = weights.dtype
        self.page_size = int(page_size)
        self.num_pages = int(num_pages)
        c = self.cfg
        self.kv = torch.zeros(
            (c.num_layers, self.num_pages, 2, c.num_kv_heads, self.page_size, c.head_dim),
            dtype=self.dtype,
            device=self.device,
        )
        self.rope = rope_table(c, max_positions, device=self.device)
        self.scale = 1.0 / math.sqrt(c.head_dim)
        if ops is None:
            if self.device.type == "cuda":
                from ..ops import cuda_ops

                ops = cuda_ops.CudaOps(self)
            else:
                ops = torch_ops
        self.ops = ops
        # CUDA: RMSNorm folded into the GEMMs and RoPE + KV append into the QKV
        # epilogue (needs head_dim 128 and 128-aligned widths).
        self.fused_norm = (
            hasattr(ops, "qkv_rope") and c.head_dim == 128 and c.hidden_size % 128 == 0
            and isinstance(weights, LlamaWeights) and os.environ.get("ATLAS_FUSED_NORM", "1") != "0"
        )
        self._folded = self._fold_norms() if self.fused_norm else None
        if hasattr(ops, "reserve_attention_workspace"):
            ops.reserve_attention_workspace(64, c.num_heads, c.num_kv_heads, int(max_positions), self.page_size)
        self.stats = ForwardStats()
        self._run_lock = threading.RLock()
        self.use_graphs = True
        self._static: dict[tuple[int, int, int], StaticBatch] = {}
        self._graphs: dict = {}
        self._graph_pool = torch.cuda.graph_pool_handle() if self.device.type == "cuda" else None
        # A forward's graph is captured as a short head (embedding + the first
        # layers) and the rest: launching a graph costs the host ~1 us per node,
        # and with one graph the GPU would wait for all of it; with two it starts
        # on the head while the host still launches the tail.
        self.graph_head_layers = int(os.environ.get("ATLAS_GRAPH_HEAD_LAYERS", "2"))
        # Scratch page for padded rows' KV writes (never part of any sequence).
        self.trash_slot = (self.num_pages - 1) * self.page_size
        # Graphs captured from now on start with the copy-on-write copy of the plan that rides in
        # the static batch (set by the drafter, whose decode forwards copy tail pages).
        self.cow_in_graph = False

    # ------------------------------------------------------------------
    def _fold_norms(self):
        """Weights with the RMSNorm gains multiplied into their input columns.

        With unit gains (random init) the weights are used as they are;
        otherwise folded copies are made once (the originals are untouched).
        """

        def fold(wt: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
            if bool(torch.all(g == 1)):
                return wt
            return (wt.float() * g.float()[None, :]).to(wt.dtype).contiguous()

        layers = [(fold(lw.wqkv, lw.attn_norm), fold(lw.wgu, lw.mlp_norm)) for lw in self.w.layers]
        return layers, fold(self.w.lm_head, self.w.final_norm)

    def graph_attention_splits(self, rows: int) -> int | None:
        """Split-KV count baked into a graph: sized for the longest context the engine holds."""
        f = getattr(self.ops, "attention_splits", None)
        if f is None:
            return None
        c = self.cfg
        return f(rows, c.num_heads, c.num_kv_heads, int(self.rope.shape[0]), self.page_size)

    def static_batch(self, rows: int, tail_stride: int = 1, mask_words: int = 1) -> "StaticBatch":
        key = (int(rows), int(tail_stride), int(mask_words))
        sb = self._static.get(key)
        if sb is None:
            sb = StaticBatch(self, *key)
            self._static[key] = sb
        return sb

    @torch.inference_mode()
    def run_rows(self, rows: int, *, tail_stride: int = 1, mask_words: int = 1, prefix_pages: torch.Tensor, **fields):
        """Forward ``len(tokens)`` rows through a CUDA graph of the padded row bucket.

        ``fields`` are host arrays (see ``StaticBatch.load``); returns fp32 logits
        [real rows, V] (a fresh tensor).  On CPU the eager forward runs instead.
        ``cow`` (optional, [n, 3] host array of (src page, dst page, tokens)) are
        copy-on-write page copies done first; they reach the device inside the
        static batch's copy.
        """
        with self._run_lock:  # sessions in several threads may share this engine's static inputs
            return self._run_rows_locked(rows, tail_stride, mask_words, prefix_pages, fields)

    def _run_rows_locked(self, rows, tail_stride, mask_words, prefix_pages, fields, topk=None):
        sb = self.static_batch(rows, tail_stride, mask_words)
        cow = fields.pop("cow", None)
        ncow = len(cow) if cow is not None else 0
        if ncow:
            if fields.get("aux") is not None:
                raise ValueError("copy-on-write page copies and auxiliary words share one region")
            if ncow > sb.M:
                raise ValueError(f"{ncow} copy-on-write pages for a bucket of {sb.M} rows")
            fields["aux"] = np.asarray(cow, dtype=np.int32).reshape(-1)
        graphed = self.device.type == "cuda" and self.use_graphs
        key = (sb.key, prefix_pages.data_ptr(), topk)
        graph = self._graphs.get(key) if graphed else None
        # A captured graph that starts with the copy-on-write node copies the plan itself (count in
        # the static batch); otherwise (eager, or the call that captures) it is copied here first.
        in_graph = graph is not None and graph.cow
        n = sb.load(**fields, cow_count=ncow if in_graph else 0)
        if ncow and not in_graph:
            # Tail-page copies (src page, dst page, tokens) before the forward appends to the copies.
            self.ops.kv_copy_pages(self.kv, sb.aux[: 3 * ncow].view(ncow, 3))
        if not graphed:
            logits = self.forward(sb.tokens, sb.positions, sb.slots, sb.desc(prefix_pages))
            return logits[sb.real_slice(n)].clone()
        if graph is None:  # a replay reads the static inputs directly; only a capture needs the descriptor
            graph = self._capture(sb, sb.desc(prefix_pages), topk)
            self._graphs[key] = graph
        if graph.cand is not None and graph.cand.pending is not None:
            graph.cand.pending.materialize()  # keep the previous replay's pack before it is overwritten
        for g in graph.graphs:
            g.replay()
        if graph.cand is not None:
            graph.cand.done.record()
            graph.cand.pending = _Replay(graph.cand, self.ops.err)
        if graph.launches:
            from ..utils import counters

            counters.launches(graph.launches)
        self.stats.calls += 1
        self.stats.rows += n
        logits = graph.out[sb.real_slice(n)].clone()
        if topk:
            return logits, CandidateReadout(graph.cand.pending, sb.real_slice(n))
        return logits

    def graph_topk_available(self) -> bool:
        """Whether ``run_rows_topk`` reads its candidates out of the captured graph."""
        return self.device.type == "cuda" and self.use_graphs and hasattr(self.ops, "topk_logprobs")

    @torch.inference_mode()
    def run_rows_topk(self, rows: int, k: int, *, tail_stride: int = 1, mask_words: int = 1,
                      prefix_pages: torch.Tensor, **fields):
        """``run_rows`` whose graph also selects each row's top-``k`` (greedy) candidates and copies
        them to the host; returns (logits, ``CandidateReadout``).  CUDA graphs only."""
        if not self.graph_topk_available():
            raise RuntimeError("run_rows_topk needs a CUDA engine with graphs")
        with self._run_lock:
            return self._run_rows_locked(rows, tail_stride, mask_words, prefix_pages, fields, topk=int(k))

    @torch.inference_mode()
    def warm_graph(self, rows: int, *, tail_stride: int = 1, mask_words: int = 1, prefix_pages: torch.Tensor,
                   topk: int | None = None) -> None:
        """Capture the graph of one row bucket now (call before concurrent serving starts).

        Padding-only rows: every row writes the trash slot and attends to
        position 0, so capture touches no live KV.
        """
        if self.device.type != "cuda" or not self.use_graphs:
            return
        sb = self.static_batch(rows, tail_stride, mask_words)
        key = (sb.key, prefix_pages.data_ptr(), topk)
        if key in self._graphs:
            return
        sb.load(tokens=[], positions=[], slots=[], shared_len=1, n_shared_pages=1, mask_base=1, row_full=[],
                row_len=[])
        self._graphs[key] = self._capture(sb, sb.desc(prefix_pages), topk)
        torch.cuda.synchronize(self.device)

    def _capture(self, sb: "StaticBatch", desc: AttnDesc, topk: int | None = None):
        from ..utils import counters

        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(2):
                self.forward(sb.tokens, sb.positions, sb.slots, desc)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        before = counters.snapshot()["launches"]
        split = self._graph_split()
        keep = ()
        cand: list = []
        cow = bool(self.cow_in_graph and hasattr(self.ops, "kv_copy_pages_counted"))

        def head(fn):
            if not cow:
                return fn
            plan = sb.aux[: 3 * sb.M].view(sb.M, 3)

            def run():
                self.ops.kv_copy_pages_counted(self.kv, plan, sb.dparams[3:4])
                return fn()
            return run
        if topk:
            # Filled by the graph on every replay (allocated before capture: pinned, fixed address).
            host = torch.zeros(sb.M * topk * 2 + 1, dtype=torch.int32, pin_memory=True)

            def tail(logits):
                lp, ids = self.ops.topk_logprobs(logits, topk)
                pack = torch.cat((ids.to(torch.int32).reshape(-1), lp.reshape(-1).view(torch.int32),
                                  self.ops.err.reshape(-1)[:1]))
                self.ops.ext.copy_to_host_async(host, pack)
                cand.append(CandidateBuffers(topk, sb.M, host, torch.cuda.Event()))
                return logits
        else:
            def tail(logits):
                return logits
        # Capture on the side stream without the device-wide synchronize that
        # ``torch.cuda.graph`` performs first: another serving thread may be
        # capturing or running at the same time (thread-local capture mode).
        with torch.cuda.stream(stream):
            if split:
                # Head: embedding + layers [0, split).  The residual stream and
                # its norm statistics carry over to the tail graph; they stay
                # referenced so no other capture reuses their memory.
                g1 = self._capture_one(head(lambda: self._fused_layers(
                    self.ops.embed_norm(sb.tokens, self.w.embed), sb.positions, sb.slots, desc, None, 0, split)))
                keep = g1[1]
                g2 = self._capture_one(lambda: tail(self._fused_end(
                    self._fused_layers(keep, sb.positions, sb.slots, desc, None, split, self.cfg.num_layers), None)))
                graphs, out = [g1[0], g2[0]], g2[1]
            else:
                g, out = self._capture_one(head(lambda: tail(self.forward(sb.tokens, sb.positions, sb.slots, desc))))
                graphs = [g]
        torch.cuda.current_stream(self.device).wait_stream(stream)
        launches = counters.snapshot()["launches"] - before
        return CapturedForward(graphs, out, launches, keep, cand[0] if cand else None, cow)

    def drop_graphs(self) -> None:
        """Release every captured graph.  Their private memory pool goes with them, so later
        captures start a new pool (a released pool cannot be captured into again)."""
        self._graphs.clear()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            self._graph_pool = torch.cuda.graph_pool_handle()

    def _capture_one(self, fn):
        g = torch.cuda.CUDAGraph()
        g.capture_begin(self._graph_pool, capture_error_mode="thread_local")
        try:
            out = fn()
        finally:
            g.capture_end()
        return g, out

    def _graph_split(self) -> int:
        """Layers in the head graph (0: one graph), for the folded-norm forward of this class."""
        if not self.fused_norm or type(self).forward is not LlamaEngine.forward:
            return 0
        k = self.graph_head_layers
        return k if 0 < k < self.cfg.num_layers else 0

    @torch.inference_mode()
    def forward(
        self,
        tokens: torch.Tensor,
        positions: torch.Tensor,
        slots: torch.Tensor,
        desc: AttnDesc,
        *,
        logits_rows: torch.Tensor | None = None,
        causal_start: int | None = None,
    ) -> torch.Tensor:
        """Run all layers for ``M`` rows; return fp32 logits for ``logits_rows`` (default: all)."""
        o = self.ops
        c = self.cfg
        self.stats.calls += 1
        self.stats.rows += int(tokens.numel())
        if self.fused_norm:
            return self._forward_fused(tokens, positions, slots, desc, logits_rows, causal_start)
        h = o.embed(tokens, self.w.embed)
        for li, lw in enumerate(self.w.layers):
            x = o.rmsnorm(h, lw.attn_norm, c.rms_eps, self.dtype)
            qkv = o.linear(x, lw.wqkv)
            q = o.rope_qkv_append(qkv, self.rope, positions, slots, self.kv[li], c.num_heads, c.num_kv_heads)
            if causal_start is None:
                a = o.attention(q, self.kv[li], desc, self.scale)
            else:
                a = o.attention_causal(q, self.kv[li], desc, causal_start, self.scale) if hasattr(
                    o, "attention_causal"
                ) else o.attention(q, self.kv[li], desc, self.scale)
            h = o.linear_residual(a, lw.wo, h)
            x = o.rmsnorm(h, lw.mlp_norm, c.rms_eps, self.dtype)
            act = o.gate_up_silu(x, lw.wgu)
            h = o.linear_residual(act, lw.wd, h)
        if logits_rows is not None:
            h = h.index_select(0, logits_rows.long())
        x = o.rmsnorm(h, self.w.final_norm, c.rms_eps, self.dtype)
        return o.lm_head(x, self.w.lm_head)

    def _attend(self, q, li, desc, causal_start):
        o = self.ops
        if causal_start is None:
            return o.attention(q, self.kv[li], desc, self.scale)
        return o.attention_causal(q, self.kv[li], desc, causal_start, self.scale)

    def _forward_fused(self, tokens, positions, slots, desc, logits_rows, causal_start):
        """CUDA forward with RMSNorm folded into the GEMMs (no norm or RoPE kernels)."""
        state = self.ops.embed_norm(tokens, self.w.embed)
        state = self._fused_layers(state, positions, slots, desc, causal_start, 0, self.cfg.num_layers)
        return self._fused_end(state, logits_rows)

    def _fused_layers(self, state, positions, slots, desc, causal_start, l0: int, l1: int):
        """Layers [l0, l1) on the residual stream ``state`` = (h fp32, hb activation copy,
        per-128-feature sums of h^2), updated in place; returns ``state``."""
        o = self.ops
        c = self.cfg
        h, hb, ss = state
        layers = self._folded[0]
        for li in range(l0, l1):
            lw = self.w.layers[li]
            wqkv, wgu = layers[li]
            q = o.qkv_rope(hb, wqkv, ss, c.rms_eps, self.rope, positions, slots, self.kv[li], c.num_heads,
                           c.num_kv_heads)
            a = self._attend(q, li, desc, causal_start)
            o.linear_residual_norm(a, lw.wo, h, hb, ss)
            act = o.gate_up_silu_norm(hb, wgu, ss, c.rms_eps)
            o.linear_residual_norm(act, lw.wd, h, hb, ss)
        return state

    def _fused_end(self, state, logits_rows):
        """Final norm (folded into the LM head) on the rows ``logits_rows`` (default: all)."""
        o = self.ops
        c = self.cfg
        _, hb, ss = state
        lm = self._folded[1]
        if logits_rows is not None:
            sel = logits_rows.long()
            hb = hb.index_select(0, sel)
            ss = ss.index_select(1, sel).contiguous()
        return o.lm_head_norm(hb, lm, ss, c.rms_eps)

    # ------------------------------------------------------------------
    def prefill_sequence(
        self,
        tokens: torch.Tensor,
        *,
        start_pos: int,
        slots: torch.Tensor,
        pages: torch.Tensor,
        chunk_size: int = 8192,
    ) -> torch.Tensor:
        """Causal prefill of ``tokens`` at positions ``start_pos..`` in one page list.

        Runs in chunks of ``chunk_size``; returns the fp32 logits of the last token.
        """
        n = int(tokens.numel())
        if n == 0:
            raise ValueError("prefill needs at least one token")
        dev = self.device
        logits = None
        self.stats.prefill_tokens += n
        for c0 in range(0, n, int(chunk_size)):
            c1 = min(n, c0 + int(chunk_size))
            pos = torch.arange(start_pos + c0, start_pos + c1, dtype=torch.int32, device=dev)
            desc = single_sequence_desc(pages, pos + 1, shared_len=start_pos + c0)
            last = torch.tensor([c1 - c0 - 1], dtype=torch.long, device=dev)
            logits = self.forward(
                tokens[c0:c1], pos, slots[c0:c1], desc, logits_rows=last, causal_start=start_pos + c0
            )
        # Tensor-parallel worker ranks get no logits (they live on the root rank).
        return None if logits is None else logits[0]

    def copy_pages(self, copies: torch.Tensor) -> None:
        if copies.numel():
            self.ops.kv_copy_pages(self.kv, copies.to(self.device))

    def move_slots(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        if src.numel():
            self.ops.kv_move_slots(self.kv, src.to(self.device), dst.to(self.device))


class CapturedForward(NamedTuple):
    """CUDA graphs of one forward (replayed in order), its static output, the kernel
    launches they contain, the tensors carried from one graph to the next, and (when
    captured with a top-k) the candidate read-out buffers."""

    graphs: list
    out: torch.Tensor | None
    launches: int
    keep: tuple
    cand: "CandidateBuffers | None" = None
    cow: bool = False  # the first graph copies the static batch's copy-on-write plan itself


@dataclass
class CandidateBuffers:
    """Top-``k`` candidates of every row of a captured forward.  The graph itself runs
    the top-k kernel on its logits, packs [ids (int32) | log-probs (fp32 bits) | the
    device error flag] and copies the pack into ``host`` (pinned), so a replay needs no
    further launch before the host reads it; ``done`` is recorded after each replay and
    ``pending`` is the last replay's read-out state."""

    k: int
    rows: int
    host: torch.Tensor
    done: torch.cuda.Event
    pending: "_Replay | None" = None


class _Replay:
    """One replay's pack in a graph's pinned buffer, copied out once: by its reader, or -- when
    another thread replays the same graph first (sessions sharing an engine) -- by that replay
    before it overwrites the buffer."""

    def __init__(self, buf: CandidateBuffers, status: torch.Tensor) -> None:
        self.buf, self.status = buf, status
        self.lock = threading.Lock()
        self.data: tuple[int, np.ndarray, np.ndarray] | None = None
        self.cleared = False

    def materialize(self) -> tuple[int, np.ndarray, np.ndarray]:
        with self.lock:
            if self.data is None:
                b = self.buf
                b.done.synchronize()
                h = b.host.numpy()
                rk = b.rows * b.k
                self.data = (int(h[2 * rk]), h[:rk].reshape(b.rows, b.k).astype(np.int64),
                             h[rk: 2 * rk].view(np.float32).reshape(b.rows, b.k).copy())
            return self.data


class CandidateReadout:
    """The candidates of one replay (rows ``real`` of the bucket)."""

    def __init__(self, replay: _Replay, real: slice) -> None:
        self.replay, self.real = replay, real
        self.buf = replay.buf
        self.words = self.buf.rows * self.buf.k * 2 + 1

    def last_row(self) -> "CandidateReadout":
        """The same replay's read-out restricted to the bucket's last row."""
        return CandidateReadout(self.replay, slice(self.buf.rows - 1, self.buf.rows))

    def get(self) -> tuple[np.ndarray, np.ndarray]:
        """(ids int64 [n, k], log-probs float32 [n, k]); raises ``KernelError`` on a device error
        (the device flag is cleared once)."""
        from ..utils import counters
        from ..utils.transfer import KernelError

        code, ids, lps = self.replay.materialize()
        if code:
            with self.replay.lock:
                if not self.replay.cleared:
                    self.replay.status.zero_()
                    self.replay.cleared = True
            raise KernelError(code, "drafter top-k")
        counters.d2h(self.words * 4)
        return ids[self.real], lps[self.real]


class StaticBatch:
    """Fixed-address inputs of one row bucket, filled by a single host->device copy.

    Layout of the int32 device buffer: dparams[4] (shared_len, n_shared_pages,
    mask_base, pad), tokens[M], positions[M], slots[M], row_full[M],
    row_len[M], tail_pages[M*T], then row masks as int64 [M*W].  The host side
    is a pair of pinned buffers used alternately (an event guards reuse).
    Rows beyond the real count are padding: token 0 at position 0 writing the
    engine's trash slot and attending to position 0 only.
    """

    def __init__(self, engine: LlamaEngine, rows: int, tail_stride: int, mask_words: int) -> None:
        self.engine = engine
        self.key = (rows, tail_stride, mask_words)
        self.M, self.T, self.W = rows, tail_stride, mask_words
        m, t, w = rows, tail_stride, mask_words
        self.offs = {}
        o = 4
        for name, size in (("tokens", m), ("positions", m), ("slots", m), ("row_full", m), ("row_len", m),
                           ("tail_pages", m * t)):
            self.offs[name] = (o, size)
            o += size
        o += o % 2
        self.offs["row_mask"] = (o, 2 * m * w)
        o += 2 * m * w
        # Free-form words that ride along in the same copy: a caller's small index arrays
        # (path log-prob gather indices, copy-on-write page copies) with no copy of their own.
        self.offs["aux"] = (o, max(128, 8 * m))
        o += self.offs["aux"][1]
        self.words = o
        dev = engine.device
        pin = dev.type == "cuda"
        self.dev = torch.zeros(o, dtype=torch.int32, device=dev)
        self.hosts = [torch.zeros(o, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        # One reusable event per host buffer: its last copy must finish before the buffer is refilled.
        self.events = [torch.cuda.Event() for _ in range(2)] if pin else [None, None]
        self._copy_pending = [False, False]
        self._upload = None
        self._event_handles = [0, 0]
        if pin and hasattr(engine.ops, "ext") and hasattr(engine.ops.ext, "upload_async"):
            for ev in self.events:
                ev.record()  # creates the CUDA event, so its handle exists
            self._event_handles = [int(getattr(ev, "cuda_event", 0) or 0) for ev in self.events]
            self._upload = engine.ops.ext.upload_async
        self.turn = 0
        self.lock = threading.Lock()
        v = self.dev
        self.dparams = v[0:4]
        self.tokens = v[self.offs["tokens"][0]: self.offs["tokens"][0] + m]
        self.positions = v[self.offs["positions"][0]: self.offs["positions"][0] + m]
        self.slots = v[self.offs["slots"][0]: self.offs["slots"][0] + m]
        self.row_full = v[self.offs["row_full"][0]: self.offs["row_full"][0] + m]
        self.row_len = v[self.offs["row_len"][0]: self.offs["row_len"][0] + m]
        a = self.offs["tail_pages"][0]
        self.tail_pages = v[a: a + m * t].view(m, t)
        a = self.offs["row_mask"][0]
        self.row_mask = v[a: a + 2 * m * w].view(torch.int64).view(m, w)
        a, size = self.offs["aux"]
        self.aux = v[a: a + size]
        self.pad_front = False
        # numpy views of each pinned host buffer, made once (load runs for every forward)
        self._host_views = []
        for hb in self.hosts:
            h = hb.numpy()
            views = {name: h[a: a + size] for name, (a, size) in self.offs.items() if name != "row_mask"}
            views["tail_pages"] = views["tail_pages"].reshape(m, t)
            a, size = self.offs["row_mask"]
            views["row_mask"] = h[a: a + size].view(np.int64).reshape(m, w)
            views["head"] = h[0:4]
            self._host_views.append(views)
        self._pad = {"tokens": 0, "positions": 0, "slots": engine.trash_slot, "row_full": 1, "row_len": 1}

    def real_slice(self, n: int) -> slice:
        return slice(self.M - n, self.M) if self.pad_front else slice(0, n)

    def load(self, *, tokens, positions, slots, shared_len, n_shared_pages, mask_base, row_full, row_len,
             tail_pages=None, row_mask=None, pad_front: bool = False, aux=None, cow_count: int = 0) -> int:
        from ..utils import counters

        n = len(tokens)
        if n > self.M:
            raise ValueError(f"{n} rows exceed the bucket of {self.M}")
        self.pad_front = bool(pad_front)
        with self.lock:
            i = self.turn
            self.turn ^= 1
            if self._copy_pending[i]:
                self.events[i].synchronize()
            hv = self._host_views[i]
            m = self.M
            r0 = m - n if pad_front else 0
            rs = slice(r0, r0 + n)
            hv["head"][:] = (int(shared_len), int(n_shared_pages), int(mask_base), int(cow_count))
            dev_tokens = isinstance(tokens, torch.Tensor) and tokens.device.type != "cpu"
            for name, vals in (("tokens", 0 if dev_tokens else tokens), ("positions", positions), ("slots", slots),
                               ("row_full", row_full), ("row_len", row_len)):
                seg = hv[name]
                if n < m:
                    seg[:] = self._pad[name]
                seg[rs] = vals
            tp = hv["tail_pages"]
            tp[:] = 0
            if tail_pages is not None:
                tp[rs, : np.asarray(tail_pages).shape[1]] = tail_pages
            mk = hv["row_mask"]
            mk[:] = -1
            if row_mask is not None:
                mk[rs, : np.asarray(row_mask).shape[1]] = row_mask
            if aux is not None:
                av = np.asarray(aux).reshape(-1)
                if av.size > hv["aux"].size:
                    raise ValueError(f"{av.size} auxiliary words exceed the bucket's {hv['aux'].size}")
                hv["aux"][: av.size] = av
            if self._upload is not None and self._event_handles[i]:
                # One native call: the copy and the event that guards this host buffer's reuse.
                self._upload(self.dev, self.hosts[i], self._event_handles[i])
                self._copy_pending[i] = True
            else:
                self.dev.copy_(self.hosts[i], non_blocking=True)
                if self.dev.is_cuda:
                    self.events[i].record(torch.cuda.current_stream(self.dev.device))
                    self._copy_pending[i] = True
            if dev_tokens:
                self.tokens[rs].copy_(tokens.reshape(-1).to(torch.int32))
        counters.h2d(self.words * 4)
        return n

    def desc(self, prefix_pages: torch.Tensor) -> AttnDesc:
        d = AttnDesc(
            prefix_pages=prefix_pages,
            n_shared_pages=int(self.hosts[self.turn ^ 1][1]),
            shared_len=max(1, int(self.hosts[self.turn ^ 1][0])),
            mask_base=int(self.hosts[self.turn ^ 1][2]),
            row_full=self.row_full,
            row_len=self.row_len,
            row_mask=self.row_mask,
            tail_pages=self.tail_pages,
        )
        d._dparams = self.dparams  # type: ignore[attr-defined]
        d._splits = self.engine.graph_attention_splits(self.M)  # type: ignore[attr-defined]
        return d


ROW_BUCKETS = (1, 2, 4, 8, 16, 32, 64)


def row_bucket(n: int) -> int:
    for b in ROW_BUCKETS:
        if n <= b:
            return b
    raise ValueError(f"{n} rows exceed the largest graph bucket ({ROW_BUCKETS[-1]})")
