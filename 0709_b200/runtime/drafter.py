"""Drafter runtime: frontier decode over the native paged route pool.

The drafter keeps one committed prefix (page list) and a view per live route
(shared prefix pages + a short list of private tail pages).  A frontier step:
1. forks pool views for routes created since the last step,
2. plans one appended token per route (in-place lease or tail-page COW),
3. runs one batched forward (COW page copies first, then the model, whose
   attention reads the shared prefix once for every row),
4. returns logits and host-reserved node ids (no device round trip for ids).

Commit promotes the selected stage-1 route's pages into the prefix without
copying KV and rebases the retained stage-2 routes; fallback drops every route
and extends the prefix with one causal EXTEND forward.

Parity: reference src/atlas_0709/flashinfer_paged/sglang_runtime.py:1120-1346
(SGLangFlashInferFrontierModelBackend), :800-959 (prepare_frontier), :1171-1251
(known-token EXTEND), :1256-1297 (commit_stage1_and_promote).
"""

from __future__ import annotations

import time
from typing import Any, Sequence

import numpy as np
import torch

from ..ops import _native
from ..utils.transfer import ids_to_device
from ..types import DraftPrefixState, FrontierDecodeOutput, PrefixKVView, RouteState
from .engine import LlamaEngine, row_bucket
from .store import KVTreeStore


# Largest k the in-graph top-k kernel takes.
GRAPH_TOPK_MAX = 8


class PrefixPageMirror:
    """Device copy of a pool's prefix page list, updated incrementally."""

    def __init__(self, capacity: int, device: torch.device) -> None:
        # Fixed capacity (the pool's page count): captured graphs keep this address.
        self.dev = torch.zeros(int(capacity), dtype=torch.int32, device=device)
        self.host: list[int] = []
        self.h2d_copies = 0
        # Called with (start, values) after each device update (tensor-parallel
        # engines forward the update to the worker ranks' copies).
        self.on_update = None

    def sync(self, pages: torch.Tensor) -> None:
        new = pages.tolist()
        if len(new) > self.dev.numel():
            raise RuntimeError(f"prefix page table of {len(new)} pages exceeds the mirror capacity {self.dev.numel()}")
        n = min(len(new), len(self.host))
        if new[:n] == self.host[:n]:  # the usual case: pages only appended or dropped at the end
            start = n
        else:
            start = 0
            while new[start] == self.host[start]:
                start += 1
        if start < len(new):
            self.dev[start: len(new)].copy_(pages[start:].to(self.dev.device, non_blocking=True))
            self.h2d_copies += 1
            if self.on_update is not None:
                self.on_update(start, new[start:])
        self.host = new

    def view(self) -> torch.Tensor:
        return self.dev[: max(1, len(self.host))]


class DrafterRuntime:
    def __init__(
        self,
        engine: LlamaEngine,
        *,
        page_pool: Any | None = None,
        prefill_chunk_size: int = 8192,
        max_tail_pages: int = 8,
    ) -> None:
        self.engine = engine
        self.host = _native.host()
        # The engine's last page is the trash page for padded graph rows.
        self.page_pool = page_pool if page_pool is not None else self.host.PagePool(engine.num_pages - 1, engine.page_size)
        self.route_pool = self.host.RoutePool(self.page_pool)
        self.page_size = engine.page_size
        self.prefill_chunk_size = int(prefill_chunk_size)
        self.max_tail_pages = int(max_tail_pages)
        self.device = engine.device
        self.mirror = PrefixPageMirror(engine.num_pages, self.device)
        self.route_store: KVTreeStore | None = None
        self.prefix_token_ids: tuple[int, ...] = ()
        self.prefix_next_token_logits: torch.Tensor | None = None
        self._prefix_candidates = None  # graph-selected children of the prefix (after an extend)
        self._graph_k: int | None = None  # the session's k (set by warm_graphs): extends select it in-graph
        self.counters = {
            "decode_steps": 0,
            "decode_rows": 0,
            "attention_metadata_page_indices": 0,
            "hot_path_host_transfer_batches": 0,
            "hot_path_host_transfer_elements": 0,
            "extend_calls": 0,
            "extend_tokens": 0,
        }
        # Decode forwards copy tail pages on write: let the engine's graphs do it from the plan that
        # rides in the static batch (one launch fewer between the host's inputs and the forward).
        if hasattr(engine, "cow_in_graph"):
            engine.cow_in_graph = True

    # ---------------------------------------------------------------- store
    def bind_store(self, store: KVTreeStore) -> None:
        self.route_store = store
        store.on_spawn(self._fork_children)

    def _fork_children(self, children: Sequence[RouteState]) -> None:
        """New child routes share their parent's pages (the tail page is copied on their first append)."""
        rp = self.route_pool
        for child in children:
            if child.parent_route_id is not None and not rp.has_route(child.route_id):
                rp.fork(int(child.route_id), int(child.parent_route_id))

    def status_flag(self) -> torch.Tensor | None:
        """The drafter device's kernel error flag (None for op tables that raise directly)."""
        return getattr(self.engine.ops, "err", None)

    # -------------------------------------------------------------- prefix
    def _sync_prefix(self) -> None:
        self.mirror.sync(self.route_pool.prefix_pages())

    def reset(self) -> None:
        self.route_pool.clear()
        self.prefix_token_ids = ()
        self.prefix_next_token_logits = None
        self._prefix_candidates = None
        self.mirror.host = []

    @torch.inference_mode()
    def prefill(self, prompt_token_ids: Sequence[int]) -> DraftPrefixState:
        toks = tuple(int(t) for t in prompt_token_ids)
        if not toks:
            raise ValueError("drafter prefill requires a non-empty prompt")
        self.reset()
        slots, copies = self.route_pool.append_prefix(len(toks))
        self.engine.copy_pages(copies)
        self._sync_prefix()
        logits = self.engine.prefill_sequence(
            ids_to_device(toks, self.device),
            start_pos=0,
            slots=slots.to(self.device),
            pages=self.mirror.view(),
            chunk_size=self.prefill_chunk_size,
        )
        self.prefix_token_ids = toks
        self.prefix_next_token_logits = logits.unsqueeze(0)
        self._prefix_candidates = None
        if self.route_store is not None:
            self.route_store.committed_token_ids = list(toks)
        return self.prefix_state()

    def prefix_state(self) -> DraftPrefixState:
        assert self.prefix_next_token_logits is not None
        return DraftPrefixState(
            token_tuple=tuple(self.prefix_token_ids),
            prefix_kv_view=PrefixKVView(committed_length=len(self.prefix_token_ids)),
            next_token_logits=self.prefix_next_token_logits,
            candidates=self._prefix_candidates,
            committed_length=len(self.prefix_token_ids),
        )

    # -------------------------------------------------------------- decode
    def _ensure_views(self, routes: Sequence[RouteState]) -> None:
        rp = self.route_pool
        for r in routes:
            rid = int(r.route_id)
            if rp.has_route(rid):
                continue
            parent = r.parent_route_id
            if parent is not None and rp.has_route(int(parent)):
                rp.fork(rid, int(parent))
            else:
                rp.fork_from_prefix(rid)
            if rp.route_len(rid) != r.kv_view.length:
                raise RuntimeError(
                    f"route {rid} physical length {rp.route_len(rid)} != logical length {r.kv_view.length}"
                )

    @property
    def supports_graph_topk(self) -> bool:
        """Whether ``decode_frontier_one_token(..., topk=k)`` selects candidates inside the forward's graph."""
        f = getattr(self.engine, "graph_topk_available", None)
        return bool(f is not None and f())

    @torch.inference_mode()
    def decode_frontier_one_token(
        self, active_routes: Sequence[RouteState], attention_backend: Any = None, topk: int | None = None
    ) -> FrontierDecodeOutput:
        """One token for every route.  With ``topk`` (greedy drafting, CUDA graphs) the forward's
        graph also selects each row's top-``topk`` children and copies them to the host, so no
        launch follows the forward before the host reads them (``FrontierDecodeOutput.candidates``)."""
        if self.route_store is None:
            raise RuntimeError("bind_store() must be called before decoding")
        t0 = time.perf_counter()
        self._ensure_views(active_routes)
        rids = [int(r.route_id) for r in active_routes]
        slots, copies = self.route_pool.prepare_append(rids)
        cow = copies.numpy() if copies.numel() else None  # copied inside the forward's input copy
        tails, lens = self.route_pool.row_tables(rids, self.max_tail_pages)
        lens_np = lens.numpy()
        plen = int(self.route_pool.prefix_len)
        fields = dict(
            tail_stride=self.max_tail_pages,
            mask_words=1,
            prefix_pages=self.mirror.dev,
            tokens=[int(r.pending_token_id) for r in active_routes],
            positions=lens_np - 1,
            slots=slots.numpy(),
            shared_len=plen,
            n_shared_pages=int(self.route_pool.prefix_full_pages),
            mask_base=plen,
            row_full=lens_np,
            row_len=lens_np,
            tail_pages=tails.numpy(),
            cow=cow,
        )
        readout = None
        if topk is not None and topk <= GRAPH_TOPK_MAX and self.supports_graph_topk:
            logits, readout = self.engine.run_rows_topk(row_bucket(len(rids)), int(topk), **fields)
        else:
            logits = self.engine.run_rows(row_bucket(len(rids)), **fields)
        node_ids = tuple(self.route_store.reserve_node_ids(len(active_routes)))
        c = self.counters
        c["decode_steps"] += 1
        c["decode_rows"] += len(rids)
        c["attention_metadata_page_indices"] += int(self.route_pool.prefix_full_pages) + int(tails.numel())
        return FrontierDecodeOutput(
            route_ids=torch.tensor(rids, dtype=torch.long),
            next_token_logits=logits,
            new_node_ids=node_ids,
            new_node_ids_cpu=node_ids,
            candidates=readout,
            model_ms=(time.perf_counter() - t0) * 1000.0,
            metadata={
                "backend": "b200_native_paged_decode",
                "paged_kv": True,
                "route_tail_page_cow": True,
                "shared_prefix_attention": True,
                "cow_pages_copied_step": int(copies.shape[0]),
                "cow_pages_copied_total": int(self.route_pool.cow_pages_copied),
                "cow_tokens_copied_total": int(self.route_pool.cow_tokens_copied),
                "attention_backend": str(attention_backend),
            },
        )

    # -------------------------------------------------------------- commit
    @torch.inference_mode()
    def commit_stage1_and_promote(
        self, *, committed_route: RouteState, retained_routes: Sequence[RouteState]
    ) -> tuple[list[RouteState], dict[str, int]]:
        store = self.route_store
        assert store is not None
        n_nodes = len(committed_route.kv_view.node_ids)
        if not n_nodes:
            raise ValueError(f"stage-1 route {committed_route.route_id} has no decoded tokens to commit")
        self._ensure_views([committed_route, *retained_routes])
        keep = [int(r.route_id) for r in retained_routes]
        # Physical: keep the survivors' views, then turn the committed route's view into the prefix.
        released_routes, freed = self.route_pool.retain([*keep, int(committed_route.route_id)])
        freed += self.route_pool.commit(int(committed_route.route_id))
        # Logical: the same commit on the node arena, survivors rebased onto the new prefix.
        tokens, promoted = store.advance_prefix(committed_route, retained_routes)
        self.prefix_token_ids = (*self.prefix_token_ids, *tokens)
        self._prefix_candidates = None
        if self.route_pool.prefix_len != len(self.prefix_token_ids):
            raise RuntimeError(f"drafter pages hold {self.route_pool.prefix_len} committed tokens, the route "
                               f"store {len(self.prefix_token_ids)}")
        self._sync_prefix()
        return promoted, {
            "committed_kv_tokens": n_nodes,
            "retained_routes": len(promoted),
            "released_route_rows": int(released_routes) + 1,
            "released_kv_pages": int(freed),
        }

    def drop_speculative(self) -> dict[str, int]:
        released, freed = self.route_pool.retain([])
        if self.route_store is not None:
            self.route_store.reset_speculative()
        return {"released_route_rows": int(released), "released_kv_pages": int(freed)}

    @torch.inference_mode()
    def append_known_tokens_as_prefix(self, token_ids: Sequence[int]) -> torch.Tensor:
        """Extend the committed prefix by known tokens with one EXTEND forward.

        Up to 64 tokens run as one graphed masked forward (the tokens see the
        old prefix fully and each other causally via row masks); longer runs use
        the chunked causal prefill.
        """
        suffix = tuple(int(t) for t in token_ids)
        if not suffix:
            raise ValueError("nothing to append to the drafter prefix")
        if self.route_pool.num_routes:
            raise RuntimeError("drop speculative routes before extending the prefix")
        start = int(self.route_pool.prefix_len)
        n = len(suffix)
        slots, copies = self.route_pool.append_prefix(n)
        self.engine.copy_pages(copies)
        self._sync_prefix()
        self._prefix_candidates = None
        if n <= 64:
            masks = np.array([(1 << (r + 1)) - 1 if r < 63 else -1 for r in range(n)], dtype=np.int64)[:, None]
            fields = dict(
                tail_stride=1,
                mask_words=1,
                prefix_pages=self.mirror.dev,
                tokens=list(suffix),
                positions=np.arange(start, start + n),
                slots=slots.numpy(),
                shared_len=start,
                n_shared_pages=len(self.mirror.host),
                mask_base=start,
                row_full=np.full(n, start),
                row_len=np.full(n, start + n),
                row_mask=masks,
                pad_front=True,
            )
            k = self._graph_k
            if k is not None and k <= GRAPH_TOPK_MAX and self.supports_graph_topk:
                rows, readout = self.engine.run_rows_topk(row_bucket(n), k, **fields)
                logits = rows[-1]
                self._prefix_candidates = readout.last_row()  # the padded bucket ends with the real rows
            else:
                logits = self.engine.run_rows(row_bucket(n), **fields)[-1]
        else:
            logits = self.engine.prefill_sequence(
                ids_to_device(suffix, self.device),
                start_pos=start,
                slots=slots.to(self.device),
                pages=self.mirror.view(),
                chunk_size=self.prefill_chunk_size,
            )
        self.prefix_token_ids = (*self.prefix_token_ids, *suffix)
        self.prefix_next_token_logits = logits.unsqueeze(0)
        self.counters["extend_calls"] += 1
        self.counters["extend_tokens"] += n
        return logits

    def warm_graphs(self, k: int, extend_tokens: int = 4) -> None:
        """Capture the decode buckets (k and k^2 routes, with and without the in-graph top-k)
        and the EXTEND bucket up front."""
        topks = [None, k] if self.supports_graph_topk and k <= GRAPH_TOPK_MAX else [None]
        self._graph_k = k if len(topks) > 1 else None
        for b in sorted({row_bucket(1), row_bucket(k), row_bucket(k * k)}):
            for t in topks:
                self.engine.warm_graph(b, tail_stride=self.max_tail_pages, mask_words=1, prefix_pages=self.mirror.dev,
                                       topk=t)
        for t in topks:
            self.engine.warm_graph(row_bucket(extend_tokens), tail_stride=1, mask_words=1, prefix_pages=self.mirror.dev,
                                   topk=t)

    # ---------------------------------------------------------- validation
    def validate_route_physical_state(self, route: RouteState) -> None:
        rid = int(route.route_id)
        if not self.route_pool.has_route(rid):
            raise RuntimeError(f"Drafter route {rid} has no physical view")
        if self.route_pool.route_len(rid) != route.kv_view.length:
            raise RuntimeError(
                f"Drafter route {rid} physical length does not match logical KV: "
                f"physical={self.route_pool.route_len(rid)}, logical={route.kv_view.length}"
            )
        self.route_pool.validate()

    def page_reference_counts(self) -> dict[int, int]:
        return dict(sorted(self.route_pool.recomputed_refcounts().items()))

    def hot_path_counters(self) -> dict[str, int]:
        return {
            **self.counters,
            "cow_pages_copied": int(self.route_pool.cow_pages_copied),
            "cow_tokens_copied": int(self.route_pool.cow_tokens_copied),
            "in_place_appends": int(self.route_pool.in_place_appends),
            "prefix_page_h2d_copies": int(self.mirror.h2d_copies),
            "pool_used_pages": int(self.page_pool.used_pages),
        }
