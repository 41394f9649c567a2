"""One frontier depth: decode, build candidates, select on device, materialize once.

Parity: reference src/atlas_0709/flashinfer_paged/frontier.py:29-403.  The
flow is the same (model call -> per-parent top-k -> deterministic selection ->
exactly one packed device-to-host transfer -> route bookkeeping); node ids are
reserved on the host by the model backend, so they never ride the transfer.
"""

from __future__ import annotations

import os
import struct
from collections import Counter
from dataclasses import dataclass
from typing import Any, Protocol, Sequence

import torch

from ..types import (
    DecodePhase,
    FrontierDecodeOutput,
    FrontierSelectionStats,
    FrontierStepOutput,
    PendingCandidate,
    PendingCandidateBatch,
    RouteState,
)
from .sampling import DrafterSamplingContext, batch_parent_token_candidates
from .selection import (
    global_topk_candidate_indices,
    global_topk_candidates,
    group_candidates_by_stage1_root,
    per_root_topk_candidate_indices,
)
from .store import KVTreeStore
from ..utils import counters


class FrontierModelBackend(Protocol):
    def decode_frontier_one_token(
        self, active_routes: Sequence[RouteState], attention_backend: Any = None
    ) -> FrontierDecodeOutput: ...


@dataclass(frozen=True)
class GlobalTopKSelection:
    """Stage-1 tree: keep the best ``k`` children over the whole frontier."""

    phase: DecodePhase = DecodePhase.STAGE1

    def select(self, candidates, *, k, active_routes):
        return global_topk_candidates(candidates, num_selected=k)

    def select_indices(self, candidates: PendingCandidateBatch, *, k: int, active_routes) -> torch.Tensor:
        return global_topk_candidate_indices(candidates, num_selected=k)


@dataclass(frozen=True)
class PerStage1RootTopKSelection:
    """Stage-2 forest: keep the best ``k`` children per stage-1 root (frontier stays k^2)."""

    phase: DecodePhase = DecodePhase.STAGE2

    def select(self, candidates, *, k, active_routes):
        roots = sorted({r.stage1_root_id for r in active_routes})
        grouped = group_candidates_by_stage1_root(candidates)
        out: list[PendingCandidate] = []
        for root in roots:
            group = grouped.get(root, [])
            if not group:
                raise ValueError(f"stage1 root {root} produced no candidates")
            out.extend(global_topk_candidates(group, num_selected=k))
        return out

    def select_indices(self, candidates: PendingCandidateBatch, *, k: int, active_routes) -> torch.Tensor:
        counts = Counter(int(r.stage1_root_id) for r in active_routes)
        root_counts = [(root, n * candidates.candidates_per_parent) for root, n in counts.items()]
        empty = [root for root, c in root_counts if c == 0]
        if empty:
            raise ValueError(f"stage1 root {min(empty)} produced no candidates")
        return per_root_topk_candidate_indices(candidates, num_selected=k, root_candidate_counts=root_counts)


def build_pending_candidate_batch(
    decoded_routes: Sequence[RouteState],
    next_token_logits: torch.Tensor,
    *,
    k: int,
    sampling: DrafterSamplingContext | None = None,
    relative_parent_paths: Sequence[Sequence[int]] | None = None,
) -> PendingCandidateBatch:
    if len(decoded_routes) != int(next_token_logits.shape[0]):
        raise ValueError("decoded_routes and next_token_logits must have the same batch size")
    if k <= 0:
        raise ValueError("k must be positive")
    if relative_parent_paths is None:
        relative_parent_paths = [() for _ in decoded_routes]
    lp, ids = batch_parent_token_candidates(
        next_token_logits, k=k, sampling=sampling, relative_parent_paths=relative_parent_paths
    )
    kk = int(ids.shape[-1])
    dev = next_token_logits.device
    b = len(decoded_routes)
    # One small host->device copy carries all per-parent scalars.
    meta = torch.tensor(
        [[int(r.route_id), int(r.stage1_root_id)] for r in decoded_routes], dtype=torch.long
    ).to(dev, non_blocking=True)
    parent_lp = torch.tensor([float(r.cumulative_logprob) for r in decoded_routes], dtype=torch.float64).to(
        dev, non_blocking=True
    )
    parent_lp = parent_lp.repeat_interleave(kk)
    return PendingCandidateBatch(
        parent_route_ids=meta[:, 0].repeat_interleave(kk),
        stage1_root_ids=meta[:, 1].repeat_interleave(kk),
        parent_row_indices=torch.arange(b, device=dev, dtype=torch.long).repeat_interleave(kk),
        pending_token_ids=ids.reshape(-1).to(torch.long),
        cumulative_logprobs=parent_lp + lp.reshape(-1).to(torch.float64),
        parent_logprobs=parent_lp,
        ranks_in_parent=torch.arange(kk, device=dev, dtype=torch.long).repeat(b),
        candidates_per_parent=kk,
    )


def _f64(bits: int) -> float:
    return struct.unpack("=d", struct.pack("=q", int(bits)))[0]


def materialize_pending_candidate_batch(
    candidates: PendingCandidateBatch,
    selected_indices: torch.Tensor,
    *,
    new_node_ids_cpu: Sequence[int] | None = None,
    new_node_ids_to_transfer: torch.Tensor | None = None,
    new_node_ids_source: str = "not_applicable",
) -> tuple[list[PendingCandidate], list[PendingCandidate], list[int], FrontierSelectionStats]:
    """Materialize candidates and the selection through exactly one packed host transfer.

    Layout of each int64 record: kind, parent, root, token, rank, score bits,
    parent-score bits, selection order (-1 when not selected).
    """
    n = candidates.candidate_count
    nsel = int(selected_indices.numel())
    dev = candidates.pending_token_ids.device
    order = torch.full((n,), -1, device=dev, dtype=torch.long)
    if nsel:
        order[selected_indices.to(dev, torch.long)] = torch.arange(nsel, device=dev, dtype=torch.long)
    rec = torch.stack(
        (
            torch.zeros(n, device=dev, dtype=torch.long),
            candidates.parent_route_ids.long(),
            candidates.stage1_root_ids.long(),
            candidates.pending_token_ids.long(),
            candidates.ranks_in_parent.long(),
            candidates.cumulative_logprobs.double().contiguous().view(torch.int64),
            candidates.parent_logprobs.double().contiguous().view(torch.int64),
            order,
        ),
        dim=1,
    )
    parts = [rec]
    moved_nodes = 0
    if new_node_ids_to_transfer is not None:
        ids = new_node_ids_to_transfer.to(dev, torch.long).reshape(-1)
        moved_nodes = int(ids.numel())
        node_rec = torch.zeros((moved_nodes, rec.shape[1]), device=dev, dtype=torch.long)
        node_rec[:, 0] = 1
        node_rec[:, 1] = ids
        parts.append(node_rec)
    packed = torch.cat(parts) if len(parts) > 1 else rec
    if packed.device.type != "cpu":
        counters.d2h(packed.numel() * 8)
    rows = packed.detach().cpu().tolist()
    cands: list[PendingCandidate] = []
    by_order: list[PendingCandidate | None] = [None] * nsel
    for row in rows[:n]:
        c = PendingCandidate(
            parent_route_id=int(row[1]),
            stage1_root_id=int(row[2]),
            pending_token_id=int(row[3]),
            cumulative_logprob=_f64(row[5]),
            rank_in_parent=int(row[4]),
            parent_logprob=_f64(row[6]),
        )
        cands.append(c)
        if row[7] >= 0:
            by_order[int(row[7])] = c
    if any(c is None for c in by_order):
        raise RuntimeError("selected candidate order was not fully materialized")
    node_ids = (
        [int(x) for x in new_node_ids_cpu] if new_node_ids_cpu is not None else [int(r[1]) for r in rows[n:]]
    )
    if new_node_ids_cpu is None and len(node_ids) != moved_nodes:
        raise RuntimeError("new node id transfer produced the wrong number of ids")
    is_transfer = packed.device.type != "cpu"
    stats = FrontierSelectionStats(
        candidate_count=n,
        selected_count=nsel,
        host_materialization_batches=1,
        host_materialization_elements=int(packed.numel()),
        host_transfer_batches=int(is_transfer),
        host_transfer_elements=int(packed.numel()) if is_transfer else 0,
        selection_device=str(dev),
        new_node_ids_source=new_node_ids_source,
    )
    return cands, [c for c in by_order if c is not None], node_ids, stats


def collect_pending_candidates(decoded_routes, next_token_logits, *, k: int) -> list[PendingCandidate]:
    batch = build_pending_candidate_batch(decoded_routes, next_token_logits, k=k)
    empty = torch.empty((0,), device=next_token_logits.device, dtype=torch.long)
    cands, _, _, _ = materialize_pending_candidate_batch(batch, empty)
    return cands


def advance_frontier_one_token(
    active_routes: Sequence[RouteState],
    *,
    k: int,
    route_store: KVTreeStore,
    model_backend: FrontierModelBackend,
    selection_policy,
    attention_backend: Any = None,
    sampling: DrafterSamplingContext | None = None,
) -> FrontierStepOutput:
    if not active_routes:
        raise ValueError("active_routes cannot be empty")
    out = model_backend.decode_frontier_one_token(active_routes, attention_backend=attention_backend)
    if HOST_SELECTION and out.new_node_ids_cpu is not None and hasattr(selection_policy, "select"):
        return _advance_host_selection(active_routes, out, k=k, route_store=route_store,
                                       selection_policy=selection_policy, sampling=sampling)
    batch = build_pending_candidate_batch(
        active_routes,
        out.next_token_logits,
        k=k,
        sampling=sampling,
        relative_parent_paths=[route_store.pending_token_path(r) for r in active_routes],
    )
    sel = selection_policy.select_indices(batch, k=k, active_routes=active_routes)
    cpu_ids, transfer_ids, source = _resolve_new_node_ids(out, expected=len(active_routes))
    cands, chosen, node_ids, stats = materialize_pending_candidate_batch(
        batch, sel, new_node_ids_cpu=cpu_ids, new_node_ids_to_transfer=transfer_ids, new_node_ids_source=source
    )
    decoded = route_store.mark_routes_materialized(list(active_routes), node_ids, phase=selection_policy.phase)
    nxt = route_store.materialize_route_descriptors(chosen, parent_routes=decoded)
    route_store.release_routes_without_descendants(decoded, nxt)
    return FrontierStepOutput(
        decoded_routes=decoded,
        next_routes=nxt,
        candidates=cands,
        selected_candidates=chosen,
        decode_output=out,
        selection_stats=stats,
    )


# Host selection: after the top-k kernel, one wait and two small copies bring the
# k candidates of every parent (ids, log-probs) to the host, where ranking (<= k^3 candidates) and route
# bookkeeping run in Python -- the same order as the device path
# (score desc, parent, rank, token), without its dozens of small GPU launches.
HOST_SELECTION = os.environ.get("ATLAS_DEVICE_SELECTION", "0") != "1"


def _advance_host_selection(active_routes, out, *, k, route_store, selection_policy, sampling) -> FrontierStepOutput:
    # Semantic parent paths key the sampling noise; greedy drafting does not read them.
    if sampling is not None and sampling.config.do_sample:
        rel = [route_store.pending_token_path(r) for r in active_routes]
    else:
        rel = [()] * len(active_routes)
    lp, ids = batch_parent_token_candidates(out.next_token_logits, k=k, sampling=sampling,
                                            relative_parent_paths=rel)
    # Two plain transfers (the first waits for the top-k kernel), no packing kernels.
    is_transfer = ids.device.type != "cpu"
    if is_transfer:
        counters.d2h(ids.numel() * ids.element_size() + lp.numel() * lp.element_size())
    id_rows = ids.cpu().tolist()
    lp_rows = lp.cpu().tolist()
    n_elems = 2 * ids.numel()
    cands: list[PendingCandidate] = []
    for r, row_ids, row_lp in zip(active_routes, id_rows, lp_rows):
        base = float(r.cumulative_logprob)
        for rank, (tok, tlp) in enumerate(zip(row_ids, row_lp)):
            cands.append(PendingCandidate(parent_route_id=int(r.route_id), stage1_root_id=int(r.stage1_root_id),
                                          pending_token_id=int(tok), cumulative_logprob=base + float(tlp),
                                          rank_in_parent=rank, parent_logprob=base))
    chosen = selection_policy.select(cands, k=k, active_routes=active_routes)
    node_ids = [int(x) for x in out.new_node_ids_cpu]
    if len(node_ids) != len(active_routes):
        raise ValueError("new_node_ids_cpu must have one id per active route")
    stats = FrontierSelectionStats(
        candidate_count=len(cands), selected_count=len(chosen), host_materialization_batches=1,
        host_materialization_elements=n_elems, host_transfer_batches=int(is_transfer),
        host_transfer_elements=n_elems if is_transfer else 0, selection_device="cpu",
        new_node_ids_source="decode_output_cpu")
    decoded = route_store.mark_routes_materialized(list(active_routes), node_ids, phase=selection_policy.phase)
    nxt = route_store.materialize_route_descriptors(chosen, parent_routes=decoded)
    route_store.release_routes_without_descendants(decoded, nxt)
    return FrontierStepOutput(decoded_routes=decoded, next_routes=nxt, candidates=cands, selected_candidates=chosen,
                              decode_output=out, selection_stats=stats)


def _resolve_new_node_ids(out: FrontierDecodeOutput, *, expected: int):
    if out.new_node_ids_cpu is not None:
        ids = [int(x) for x in out.new_node_ids_cpu]
        if len(ids) != expected:
            raise ValueError("new_node_ids_cpu must have one id per active route")
        return ids, None, "decode_output_cpu"
    if not isinstance(out.new_node_ids, torch.Tensor):
        ids = [int(x) for x in out.new_node_ids]
        if len(ids) != expected:
            raise ValueError("new_node_ids must have one id per active route")
        return ids, None, "decode_output_sequence"
    if int(out.new_node_ids.numel()) != expected:
        raise ValueError("new_node_ids must have one id per active route")
    return None, out.new_node_ids, "packed_transfer"
