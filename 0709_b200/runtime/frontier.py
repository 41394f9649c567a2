"""One frontier depth of the drafter: decode the active routes, rank their children, grow the tree.

A depth is four moves:

1. ``decode``: the model backend runs one graphed forward over every active
   route (their pending tokens), writing their KV and reserving one node id
   per route;
2. ``propose``: the fused top-k kernel turns each route's logits into ``k``
   candidate children (greedy, or keyed Gumbel-top-k sampling), and a single
   device-to-host copy brings back their ids and log-probs together with the
   device's kernel error flag -- the host's only wait of the depth.  For greedy
   drafting on a CUDA-graph backend the top-k and that copy are part of the
   forward's graph (``decode_frontier_one_token(..., topk=k)``), so nothing is
   launched between the forward and the host's read;
3. ``rank``: the selection policy picks the next frontier on the host (a
   stage-1 tree keeps the best ``k`` overall, a stage-2 forest the best ``k``
   per stage-1 root; at most k^3 candidates);
4. ``grow``: the store turns the decoded routes' pending tokens into nodes
   and spawns one child route per pick (the drafter's page pool forks their
   physical views).

A kernel error raises before step 4, so no route is grown or spawned from a
depth whose device work failed.

Behaviour matches the reference's frontier step
(src/atlas_0709/flashinfer_paged/frontier.py:29-403); there the ranking runs on
the device and the selection is materialized through one packed transfer.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Protocol, Sequence

import numpy as np
import torch

from ..types import DecodePhase, FrontierDecodeOutput, FrontierSelectionStats, FrontierStepOutput, PendingCandidate
from ..types import RouteState
from ..utils.transfer import read_back
from .sampling import DrafterSamplingContext, batch_parent_token_candidates
from .selection import best_per_root, global_topk_candidates
from .store import KVTreeStore


class FrontierModelBackend(Protocol):
    def decode_frontier_one_token(
        self, active_routes: Sequence[RouteState], attention_backend: Any = None
    ) -> FrontierDecodeOutput: ...


@dataclass(frozen=True)
class BestKOverall:
    """Stage-1 tree: the next frontier is the best ``k`` children of the whole frontier."""

    phase: DecodePhase = DecodePhase.STAGE1

    def select(self, candidates, *, k, active_routes):
        return global_topk_candidates(candidates, k)


@dataclass(frozen=True)
class BestKPerRoot:
    """Stage-2 forest: the best ``k`` children under every stage-1 root (the forest stays k^2 wide)."""

    phase: DecodePhase = DecodePhase.STAGE2

    def select(self, candidates, *, k, active_routes):
        return best_per_root(candidates, k, [r.stage1_root_id for r in active_routes])


def propose_children(
    parents: Sequence[RouteState | None],
    logits: torch.Tensor,
    *,
    k: int,
    sampling: DrafterSamplingContext | None = None,
    history: Callable[[RouteState | None], Sequence[int]] | None = None,
    status: torch.Tensor | None = None,
    root_of: Callable[[RouteState | None], int] | None = None,
    readout: Any = None,
) -> tuple[list[PendingCandidate], int]:
    """``k`` candidate children for each parent (one row of ``logits`` each).

    ``history(parent)`` is the parent's token history relative to the committed
    prefix; only keyed sampling reads it.  A candidate's score is the parent's
    cumulative draft log-prob (0 for the committed prefix, ``parent`` None)
    plus its own log-prob, and its stage-1 root is ``root_of(parent)``
    (default: the parent's root).  Returns the candidates and the number of
    32-bit words copied back.
    """
    rows = logits.reshape(-1, logits.shape[-1])
    if len(parents) != int(rows.shape[0]):
        raise ValueError(f"{len(parents)} parents for {int(rows.shape[0])} rows of logits")
    keyed = sampling is not None and sampling.config.do_sample
    if keyed and history is None:
        raise ValueError("keyed sampling needs each parent's token history")
    if readout is not None and not keyed and readout.buf.k >= k:
        # Selected inside the forward's graph (greedy): only the host read remains.
        ids_h, lp_h = readout.get()
        ids_h, lp_h = ids_h[:, :k], lp_h[:, :k]
        words = int(readout.words)
    else:
        paths = [tuple(history(p)) for p in parents] if keyed else [()] * len(parents)
        lp, ids = batch_parent_token_candidates(rows, k=k, sampling=sampling, relative_parent_paths=paths)
        ids_h, lp_h = read_back([ids, lp.float()], status, where="drafter top-k")
        words = int(ids.numel() + lp.numel()) + (1 if status is not None else 0)
    id_rows, lp_rows = ids_h.tolist(), lp_h.astype(np.float64).tolist()
    out: list[PendingCandidate] = []
    for parent, row_ids, row_lps in zip(parents, id_rows, lp_rows):
        if parent is None:
            pid, root, base = 0, 0, 0.0
        else:
            pid, root, base = parent.route_id, parent.stage1_root_id, parent.cumulative_logprob
        if root_of is not None:
            root = root_of(parent)
        for rank, (tok, tlp) in enumerate(zip(row_ids, row_lps)):
            out.append(PendingCandidate(pid, root, tok, base + tlp, rank, base))
    return out, words


def backend_status(backend) -> torch.Tensor | None:
    """The backend's device error flag, if it has one."""
    return backend.status_flag() if backend is not None and hasattr(backend, "status_flag") else None


def _decoded_node_ids(out: FrontierDecodeOutput, count: int) -> list[int]:
    ids = out.new_node_ids_cpu if out.new_node_ids_cpu is not None else out.new_node_ids
    if isinstance(ids, torch.Tensor):
        ids = ids.tolist()
    ids = [int(x) for x in ids]
    if len(ids) != count:
        raise ValueError(f"the decode step reserved {len(ids)} node ids for {count} routes")
    return ids


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
    """Decode one token for every active route and grow the next frontier (see module doc)."""
    if not active_routes:
        raise ValueError("a frontier step needs at least one active route")
    routes = list(active_routes)
    keyed = sampling is not None and sampling.config.do_sample
    if not keyed and getattr(model_backend, "supports_graph_topk", False):
        out = model_backend.decode_frontier_one_token(routes, attention_backend=attention_backend, topk=k)
    else:
        out = model_backend.decode_frontier_one_token(routes, attention_backend=attention_backend)
    node_ids = _decoded_node_ids(out, len(routes))
    cands, words = propose_children(routes, out.next_token_logits, k=k, sampling=sampling,
                                    history=route_store.pending_token_path, status=backend_status(model_backend),
                                    readout=getattr(out, "candidates", None))
    picks = selection_policy.select(cands, k=k, active_routes=routes)
    grown = route_store.grow(routes, node_ids, selection_policy.phase)
    nxt = route_store.spawn(picks, grown)
    on_device = out.next_token_logits.device.type != "cpu"
    stats = FrontierSelectionStats(
        candidate_count=len(cands),
        selected_count=len(picks),
        host_materialization_batches=1,
        host_materialization_elements=words,
        host_transfer_batches=int(on_device),
        host_transfer_elements=words if on_device else 0,
        selection_device="cpu",
        new_node_ids_source="decode_output_cpu" if out.new_node_ids_cpu is not None else "decode_output",
    )
    return FrontierStepOutput(decoded_routes=grown, next_routes=nxt, candidates=cands, selected_candidates=picks,
                              decode_output=out, selection_stats=stats)
