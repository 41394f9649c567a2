"""Edge-observed timeline: spans, per-round overlap, exposed wait, JSON and SVG output.

The coordinator records host ``perf_counter`` spans (verify black box, forest
steps, post-prune tree steps, handoff) and summarizes how much of the Target's
verify time the forest hid.  The SVG is plain text written here (no graphics
API).  Parity: reference src/atlas_0709/edge_timeline.py:11-475 (span model,
``cloud_edge_overlap_s``, ``exposed_cloud_wait_s``, summary fields).
"""

from __future__ import annotations

import html
import json
import statistics
from dataclasses import dataclass, field
from pathlib import Path


@dataclass(frozen=True)
class EdgeSpan:
    name: str
    start_s: float
    end_s: float

    @property
    def elapsed_s(self) -> float:
        return max(0.0, float(self.end_s) - float(self.start_s))

    def to_dict(self) -> dict[str, object]:
        return {"name": self.name, "start_s": float(self.start_s), "end_s": float(self.end_s), "elapsed_s": self.elapsed_s}


@dataclass
class EdgeRoundTimeline:
    round_index: int
    verify_blackbox: EdgeSpan
    forest_steps: list[EdgeSpan]
    post_prune_tree_steps: list[EdgeSpan]
    handoff: EdgeSpan | None
    forest_depth: int
    accepted_tokens: int
    generated_tokens: int
    handoff_mode: str
    verify_returned_before_forest_done: bool

    @property
    def forest_end_s(self) -> float:
        return self.forest_steps[-1].end_s if self.forest_steps else self.verify_blackbox.start_s

    @property
    def cloud_edge_overlap_s(self) -> float:
        v = self.verify_blackbox
        return sum(max(0.0, min(v.end_s, s.end_s) - max(v.start_s, s.start_s)) for s in self.forest_steps)

    @property
    def exposed_cloud_wait_s(self) -> float:
        return max(0.0, self.verify_blackbox.end_s - self.forest_end_s)

    def to_dict(self) -> dict[str, object]:
        return {
            "round_index": int(self.round_index),
            "verify_blackbox": self.verify_blackbox.to_dict(),
            "forest_steps": [s.to_dict() for s in self.forest_steps],
            "post_prune_tree_steps": [s.to_dict() for s in self.post_prune_tree_steps],
            "handoff": None if self.handoff is None else self.handoff.to_dict(),
            "forest_depth": int(self.forest_depth),
            "accepted_tokens": int(self.accepted_tokens),
            "generated_tokens": int(self.generated_tokens),
            "handoff_mode": self.handoff_mode,
            "verify_returned_before_forest_done": bool(self.verify_returned_before_forest_done),
            "cloud_edge_overlap_s": self.cloud_edge_overlap_s,
            "exposed_cloud_wait_s": self.exposed_cloud_wait_s,
        }


@dataclass
class EdgeBlackboxTimeline:
    edge_prefill: EdgeSpan
    cloud_prefill_blackbox: EdgeSpan
    initial_tree: EdgeSpan
    rounds: list[EdgeRoundTimeline] = field(default_factory=list)
    elapsed_s: float = 0.0
    generated_tokens: int = 0

    def summary(self) -> dict[str, object]:
        verify = [r.verify_blackbox.elapsed_s for r in self.rounds]
        overlap = [r.cloud_edge_overlap_s for r in self.rounds]
        waits = [r.exposed_cloud_wait_s for r in self.rounds]
        tv = sum(verify)
        return {
            "measurement_view": "edge_observed_cloud_blackbox",
            "cloud_blackbox_definition": (
                "request handoff + target queue + target verify + target KV commit + response handoff"
            ),
            "cloud_internal_timings_used": False,
            "rounds": len(self.rounds),
            "generated_tokens": int(self.generated_tokens),
            "elapsed_s": float(self.elapsed_s),
            "tokens_per_second": float(self.generated_tokens) / max(float(self.elapsed_s), 1e-12),
            "mean_verify_blackbox_s": statistics.fmean(verify) if verify else 0.0,
            "total_verify_blackbox_s": tv,
            "total_cloud_edge_overlap_s": sum(overlap),
            "cloud_hidden_ratio": sum(overlap) / max(tv, 1e-12),
            "total_exposed_cloud_wait_s": sum(waits),
            "early_return_rounds": sum(int(r.verify_returned_before_forest_done) for r in self.rounds),
        }

    def to_dict(self) -> dict[str, object]:
        return {
            "edge_prefill": self.edge_prefill.to_dict(),
            "cloud_prefill_blackbox": self.cloud_prefill_blackbox.to_dict(),
            "initial_tree": self.initial_tree.to_dict(),
            "rounds": [r.to_dict() for r in self.rounds],
            "summary": self.summary(),
        }


def write_timeline_json(path: str | Path, timeline: EdgeBlackboxTimeline) -> None:
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(timeline.to_dict(), indent=2, sort_keys=True) + "\n", encoding="utf-8")


_COLORS = {
    "verify": "#d9534f",
    "forest": "#5bc0de",
    "tree": "#5cb85c",
    "handoff": "#f0ad4e",
    "prefill": "#777777",
}


def render_timeline_svg(timeline: EdgeBlackboxTimeline, *, width: int = 1600) -> str:
    """Two-lane Gantt chart (Cloud black box vs Edge work) as SVG text."""
    spans: list[tuple[str, str, EdgeSpan]] = [
        ("edge", "prefill", timeline.edge_prefill),
        ("cloud", "prefill", timeline.cloud_prefill_blackbox),
        ("edge", "tree", timeline.initial_tree),
    ]
    for r in timeline.rounds:
        spans.append(("cloud", "verify", r.verify_blackbox))
        spans += [("edge", "forest", s) for s in r.forest_steps]
        spans += [("edge", "tree", s) for s in r.post_prune_tree_steps]
        if r.handoff is not None:
            spans.append(("edge", "handoff", r.handoff))
    end = max([timeline.elapsed_s] + [s.end_s for _, _, s in spans] + [1e-9])
    left, right, lane_h, top = 90, 20, 34, 40
    plot_w = max(100, int(width) - left - right)
    height = top + 2 * lane_h + 70

    def x(t: float) -> float:
        return left + plot_w * max(0.0, t) / end

    lanes = {"cloud": top, "edge": top + lane_h + 8}
    parts = [
        f'<svg xmlns="http://www.w3.org/2000/svg" width="{int(width)}" height="{height}" font-family="monospace" font-size="12">',
        f'<text x="{left}" y="20">Edge-observed timeline: {len(timeline.rounds)} rounds, '
        f"{timeline.generated_tokens} tokens, {timeline.elapsed_s * 1e3:.1f} ms</text>",
    ]
    for lane, y in lanes.items():
        parts.append(f'<text x="8" y="{y + lane_h / 2 + 4}">{lane}</text>')
        parts.append(f'<rect x="{left}" y="{y}" width="{plot_w}" height="{lane_h}" fill="#f7f7f7" stroke="#ccc"/>')
    for lane, kind, s in spans:
        y = lanes[lane]
        w = max(0.5, x(s.end_s) - x(s.start_s))
        title = html.escape(f"{s.name}: {s.elapsed_s * 1e3:.3f} ms")
        parts.append(
            f'<rect x="{x(s.start_s):.2f}" y="{y + 3}" width="{w:.2f}" height="{lane_h - 6}" '
            f'fill="{_COLORS[kind]}" opacity="0.85"><title>{title}</title></rect>'
        )
    ly = top + 2 * lane_h + 30
    for i, (kind, color) in enumerate(_COLORS.items()):
        parts.append(f'<rect x="{left + i * 110}" y="{ly}" width="12" height="12" fill="{color}"/>')
        parts.append(f'<text x="{left + i * 110 + 16}" y="{ly + 11}">{kind}</text>')
    summ = timeline.summary()
    parts.append(
        f'<text x="{left}" y="{ly + 32}">hidden ratio {summ["cloud_hidden_ratio"]:.3f}, '
        f'exposed wait {summ["total_exposed_cloud_wait_s"] * 1e3:.2f} ms</text>'
    )
    parts.append("</svg>")
    return "\n".join(parts) + "\n"


def write_timeline_svg(path: str | Path, timeline: EdgeBlackboxTimeline, *, width: int = 1600) -> None:
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(render_timeline_svg(timeline, width=width), encoding="utf-8")
