"""Session timeline: a Gantt chart of SessionTimer spans (one row per session, one colour per
execution kind), written as a self-contained SVG/HTML file.

Reference: ``axrl/utils/visualize_session_timer.py:323`` (plotly timeline of the JSON-tagged
timer log).  Input: the JSON-lines file written when ``AXRL_SESSION_TIMELINE`` is set.

Usage: ``python -m axrl_b200.utils.visualize_session_timer timeline.jsonl out.html``
"""

from __future__ import annotations

import json
import sys
from html import escape
from pathlib import Path

PALETTE = ["#4e79a7", "#f28e2b", "#e15759", "#76b7b2", "#59a14f", "#edc948", "#b07aa1", "#ff9da7", "#9c755f", "#bab0ac"]


def load_spans(path: str | Path) -> list[dict]:
    spans = []
    for line in Path(path).read_text().splitlines():
        line = line.strip()
        if line:
            spans.append(json.loads(line))
    return spans


def render(spans: list[dict], width: int = 1200, row_h: int = 18) -> str:
    if not spans:
        return "<html><body>no spans</body></html>"
    t0 = min(s["start"] for s in spans)
    t1 = max(s["end"] for s in spans)
    span = max(t1 - t0, 1e-9)
    sessions = sorted({s["session_id"] for s in spans})
    kinds = sorted({s["execution_kind"] for s in spans})
    color = {k: PALETTE[i % len(PALETTE)] for i, k in enumerate(kinds)}
    left, top = 180, 30
    H = top + row_h * len(sessions) + 40
    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{left + width + 20}" height="{H}" font-family="monospace" font-size="11">']
    for i, sid in enumerate(sessions):
        y = top + i * row_h
        parts.append(f'<text x="4" y="{y + row_h - 5}">{escape(str(sid))[:24]}</text>')
    for s in spans:
        i = sessions.index(s["session_id"])
        x = left + width * (s["start"] - t0) / span
        w = max(1.0, width * (s["end"] - s["start"]) / span)
        y = top + i * row_h + 2
        tip = f'{s["function_name"]} ({s["execution_kind"]}): {s["end"] - s["start"]:.3f}s'
        parts.append(f'<rect x="{x:.1f}" y="{y}" width="{w:.1f}" height="{row_h - 4}" fill="{color[s["execution_kind"]]}">'
                     f"<title>{escape(tip)}</title></rect>")
    for j, k in enumerate(kinds):
        parts.append(f'<rect x="{left + 120 * j}" y="{H - 25}" width="10" height="10" fill="{color[k]}"/>'
                     f'<text x="{left + 120 * j + 14}" y="{H - 16}">{escape(k)}</text>')
    parts.append(f'<text x="{left}" y="15">0 s</text><text x="{left + width - 60}" y="15">{span:.2f} s</text></svg>')
    return "<html><body>" + "".join(parts) + "</body></html>"


def main(argv: list[str] | None = None) -> None:
    a = argv if argv is not None else sys.argv[1:]
    Path(a[1]).write_text(render(load_spans(a[0])))


if __name__ == "__main__":
    main()
