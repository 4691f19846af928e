#!/usr/bin/env python3
"""Four-lane Gantt chart (A, A->F, F, F->A) of a DBO run as a PNG.

Reference: scripts/visualize_dbo_pipeline.py (matplotlib). This one draws
with ``afd_demo_b200.utils.png`` (no plotting library needed).

Clock alignment: attention and FFN events come from different clocks (two
processes, or two trackers). The FFN lane is shifted by the smallest
``ffn recv_wait end - attention hand-off end`` over the (layer, micro-batch)
pairs shown, where the hand-off end is the A2F send span's end when the run
recorded one, else the attention compute end (the fused transport stores
the tile inside the o_proj kernel, so data is on the FFN GPU when the
attention span ends). Micro-batch 0 is blue, 1 orange; layer numbers are
printed in the bars.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Dict, List, Optional, Tuple

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from afd_demo_b200.scripts.experiment_baselines import normalize_mode, resolve_serial_baseline
from afd_demo_b200.utils.png import Canvas

MB_COLORS = [(66, 133, 244), (255, 153, 51), (52, 168, 83), (234, 67, 53)]
LANES = ["A", "A2F", "F", "F2A"]


def _end_ms(e) -> float:
    return e["start"] * 1000 + e["duration_ms"]


def clock_offset(attn: dict, ffn: dict, layers: range) -> float:
    hand = {}
    sends = [e for e in attn["events"] if e["type"] == "send_transfer"]
    src = sends if sends else [e for e in attn["events"] if e["type"] == "attn_compute"]
    for e in src:
        hand[(e["layer"], e["mb"])] = _end_ms(e)
    offs = [_end_ms(e) - hand[(e["layer"], e["mb"])] for e in ffn["events"]
            if e["type"] == "recv_wait" and e["layer"] in layers and (e["layer"], e["mb"]) in hand]
    return min(offs) if offs else 0.0


def auto_start_layer(attn: dict, start: int) -> int:
    """Skip leading layers whose mb-0 attention span is > 5x the median."""
    durs = {e["layer"]: e["duration_ms"] for e in attn["events"]
            if e["type"] == "attn_compute" and e["mb"] == 0}
    if len(durs) < 3:
        return start
    med = sorted(durs.values())[len(durs) // 2]
    while start in durs and durs[start] > 5 * med:
        start += 1
    return start


def lanes(attn: dict, ffn: dict, start: int, n: int) -> Tuple[Dict[str, List], float]:
    layers = range(start, start + n)
    off = clock_offset(attn, ffn, layers)
    evs = []
    for e in attn["events"]:
        if e["layer"] in layers and e["type"] in ("attn_compute", "send_transfer"):
            evs.append(("A" if e["type"] == "attn_compute" else "A2F", e["start"] * 1000, e))
    for e in ffn["events"]:
        if e["layer"] in layers and e["type"] in ("ffn_compute", "send_transfer"):
            evs.append(("F" if e["type"] == "ffn_compute" else "F2A", e["start"] * 1000 - off, e))
    t0 = min((t for _, t, _ in evs), default=0.0)
    out: Dict[str, List] = {k: [] for k in LANES}
    for lane, t, e in evs:
        out[lane].append((t - t0, e["duration_ms"], e["layer"] - start, e["mb"]))
    return out, off


def draw(data: Dict[str, List], path: str, title: str, note: str = "") -> None:
    W, H, left, top, lane_h = 1400, 120 + 60 * len(LANES), 80, 60, 50
    c = Canvas(W, H)
    c.text(10, 10, title, scale=2)
    if note:
        c.text(10, 34, note)
    span = max((s + d for v in data.values() for s, d, _, _ in v), default=1.0) or 1.0
    sx = (W - left - 20) / span
    for i, lane in enumerate(LANES):
        y = top + i * 60
        c.text(10, y + 20, lane, scale=2)
        c.rect(left, y + lane_h + 4, W - 20, y + lane_h + 5, (200, 200, 200))
        for s, d, layer, mb in data[lane]:
            x0 = left + int(s * sx)
            x1 = max(x0 + 1, left + int((s + d) * sx))
            c.rect(x0, y, x1, y + lane_h, MB_COLORS[mb % len(MB_COLORS)])
            c.frame(x0, y, x1, y + lane_h, (40, 40, 40))
            if x1 - x0 > 14:
                c.text(x0 + 3, y + 4, f"L{layer}", (255, 255, 255))
    ty = top + len(LANES) * 60 + 10
    for k in range(6):
        x = left + int((W - left - 20) * k / 5)
        c.rect(x, ty - 6, x + 1, ty, (0, 0, 0))
        c.text(x - 10, ty + 2, f"{span * k / 5:.2f}")
    c.text(left, ty + 16, "MS   BLUE=MB0  ORANGE=MB1")
    c.save(path)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--attn-timing", default="results/prefill_dbo/timing_attention.json")
    ap.add_argument("--ffn-timing", default="results/prefill_dbo/timing_ffn.json")
    ap.add_argument("--output", default="results/prefill_dbo/dbo_pipeline_4lanes.png")
    ap.add_argument("--start-layer", type=int, default=0)
    ap.add_argument("--auto-skip-warmup", dest="auto_skip", action="store_true", default=True)
    ap.add_argument("--no-auto-skip-warmup", dest="auto_skip", action="store_false")
    ap.add_argument("--num-layers", type=int, default=2)
    ap.add_argument("--serial-time", type=float, default=None)
    ap.add_argument("--serial-timing", default=None)
    ap.add_argument("--mode", default="auto")
    a = ap.parse_args(argv)
    attn = json.loads(Path(a.attn_timing).read_text())
    ffn = json.loads(Path(a.ffn_timing).read_text())
    start = auto_start_layer(attn, a.start_layer) if a.auto_skip else a.start_layer
    data, off = lanes(attn, ffn, start, a.num_layers)
    mode = normalize_mode(a.attn_timing if a.mode == "auto" else a.mode)
    note = f"CLOCK OFFSET FFN-ATT {off:.3f} MS"
    serial: Optional[float] = a.serial_time
    if serial is None and a.serial_timing and Path(a.serial_timing).exists():
        b = resolve_serial_baseline(json.loads(Path(a.serial_timing).read_text()), mode)
        serial = b.value_ms if b.available else None
    if serial:
        cur = attn.get("decode_tpot_ms") if mode == "decode" else attn.get("total_time_ms")
        note += f"   SERIAL {serial:.2f} MS" + (f"  DBO {cur:.2f} MS  SPEEDUP {serial / cur:.2f}X"
                                                  if cur else "")
    Path(a.output).parent.mkdir(parents=True, exist_ok=True)
    draw(data, a.output, f"DBO PIPELINE L{start}-L{start + a.num_layers - 1}", note)
    print(f"Wrote {a.output}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
