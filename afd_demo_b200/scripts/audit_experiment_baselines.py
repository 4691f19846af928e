#!/usr/bin/env python3
"""Audit that every DBO result has a mode-matched serial baseline.

Reference: scripts/audit_experiment_baselines.py. Scans
``<root>/{decode-dbo,decode-dbo-crosslayer,prefill-dbo}/timing_attention_*.json``,
pairs each with ``<root>/serial/cache/b{B}_s{S}_t{T}.json``, and reports
(root, mode, tag, batch, seq, tokens, status, serial_cache,
serial_baseline_ms, dbo_ms, speedup, note) rows; ``--output-csv`` writes them.
Statuses: ok, unparseable-tag, serial-cache-missing, serial-cache-invalid,
baseline-missing.
"""

from __future__ import annotations

import argparse
import csv
import json
import re
import sys
from dataclasses import asdict, dataclass, fields
from pathlib import Path
from typing import List, Optional

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from afd_demo_b200.scripts.experiment_baselines import infer_mode_from_path, resolve_serial_baseline

SUBDIRS = ("decode-dbo", "decode-dbo-crosslayer", "prefill-dbo")
NAME_RE = re.compile(r"timing_attention_(?P<tag>.+)\.json$")
CFG_RE = re.compile(r"b(?P<batch>\d+)_s(?P<seq>\d+)_t(?P<tokens>\d+)")


@dataclass
class Row:
    root: str
    mode: str
    tag: str
    batch: str
    seq: str
    tokens: str
    status: str
    serial_cache: str
    serial_baseline_ms: str
    dbo_ms: str
    speedup: str
    note: str


def _f(v: Optional[float]) -> str:
    return "" if v is None else f"{v:.6f}"


def audit_root(root: Path) -> List[Row]:
    rows: List[Row] = []
    cache = root / "serial" / "cache"
    for sub in SUBDIRS:
        d = root / sub
        if not d.is_dir():
            continue
        mode = infer_mode_from_path(sub) or "unknown"
        for p in sorted(d.glob("timing_attention_*.json")):
            m = NAME_RE.match(p.name)
            if not m:
                continue
            tag = m.group("tag")
            c = CFG_RE.search(tag)
            dbo = None
            try:
                data = json.loads(p.read_text())
                dbo = float(data.get("decode_tpot_ms" if mode == "decode" else "total_time_ms") or 0)
            except (OSError, ValueError, TypeError):
                pass
            if not c:
                rows.append(Row(root.name, mode, tag, "", "", "", "unparseable-tag", "", "", _f(dbo),
                                "", "could not parse b/s/t"))
                continue
            b, s, t = c.group("batch"), c.group("seq"), c.group("tokens")
            sp = cache / f"b{b}_s{s}_t{t}.json"
            if not sp.exists():
                rows.append(Row(root.name, mode, tag, b, s, t, "serial-cache-missing", str(sp), "",
                                _f(dbo), "", "matching serial cache not found"))
                continue
            try:
                base = resolve_serial_baseline(json.loads(sp.read_text()), mode)
            except (OSError, ValueError, TypeError) as e:
                rows.append(Row(root.name, mode, tag, b, s, t, "serial-cache-invalid", str(sp), "",
                                _f(dbo), "", str(e)))
                continue
            if not base.available:
                rows.append(Row(root.name, mode, tag, b, s, t, "baseline-missing", str(sp), "",
                                _f(dbo), "", base.warning or "mode-matched baseline missing"))
                continue
            speed = base.value_ms / dbo if dbo else None
            rows.append(Row(root.name, mode, tag, b, s, t, "ok", str(sp), _f(base.value_ms),
                            _f(dbo), _f(speed), base.source))
    return rows


def write_csv(rows: List[Row], out: Path) -> None:
    out.parent.mkdir(parents=True, exist_ok=True)
    with out.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=[x.name for x in fields(Row)], lineterminator="\n")
        w.writeheader()
        for r in rows:
            w.writerow(asdict(r))


def summary(rows: List[Row]) -> str:
    counts = {}
    for r in rows:
        counts[(r.root, r.mode, r.status)] = counts.get((r.root, r.mode, r.status), 0) + 1
    lines = ["| Root | Mode | Status | Count |", "|---|---|---|---:|"]
    lines += [f"| {a} | {b} | {c} | {n} |" for (a, b, c), n in sorted(counts.items())]
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--root", action="append", default=[])
    ap.add_argument("--output-csv", default="")
    a = ap.parse_args(argv)
    roots = [Path(r) for r in a.root] or [Path("results")]
    rows: List[Row] = []
    for r in roots:
        if r.is_dir():
            rows += audit_root(r)
        else:
            print(f"Warning: results root not found: {r}", file=sys.stderr)
    print(summary(rows))
    if a.output_csv:
        write_csv(rows, Path(a.output_csv))
        print(f"\nWrote detail CSV: {a.output_csv}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
