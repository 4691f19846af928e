#!/usr/bin/env python3
"""Add the prefill/decode split to serial cache entries.

Reference: scripts/capture_serial_split.py and capture_serial_prefill.sh. For
each ``<root>/serial/cache/b{B}_s{S}_t{T}.json`` it re-runs a serial,
prefill-only run through run_single.sh and merges the measured
``prefill_ms`` into the cache, with ``decode_tpot_ms = decode_step_ms =
(total_time_ms - prefill_ms) / (tokens - 1)`` and ``decode_steps``.

Serial generation runs of this framework already record device-timed
``prefill_ms`` and ``decode_tpot_ms``; entries that have both are skipped with
``--skip-existing``.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
from dataclasses import dataclass
from pathlib import Path
from typing import List, Optional, Set

ROOT = Path(__file__).resolve().parents[2]
CACHE_RE = re.compile(r"^b(?P<b>\d+)_s(?P<s>\d+)_t(?P<t>\d+)\.json$")


@dataclass
class Config:
    batch: int
    seq: int
    tokens: int
    cache_path: Path


def parse_list(s: str) -> Optional[Set[int]]:
    return {int(x) for x in s.split(",") if x.strip()} if s else None


def iter_configs(cache_dir: Path, batches=None, seqs=None, tokens=None) -> List[Config]:
    out = []
    for p in sorted(cache_dir.glob("b*_s*_t*.json")):
        m = CACHE_RE.match(p.name)
        if not m:
            continue
        c = Config(int(m["b"]), int(m["s"]), int(m["t"]), p)
        if (batches and c.batch not in batches) or (seqs and c.seq not in seqs) or \
                (tokens and c.tokens not in tokens):
            continue
        out.append(c)
    return out


def has_split(path: Path) -> bool:
    try:
        d = json.loads(path.read_text())
    except (OSError, ValueError):
        return False
    return "prefill_ms" in d and "decode_tpot_ms" in d


def merge_split(cache_path: Path, raw_path: Path):
    cache = json.loads(cache_path.read_text())
    prefill = float(json.loads(raw_path.read_text())["total_time_ms"])
    total = float(cache["total_time_ms"])
    tokens = int(cache.get("max_new_tokens") or 0)
    steps = max(tokens - 1, 0)
    if steps <= 0:
        raise ValueError(f"{cache_path}: no decode-loop steps")
    if total < prefill:
        raise ValueError(f"{cache_path}: total_time_ms {total:.3f} < prefill {prefill:.3f}")
    step = (total - prefill) / steps
    cache.update(prefill_ms=prefill, decode_step_ms=step, decode_tpot_ms=step, decode_steps=steps)
    cache_path.write_text(json.dumps(cache, indent=2) + "\n")
    return prefill, step


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--root", default="results")
    ap.add_argument("--deployment", default="local")
    ap.add_argument("--batches", default="")
    ap.add_argument("--seqs", default="")
    ap.add_argument("--tokens", default="")
    ap.add_argument("--skip-batches", default="")
    ap.add_argument("--skip-existing", action="store_true")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--warmup-rounds", type=int, default=3)
    a = ap.parse_args(argv)
    root = Path(a.root)
    cache_dir = root / "serial" / "cache"
    if not cache_dir.is_dir():
        print(f"Missing serial cache directory: {cache_dir}", file=sys.stderr)
        return 2
    skip = parse_list(a.skip_batches) or set()
    failures = 0
    for c in iter_configs(cache_dir, parse_list(a.batches), parse_list(a.seqs),
                          parse_list(a.tokens)):
        name = c.cache_path.stem
        if c.batch in skip:
            print(f"[skip-batch] {name}")
            continue
        if a.skip_existing and has_split(c.cache_path):
            print(f"[skip-existing] {name}")
            continue
        sfx = f"warmup_serial_{a.deployment}_b{c.batch}_s{c.seq}_t{c.tokens}"
        raw = root / "prefill_dbo" / f"timing_attention_{sfx}.json"
        cmd = ["bash", str(ROOT / "afd_demo_b200/scripts/run_single.sh"), a.deployment,
               str(c.batch), str(c.seq), "--tokens", str(c.tokens), "--no-dbo", "--warmup-p2p",
               "--warmup-rounds", str(a.warmup_rounds)]
        print(f"\n=== capture serial split: {name} ===\n{' '.join(cmd)}")
        if a.dry_run:
            continue
        raw.unlink(missing_ok=True)
        env = dict(os.environ, RESULTS_DIR=str(root))
        env.setdefault("MASTER_PORT", str(29500 + os.getpid() % 2000))
        if subprocess.run(cmd, env=env).returncode != 0 or not raw.exists():
            print(f"[FAIL] {name}", file=sys.stderr)
            failures += 1
            continue
        p, s = merge_split(c.cache_path, raw)
        print(f"  merged: prefill={p:.1f}ms decode_tpot={s:.1f}ms")
    return 1 if failures else 0


if __name__ == "__main__":
    raise SystemExit(main())
