#!/usr/bin/env python3
"""Gantt PNG for every DBO run under a results root, plus a
``pipelines_index.md`` per mode directory (reference:
scripts/plot_all_pipelines.py). Decode modes show layers 0-2, prefill
layers 1-4."""

from __future__ import annotations

import argparse
import re
import sys
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from afd_demo_b200.scripts import visualize_dbo_pipeline as vis

TARGETS = [("decode-dbo", 0, 3), ("decode-dbo-crosslayer", 0, 3), ("prefill-dbo", 1, 4)]
NAME_RE = re.compile(r"timing_attention_(?P<tag>.+)\.json$")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--root", default="results")
    a = ap.parse_args(argv)
    root = Path(a.root)
    ok = fail = 0
    for sub, start, n in TARGETS:
        d = root / sub
        if not d.is_dir():
            continue
        index = [f"# Pipeline figures — {sub}\n"]
        for attn in sorted(d.glob("timing_attention_*.json")):
            m = NAME_RE.search(attn.name)
            if not m:
                continue
            tag = m["tag"]
            ffn = d / f"timing_ffn_{tag}.json"
            if not ffn.exists():
                print(f"  ! missing ffn for {tag}")
                continue
            args = ["--attn-timing", str(attn), "--ffn-timing", str(ffn),
                    "--output", str(d / f"pipeline_{tag}.png"), "--start-layer", str(start),
                    "--num-layers", str(n)]
            bm = re.search(r"b(\d+)_s(\d+)_t(\d+)", tag)
            if bm:
                cache = root / "serial" / "cache" / f"b{bm[1]}_s{bm[2]}_t{bm[3]}.json"
                if cache.exists():
                    args += ["--serial-timing", str(cache)]
            try:
                vis.main(args)
                ok += 1
                index.append(f"## {tag}\n\n![{tag}](pipeline_{tag}.png)\n")
            except Exception as e:  # keep going over the other runs
                print(f"  x {tag}: {e}")
                fail += 1
        (d / "pipelines_index.md").write_text("\n".join(index))
    print(f"plotted {ok}, failed {fail}")
    return 0 if fail == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
