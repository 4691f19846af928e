#!/usr/bin/env python3
"""Markdown report of one run from its attention + FFN timing JSON files.

Reference: scripts/gen_experiment_report.py. Same inputs (``--attn-timing``,
``--ffn-timing``, ``--output``, ``--mode``, ``--batch``, ``--seq``,
``--tokens``, ``--model``, ``--dtype``, ``--comm-timing-mode``,
``--serial-baseline``) and the same sections: configuration, model-side
timing (TTFT for prefill, exact TPOT for decode), comparison with the
mode-matched serial baseline, layer averages, per-layer table
(attention / A2F / FFN / F2A / recv-wait, mean/min/max over micro-batches).

Timing JSON written by this framework is device-timed (CUDA events); the
report says so when ``device_timed`` is set. With the fused transport the
A2F/F2A transfer happens inside the o_proj / combine kernels, so there are no
separate send spans and the transfer shows up in the compute columns.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
from collections import defaultdict
from pathlib import Path
from typing import Dict, List, Optional

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from afd_demo_b200.scripts.experiment_baselines import normalize_mode, resolve_serial_baseline


def load(path: str) -> Optional[dict]:
    if not path or not os.path.isfile(path):
        return None
    with open(path) as f:
        return json.load(f)


def by_layer(events: List[dict]) -> Dict[int, Dict[str, List[float]]]:
    out: Dict[int, Dict[str, List[float]]] = defaultdict(lambda: defaultdict(list))
    for e in events or []:
        if e.get("layer") is None or e.get("type") is None or e.get("duration_ms") is None:
            continue
        out[int(e["layer"])][e["type"]].append(float(e["duration_ms"]))
    return out


def stats3(v: List[float]) -> str:
    if not v:
        return "-"
    if len(v) == 1:
        return f"{v[0]:.3f}"
    return f"{statistics.mean(v):.3f} / {min(v):.3f} / {max(v):.3f}"


def comm_mode(attn, ffn) -> str:
    for d in (attn, ffn):
        if d and d.get("comm_timing_mode"):
            return str(d["comm_timing_mode"])
    return "enqueue"


def send_label(attn, ffn) -> str:
    return "send completion" if comm_mode(attn, ffn) == "completion" else "send enqueue"


def timed_step(attn, ffn):
    for d in (attn, ffn):
        if d and d.get("timed_decode_step") is not None:
            return int(d["timed_decode_step"]), False
    return 1, True


def merge_serial_cache(attn, serial, mode):
    """Serial reports borrow missing display fields from the cache entry."""
    if normalize_mode(mode) is not None or not attn or not serial:
        return attn
    m = dict(attn)
    for k in ("prefill_ms", "decode_loop_ms", "decode_steps", "decode_tpot_ms", "decode_step_ms"):
        if m.get(k) is None and serial.get(k) is not None:
            m[k] = serial[k]
    if m != attn:
        m["_serial_cache_merged"] = True
    return m


def metadata(attn, ffn, a) -> str:
    md = attn or ffn or {}
    lines = [f"- **Mode**: `{a.mode or 'unknown'}`", f"- **Batch size**: {a.batch}",
             f"- **Prefill seq**: {a.seq}", f"- **Decode tokens**: {a.tokens}",
             f"- **Layers**: {md.get('num_layers', '?')}",
             f"- **Micro-batches**: {md.get('num_micro_batches', '?')}",
             f"- **Comm timing mode**: `{a.comm_timing_mode or comm_mode(attn, ffn)}`"]
    for key, label in (("prefill_seq_len", "Requested prefill seq"),
                       ("actual_prompt_len", "Actual prompt len"), ("topology", "Topology"),
                       ("gpus", "GPUs")):
        if md.get(key) is not None:
            lines.append(f"- **{label}**: {md[key]}")
    if md.get("device_timed"):
        lines.append("- **Clock**: device (CUDA events on the streams that ran the work)")
    if a.model:
        lines.append(f"- **Model**: `{a.model}`")
    if a.dtype:
        lines.append(f"- **Dtype**: `{a.dtype}`")
    return "\n".join(lines)


def timing_table(attn, ffn, mode) -> str:
    nm = normalize_mode(mode)
    if nm == "prefill":
        total = "Model-side prefill total / TTFT-path"
    elif nm == "decode":
        s, _ = timed_step(attn, ffn)
        total = f"Decode step {s} timing total (0-based)"
    else:
        total = "Model-side generation total"
    rows = ["| Metric | Attention rank view | FFN rank view |", "|---|---:|---:|"]

    def fmt(v, unit):
        if v is None:
            return "-"
        return f"{v:.3f} {unit}".strip() if isinstance(v, float) else str(v)

    for label, key, unit in [(total, "total_time_ms", "ms"), ("Prefill / TTFT-path", "prefill_ms", "ms"),
                             ("Decode loop total", "decode_loop_ms", "ms"),
                             ("Decode steps", "decode_steps", ""), ("Decode TPOT", "decode_tpot_ms", "ms"),
                             ("Legacy decode step (not exact TPOT)", "decode_step_ms", "ms"),
                             ("Compute", "total_compute_ms", "ms"),
                             ("Recv wait", "total_recv_wait_ms", "ms"),
                             ("MoE router", "total_moe_router_ms", "ms"),
                             ("MoE experts", "total_moe_experts_ms", "ms"),
                             ("MoE shared/dense", "total_moe_shared_or_dense_ms", "ms"),
                             ("Compute ratio", "compute_ratio", ""),
                             ("Max over ranks", "rank_max_ms", "ms")]:
        av = attn.get(key) if attn else None
        fv = ffn.get(key) if ffn else None
        rows.append(f"| {label} | {fmt(av, unit)} | {fmt(fv, unit)} |")
    if attn and "tokens_per_sec" in attn:
        rows.append(f"| Tokens/sec | {attn['tokens_per_sec']:.2f} | - |")
    return "\n".join(rows)


def notes(attn, ffn, mode) -> str:
    nm = normalize_mode(mode)
    out = []
    if nm is None:
        out += ["- `Model-side generation total` is `total_time_ms` for the full generation call.",
                "- `Decode TPOT` is the serial decode baseline used for decode speedup."]
        if attn and attn.get("_serial_cache_merged"):
            out.append("- Missing serial display fields were filled from the matching serial cache JSON.")
    elif nm == "decode" and ((attn and attn.get("events")) or (ffn and ffn.get("events"))):
        s, inferred = timed_step(attn, ffn)
        out += [f"- Pipeline detail is recorded for 0-based decode step **{s}** "
                f"({'inferred' if inferred else 'recorded in timing JSON'}).",
                "- Decode speedup uses exact `decode_tpot_ms` over all decode-loop steps."]
        if comm_mode(attn, ffn) == "completion":
            out.append("- A2F/F2A spans are effective send completion latency, not pure wire time.")
        else:
            out.append("- A2F/F2A spans are isend enqueue overhead; with the fused transport the "
                       "transfer runs inside the o_proj / combine kernels and has no span.")
    elif nm == "prefill":
        out.append("- Prefill speedup uses model-side TTFT-path: serial `prefill_ms` / DBO `total_time_ms`.")
    return "\n".join(out)


def compare(cur, serial, mode, path="") -> str:
    nm = normalize_mode(mode)
    if not cur or not serial or nm is None:
        return ""
    v = cur.get("total_time_ms") if nm == "prefill" else cur.get("decode_tpot_ms")
    metric = "TTFT" if nm == "prefill" else "exact TPOT"
    if v is None:
        return (f"\n## Compared to serial baseline\n\n- This run {metric}: **N/A** (missing "
                "required timing field)\n- Speedup: **N/A**\n")
    v = float(v)
    b = resolve_serial_baseline(serial, nm)
    src = f" from `{path}`" if path else ""
    if not b.available:
        return (f"\n## Compared to serial baseline\n\n- Serial baseline: **N/A** ({b.warning})\n"
                f"- This run {metric}: **{v:.3f} ms**\n- Speedup: **N/A**\n")
    sp = b.value_ms / v if v > 0 else float("nan")
    note = b.source + (f"; {b.warning}" if b.warning else "")
    return (f"\n## Compared to serial baseline\n\n"
            f"- Serial {b.unit}: **{b.value_ms:.3f} ms**  ({note}{src})\n"
            f"- This run {metric}: **{v:.3f} ms**\n"
            f"- Δ: {v - b.value_ms:+.3f} ms   |   {'TTFT' if nm == 'prefill' else 'TPOT'} "
            f"speedup: **{sp:.3f}×**\n")


def layer_summary(attn, ffn) -> str:
    ab = by_layer((attn or {}).get("events"))
    fb = by_layer((ffn or {}).get("events"))
    layers = sorted(set(ab) | set(fb))
    if not layers:
        return "_No per-layer events recorded._"

    def avg(sel, b, t):
        vals = [statistics.mean(b[l][t]) if b.get(l, {}).get(t) else 0.0 for l in sel]
        return statistics.mean(vals) if vals else 0.0

    sl = send_label(attn, ffn)
    rows = [f"| Scope | Layers | Attention avg/layer (ms) | A2F {sl} avg/layer (ms) | FFN avg/layer (ms) "
            f"| F2A {sl} avg/layer (ms) | F2A recv-wait avg/layer (ms) |",
            "|---|---:|---:|---:|---:|---:|---:|"]
    scopes = [("All layers", layers)]
    if [l for l in layers if l != 0]:
        scopes.append(("Excl. L0", [l for l in layers if l != 0]))
    for label, sel in scopes:
        rows.append(f"| {label} | {len(sel)} | {avg(sel, ab, 'attn_compute'):.3f} | "
                    f"{avg(sel, ab, 'send_transfer'):.3f} | {avg(sel, fb, 'ffn_compute'):.3f} | "
                    f"{avg(sel, fb, 'send_transfer'):.3f} | {avg(sel, ab, 'recv_wait'):.3f} |")
    rows += ["", "_Each value averages across micro-batches within a layer, then across layers._"]
    return "\n".join(rows)


def per_layer(attn, ffn) -> str:
    ae = (attn or {}).get("events") or []
    fe = (ffn or {}).get("events") or []
    ab, fb = by_layer(ae), by_layer(fe)
    layers = sorted(set(ab) | set(fb))
    if not layers:
        return "_No per-layer events recorded._"

    def mib(events, l):
        return stats3([float(e["tensor_mib"]) for e in events if e.get("layer") == l and
                       e.get("type") == "send_transfer" and e.get("tensor_mib") is not None])

    sl = send_label(attn, ffn)
    rows = [f"| Layer | Attention (ms) | A2F {sl} (ms) | A2F payload (MiB) | FFN (ms) | F2A {sl} (ms) "
            "| F2A payload (MiB) | F2A recv-wait (ms) |",
            "|------:|---------------:|---------:|---------:|---------:|---------:|---------:|---------:|"]
    for l in layers:
        a, f = ab.get(l, {}), fb.get(l, {})
        rows.append(f"| {l} | {stats3(a.get('attn_compute', []))} | {stats3(a.get('send_transfer', []))} "
                    f"| {mib(ae, l)} | {stats3(f.get('ffn_compute', []))} | "
                    f"{stats3(f.get('send_transfer', []))} | {mib(fe, l)} | "
                    f"{stats3(a.get('recv_wait', []))} |")

    def tot(b, t):
        return sum(statistics.mean(m[t]) for l, m in b.items() if l != 0 and m.get(t))

    rows.append(f"| **Σ (excl. L0)** | **{tot(ab, 'attn_compute'):.3f}** | "
                f"**{tot(ab, 'send_transfer'):.3f}** | - | **{tot(fb, 'ffn_compute'):.3f}** | "
                f"**{tot(fb, 'send_transfer'):.3f}** | - | **{tot(ab, 'recv_wait'):.3f}** |")
    rows += ["", "_Cells with three values are **mean / min / max across micro-batches**._",
             "_L0 is skipped in the Σ row because layer 0 contains pipeline warmup._"]
    return "\n".join(rows)


def build_report(attn, ffn, a, serial=None) -> str:
    attn = merge_serial_cache(attn, serial, a.mode)
    nm = normalize_mode(a.mode)
    title = {"prefill": "Model-side TTFT timing (prefill path)",
             "decode": "Decode timing (exact TPOT + decode step detail)"}.get(
        nm, "Serial timing (model-side total + decode fields)")
    parts = [f"# Experiment report — {a.mode or 'run'} b{a.batch} s{a.seq} t{a.tokens}\n",
             "## Configuration\n", metadata(attn, ffn, a), "", f"## {title}\n",
             timing_table(attn, ffn, a.mode)]
    n = notes(attn, ffn, a.mode)
    if n:
        parts += ["", n]
    parts.append("")
    c = compare(attn, serial, a.mode, a.serial_baseline)
    if c:
        parts.append(c)
    parts += ["## Layer averages summary\n", layer_summary(attn, ffn), "",
              "## Per-layer breakdown\n", per_layer(attn, ffn), "", "---",
              f"_Generated from `{os.path.basename(a.attn_timing)}` + "
              f"`{os.path.basename(a.ffn_timing)}`._"]
    return "\n".join(parts) + "\n"


def parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--attn-timing", required=True)
    ap.add_argument("--ffn-timing", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--mode", default="")
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--seq", type=int, default=0)
    ap.add_argument("--tokens", type=int, default=0)
    ap.add_argument("--model", default="")
    ap.add_argument("--dtype", default="")
    ap.add_argument("--comm-timing-mode", default="")
    ap.add_argument("--serial-baseline", default="")
    return ap


def main(argv=None) -> int:
    a = parser().parse_args(argv)
    attn, ffn = load(a.attn_timing), load(a.ffn_timing)
    if attn is None and ffn is None:
        raise SystemExit(f"ERROR: neither {a.attn_timing} nor {a.ffn_timing} exist")
    serial = load(a.serial_baseline) if a.serial_baseline else None
    Path(a.output).parent.mkdir(parents=True, exist_ok=True)
    with open(a.output, "w") as f:
        f.write(build_report(attn, ffn, a, serial))
    print(f"Report written: {a.output}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
