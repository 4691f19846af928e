#!/usr/bin/env python3
"""Kernel timeline of CUDA-graph-replayed decode steps, per rank.

Runs the model at its benchmark shape (random-init weights, 32 sequences per
GPU, prompt 256), warms up the decode graphs, then records ``--steps`` graph
replays with ``torch.profiler`` (CUPTI kernel records, which include kernels
launched from CUDA graphs) and writes, per rank, the kernel list
(name, start, duration in us) to ``<out>/trace_<schedule>_r<rank>.json``.
``--summary`` prints, per kernel name, the critical-path time of the last
step: on one stream each kernel is charged from the previous kernel's end to
its own end, which removes the overlap that programmatic dependent launch
creates (a kernel launched early is "running" while it waits). The charge is
exact for the serial schedule, which runs on one stream; with two streams
(co-located DBO) kernels of the two micro-batches interleave and the per-name
split is only indicative, but the step total still holds.

With ``--standalone-waits`` every receive is its own one-CTA wait kernel
instead of being folded into the consuming kernel (the RMSNorm on an
attention rank, the MoE gate on an FFN rank), so the summary separates the
time a rank spends waiting for its peers (F2A waits on attention ranks, A2F
waits on FFN ranks) from its kernels' own time. The extra launch per receive
adds about a microsecond per layer and micro-batch.

This is a diagnostic: profiler timings are not benchmark numbers (bench.py
times with CUDA events and no profiler).

    torchrun --nproc-per-node N -m afd_demo_b200.scripts.trace_decode \
        --schedule dbo|serial [--steps 2] [--out results/trace] [--summary] \
        [--standalone-waits] [--attn-gpus A]
"""

from __future__ import annotations

import argparse
import collections
import json
import os
import sys
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))


WAIT_KERNEL = "wait_flags_kernel"


def summarize(path: str) -> str:
    """Critical-path time per kernel name over the last recorded step, and
    the step split into peer waits (stand-alone wait kernels), kernel time
    and idle gaps, per layer."""
    d = json.load(open(path))
    ev = sorted(d["events"], key=lambda e: e[1])
    if not ev:
        return f"{path}: no kernels"
    # every step launches the same kernels: the last step is the last 1/steps
    per_step = len(ev) // max(1, d.get("steps", 1))
    last = sorted(ev[len(ev) - per_step:], key=lambda e: e[1] + e[2])
    agg = collections.defaultdict(lambda: [0, 0.0])
    prev = last[0][1]
    for name, s, du in last:
        end = s + du
        agg[name.split("(")[0][:60]][0] += 1
        agg[name.split("(")[0][:60]][1] += max(0.0, end - prev)
        prev = max(prev, end)
    total = sum(t for _, t in agg.values())
    out = [f"{path} ({d['role']}): last step {total / 1e3:.2f} ms, {len(last)} kernels"]
    for k, (c, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        out.append(f"  {k:60s} {c:4d} {t / 1e3:7.3f} ms {100 * t / total:5.1f}%  "
                   f"{t / c:7.1f} us each")
    wait = sum(t for k, (c, t) in agg.items() if WAIT_KERNEL in k)
    layers = max(1, int(d.get("layers", 1)))
    peer = "F2A" if d["role"] == "attention" else ("A2F" if d["role"] == "ffn" else "peer")
    busy = _busy_union(last)
    span = last[-1][1] + last[-1][2] - min(e[1] for e in last)
    out.append(f"  split per layer ({layers} layers): {peer} waits {wait / layers:7.1f} us, "
               f"kernels {(total - wait) / layers:7.1f} us; GPU busy {100 * busy / span:5.1f}% "
               f"of the step")
    return "\n".join(out)


def _busy_union(ev) -> float:
    """Time covered by at least one kernel (overlaps counted once)."""
    iv = sorted((s, s + du) for _, s, du in ev)
    tot, cur_s, cur_e = 0.0, None, None
    for s, e in iv:
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                tot += cur_e - cur_s
            cur_s, cur_e = s, e
        else:
            cur_e = max(cur_e, e)
    if cur_e is not None:
        tot += cur_e - cur_s
    return tot


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--schedule", choices=["dbo", "serial"], default="dbo")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--batch-per-gpu", type=int, default=32)
    ap.add_argument("--seq", type=int, default=256)
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--out", default="results/trace")
    ap.add_argument("--summary", action="store_true")
    ap.add_argument("--standalone-waits", action="store_true",
                    help="one wait kernel per receive (separates peer waits from kernel time)")
    ap.add_argument("--attn-gpus", type=int, default=None,
                    help="attention ranks (default: half the world)")
    ap.add_argument("--comm-impl", default="auto", choices=["auto", "fused", "nccl"])
    a = ap.parse_args(argv)
    if a.standalone_waits:
        # read by the engine at import time
        os.environ["AFD_DEFER_WAITS"] = "0"

    import torch
    from torch.profiler import ProfilerActivity, profile

    from afd_demo_b200 import ops
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    devmod.init_backend("cuda")
    torch.cuda.set_device(local)
    ctx = get_distributed_context()
    ctx.initialize(DistributedConfig(world_size=world, rank=rank, local_rank=local,
                                     backend="nccl", timeout_s=120, n_attn=a.attn_gpus,
                                     master_addr=os.environ.get("MASTER_ADDR", "127.0.0.1"),
                                     master_port=os.environ.get("MASTER_PORT", "29500")))
    B, S = a.batch_per_gpu * world, a.seq
    m = DisaggregatedQwenModel.from_pretrained(
        a.model, device=f"cuda:{local}", dtype=torch.bfloat16,
        max_seq_len=S + a.warmup + a.steps + 8, max_batch_size=B, random_init=True, seed=0,
        num_micro_batches=2, comm_impl=a.comm_impl)
    ids = torch.randint(0, m.config.vocab_size, (B, S),
                        generator=torch.Generator().manual_seed(1234)).to(f"cuda:{local}")
    logits = m.run_forward(ids, "dbo", 2, crosslayer=True, reset_cache=True)
    tok = torch.zeros(B, 1, dtype=torch.long, device=f"cuda:{local}")
    r = m.local_batch(B)
    nmb, xl = (2, True) if a.schedule == "dbo" else (1, False)
    state = {"logits": logits}

    def step():
        if m.ctx.is_attention_node:
            tok[r.start:r.stop, 0] = ops.argmax(state["logits"])
        state["logits"] = m.decode_step(tok, a.schedule, nmb, xl, True)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    ctx.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.steps):
            step()
        torch.cuda.synchronize()
    ctx.barrier()
    events = [(e.name, e.time_range.start, e.time_range.end - e.time_range.start)
              for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    path = out / f"trace_{a.schedule}_r{rank}.json"
    role = "both" if (m.ctx.is_attention_node and m.ctx.is_ffn_node) else m.ctx.role
    path.write_text(json.dumps({"rank": rank, "role": role, "schedule": a.schedule,
                                "steps": a.steps, "layers": m.num_layers,
                                "topology": m.topology.tag(), "batch": B,
                                "standalone_waits": a.standalone_waits, "events": events}))
    if a.summary:
        print(summarize(str(path)), flush=True)
    m.release_graphs()
    ctx.barrier()
    ctx.cleanup()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
