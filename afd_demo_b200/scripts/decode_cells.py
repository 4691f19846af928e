#!/usr/bin/env python3
"""Serial and DBO cells of the experiment matrix on one loaded model.

The reference's matrix (scripts/run_experiment_matrix.sh:72-84) starts one
process per (mode, batch, prompt) cell and reloads the checkpoint each time;
this script loads the model once per job and runs every cell through
`generate`, so a whole table of TPOT / TTFT cells costs seconds per cell:

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m afd_demo_b200.scripts.decode_cells --batches 2,4,16,64 --seqs 128,512,2048

Per cell and mode: decode TPOT (`decode_tpot_ms`, the reference's
decode_loop_ms / (tokens - 1)) and prefill TTFT (`prefill_ms`), device-timed,
max over ranks, measured after warm-up runs (the first captures the CUDA graphs;
more follow while the caching allocator is still growing).
Modes: serial (serial prefill and decode), dbo (prefill DBO, decode DBO),
dbo-crosslayer (prefill DBO, cross-layer decode DBO). A cell whose batch the
attention ranks cannot split into two micro-batches runs serial only. Rank 0
prints one JSON line per cell and, with --output, writes them all as a list.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

if __package__ in (None, ""):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

MODES = {"serial": (False, False), "dbo": (True, False), "dbo-crosslayer": (True, True)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="qwen3-30b-a3b")
    ap.add_argument("--batches", default="2,4,8,16,32,64")
    ap.add_argument("--seqs", default="128,256,512")
    ap.add_argument("--tokens", type=int, default=20)
    ap.add_argument("--modes", default="serial,dbo-crosslayer")
    ap.add_argument("--attn-gpus", type=int, default=None)
    ap.add_argument("--comm-impl", default="auto")
    ap.add_argument("--output", default="")
    a = ap.parse_args(argv)

    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        # one GPU: both roles' streams hand tensors to each other; expandable
        # segments keep the caching allocator from fragmenting (set before the
        # first CUDA allocation)
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    devmod.init_backend("cuda")
    torch.cuda.set_device(local)
    ctx = get_distributed_context()
    ctx.initialize(DistributedConfig(world_size=world, rank=rank, local_rank=local,
                                     backend="nccl", timeout_s=120, n_attn=a.attn_gpus,
                                     master_addr=os.environ.get("MASTER_ADDR", "127.0.0.1"),
                                     master_port=os.environ.get("MASTER_PORT", "29500")))
    batches = [int(b) for b in a.batches.split(",")]
    seqs = [int(s) for s in a.seqs.split(",")]
    modes = a.modes.split(",")
    for m in modes:
        if m not in MODES:
            raise SystemExit(f"unknown mode {m!r}; choose from {sorted(MODES)}")
    dev = f"cuda:{local}"
    model = DisaggregatedQwenModel.from_pretrained(
        a.model, device=dev, dtype=torch.bfloat16, max_seq_len=max(seqs) + a.tokens + 8,
        max_batch_size=max(batches), comm_impl=a.comm_impl, random_init=True, seed=0,
        num_micro_batches=2)
    V = model.config.vocab_size
    n_attn = model.topology.n_attn

    def mx(vals):
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    rows = []
    for s in seqs:
        for b in batches:
            ids = torch.randint(0, V, (b, s), generator=torch.Generator().manual_seed(b * 7 + s))
            ids = ids.to(dev)
            # DBO needs two micro-batches on every attention rank
            splittable = b >= 2 * n_attn
            for mode in modes:
                dbo, xl = MODES[mode]
                if dbo and not splittable:
                    continue
                kw = dict(max_new_tokens=a.tokens, do_sample=False, use_decode_dbo=dbo,
                          num_decode_micro_batches=2, decode_use_crosslayer=xl,
                          prefill_mode="dbo" if dbo else "serial",
                          num_prefill_micro_batches=2 if dbo else 1, use_cuda_graph=True)
                # warm-up: captures this batch's graphs, and repeats (at most 4
                # times, every rank agreeing) while the caching allocator still
                # adds device segments, whose cudaMalloc stalls would land in
                # the measured call
                last = -1
                for i in range(4):
                    model.generate(ids, **kw)
                    torch.cuda.synchronize()
                    n = int(torch.cuda.memory_stats().get("num_device_alloc", 0))
                    grew = mx([1.0 if (i < 1 or n != last) else 0.0])[0]
                    last = n
                    if grew == 0.0:
                        break
                model.generate(ids, **kw)
                m = model._last_generation_metrics
                pf, tp = mx([m["prefill_ms"], m["decode_tpot_ms"]])
                row = {"mode": mode, "batch": b, "seq": s, "tokens": a.tokens, "n_gpus": world,
                       "topology": model.topology.tag(),
                       "prefill_ms": pf, "decode_tpot_ms": tp, "decode_tok_s": 1000.0 * b / tp}
                rows.append(row)
                if rank == 0:
                    print(json.dumps(row), flush=True)
            model.release_graphs()
    if rank == 0 and a.output:
        os.makedirs(os.path.dirname(os.path.abspath(a.output)) or ".", exist_ok=True)
        with open(a.output, "w") as f:
            json.dump(rows, f, indent=1)
    model.release_graphs()
    ctx.cleanup()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
