#!/usr/bin/env python
"""Headline benchmark: Qwen3-30B-A3B bf16 decode throughput with
cross-layer decode DBO (plus serial decode TPOT and prefill TTFT, DBO vs
serial), random-init weights, synthetic token ids.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

N = 1 co-locates the attention and FFN roles on one GPU (two streams);
N > 1 runs one rank per GPU under torchrun: N/2 attention ranks (data parallel
over the batch) and N/2 FFN ranks (expert parallel, 128/(N/2) experts each),
with the fused peer-memory A2F/F2A path. Weak scaling: 32 sequences per GPU
(global batch 32 * N; 256 at 8 GPUs), prompt 256 tokens.

Timing: W untimed decode steps, then exactly K decode steps between a barrier
and a device synchronize, measured with CUDA events on the launching stream,
max over ranks. Each step reads the 61 GB of weights (far above the 126 MB
L2), so no L2 flush is needed. nvidia-smi clocks are sampled during the timed
region. The e2e number runs the public ``generate`` API with per-step
host->device token input and device->host token output from pinned memory.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = ("Qwen3-30B-A3B decode TPOT ms & prefill TTFT ms, DBO vs serial, at 1/2/4/8 B200")
# published cross-layer decode TPOT (ms) of the reference at seq 256, by batch,
# measured on 4xV100 (reference results/baseline_audit.csv, decode-dbo-crosslayer
# rows); vs_baseline = value / (1000 * b / TPOT)
REF_XL_TPOT_S256 = {2: 243.7, 4: 417.1, 8: 502.9, 16: 739.4, 32: 884.2, 64: 1274.1,
                    96: 1596.4, 128: 1757.4, 192: 1873.6}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", default="qwen3-30b-a3b")
    p.add_argument("--batch-per-gpu", type=int, default=32)
    p.add_argument("--batch", type=int, default=None, help="global batch (default 32 * gpus)")
    p.add_argument("--seq", type=int, default=256)
    p.add_argument("--tokens", type=int, default=20)
    p.add_argument("--comm-impl", default="auto", choices=["auto", "fused", "nccl"])
    p.add_argument("--no-serial", action="store_true", help="skip the serial comparison")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--profile", type=int, default=0, metavar="STEPS",
                   help="profiling run: prefill, then STEPS eager decode steps (DBO, cross-"
                        "layer); the last one inside the NVTX range 'profile_step'; no JSON")
    p.add_argument("--layers", type=int, default=None,
                   help="override the layer count (profiling small cases only)")
    p.add_argument("--attn-gpus", type=int, default=None,
                   help="attention ranks for N > 1 (default N/2; the rest are FFN ranks)")
    p.add_argument("--cells", choices=["auto", "none"], default="auto",
                   help="auto: also measure the benchmark configs' cells that match this N "
                        "(2 GPUs: serial b4 s128; 8 GPUs: prefill b32 s512, decode batch "
                        "16/64/256) and, for N > 1, the decode step over NCCL isend/irecv")
    return p.parse_args()


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons (every 50 ms).

    Started before the warm-up steps, so that nvidia-smi is already sampling
    when the timed region opens; `mark_start` / `mark_end` bracket the timed
    region on the host clock, and only samples stamped inside it are
    summarised. A region shorter than the sampling interval keeps the
    nearest sample on each side (`samples_in_region` says how many fell
    inside)."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.p = None

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    @staticmethod
    def _stamp(text: str):
        # nvidia-smi timestamp: "YYYY/MM/DD HH:MM:SS.mmm" in local time
        import datetime
        try:
            return datetime.datetime.strptime(text.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    @classmethod
    def summarise(cls, rows, t0=None, t1=None) -> dict:
        """rows: split CSV rows of Q. Samples inside [t0, t1] when given (else
        all); with none inside, the nearest one before and after."""
        parsed = []
        for r in rows:
            try:
                parsed.append((cls._stamp(r[0]), float(r[2]), float(r[3]),
                               [v.strip().lower() == "active" for v in r[6:10]]))
            except (ValueError, IndexError):
                continue
        inside = parsed
        n_in = len(parsed)
        if t0 is not None and t1 is not None and all(p[0] is not None for p in parsed):
            inside = [p for p in parsed if t0 <= p[0] <= t1]
            n_in = len(inside)
            if not inside:
                before = [p for p in parsed if p[0] < t0]
                after = [p for p in parsed if p[0] > t1]
                inside = before[-1:] + after[:1]
        sm = [p[1] for p in inside]
        reasons = sorted({n for p in inside for n, a in zip(cls.NAMES, p[3]) if a})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": inside[-1][2] if inside else None,
                "reasons": reasons, "samples": len(sm), "samples_in_region": n_in}

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        self.f.seek(0)
        rows = [r.strip().split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        return self.summarise(rows, self.t0, self.t1)


def reference_arm(args, rank):
    from afd_demo_b200.scripts.reference_arm import run_reference

    line = run_reference(args)
    if rank == 0:
        print(json.dumps(line), flush=True)


def measure_cells(model, args, B, S, T, local, world, timed, ctx):
    """The benchmark configs' cells that match this GPU count, measured on
    the same loaded model (device time, max over ranks):

    * 2 GPUs: serial prefill + serial decode, batch 4, prompt 128, 20 tokens,
      through ``generate`` (the reference's serial A/F baseline cell);
    * 8 GPUs: prefill TTFT at batch 32, prompt 512, DBO (2 micro-batches)
      and serial; cross-layer DBO and serial decode TPOT at batch 16, 64 and
      256, prompt 256, 20 tokens, through ``generate``;
    * N > 1: one prefill over the fused transport and over NCCL, compared
      (largest logit difference, share of equal greedy tokens);
    * N > 1: the headline decode step with the A2F/F2A hand-offs over NCCL
      isend/irecv (the reference's mechanism) instead of the fused
      peer-memory path, both run eagerly (the NCCL path keeps host-side work
      handles and is not graph-captured), next to the fused path's eager
      step, so the transport's own gain is visible.
    """
    import torch
    import torch.distributed as dist

    from afd_demo_b200 import ops
    from afd_demo_b200.parallel.transport import NcclTransport

    dev = f"cuda:{local}"
    V = model.config.vocab_size
    out = {}

    def mx(vals):
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def ids_of(b, s, seed):
        return torch.randint(0, V, (b, s), generator=torch.Generator().manual_seed(seed)).to(dev)

    def gen(ids, dbo, graph=True):
        model.generate(ids, max_new_tokens=T, do_sample=False, use_decode_dbo=dbo,
                       num_decode_micro_batches=2, decode_use_crosslayer=dbo,
                       prefill_mode="serial" if not dbo else "dbo",
                       num_prefill_micro_batches=1 if not dbo else 2, use_cuda_graph=graph)
        m = model._last_generation_metrics
        return m["prefill_ms"], m["decode_tpot_ms"]

    if args.gpus == 2 and B >= 4:
        ids = ids_of(4, 128, 7)
        gen(ids, False)  # warm: graphs for this batch
        pf, tp = mx(list(gen(ids, False)))
        out["serial_b4_s128_2gpu"] = {"prefill_ms": pf, "decode_tpot_ms": tp,
                                      "tok_s": 1000.0 * 4 / tp}
        model.release_graphs()
    if args.gpus == 8 and B >= 256:
        ids = ids_of(32, 512, 8)
        run = lambda mode, nmb: model.run_forward(ids, mode, nmb, crosslayer=True,  # noqa: E731
                                                  reset_cache=True)
        run("dbo", 2)
        run("serial", 1)
        t_dbo = timed(lambda: run("dbo", 2), 3) / 3
        t_ser = timed(lambda: run("serial", 1), 3) / 3
        out["prefill_b32_s512_8gpu"] = {"dbo_ms": t_dbo, "serial_ms": t_ser,
                                        "dbo_speedup": t_ser / t_dbo}
        sweep = {}
        for b in (16, 64, 256):
            ids = ids_of(b, S, 9 + b)
            row = {}
            for name, dbo in (("dbo_crosslayer", True), ("serial", False)):
                gen(ids, dbo)  # warm: graphs for this batch
                tp = mx([gen(ids, dbo)[1]])[0]
                row[name + "_tpot_ms"] = tp
                row[name + "_tok_s"] = 1000.0 * b / tp
            row["dbo_speedup"] = row["serial_tpot_ms"] / row["dbo_crosslayer_tpot_ms"]
            sweep[str(b)] = row
            model.release_graphs()
        out["decode_s256_8gpu"] = sweep
    if world > 1:
        # correctness record: the same prefill over the fused transport and
        # over NCCL isend/irecv, greedy tokens and logits compared
        agree = model.transport_agreement(ids_of(B, S, 1234), "dbo", 2, crosslayer=True)
        out["transport_agreement"] = dict(agree, batch=B, seq_len=S,
                                          mode="prefill DBO, cross-layer, fused vs NCCL")
        # eager decode steps: fused peer-memory transport vs NCCL isend/irecv
        logits = model.run_forward(ids_of(B, S, 1234), "dbo", 2, crosslayer=True,
                                   reset_cache=True)
        tok = torch.zeros(B, 1, dtype=torch.long, device=dev)
        r = model.local_batch(B)
        hold = {"l": logits}

        def step():
            if model.ctx.is_attention_node:
                tok[r.start:r.stop, 0] = ops.argmax(hold["l"])
            hold["l"] = model.decode_step(tok, "dbo", 2, True, False)

        for _ in range(2):
            step()
        fused_eager = timed(step, 5) / 5
        saved = (model.transport, model.comm_impl)
        model.transport = NcclTransport(ctx, model.hidden_size, model.dtype, model.device,
                                        crosslayer=True)
        model.comm_impl = "nccl"
        try:
            for _ in range(2):
                step()
            nccl_eager = timed(step, 5) / 5
        finally:
            model.transport, model.comm_impl = saved
        out["transport_decode_tpot_ms"] = {
            "batch": B, "mode": "decode DBO, cross-layer, eager (no CUDA graph)",
            "fused_peer_memory": fused_eager, "nccl_isend_irecv": nccl_eager,
            "fused_speedup": nccl_eager / fused_eager}
    return out


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world != args.gpus:
        if args.gpus > 1 and world == 1:
            raise SystemExit("run N > 1 under torchrun (one rank per GPU)")
    if args.impl == "reference":
        return reference_arm(args, rank)

    # one GPU: expandable segments let the caching allocator grow in place. With
    # both roles' streams handing tensors to each other, fixed-size segments
    # fragment and the pool keeps calling cudaMalloc for a dozen forwards.
    if world == 1:
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    from afd_demo_b200 import ops
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cuda")
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    ctx = get_distributed_context()
    ctx.initialize(DistributedConfig(world_size=world, rank=rank, local_rank=local,
                                     backend="nccl", timeout_s=120, n_attn=args.attn_gpus,
                                     master_addr=os.environ.get("MASTER_ADDR", "127.0.0.1"),
                                     master_port=os.environ.get("MASTER_PORT", "29500")))
    B = args.batch or args.batch_per_gpu * args.gpus
    S, T = args.seq, args.tokens
    cells_on = args.cells == "auto" and not args.profile and args.model == "qwen3-30b-a3b"
    # the 8-GPU prefill cell runs a 512-token prompt
    s_cells = 512 if (cells_on and args.gpus == 8) else S
    max_seq = max(S, s_cells) + max(T, args.warmup + args.steps + 2, args.profile + 2) + 8
    # only the full model is the benchmark's config; anything else is labelled
    # as what it is and gets no baseline ratio
    headline = args.model == "qwen3-30b-a3b" and args.layers is None
    model_name = args.model
    if args.layers is not None:
        from afd_demo_b200.config import PRESETS
        cfg = PRESETS[args.model]()
        cfg.num_hidden_layers = args.layers
        from afd_demo_b200 import config as _cfgmod
        _cfgmod.PRESETS["_bench"] = lambda: cfg
        args.model = "_bench"
    model = DisaggregatedQwenModel.from_pretrained(
        args.model, device=f"cuda:{local}", dtype=torch.bfloat16, max_seq_len=max_seq,
        max_batch_size=B, comm_impl=args.comm_impl, random_init=True, seed=0,
        num_micro_batches=2)
    # the model's tensors and modules are long-lived: move them out of the cyclic
    # collector's generations so a collection between timed regions stays short
    gc.collect()
    gc.freeze()
    V = model.config.vocab_size
    g = torch.Generator().manual_seed(1234)
    ids_host = torch.randint(0, V, (B, S), generator=g).pin_memory()
    ids = ids_host.to(f"cuda:{local}", non_blocking=True)
    torch.cuda.synchronize()

    if args.profile:
        # greedy tokens from the model, so the routing is that of real decoding;
        # the prefill of the second pass is NVTX range 'profile_prefill'
        model.run_forward(ids, "dbo", 2, crosslayer=True, reset_cache=True)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("profile_prefill")
        logits = model.run_forward(ids, "dbo", 2, crosslayer=True, reset_cache=True)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        tok = torch.zeros(B, 1, dtype=torch.long, device=f"cuda:{local}")
        r = model.local_batch(B)
        for i in range(args.profile):
            if model.ctx.is_attention_node:
                tok[r.start:r.stop, 0] = ops.argmax(logits)
            if i == args.profile - 1:
                torch.cuda.synchronize()
                torch.cuda.nvtx.range_push("profile_step")
            logits = model.run_forward(tok, "dbo", 2, crosslayer=True)
            if i == args.profile - 1:
                torch.cuda.synchronize()
                torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ctx.barrier()
        ctx.cleanup()
        return

    def bar():
        torch.cuda.synchronize()
        ctx.barrier()

    def timed(fn, n, clocks=None):
        bar()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        # no cyclic-GC pause inside the timed region (as in generate)
        gc.disable()
        if clocks is not None:
            clocks.mark_start()
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        if clocks is not None:
            clocks.mark_end()
        gc.enable()
        ctx.barrier()
        ms = s.elapsed_time(e)
        if world > 1:
            t = torch.tensor([ms], device=f"cuda:{local}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # ---------------- prefill TTFT: serial vs DBO (2 micro-batches)
    def prefill(mode, nmb):
        return model.run_forward(ids, mode, nmb, crosslayer=True, reset_cache=True)

    # warm-up until the caching allocator stops growing (every rank agrees):
    # a DBO prefill hands tensors between streams, and the first forwards add
    # device segments (cudaMalloc stalls of up to hundreds of ms) for several
    # rounds; at most 12 rounds
    last = -1
    for i in range(12):
        prefill("dbo", 2)
        prefill("serial", 1)
        torch.cuda.synchronize()
        n = int(torch.cuda.memory_stats().get("num_device_alloc", 0))
        grew = torch.tensor([1 if (i < 1 or n != last) else 0], device=f"cuda:{local}")
        if world > 1:
            dist.all_reduce(grew, op=dist.ReduceOp.MAX)
        last = n
        if int(grew.item()) == 0:
            break
    ttft_dbo = timed(lambda: prefill("dbo", 2), 3) / 3
    ttft_serial = timed(lambda: prefill("serial", 1), 3) / 3

    # ---------------- decode: device-timed graph replays
    def decode_run(mode, nmb, crosslayer, warm, steps):
        logits = prefill("dbo", 2)
        tok = torch.zeros(B, 1, dtype=torch.long, device=f"cuda:{local}")
        r = model.local_batch(B)
        holder = {}

        def step():
            if model.ctx.is_attention_node:
                tok[r.start:r.stop, 0] = ops.argmax(holder.get("logits", logits))
            holder["logits"] = model.decode_step(tok, mode, nmb, crosslayer, True)

        # the sampler starts before the warm-up, so it is sampling when the
        # timed region opens; only its samples inside the region are kept
        clocks = ClockSampler(local)
        clocks.start()
        for _ in range(warm):
            step()
        ops.LAUNCHES.reset()
        ms = timed(step, steps, clocks)
        clk = clocks.stop()
        # kernels of this package in the timed region: graph contents per
        # replay plus the argmax launched outside the graph each step
        per_graph = sum(gr.launches for gr in model._graphs.values())
        launches = steps * per_graph + ops.LAUNCHES.reset()
        model.release_graphs()
        return ms / steps, clk, launches

    tpot_xl, clk, launches = decode_run("dbo", 2, True, args.warmup, args.steps)
    tpot_serial = None
    if not args.no_serial:
        tpot_serial, _, _ = decode_run("serial", 1, False, 2, max(3, min(args.steps, 10)))

    # ---------------- e2e through the public generate API (host I/O per step)
    e2e = None
    if not args.no_e2e:
        def gen():
            ids_dev = ids_host.to(f"cuda:{local}", non_blocking=True)
            model.generate(ids_dev, max_new_tokens=T, do_sample=False, use_decode_dbo=True,
                           num_decode_micro_batches=2, decode_use_crosslayer=True,
                           prefill_mode="dbo", num_prefill_micro_batches=2,
                           use_cuda_graph=True, host_io=True)
            return model._last_generation_metrics

        met0 = gen()  # warm (graphs for this batch)
        dbg = os.environ.get("AFD_BENCH_DEBUG")
        keys = ("num_device_alloc", "num_device_free", "num_alloc_retries", "num_sync_all_streams")
        st0 = torch.cuda.memory_stats() if dbg else {}
        t0 = time.perf_counter()
        met = gen()
        if dbg:
            st1 = torch.cuda.memory_stats()
            print(f"[rank {rank}] e2e warm {met0} timed {met} wall {1e3 * (time.perf_counter() - t0):.0f} ms "
                  f"alloc-stats {[(k, st1.get(k, 0) - st0.get(k, 0)) for k in keys]}",
                  file=sys.stderr, flush=True)
        tp = torch.tensor([met["decode_tpot_ms"], met["prefill_ms"]], device=f"cuda:{local}")
        if world > 1:
            dist.all_reduce(tp, op=dist.ReduceOp.MAX)
        e2e_tpot = float(tp[0])
        e2e = {"value": 1000.0 * B / e2e_tpot, "unit": "tok/s", "decode_tpot_ms": e2e_tpot,
               "prefill_ms": float(tp[1]),
               "h2d_bytes_per_step": int(len(model.local_batch(B)) * 8)
               if model.ctx.is_attention_node else 0,
               "d2h_bytes_per_step": int(len(model.local_batch(B)) * 8)
               if model.ctx.is_attention_node else 0,
               "api": "DisaggregatedQwenModel.generate(host_io=True, use_cuda_graph=True)"}

    cells = None
    if cells_on:
        # the cells are extra keys: an error in one (the same on every rank,
        # e.g. a batch the topology cannot split) must not cost the headline line
        try:
            cells = measure_cells(model, args, B, S, T, local, world, timed, ctx)
        except Exception as e:  # noqa: BLE001
            print(f"bench: cells skipped: {type(e).__name__}: {e}", file=sys.stderr)
            cells = {"error": f"{type(e).__name__}: {e}"[:300]}
            model.release_graphs()

    value = 1000.0 * B / tpot_xl
    ref = REF_XL_TPOT_S256.get(B) if (S == 256 and headline) else None
    mc = model.config
    model_label = ("Qwen3-30B-A3B" if headline else
                   f"{model_name} ({mc.num_hidden_layers} layers, hidden {mc.hidden_size}, "
                   f"{mc.num_experts} experts)")
    topo = model.topology
    par = ("colocated attention+FFN on 1 GPU" if topo.colocated else
           f"{topo.n_attn}A{topo.n_ffn}F: attention dp{topo.n_attn}, FFN ep{topo.n_ffn}")
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tok/s (decode, 1000*batch/TPOT)",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tpot_xl,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": (value / (1000.0 * B / ref)) if ref else None,
        "vs_baseline_basis": ("the reference's published cross-layer decode throughput at the "
                              "same batch and prompt, measured on 4x V100-32GB (other "
                              "hardware); not a same-box comparison") if ref else None,
        "dtype": "bf16",
        "data": "synthetic token ids uniform in [0, vocab), random-init weights",
        "config": {"model": model_label, "global_batch": B, "seq_len": S,
                   "decode_tokens": T, "parallelism": par,
                   "mode": "decode DBO, cross-layer, 2 micro-batches, CUDA graph per step",
                   "comm_impl": model.comm_impl,
                   "l2": ("inputs larger than L2 (all expert weights read every step)"
                          if headline else "small model: weights may stay in L2 (contract "
                          "and smoke runs only, not a benchmark number)")},
        "decode_tpot_ms": {"dbo_crosslayer": tpot_xl, "serial": tpot_serial},
        "dbo_speedup_decode": (tpot_serial / tpot_xl) if tpot_serial else None,
        "prefill_ttft_ms": {"dbo": ttft_dbo, "serial": ttft_serial,
                            "speedup": ttft_serial / ttft_dbo},
        "clocks": clk,
        "cells": cells,
        "e2e": e2e,
        "gpu_launches": launches,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.release_graphs()
    ctx.barrier()
    ctx.cleanup()


if __name__ == "__main__":
    main()
