#!/usr/bin/env python3
"""A2F / F2A transfer benchmark: NCCL isend/irecv vs the fused peer-store path.

Reference: scripts/bench_comm_transfer.py (2 ranks, host-observed NCCL
isend/irecv timings). Here rank 0 is the attention GPU and ranks 1..N-1 are
FFN GPUs (1, 2, 4 or 7 of them); every number is device time (CUDA events on
each rank's stream between a barrier and a synchronize), max over ranks.

Payload per transfer: bf16 hidden states [tokens, 2048] of normal(0, 1)
values plus int32 top-8 expert ids [tokens, 8] uniform in [0, 128), sized
from --sizes-mib (hidden part). Directions:

* a2f: rank 0 -> every FFN rank (the attention o_proj hand-off);
* f2a: every FFN rank -> rank 0, each into its own slot (the combine return).

Implementations:

* nccl:  one isend per (iteration, peer), matching irecvs;
* fused: a peer-store kernel writes the payload into the peers' IPC-mapped
  buffers with 16-byte NVLink stores and its last CTA raises a release flag;
  receivers run the bounded flag-wait kernel;
* gemm (a2f only): the real fused path -- the o_proj tcgen05 GEMM
  ([tokens, 4096] x [4096, 2048] + residual) whose epilogue stores the output
  tile into every FFN GPU -- against the same GEMM stored locally followed by
  NCCL isends;
* moe (f2a only): the real fused return -- every FFN rank runs its slice of
  the Qwen3-30B-A3B expert layer (128 / n_ffn experts, top-8 routing) whose
  combine stores each token's partial sum (FFN rank 0 adds the residual)
  straight into the attention GPU's slot for that rank -- against the same
  layer stored locally followed by NCCL isends. Its roofline is the slowest
  of the local expert weights over HBM, the FLOPs over the GEMM peak and the
  returned rows over NVLink.

Roofline of a transfer: bytes crossing the busiest GPU's NVLink ports
(tokens * row bytes * peers) / 770 GB/s (measured peer copy bandwidth per
direction); of the fused GEMM: the slower of that and FLOPs / 1656.5 TFLOP/s.

Launch: torchrun --nproc-per-node N -m afd_demo_b200.scripts.bench_comm_transfer
"""

from __future__ import annotations

import argparse
import csv
import json
import os
import statistics
import sys
from pathlib import Path
from typing import Dict, List

import torch
import torch.distributed as dist

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

H = 2048
TOPK = 8
LINK_GBS = 770.0


def _peaks():
    """HBM bytes/s and bf16 FLOP/s: MEASURED_PEAKS.json when present."""
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]) * 1e9, float(d["bf16_tflops"]) * 1e12
    return 6.65e12, 1.59e15


HBM_BPS, GEMM_FLOPS = _peaks()
GEMM_TFLOPS = GEMM_FLOPS / 1e12


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--sizes-mib", default="0.004,0.031,1,16,32")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--impls", default="nccl,fused,gemm,moe")
    ap.add_argument("--directions", default="a2f,f2a")
    ap.add_argument("--output", default="results/comm_bench/comm_transfer.json")
    ap.add_argument("--csv-output", default="")
    ap.add_argument("--timeout-ms", type=float, default=20000.0)
    return ap.parse_args()


def main() -> int:
    a = parse()
    from afd_demo_b200 import ops

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world < 2:
        raise SystemExit("needs >= 2 ranks (1 attention + FFN ranks)")
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    dist.init_process_group("nccl", device_id=dev)
    C = ops.ext()
    n_ffn = world - 1
    sizes = [float(s) for s in a.sizes_mib.split(",") if s]
    max_tok = max(1, int(max(sizes) * 2**20) // (H * 2))
    row_bytes = H * 2 + TOPK * 4
    slot = ((max_tok * row_bytes + 255) // 256) * 256
    # region: flags (4 KiB) | n_ffn slots (rank 0 receives F2A) or 1 slot
    region = C.ipc_alloc(4096 + slot * max(1, n_ffn), local)
    base = region.data_ptr()
    handles: List[bytes] = [None] * world  # type: ignore
    dist.all_gather_object(handles, bytes(C.ipc_handle(region)))
    peer = {r: int(C.ipc_open(handles[r])) for r in range(world) if r != rank}
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(rank)
    results = []

    def timed(fn, iters) -> float:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(iters):
            fn(i)
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    flag_value = [0]

    for size in sizes:
        tokens = max(1, int(size * 2**20) // (H * 2))
        hidden = torch.randn(tokens, H, generator=g, device=dev).to(torch.bfloat16)
        ids = torch.randint(0, 128, (tokens, TOPK), generator=g, device=dev, dtype=torch.int32)
        payload = torch.cat([hidden.view(torch.uint8).view(-1), ids.view(torch.uint8).view(-1)])
        nbytes = payload.numel()
        pad = (-nbytes) % 16
        if pad:
            payload = torch.cat([payload, torch.zeros(pad, dtype=torch.uint8, device=dev)])
        recv = torch.empty_like(payload)
        for direction in a.directions.split(","):
            senders = [0] if direction == "a2f" else list(range(1, world))
            receivers = list(range(1, world)) if direction == "a2f" else [0]
            link_bytes = nbytes * n_ffn  # through rank 0's ports either way
            row = {"direction": direction, "n_ffn": n_ffn, "size_mib_requested": size,
                   "tokens": tokens, "tensor_bytes": nbytes, "tensor_mib": nbytes / 2**20,
                   "roofline_ms": link_bytes / (LINK_GBS * 1e9) * 1e3}
            if "nccl" in a.impls:
                def nccl_step(i):
                    works = []
                    if rank in senders:
                        for r in receivers:
                            works.append(dist.isend(payload, dst=r))
                    if rank in receivers:
                        for r in senders:
                            works.append(dist.irecv(recv, src=r))
                    for w in works:
                        w.wait()

                for i in range(a.warmup):
                    nccl_step(i)
                row["nccl_ms"] = timed(nccl_step, a.iters)
            if "fused" in a.impls:
                def dst_addr(r_recv: int, r_send: int) -> int:
                    slot_idx = 0 if direction == "a2f" else r_send - 1
                    return peer[r_recv] + 4096 + slot_idx * slot

                def flag_addr(b: int, r_send: int) -> int:
                    return b + 4 * (0 if direction == "a2f" else r_send)

                def fused_step(i):
                    flag_value[0] += 1
                    v = flag_value[0]
                    if rank in senders:
                        grid = max(1, min(4 * 148, payload.numel() // (16 * 512)))
                        C.peer_copy(payload, [dst_addr(r, rank) for r in receivers],
                                    [flag_addr(peer[r], rank) for r in receivers], v, counter,
                                    None, grid)
                    if rank in receivers:
                        C.wait_flags([flag_addr(base, r) for r in senders], v, status,
                                     int(a.timeout_ms * 1e6), None)

                for i in range(a.warmup):
                    fused_step(i)
                row["fused_ms"] = timed(fused_step, a.iters)
            if "gemm" in a.impls and direction == "a2f":
                K = 4096
                x = torch.randn(tokens, K, generator=g, device=dev).to(torch.bfloat16)
                w = (torch.randn(H, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
                res = hidden
                out = torch.empty(tokens, H, device=dev, dtype=torch.bfloat16)

                def gemm_fused(i):
                    flag_value[0] += 1
                    v = flag_value[0]
                    if rank == 0:
                        ops.linear(x, w, residual=res, out=out,
                                   peers=[peer[r] + 4096 for r in receivers],
                                   flags=[peer[r] for r in receivers], signal_value=v,
                                   done_counter=counter, status=status)
                    else:
                        C.wait_flags([base], v, status, int(a.timeout_ms * 1e6), None)

                def gemm_nccl(i):
                    works = []
                    if rank == 0:
                        ops.linear(x, w, residual=res, out=out)
                        works = [dist.isend(out, dst=r) for r in receivers]
                    else:
                        works = [dist.irecv(recv[:out.numel() * 2].view(torch.bfloat16), src=0)]
                    for wk in works:
                        wk.wait()

                for i in range(a.warmup):
                    gemm_fused(i)
                    gemm_nccl(i)
                row["gemm_fused_ms"] = timed(gemm_fused, a.iters)
                row["gemm_nccl_ms"] = timed(gemm_nccl, a.iters)
                flops = 2.0 * tokens * K * H
                row["gemm_roofline_ms"] = max(flops / (GEMM_TFLOPS * 1e12),
                                              tokens * H * 2 * n_ffn / (LINK_GBS * 1e9)) * 1e3
                row["gemm_fused_roofline_frac"] = row["gemm_roofline_ms"] / row["gemm_fused_ms"]
            if "moe" in a.impls and direction == "f2a":
                E, I, Ek = 128, 768, 128 // n_ffn
                fi = rank - 1
                if rank > 0:
                    w_gu = (torch.randn(Ek, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
                    w_dn = (torch.randn(Ek, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
                gl = torch.Generator(device=dev).manual_seed(7)  # same routing on every rank
                rid = torch.stack([torch.randperm(E, device=dev, generator=gl)[:TOPK]
                                   for _ in range(min(tokens, 4096))])
                rid = rid.repeat((tokens + rid.shape[0] - 1) // rid.shape[0], 1)[:tokens]
                rid = rid.to(torch.int32).contiguous()
                rw = torch.full((tokens, TOPK), 1.0 / TOPK, device=dev)
                xn = hidden
                res = hidden if rank == 1 else None
                out_loc = torch.empty(tokens, H, device=dev, dtype=torch.bfloat16)

                def moe_fused(i):
                    flag_value[0] += 1
                    v = flag_value[0]
                    if rank > 0:
                        ops.moe_experts(xn, rid, rw, w_gu, w_dn, fi * Ek, residual=res,
                                        peers=[dst_addr(0, rank)], seg_offsets=[0, tokens],
                                        flags=[flag_addr(peer[0], rank)], signal_value=v,
                                        done_counter=counter)
                    else:
                        C.wait_flags([flag_addr(base, r) for r in senders], v, status,
                                     int(a.timeout_ms * 1e6), None)

                def moe_nccl(i):
                    works = []
                    if rank > 0:
                        ops.moe_experts(xn, rid, rw, w_gu, w_dn, fi * Ek, residual=res,
                                        out=out_loc)
                        works = [dist.isend(out_loc, dst=0)]
                    else:
                        works = [dist.irecv(recv[:tokens * H * 2].view(torch.bfloat16), src=r)
                                 for r in senders]
                    for wk in works:
                        wk.wait()

                for i in range(a.warmup):
                    moe_fused(i)
                    moe_nccl(i)
                row["moe_fused_ms"] = timed(moe_fused, a.iters)
                row["moe_nccl_ms"] = timed(moe_nccl, a.iters)
                hit = torch.zeros(E, dtype=torch.bool, device=dev)
                hit[rid.view(-1).long()] = True
                loc_hit = max(int(hit[r * Ek:(r + 1) * Ek].sum()) for r in range(n_ffn))
                wbytes = loc_hit * 3 * I * H * 2
                flops = 2.0 * tokens * TOPK * 3 * I * H / n_ffn
                row["moe_local_experts_hit"] = loc_hit
                row["moe_roofline_ms"] = max(wbytes / HBM_BPS, flops / GEMM_FLOPS,
                                             tokens * H * 2 * n_ffn / (LINK_GBS * 1e9)) * 1e3
                row["moe_fused_roofline_frac"] = row["moe_roofline_ms"] / row["moe_fused_ms"]
            for k in ("nccl_ms", "fused_ms"):
                if k in row:
                    row[k.replace("_ms", "_gbs")] = link_bytes / (row[k] * 1e-3) / 1e9
                    row[k.replace("_ms", "_roofline_frac")] = row["roofline_ms"] / row[k]
            results.append(row)
            if rank == 0:
                print(json.dumps(row), flush=True)
    torch.cuda.synchronize()
    st = status.cpu()
    ok = torch.tensor([int(st[0])], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MAX)
    if rank == 0:
        out = {"world": world, "n_ffn": n_ffn, "iters": a.iters, "warmup": a.warmup,
               "device_timed": True, "status_ok": int(ok) == 0, "results": results}
        p = Path(a.output)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(json.dumps(out, indent=2))
        csv_path = Path(a.csv_output) if a.csv_output else p.with_suffix(".csv")
        keys = sorted({k for r in results for k in r})
        with csv_path.open("w", newline="") as f:
            wr = csv.DictWriter(f, fieldnames=keys)
            wr.writeheader()
            wr.writerows(results)
        print(f"wrote {p} and {csv_path}")
    for p_ in peer.values():
        C.ipc_close(p_)
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
