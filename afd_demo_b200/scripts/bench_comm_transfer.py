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

Host-timed section (2 ranks; also the only section with ``--backend cpu``,
gloo): the reference's own measurement and output schema -- per payload size
the sender's isend enqueue time, isend start -> Work.wait return, the
receiver's irecv post -> Work.wait return and, with ``--blocking``, blocking
send / recv, each summarised as mean / median / p95 / min / max over
``--iters`` host perf_counter samples after a barrier and a ``--sender-delay-ms``
pause. With NCCL, Work.wait only orders the stream, so these spans are host
enqueue figures, not transfer times; the device-timed section above is the
measurement. JSON: ``{"meta", "results"}`` as the reference writes it, plus
``"device"`` for the device-timed rows; CSV: the reference's nine columns
(device rows go to ``<stem>_device.csv``).

Launch: torchrun --nproc-per-node N -m afd_demo_b200.scripts.bench_comm_transfer
"""

from __future__ import annotations

import argparse
import csv
import json
import os
import statistics
import sys
import time
from pathlib import Path
from typing import Dict, List, Optional

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
    # host-timed section (the reference's flags and defaults)
    ap.add_argument("--backend", choices=["auto", "cuda", "cpu"], default="auto")
    ap.add_argument("--dtype", choices=sorted(HOST_DTYPES), default="float16")
    ap.add_argument("--sender-delay-ms", type=float, default=1.0)
    ap.add_argument("--blocking", action="store_true")
    ap.add_argument("--host-only", action="store_true", help="skip the device-timed section")
    ap.add_argument("--device-only", action="store_true", help="skip the host-timed section")
    return ap.parse_args()


HOST_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
               "uint8": torch.uint8}
HOST_CSV_COLUMNS = ("size_mib_requested", "tensor_mib", "tensor_bytes", "sender_enqueue_mean_ms",
                    "sender_completion_mean_ms", "receiver_wait_mean_ms", "blocking_send_mean_ms",
                    "blocking_recv_mean_ms", "completion_bandwidth_mib_s")


def _summary(samples: List[float]) -> Dict[str, float]:
    """mean / median / p95 (linear interpolation between order statistics) /
    min / max of host-timed samples in ms."""
    if not samples:
        return {"mean": 0.0, "median": 0.0, "p95": 0.0, "min": 0.0, "max": 0.0}
    t = sorted(samples)
    pos = 0.95 * (len(t) - 1)
    i = int(pos)
    p95 = t[i] + (t[min(i + 1, len(t) - 1)] - t[i]) * (pos - i)
    return {"mean": statistics.fmean(t), "median": statistics.median(t), "p95": p95,
            "min": t[0], "max": t[-1]}


def host_timed(a, rank: int, device: torch.device, backend: str, dist_backend: str
               ) -> Optional[dict]:
    """The reference's two-rank host-timed p2p measurement (rank 0 sends to
    rank 1). Returns the merged {"meta", "results"} dict on rank 0."""
    sync = torch.cuda.synchronize if device.type == "cuda" else (lambda: None)
    dt = HOST_DTYPES[a.dtype]
    el = torch.empty((), dtype=dt).element_size()
    delay = a.sender_delay_ms / 1e3
    peer = 1 - rank
    local = []
    for si, size in enumerate(float(x) for x in a.sizes_mib.split(",") if x):
        x = torch.empty(max(1, -(-max(1, int(size * 2**20)) // el)), dtype=dt, device=device)
        recv = torch.empty_like(x)
        nbytes = x.numel() * el

        def exchange(tag: int, blocking: bool) -> float:
            dist.barrier()
            sync()
            if rank == 0:
                if delay > 0:
                    time.sleep(delay)
                t0 = time.perf_counter()
                if blocking:
                    dist.send(x, dst=peer, tag=tag)
                    return (time.perf_counter() - t0) * 1e3, None
                w = dist.isend(x, dst=peer, tag=tag)
                t1 = time.perf_counter()
                w.wait()
                return (t1 - t0) * 1e3, (time.perf_counter() - t0) * 1e3
            t0 = time.perf_counter()
            if blocking:
                dist.recv(recv, src=peer, tag=tag)
            else:
                dist.irecv(recv, src=peer, tag=tag).wait()
            return (time.perf_counter() - t0) * 1e3, None

        for i in range(a.warmup):
            exchange(10_000 + i, False)
        dist.barrier()
        enq, comp, rwait, bsend, brecv = [], [], [], [], []
        for i in range(a.iters):
            t_a, t_b = exchange(20_000 + si * 10_000 + i, False)
            if rank == 0:
                enq.append(t_a)
                comp.append(t_b)
            else:
                rwait.append(t_a)
        dist.barrier()
        if a.blocking:
            for i in range(a.iters):
                t_a, _ = exchange(200_000 + si * 10_000 + i, True)
                (bsend if rank == 0 else brecv).append(t_a)
            dist.barrier()
        local.append({"size_mib_requested": size, "tensor_bytes": nbytes,
                      "tensor_mib": nbytes / 2**20, "enq": enq, "comp": comp, "rwait": rwait,
                      "bsend": bsend, "brecv": brecv})
    both: List[Optional[list]] = [None, None]
    dist.all_gather_object(both, local)
    if rank != 0:
        return None
    rows = []
    for snd, rcv in zip(both[0], both[1]):
        comp = _summary(snd["comp"])
        row = {"size_mib_requested": snd["size_mib_requested"], "tensor_bytes": snd["tensor_bytes"],
               "tensor_mib": snd["tensor_mib"], "sender_enqueue_ms": _summary(snd["enq"]),
               "sender_completion_ms": comp, "receiver_wait_ms": _summary(rcv["rwait"]),
               "completion_bandwidth_mib_s": (snd["tensor_mib"] * 1e3 / comp["mean"]
                                              if comp["mean"] > 0 else 0.0)}
        if a.blocking:
            row["blocking_send_ms"] = _summary(snd["bsend"])
            row["blocking_recv_ms"] = _summary(rcv["brecv"])
        rows.append(row)
    meta = {"backend": backend, "dist_backend": dist_backend, "dtype": a.dtype,
            "warmup": a.warmup, "iters": a.iters, "sender_delay_ms": a.sender_delay_ms,
            "world_size": 2,
            "note": ("host perf_counter spans: isend start -> Work.wait return (sender), "
                     "irecv post -> Work.wait return (receiver); with NCCL, Work.wait only "
                     "orders the stream, so see 'device' for device-timed transfers")}
    return {"meta": meta, "results": rows}


def write_host_csv(path: Path, host: dict) -> None:
    with path.open("w", newline="") as f:
        wr = csv.DictWriter(f, fieldnames=list(HOST_CSV_COLUMNS))
        wr.writeheader()
        for r in host["results"]:
            wr.writerow({
                "size_mib_requested": r["size_mib_requested"], "tensor_mib": r["tensor_mib"],
                "tensor_bytes": r["tensor_bytes"],
                "sender_enqueue_mean_ms": r["sender_enqueue_ms"]["mean"],
                "sender_completion_mean_ms": r["sender_completion_ms"]["mean"],
                "receiver_wait_mean_ms": r["receiver_wait_ms"]["mean"],
                "blocking_send_mean_ms": r.get("blocking_send_ms", {}).get("mean", ""),
                "blocking_recv_mean_ms": r.get("blocking_recv_ms", {}).get("mean", ""),
                "completion_bandwidth_mib_s": r["completion_bandwidth_mib_s"]})


def main() -> int:
    a = parse()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world < 2:
        raise SystemExit("needs >= 2 ranks (1 attention + FFN ranks)")
    backend = a.backend
    if backend == "auto":
        backend = "cuda" if torch.cuda.is_available() else "cpu"
    out_path = Path(a.output)
    csv_path = Path(a.csv_output) if a.csv_output else out_path.with_suffix(".csv")
    if backend == "cpu":
        if world != 2:
            raise SystemExit("the host-timed (cpu/gloo) benchmark runs on exactly 2 ranks")
        dist.init_process_group("gloo")
        host = host_timed(a, rank, torch.device("cpu"), "cpu", "gloo")
        if rank == 0:
            out_path.parent.mkdir(parents=True, exist_ok=True)
            out_path.write_text(json.dumps(host, indent=2))
            write_host_csv(csv_path, host)
            print(f"wrote {out_path} and {csv_path}")
        dist.barrier()
        dist.destroy_process_group()
        return 0

    from afd_demo_b200 import ops

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    dist.init_process_group("nccl", device_id=dev)
    host = None
    if world == 2 and not a.device_only:
        host = host_timed(a, rank, dev, "cuda", "nccl")
    if a.host_only:
        if rank == 0:
            out_path.parent.mkdir(parents=True, exist_ok=True)
            out_path.write_text(json.dumps(host, indent=2))
            write_host_csv(csv_path, host)
            print(f"wrote {out_path} and {csv_path}")
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
        return 0
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
        device = {"world": world, "n_ffn": n_ffn, "iters": a.iters, "warmup": a.warmup,
                  "device_timed": True, "status_ok": int(ok) == 0, "results": results}
        out = dict(host) if host is not None else {}
        out["device"] = device
        out_path.parent.mkdir(parents=True, exist_ok=True)
        out_path.write_text(json.dumps(out, indent=2))
        dev_csv = csv_path.with_name(csv_path.stem + "_device.csv")
        keys = sorted({k for r in results for k in r})
        with dev_csv.open("w", newline="") as f:
            wr = csv.DictWriter(f, fieldnames=keys)
            wr.writeheader()
            wr.writerows(results)
        if host is not None:
            write_host_csv(csv_path, host)
        print(f"wrote {out_path}, {dev_csv}" + (f" and {csv_path}" if host is not None else ""))
    for p_ in peer.values():
        C.ipc_close(p_)
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
