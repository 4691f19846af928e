"""P2P warmup between the attention and FFN ranks.

Reference: ``warmup_p2p`` (src/distributed/warmup.py:11-96): a few rounds of
1 KiB bidirectional isend/irecv, lower rank sending first, reporting cold and
warm latency. Here every attention rank exchanges with every FFN rank, on the
world group and on any extra (directional) groups, and latencies are taken
with a device synchronize only on CUDA (the reference calls
``torch.cuda.synchronize`` unconditionally, which fails without a GPU).
"""

from __future__ import annotations

import time
from typing import List, Optional

import torch
import torch.distributed as dist

from ..utils import device as devmod


def _pairs(ctx) -> List[int]:
    if ctx.role == "attention":
        return ctx.ffn_ranks()
    if ctx.role == "ffn":
        return ctx.attn_ranks()
    return []


def warmup_p2p(ctx, num_rounds: int = 3, tensor_size: int = 1024, dtype=torch.float16,
               groups: Optional[list] = None) -> dict:
    if ctx.world_size == 1 or not dist.is_initialized():
        return {"cold_latency_ms": 0.0, "warm_latency_ms": 0.0, "num_rounds": 0,
                "all_latencies_ms": []}
    device = ctx.device
    n = max(1, tensor_size // torch.tensor([], dtype=dtype).element_size())
    peers = _pairs(ctx)
    groups = groups if groups else [None]
    lat: List[float] = []
    for group in groups:
        for _ in range(num_rounds):
            devmod.synchronize()
            t0 = time.perf_counter()
            works = []
            for p in peers:
                s = torch.ones(n, dtype=dtype, device=device)
                r = torch.empty(n, dtype=dtype, device=device)
                if ctx.rank < p:
                    works.append(dist.isend(s, dst=p, group=group))
                    works.append(dist.irecv(r, src=p, group=group))
                else:
                    works.append(dist.irecv(r, src=p, group=group))
                    works.append(dist.isend(s, dst=p, group=group))
            for w in works:
                w.wait()
            devmod.synchronize()
            lat.append((time.perf_counter() - t0) * 1000)
    return {
        "cold_latency_ms": lat[0] if lat else 0.0,
        "warm_latency_ms": (sum(lat[1:]) / max(1, len(lat) - 1)) if len(lat) > 1 else 0.0,
        "num_rounds": num_rounds,
        "all_latencies_ms": lat,
    }
