#!/usr/bin/env python3
"""Runs one kernel of the decode step a few times on random inputs of the
Qwen3-30B-A3B shapes, for a profiler (ncu) to capture one launch:

    python -m afd_demo_b200.scripts.kernel_probe decode_attn 64 2048   # batch, kv length
    python -m afd_demo_b200.scripts.kernel_probe linear qkv 128         # or o_proj; tokens
    python -m afd_demo_b200.scripts.kernel_probe gate 128 32            # tokens, local experts
    python -m afd_demo_b200.scripts.kernel_probe moe 8192               # tokens (MoE block)
    python -m afd_demo_b200.scripts.kernel_probe prefill_attn 2048 4    # prompt length, batch

    ncu --set full --clock-control none -k regex:<kernel> -s 2 -c 1 -o out \\
        python -m afd_demo_b200.scripts.kernel_probe ...

Four calls, then a synchronize; no timing (times come from bench_kernels).
"""

from __future__ import annotations

import argparse
import os
import sys

if __package__ in (None, ""):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402

from afd_demo_b200 import ops  # noqa: E402

H, I, E, TOPK, NQ, NKV, D = 2048, 768, 128, 8, 32, 4, 128


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("op", choices=["decode_attn", "linear", "gate", "moe", "prefill_attn"])
    ap.add_argument("args", nargs="*")
    ap.add_argument("--calls", type=int, default=4)
    a = ap.parse_args(argv)
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*s, scale=1.0):
        return (torch.randn(*s, generator=g, device=dev) * scale).to(torch.bfloat16)

    if a.op == "decode_attn":
        B, kv = int(a.args[0]), int(a.args[1])
        kc, vc, q = rnd(B, NKV, kv + 8, D), rnd(B, NKV, kv + 8, D), rnd(B, NQ, D)
        pos = torch.tensor([kv - 1], device=dev, dtype=torch.int32)
        fn = lambda: ops.decode_attention_tc(q, kc, vc, 0, kv - 1, pos)  # noqa: E731
    elif a.op == "linear":
        which, T = a.args[0], int(a.args[1])
        if which == "qkv":
            w, x = rnd((NQ + 2 * NKV) * D, H, scale=0.02), rnd(T, H)
            fn = lambda: ops.linear(x, w)  # noqa: E731
        else:
            w, x, r = rnd(H, NQ * D, scale=0.02), rnd(T, NQ * D), rnd(T, H)
            fn = lambda: ops.linear(x, w, residual=r)  # noqa: E731
    elif a.op == "moe":
        T, I_ = int(a.args[0]), 768
        h, wr = rnd(T, H), rnd(E, H, scale=0.02)
        pn = torch.ones(H, device=dev, dtype=torch.bfloat16)
        wgu, wdn = rnd(E, 2 * I_, H, scale=0.02), rnd(E, H, I_, scale=0.02)
        fn = lambda: ops.moe_ffn(h, pn, wr, wgu, wdn, TOPK, 1e-6)  # noqa: E731
    elif a.op == "prefill_attn":
        S, B = int(a.args[0]), int(a.args[1]) if len(a.args) > 1 else 1
        q, kc, vc = rnd(B * S, NQ, D), rnd(B, NKV, S, D), rnd(B, NKV, S, D)
        pos = torch.zeros(1, device=dev, dtype=torch.int32)
        fn = lambda: ops.attention(q, kc, vc, 0, S, 0, pos)  # noqa: E731
    else:
        T, e_loc = int(a.args[0]), int(a.args[1]) if len(a.args) > 1 else E
        h, wr = rnd(T, H), rnd(E, H, scale=0.02)
        pn = torch.ones(H, device=dev, dtype=torch.bfloat16)
        fn = lambda: ops.moe_gate(h, pn, wr, TOPK, 1e-6, True, 0, e_loc)  # noqa: E731
    for _ in range(a.calls):
        fn()
    torch.cuda.synchronize()
    print("probe ok", a.op, *a.args)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
