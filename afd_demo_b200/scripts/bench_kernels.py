#!/usr/bin/env python3
"""Per-kernel timings on Qwen3-30B-A3B shapes with roofline fractions.

Each op is timed with CUDA events around one replay of a CUDA graph holding
`--iters` back-to-back calls (after `--warmup` eager calls), on the launching
stream, with a device synchronize on both sides: device time per call, as in
the captured decode step. Weights rotate over enough distinct copies that every launch
reads them from HBM (the set of copies is larger than the 126 MB L2), as the
48 distinct layers of the model do. Achieved bandwidth = algorithmic bytes /
time; achieved FLOP rate = algorithmic FLOPs / time; fractions are of the
measured peaks in MEASURED_PEAKS.json when present (HBM copy bandwidth and
cuBLAS bf16 burst throughput), else of earlier B200 measurements (6.65 TB/s,
1.59 PFLOP/s).

    python -m afd_demo_b200.scripts.bench_kernels [--tokens 16,32,64,128] [--json out.json]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
if __package__ in (None, ""):
    sys.path.insert(0, REPO)

from afd_demo_b200 import ops  # noqa: E402

L2_BYTES = 126 * 2**20


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]) * 1e9, float(d["bf16_tflops"]) * 1e12, "of measured"
    return 6.65e12, 1.59e15, "of fallback"


def copies_for(nbytes: int) -> int:
    return max(2, -(-2 * L2_BYTES // max(nbytes, 1)))


def timeit(fn, iters: int, warmup: int, graph: bool = True) -> float:
    """Device time per call. With `graph`, the `iters` calls are captured in
    one CUDA graph and the replay is timed, as the decode step replays them;
    otherwise host launch time is included."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            for i in range(warmup):  # allocations of the capture stream
                fn(i)
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for i in range(iters):
                fn(i)
        g.replay()  # first replay uploads the graph
        torch.cuda.synchronize()
        s.record()
        g.replay()
        e.record()
    else:
        s.record()
        for i in range(iters):
            fn(i)
        e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / iters  # us


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--tokens", default="16,32,64,128")
    ap.add_argument("--kv-len", type=int, default=276)
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--json", default="")
    ap.add_argument("--sections", default="decode,attention,prefill",
                    help="comma list of: decode (per-layer decode kernels by token count), "
                         "attention (decode attention over long caches), prefill (prefill "
                         "GEMMs and attention), prefill_attn (prefill attention only), tiling "
                         "(every token-block / split-K choice of the qkv and o_proj GEMMs)")
    ap.add_argument("--attn-batches", default="16,64")
    ap.add_argument("--attn-kv", default="256,1024,2048,4096")
    ap.add_argument("--prefill-attn-seqs", default="256",
                    help="prompt lengths of the prefill attention rows (batch = tokens / length)")
    ap.add_argument("--prefill-attn-variants", default=None,
                    help="prefill attention kernels to time: tc (two heads per CTA), tc1, mma "
                         "(default: the op layer's choice)")
    a = ap.parse_args(argv)
    sections = set(a.sections.split(","))
    if a.prefill_attn_variants is None:
        a.prefill_attn_variants = ops._PREFILL_ATTN
    dev = torch.device("cuda")
    bw, fl, tag = peaks()
    H, I, E, k, nq, nkv, D = 2048, 768, 128, 8, 32, 4, 128
    QKV = (nq + 2 * nkv) * D
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*s, scale=0.02):
        return (torch.randn(*s, generator=g, device=dev) * scale).to(torch.bfloat16)

    rows = []

    def report(name, T, us, nbytes, flops):
        r = {"op": name, "tokens": T, "us": round(us, 2),
             "GB/s": round(nbytes / us / 1e3, 1), "hbm_frac": round(nbytes / us / 1e-6 / bw, 3),
             "TFLOP/s": round(flops / us / 1e6, 1), "tc_frac": round(flops / us / 1e-6 / fl, 3)}
        rows.append(r)
        print(f"{name:28s} T={T:5d} {us:9.2f} us  {r['GB/s']:8.1f} GB/s ({r['hbm_frac']:.2f} {tag})"
              f"  {r['TFLOP/s']:7.1f} TFLOP/s ({r['tc_frac']:.3f} {tag})", flush=True)

    n_qkv = copies_for(QKV * H * 2)
    w_qkv = [rnd(QKV, H) for _ in range(n_qkv)]
    n_o = copies_for(H * nq * D * 2)
    w_o = [rnd(H, nq * D) for _ in range(n_o)]
    n_e = 2  # one layer of experts is 1.2 GB: two copies alternate
    w_gu = [rnd(E, 2 * I, H) for _ in range(n_e)]
    w_dn = [rnd(E, H, I) for _ in range(n_e)]
    w_r = [rnd(E, H) for _ in range(n_qkv)]
    pn = (1 + 0.1 * torch.randn(H, device=dev)).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
    rope = ops.rope_table(4096, D, 1e6, dev)

    for T in ([int(t) for t in a.tokens.split(",")] if "decode" in sections else []):
        x = rnd(T, H, scale=1.0)
        o_in = rnd(T, nq * D, scale=1.0)
        report("sum_rmsnorm (2 parts)", T,
               timeit(lambda i: ops.sum_rmsnorm([x, x], pn, 1e-6), a.iters, a.warmup),
               3 * T * H * 2, 0)
        report("linear qkv", T,
               timeit(lambda i: ops.linear(x, w_qkv[i % n_qkv]), a.iters, a.warmup),
               QKV * H * 2 + T * (H + QKV) * 2, 2 * T * H * QKV)
        report("linear o_proj + residual", T,
               timeit(lambda i: ops.linear(o_in, w_o[i % n_o], residual=x), a.iters, a.warmup),
               H * nq * D * 2 + T * (nq * D + 2 * H) * 2, 2 * T * H * nq * D)
        kc = rnd(T, nkv, a.kv_len + 8, D, scale=1.0)
        vc = rnd(T, nkv, a.kv_len + 8, D, scale=1.0)
        qkv = rnd(T, QKV, scale=1.0)
        start = a.kv_len - 1
        pos = torch.tensor([start], device=dev, dtype=torch.int32)
        report("decode attention (fused)", T,
               timeit(lambda i: ops.decode_attention_fused(qkv, qn, qn, rope, kc, vc, start, pos, 0,
                                                           nq, nkv, 1e-6), a.iters, a.warmup),
               2 * T * nkv * a.kv_len * D * 2, 4 * T * nq * a.kv_len * D)
        h = rnd(T, H, scale=1.0)
        ids = torch.stack([torch.randperm(E, device=dev)[:k] for _ in range(T)]).to(torch.int32)
        distinct = int(torch.unique(ids).numel())
        wts = torch.full((T, k), 1.0 / k, device=dev)
        eb = distinct * 3 * I * H * 2
        report(f"moe experts ({distinct} hit)", T,
               timeit(lambda i: ops.moe_experts(x, ids, wts, w_gu[i % n_e], w_dn[i % n_e], 0,
                                                residual=h), a.iters, a.warmup),
               eb, 2 * T * k * 3 * I * H)
        for e_loc in (32, 64):
            # one FFN rank of expert parallelism (4 or 2 FFN ranks): experts 0..e_loc-1
            # of the same routing; bytes = the local experts hit
            hit = int((torch.unique(ids) < e_loc).sum())
            wg, wdn = w_gu[0][:e_loc].contiguous(), w_dn[0][:e_loc].contiguous()
            wg2, wdn2 = w_gu[1][:e_loc].contiguous(), w_dn[1][:e_loc].contiguous()
            pair = [(wg, wdn), (wg2, wdn2)]
            report(f"moe experts EP{e_loc} ({hit} hit)", T,
                   timeit(lambda i: ops.moe_experts(x, ids, wts, pair[i % 2][0], pair[i % 2][1], 0,
                                                    residual=h), a.iters, a.warmup),
                   hit * 3 * I * H * 2, 2 * T * k * 3 * I * H * e_loc / E)
            del wg, wdn, wg2, wdn2, pair
        report("moe gate (norm+router+top-k+routing)", T,
               timeit(lambda i: ops.moe_gate(h, pn, w_r[i % n_qkv], k, 1e-6), a.iters, a.warmup),
               E * H * 2 + 2 * T * H * 2, 2 * T * E * H)
        report("moe block (gate+experts)", T,
               timeit(lambda i: ops.moe_ffn(h, pn, w_r[i % n_qkv], w_gu[i % n_e], w_dn[i % n_e], k,
                                            1e-6), a.iters, a.warmup),
               eb + E * H * 2, 2 * T * k * 3 * I * H + 2 * T * E * H)

    # token-block / split-K sweep of the decode-sized dense GEMMs (the table the
    # tiling rule of ops.linear was read from)
    if "tiling" in sections:
        C = ops.ext()
        for name, (N, K) in {"qkv": (QKV, H), "o_proj": (H, nq * D)}.items():
            n_w = copies_for(N * K * 2)
            wl = [rnd(N, K) for _ in range(n_w)]
            for T in [int(t) for t in a.tokens.split(",")]:
                x = rnd(T, K, scale=1.0)
                out = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
                res = {}
                for bn in (64, 128, 256):
                    if bn > 64 and bn // 2 >= T:
                        continue
                    tiles = ((T + bn - 1) // bn) * (N // 128)
                    for sp in (1, 2, 4, 8, 16):
                        if (K // 64) % sp or K // 64 // sp < 2 or tiles * sp > 4 * 148:
                            continue
                        wsp = cnt = None
                        if sp > 1:
                            wsp, cnt = ops._SplitKWorkspace.get(x.device, tiles, bn, sp)

                        def f(i, bn=bn, sp=sp, tiles=tiles, wsp=wsp, cnt=cnt):
                            C.gemm(wl[i % n_w], x, out, N // 128, N, 0, None, None, T, None, None,
                                   False, bn, tiles * sp, [], 0, [], 0, None, None, None, sp, wsp,
                                   cnt, None, False, False)
                        res[(bn, sp)] = timeit(f, 20, 3)
                chosen = ops._decode_tiling(T, N, K) if T <= 256 else None
                best = min(res, key=res.get)
                print(f"tiling {name:6s} T={T:4d} chosen {chosen} "
                      f"{res.get(chosen, float('nan')):6.2f} us, best {best} {res[best]:6.2f} us | "
                      + " ".join(f"{b}/{sp}:{u:.1f}" for (b, sp), u in sorted(res.items())),
                      flush=True)
                rows.append({"op": f"tiling {name}", "tokens": T, "chosen": list(chosen or ()),
                             "best": list(best),
                             "us": {f"{b}/{sp}": round(u, 2) for (b, sp), u in res.items()}})

    # decode attention over long caches: tcgen05 kernel vs the mma.sync kernel
    for B in ([int(b) for b in a.attn_batches.split(",")] if "attention" in sections else []):
        for kv in [int(v) for v in a.attn_kv.split(",")]:
            S = kv + 8
            cache_bytes = 2 * B * nkv * S * D * 2
            n_c = copies_for(cache_bytes // 2)
            kcs = [rnd(B, nkv, S, D, scale=1.0) for _ in range(n_c)]
            vcs = [rnd(B, nkv, S, D, scale=1.0) for _ in range(n_c)]
            q = rnd(B, nq, D, scale=1.0)
            pos = torch.tensor([kv - 1], device=dev, dtype=torch.int32)
            nbytes = 2 * B * nkv * kv * D * 2 + 2 * B * nq * D * 2
            flops = 4 * B * nq * kv * D
            sp = ops.decode_splits(B, nkv, kv)
            report(f"decode attn tcgen05 kv={kv} s={sp}", B,
                   timeit(lambda i: ops.decode_attention_tc(q, kcs[i % n_c], vcs[i % n_c], 0,
                                                            kv - 1, pos), a.iters, a.warmup),
                   nbytes, flops)
            saved = ops._DECODE_ATTN
            ops._DECODE_ATTN = "mma"
            try:
                qkv = rnd(B, QKV, scale=1.0)
                report(f"decode attn mma.sync kv={kv}", B,
                       timeit(lambda i: ops.decode_attention_fused(
                           qkv, qn, qn, rope, kcs[i % n_c], vcs[i % n_c], kv - 1, pos, 0, nq, nkv,
                           1e-6), a.iters, a.warmup),
                       nbytes, flops)
            finally:
                ops._DECODE_ATTN = saved
            del kcs, vcs

    if "prefill" not in sections and "prefill_attn" not in sections:
        if a.json:
            os.makedirs(os.path.dirname(os.path.abspath(a.json)), exist_ok=True)
            json.dump({"peaks": {"hbm_Bps": bw, "bf16_flops": fl, "basis": tag}, "rows": rows},
                      open(a.json, "w"), indent=1)
        return 0
    # prefill-sized dense GEMM and attention
    T = a.prefill_tokens
    if "prefill" in sections:
        xp = rnd(T, H, scale=1.0)
        report("linear qkv (prefill)", T,
               timeit(lambda i: ops.linear(xp, w_qkv[i % n_qkv]), max(5, a.iters // 5), 2),
               QKV * H * 2 + T * (H + QKV) * 2, 2 * T * H * QKV)
        op = rnd(T, nq * D, scale=1.0)
        report("linear o_proj + residual (prefill)", T,
               timeit(lambda i: ops.linear(op, w_o[i % n_o], residual=xp), max(5, a.iters // 5), 2),
               H * nq * D * 2 + T * (nq * D + 2 * H) * 2, 2 * T * H * nq * D)
        hp = rnd(T, H, scale=1.0)
        report("moe block (prefill)", T,
               timeit(lambda i: ops.moe_ffn(hp, pn, w_r[i % n_qkv], w_gu[i % n_e], w_dn[i % n_e],
                                            k, 1e-6), max(5, a.iters // 5), 2),
               E * 3 * I * H * 2 + E * H * 2, 2 * T * k * 3 * I * H + 2 * T * E * H)
        del xp, op, hp
    # prefill attention at each prompt length, each kernel variant
    pos0 = torch.zeros(1, device=dev, dtype=torch.int32)
    default_variant = ops._PREFILL_ATTN
    for S in [int(v) for v in a.prefill_attn_seqs.split(",")]:
        B = max(1, T // S)
        q = rnd(B * S, nq, D, scale=1.0)
        kc = rnd(B, nkv, S, D, scale=1.0)
        vc = rnd(B, nkv, S, D, scale=1.0)
        for variant in a.prefill_attn_variants.split(","):
            ops._PREFILL_ATTN = variant
            # causal: half of the S x S score matrix, two products (QK^T and PV)
            report(f"prefill attention S={S} [{variant}]", B * S,
                   timeit(lambda i: ops.attention(q, kc, vc, 0, S, 0, pos0), max(5, a.iters // 5),
                          2),
                   (B * S * nq * D * 2) * 2 + 2 * B * nkv * S * D * 2,
                   2 * 2 * B * nq * S * S * D / 2)
        ops._PREFILL_ATTN = default_variant
        del q, kc, vc
    if a.json:
        os.makedirs(os.path.dirname(os.path.abspath(a.json)), exist_ok=True)
        json.dump({"peaks": {"hbm_Bps": bw, "bf16_flops": fl, "basis": tag}, "rows": rows},
                  open(a.json, "w"), indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
