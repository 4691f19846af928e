"""sm_100a kernels against PyTorch fp32 statements of the same ops."""

import pytest
import torch

from afd_demo_b200 import ops
from afd_demo_b200.ops import torch_ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


def _randn(*s, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*s, generator=g, device=DEV) * scale).to(torch.bfloat16)


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ops.ext()  # must load: no silent fallback


@pytest.mark.parametrize("T", [1, 5, 32, 37, 64, 100, 300, 513])
@pytest.mark.parametrize("N,K", [(256, 2048), (5120, 2048), (2048, 4096), (128, 2048)])
def test_dense_gemm(T, N, K):
    x = _randn(T, K, seed=1)
    w = _randn(N, K, scale=0.02, seed=2)
    ref = x.float() @ w.float().t()
    out = ops.linear(x, w)
    torch.cuda.synchronize()
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("T", [300, 1000, 4096])
def test_dense_gemm_token_major(T, monkeypatch):
    """Prefill-sized dense GEMM (+ residual) on the token-major kernel, ragged
    last row block included."""
    monkeypatch.setattr(ops, "_DENSE_TM", "all")
    K, N = 4096, 2048
    x = _randn(T, K, seed=29)
    w = _randn(N, K, scale=0.02, seed=30)
    r = _randn(T, N, seed=31)
    ref = x.float() @ w.float().t() + r.float()
    assert _rel(ops.linear(x, w, residual=r), ref) < 1e-2
    ref = x.float() @ w.float().t()
    assert _rel(ops.linear(x, w), ref) < 1e-2


@pytest.mark.parametrize("T", [3, 64, 200])
def test_dense_gemm_residual(T):
    K, N = 4096, 2048
    x = _randn(T, K, seed=3)
    w = _randn(N, K, scale=0.02, seed=4)
    r = _randn(T, N, seed=5)
    ref = x.float() @ w.float().t() + r.float()
    out = ops.linear(x, w, residual=r)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("T,E,k", [(1, 128, 8), (16, 128, 8), (64, 128, 8), (333, 128, 8),
                                   (2048, 128, 8), (40, 32, 8)])
def test_moe_experts(T, E, k):
    H, I = 2048, 768
    torch.manual_seed(0)
    xn = _randn(T, H, seed=6)
    wgu = _randn(E, 2 * I, H, scale=0.02, seed=7)
    wd = _randn(E, H, I, scale=0.02, seed=8)
    logits = torch.randn(T, 128, device=DEV)
    probs = logits.softmax(-1)
    w, ids = probs.topk(k, -1)
    w = (w / w.sum(-1, keepdim=True)).float()
    ids = ids.to(torch.int32)
    start = 0 if E == 128 else 32  # expert-parallel slice [32, 64)
    ref = torch_ref.moe_experts(xn, ids, w, wgu, wd, start)
    out = ops.moe_experts(xn, ids, w, wgu, wd, start)
    assert _rel(out, ref) < 2e-2


@pytest.mark.parametrize("sk", [True, False])
@pytest.mark.parametrize("T,E_loc,start,sms", [(128, 32, 32, 0), (128, 32, 96, 128), (16, 128, 0, 0),
                                               (64, 128, 0, 100), (256, 64, 64, 0), (5, 32, 0, 0)])
def test_moe_experts_decode_stream_k(T, E_loc, start, sms, sk, monkeypatch):
    """Decode-sized expert GEMMs with stream-K ranges (boundary tiles reduced in
    two pieces) and with round-robin tiles, full grid and a capped grid,
    against the fp32 statement; twice, so the piece counters are seen reset."""
    monkeypatch.setattr(ops, "_STREAM_K", sk)
    H, I, E, k = 2048, 768, 128, 8
    xn = _randn(T, H, seed=32)
    h = _randn(T, H, seed=33)
    wgu = _randn(E_loc, 2 * I, H, scale=0.02, seed=34)
    wd = _randn(E_loc, H, I, scale=0.02, seed=35)
    probs = torch.randn(T, E, device=DEV).softmax(-1)
    w, ids = probs.topk(k, -1)
    w = (w / w.sum(-1, keepdim=True)).float()
    ids = ids.to(torch.int32)
    ref = torch_ref.moe_experts(xn, ids, w, wgu, wd, start).float() + h.float()
    for _ in range(2):
        with ops.sm_budget(sms):
            out = ops.moe_experts(xn, ids, w, wgu, wd, start, residual=h)
        assert _rel(out, ref) < 2e-2


@pytest.mark.parametrize("tm", [True, False])
@pytest.mark.parametrize("T,E_loc,start", [(2048, 128, 0), (1600, 128, 0), (3000, 32, 32),
                                           (4096, 64, 64)])
def test_moe_experts_prefill_kernels(T, E_loc, start, tm, monkeypatch):
    """Prefill-sized expert GEMMs on the token-major kernel (128 x 256 MMAs,
    one token row per TMEM lane) and on the swap-AB kernel, against the fp32
    statement: full and ragged 128-row blocks, expert-parallel slices."""
    monkeypatch.setattr(ops, "_MOE_TM", tm)
    H, I, E, k = 2048, 768, 128, 8
    xn = _randn(T, H, seed=25)
    h = _randn(T, H, seed=26)
    wgu = _randn(E_loc, 2 * I, H, scale=0.02, seed=27)
    wd = _randn(E_loc, H, I, scale=0.02, seed=28)
    probs = torch.randn(T, E, device=DEV).softmax(-1)
    w, ids = probs.topk(k, -1)
    w = (w / w.sum(-1, keepdim=True)).float()
    ids = ids.to(torch.int32)
    ref = torch_ref.moe_experts(xn, ids, w, wgu, wd, start).float() + h.float()
    out = ops.moe_experts(xn, ids, w, wgu, wd, start, residual=h)
    assert _rel(out, ref) < 2e-2


@pytest.mark.parametrize("T,E_loc,start", [(1, 128, 0), (16, 128, 0), (64, 128, 0), (300, 128, 0),
                                           (1024, 128, 0), (48, 32, 32), (2048, 128, 0)])
def test_moe_ffn_block(T, E_loc, start):
    """RMSNorm + router + fused top-k/routing + gathered grouped GEMMs + combine."""
    H, I, E = 2048, 768, 128
    h = _randn(T, H, seed=13)
    pw = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    wr = _randn(E, H, scale=0.02, seed=14)
    wgu = _randn(E_loc, 2 * I, H, scale=0.02, seed=15)
    wd = _randn(E_loc, H, I, scale=0.02, seed=16)
    ref = torch_ref.ffn_layer(h, pw, wr, wgu, wd, 8, 1e-6, expert_start=start,
                              add_residual=(start == 0))
    out = ops.moe_ffn(h, pw, wr, wgu, wd, 8, 1e-6, True, start, add_residual=(start == 0))
    assert _rel(out, ref) < 2e-2


@pytest.mark.parametrize("T,E_loc,start", [(1, 128, 0), (16, 128, 0), (200, 128, 0), (24, 32, 32)])
def test_moe_ffn_block_fused_combine(T, E_loc, start, monkeypatch):
    """The A/B variant that runs the top-k combine inside the down GEMM's
    epilogue (off by default) against the same fp32 statement."""
    monkeypatch.setattr(ops, "_FUSED_COMBINE", True)
    H, I, E = 2048, 768, 128
    h = _randn(T, H, seed=17)
    pw = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    wr = _randn(E, H, scale=0.02, seed=18)
    wgu = _randn(E_loc, 2 * I, H, scale=0.02, seed=19)
    wd = _randn(E_loc, H, I, scale=0.02, seed=20)
    ref = torch_ref.ffn_layer(h, pw, wr, wgu, wd, 8, 1e-6, expert_start=start,
                              add_residual=(start == 0))
    out = ops.moe_ffn(h, pw, wr, wgu, wd, 8, 1e-6, True, start, add_residual=(start == 0))
    assert _rel(out, ref) < 2e-2


@pytest.mark.parametrize("T,E_loc,start", [(16, 128, 0), (300, 128, 0), (1024, 32, 32)])
def test_routing_tables_pass_bounds_check(T, E_loc, start, monkeypatch):
    """AFD_BOUNDS_CHECK=1 validates the routing tables of the fused gate (16
    tokens), the one-CTA route kernel (300) and the multi-CTA align (1024) on
    the host; the layer output is unchanged."""
    monkeypatch.setattr(ops, "_BOUNDS_CHECK", True)
    H, I, E = 2048, 768, 128
    h = _randn(T, H, seed=21)
    pw = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    wr = _randn(E, H, scale=0.02, seed=22)
    wgu = _randn(E_loc, 2 * I, H, scale=0.02, seed=23)
    wd = _randn(E_loc, H, I, scale=0.02, seed=24)
    ref = torch_ref.ffn_layer(h, pw, wr, wgu, wd, 8, 1e-6, expert_start=start,
                              add_residual=(start == 0))
    out = ops.moe_ffn(h, pw, wr, wgu, wd, 8, 1e-6, True, start, add_residual=(start == 0))
    assert _rel(out, ref) < 2e-2


def test_moe_residual_and_ep_partials_sum():
    T, H, I, E = 48, 2048, 768, 128
    xn = _randn(T, H, seed=9)
    h = _randn(T, H, seed=10)
    wgu = _randn(E, 2 * I, H, scale=0.02, seed=11)
    wd = _randn(E, H, I, scale=0.02, seed=12)
    w, ids = torch.rand(T, 128, device=DEV).softmax(-1).topk(8, -1)
    w = (w / w.sum(-1, keepdim=True)).float()
    ids = ids.to(torch.int32)
    full = ops.moe_experts(xn, ids, w, wgu, wd, 0, residual=h).float()
    parts = [ops.moe_experts(xn, ids, w, wgu[e0:e0 + 32], wd[e0:e0 + 32], e0,
                             residual=h if e0 == 0 else None).float() for e0 in (0, 32, 64, 96)]
    assert _rel(sum(parts), full) < 1e-2


@pytest.mark.parametrize("T", [37, 300])
@pytest.mark.parametrize("parts", [1, 2, 4])
def test_sum_rmsnorm(parts, T):
    H = 2048
    xs = [_randn(T, H, seed=20 + i) for i in range(parts)]
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    x_ref, y_ref = torch_ref.sum_rmsnorm(xs, w, 1e-6)
    x, y = ops.sum_rmsnorm(xs, w, 1e-6)
    assert _rel(x, x_ref) < 5e-3
    assert _rel(y, y_ref) < 1e-2


@pytest.mark.parametrize("q_len,start", [(1, 0), (1, 200), (7, 0), (64, 0), (100, 30)])
def test_qk_norm_rope_cache(q_len, start):
    B, nq, nkv, D, S = 3, 32, 4, 128, 512
    T = B * q_len
    qkv = _randn(T, (nq + 2 * nkv) * D, seed=30)
    qn = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    rope = ops.rope_table(S, D, 1e6, DEV)
    kc = torch.zeros(4, nkv, S, D, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    q_ref = torch_ref.qk_norm_rope_cache(qkv.float(), qn.float(), kn.float(), rope, kc2, vc2, 1,
                                         q_len, start, nq, nkv, 1e-6)
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    q = ops.qk_norm_rope_cache(qkv, qn, kn, rope, kc, vc, start, pos, q_len, 1, nq, nkv, 1e-6)
    assert _rel(q, q_ref) < 1e-2
    sl = slice(start, start + q_len)
    assert _rel(kc[1:1 + B, :, sl], kc2[1:1 + B, :, sl]) < 1e-2
    assert torch.equal(vc[1:1 + B, :, sl], vc2[1:1 + B, :, sl])


@pytest.mark.parametrize("B,kv_len", [(1, 1), (3, 77), (16, 276), (64, 300), (2, 2049)])
def test_decode_attention(B, kv_len):
    nq, nkv, D, S = 32, 4, 128, 2304
    kc = _randn(B + 1, nkv, S, D, seed=40)
    vc = _randn(B + 1, nkv, S, D, seed=41)
    q = _randn(B, nq, D, seed=42)
    start = kv_len - 1
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), 1, 1, start)
    out = ops.attention(q, kc, vc, 1, 1, start, pos)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("B", [16, 64])
@pytest.mark.parametrize("kv_len", [256, 1024, 2048, 4096])
def test_decode_attention_tc_long_kv(B, kv_len):
    """tcgen05 decode attention at the cache lengths where it dominates."""
    nq, nkv, D, S = 32, 4, 128, 4104
    kc = _randn(B + 1, nkv, S, D, seed=50)
    vc = _randn(B + 1, nkv, S, D, seed=51)
    q = _randn(B, nq, D, seed=52)
    start = kv_len - 1
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), 1, 1, start)
    out = ops.decode_attention_tc(q, kc, vc, 1, start, pos).view(B, nq * D)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("nsplit", [1, 2, 3, 7, 16, 40])
@pytest.mark.parametrize("G", [8, 4])
def test_decode_attention_tc_splits(nsplit, G):
    """Every split count merges to the same result, including splits that
    own no key tile (more splits than tiles), for 8 and 4 query heads per
    kv head."""
    nkv, D, S, B, kv_len = 4, 128, 2304, 5, 1500
    nq = G * nkv
    kc = _randn(B, nkv, S, D, seed=53)
    vc = _randn(B, nkv, S, D, seed=54)
    q = _randn(B, nq, D, seed=55)
    pos = torch.tensor([kv_len - 1], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), 0, 1, kv_len - 1)
    for _ in range(2):  # the merge counters must be left at zero
        out = ops.decode_attention_tc(q, kc, vc, 0, kv_len - 1, pos, nsplit=nsplit)
        assert _rel(out.view(B, nq * D), ref) < 1e-2


def test_decode_attention_tc_nan_past_the_end():
    """Cache rows past the sequence end may hold anything (here NaN): they
    must not reach the output."""
    nq, nkv, D, S, B, kv_len = 32, 4, 128, 512, 3, 200
    kc = _randn(B, nkv, S, D, seed=56)
    vc = _randn(B, nkv, S, D, seed=57)
    kc[:, :, kv_len:] = float("nan")
    vc[:, :, kv_len:] = float("nan")
    q = _randn(B, nq, D, seed=58)
    pos = torch.tensor([kv_len - 1], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), 0, 1, kv_len - 1)
    out = ops.decode_attention_tc(q, kc, vc, 0, kv_len - 1, pos).view(B, nq * D)
    assert torch.isfinite(out.float()).all()
    assert _rel(out, ref) < 1e-2


def test_decode_attention_tc_bad_position_reads_nothing():
    nq, nkv, D, S, B = 32, 4, 128, 256, 2
    kc = _randn(B + 2, nkv, S, D, seed=59)
    q = _randn(B, nq, D, seed=60)
    for p in (S, -5):
        pos = torch.tensor([p], device=DEV, dtype=torch.int32)
        st = torch.zeros(2, device=DEV, dtype=torch.int32)
        out = ops.decode_attention_tc(q, kc, kc, 0, 100, pos, status=st)
        torch.cuda.synchronize()
        assert int(st[0]) == 3 and torch.count_nonzero(out) == 0


@pytest.mark.parametrize("B,kv_len", [(3, 77), (16, 276), (2, 2049)])
def test_decode_attention_mma_kernels(B, kv_len, monkeypatch):
    """The mma.sync / SIMT decode kernels (AFD_DECODE_ATTN=mma) stay correct."""
    monkeypatch.setattr(ops, "_DECODE_ATTN", "mma")
    nq, nkv, D, S = 32, 4, 128, 2304
    kc = _randn(B + 1, nkv, S, D, seed=61)
    vc = _randn(B + 1, nkv, S, D, seed=62)
    q = _randn(B, nq, D, seed=63)
    start = kv_len - 1
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), 1, 1, start)
    assert _rel(ops.attention(q, kc, vc, 1, 1, start, pos), ref) < 1e-2
    qkv = _randn(B, (nq + 2 * nkv) * D, seed=64)
    qn = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    rope = ops.rope_table(S, D, 1e6, DEV)
    kc2, vc2 = kc.clone(), vc.clone()
    q_ref = torch_ref.qk_norm_rope_cache(qkv.float(), qn.float(), kn.float(), rope, kc2, vc2, 1,
                                         1, start, nq, nkv, 1e-6)
    ref = torch_ref.attention(q_ref, kc2.float(), vc2.float(), 1, 1, start)
    out = ops.decode_attention_fused(qkv, qn, kn, rope, kc, vc, start, pos, 1, nq, nkv, 1e-6)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("B,kv_len,G,D", [(1, 1, 8, 128), (3, 77, 8, 128), (16, 276, 8, 128),
                                           (64, 300, 8, 128), (2, 2049, 8, 128), (5, 100, 2, 64),
                                           (4, 500, 8, 64)])
def test_decode_attention_fused(B, kv_len, G, D):
    nkv = 4 if D == 128 else 2
    nq = G * nkv
    S = 2304
    kc = _randn(B + 1, nkv, S, D, seed=43)
    vc = _randn(B + 1, nkv, S, D, seed=44)
    qkv = _randn(B, (nq + 2 * nkv) * D, seed=45)
    qn = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16)
    rope = ops.rope_table(S, D, 1e6, DEV)
    start = kv_len - 1
    kc2, vc2 = kc.clone(), vc.clone()
    q_ref = torch_ref.qk_norm_rope_cache(qkv.float(), qn.float(), kn.float(), rope, kc2, vc2, 1,
                                         1, start, nq, nkv, 1e-6)
    ref = torch_ref.attention(q_ref, kc2.float(), vc2.float(), 1, 1, start)
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    out = ops.decode_attention_fused(qkv, qn, kn, rope, kc, vc, start, pos, 1, nq, nkv, 1e-6)
    assert _rel(out, ref) < 1e-2
    assert _rel(kc[1:1 + B, :, start], kc2[1:1 + B, :, start]) < 1e-2
    assert torch.equal(vc[1:1 + B, :, start], vc2[1:1 + B, :, start])


@pytest.mark.parametrize("B,q_len,start,off", [(1, 16, 0, 0), (2, 128, 0, 0), (3, 100, 0, 0),
                                               (2, 64, 40, 0), (1, 512, 0, 0), (2, 300, 0, 1),
                                               (1, 257, 100, 0), (2, 129, 383, 1)])
def test_prefill_attention(B, q_len, start, off):
    """Causal prefill over a cache holding `start` earlier keys; sequences
    sit at cache rows off .. off + B - 1."""
    nq, nkv, D, S = 32, 4, 128, 1024
    kc = _randn(B + off, nkv, S, D, seed=50)
    vc = _randn(B + off, nkv, S, D, seed=51)
    q = _randn(B * q_len, nq, D, seed=52)
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), off, q_len, start)
    out = ops.attention(q, kc, vc, off, q_len, start, pos)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("T", [1, 9, 256])
def test_router_topk(T):
    H, E = 2048, 128
    h = _randn(T, H, seed=60)
    pw = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    wr = _randn(E, H, scale=0.02, seed=61)
    xn_r, ids_r, w_r = torch_ref.router_topk(h, pw, wr, 8, 1e-6)
    xn, ids, w = ops.router_topk(h, pw, wr, 8, 1e-6)
    assert _rel(xn, xn_r) < 1e-2
    # compare as (expert -> weight) maps: near-ties may swap order
    dense = torch.zeros(T, E, device=DEV).scatter_(1, ids.long(), w)
    dense_r = torch.zeros(T, E, device=DEV).scatter_(1, ids_r.long(), w_r)
    assert (dense - dense_r).abs().max() < 2e-2


def test_argmax():
    x = _randn(5, 151936, seed=70)
    x[2, 12345] = 100.0
    assert torch.equal(ops.argmax(x), x.float().argmax(-1))
    assert torch.equal(ops.argmax(x), x.float().argmax(-1))  # workspace counters reset


def test_argmax_row_counts_change_between_calls():
    """32 rows, then 8, then 32 again on one stream: the per-row counters of the
    split kernel must not inherit the 8-row call's partial maxima (they once
    shared a buffer, and the third call returned unwritten indices)."""
    for rows in (32, 8, 32, 5, 32):
        x = _randn(rows, 151936, seed=76 + rows)
        assert torch.equal(ops.argmax(x), x.float().argmax(-1)), rows


@pytest.mark.parametrize("V", [100, 151936])
def test_argmax_all_nan_row_gives_a_valid_index(V):
    """A row with no comparable value (all NaN) returns 0, both kernels: the
    index always stays a valid token id for the next embedding lookup."""
    x = _randn(3, V, seed=74)
    x[1] = float("nan")
    got = ops.argmax(x)
    assert int(got[1]) == 0
    assert int(got[0]) == int(x[0].float().argmax()) and int(got[2]) == int(x[2].float().argmax())
    view = _randn(3, V + 3, seed=75)[:, 1:V + 1]  # unaligned rows: the one-CTA kernel
    view[0] = float("nan")
    assert int(ops.argmax(view)[0]) == 0


@pytest.mark.parametrize("V", [100, 8192, 8200, 151936, 151937])
def test_argmax_ties_and_strided_rows(V):
    """Ties across chunks go to the first index; a ragged tail, a NaN (never
    chosen, as in the one-CTA kernel) and row views of a wider matrix (the
    one-CTA fallback when the rows are not 16-byte aligned)."""
    x = _randn(3, V, seed=71)
    x[0, V - 1] = 50.0
    x[0, V // 3] = 50.0  # tie: the first index wins
    x[1, 7] = float("nan")
    x[1, V // 2] = 60.0
    ref = x.float().nan_to_num(-1e30).argmax(-1)
    assert torch.equal(ops.argmax(x), ref)
    wide = _randn(3, V + 3, seed=72)
    view = wide[:, 1:V + 1]
    assert torch.equal(ops.argmax(view), view.float().argmax(-1))
    # aligned rows whose length is not a multiple of 8: scalar tail of the last chunk
    wide = _randn(3, V + 16, seed=73)
    view = wide[:, :V + 3]
    view[2, V + 2] = 70.0
    assert torch.equal(ops.argmax(view), view.float().argmax(-1))


def test_flags_roundtrip_and_timeout():
    C = ops.ext()
    buf = C.ipc_alloc(4096, torch.cuda.current_device())
    base = buf.data_ptr()
    status = torch.zeros(2, dtype=torch.int32, device=DEV)
    C.signal_flags([base, base + 4], 7, None)
    C.wait_flags([base, base + 4], 7, status, 1_000_000_000, None)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    # a flag nobody raises: the bounded wait gives up and reports
    C.wait_flags([base + 8], 1, status, 50_000_000, None)
    torch.cuda.synchronize()
    assert int(status[0]) == 2


@pytest.mark.parametrize("with_residual", [True, False])
def test_moe_experts_no_local_rows(with_residual):
    """Every routed expert lives on another rank: the output is the residual
    (or zeros) and the fused combine still writes every token."""
    T, H, I = 3, 2048, 768
    xn = _randn(T, H, seed=80)
    h = _randn(T, H, seed=81)
    wgu = _randn(32, 2 * I, H, scale=0.02, seed=82)
    wd = _randn(32, H, I, scale=0.02, seed=83)
    ids = torch.arange(64, 72, device=DEV, dtype=torch.int32).repeat(T, 1)
    w = torch.full((T, 8), 0.125, device=DEV)
    out = ops.moe_experts(xn, ids, w, wgu, wd, 0, residual=h if with_residual else None)
    want = h if with_residual else torch.zeros_like(h)
    assert torch.equal(out, want)


@pytest.mark.parametrize("variant", ["tc", "tc1", "mma"])
@pytest.mark.parametrize("B,q_len,start,off", [(2, 300, 0, 1), (1, 257, 100, 0), (1, 2048, 0, 0)])
def test_prefill_attention_kernels(B, q_len, start, off, variant, monkeypatch):
    """Each prefill kernel against the fp32 oracle: tcgen05 with two query
    heads per CTA (P in TMEM), tcgen05 with one head per CTA, mma.sync."""
    monkeypatch.setattr(ops, "_PREFILL_ATTN", variant)
    nq, nkv, D = 32, 4, 128
    S = max(1024, start + q_len)
    kc = _randn(B + off, nkv, S, D, seed=53)
    vc = _randn(B + off, nkv, S, D, seed=54)
    q = _randn(B * q_len, nq, D, seed=55)
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), off, q_len, start)
    out = ops.attention(q, kc, vc, off, q_len, start, pos)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("nq,nkv", [(8, 8), (12, 4), (16, 2)])
@pytest.mark.parametrize("variant", ["tc", "tc1"])
def test_prefill_attention_gqa_groups(nq, nkv, variant, monkeypatch):
    """Group sizes 1 and 3 (one head per CTA) and 8 (head pairs) with a
    query tile that straddles the cache's earlier keys."""
    monkeypatch.setattr(ops, "_PREFILL_ATTN", variant)
    B, q_len, start, D, S = 2, 200, 60, 128, 512
    kc = _randn(B, nkv, S, D, seed=56)
    vc = _randn(B, nkv, S, D, seed=57)
    q = _randn(B * q_len, nq, D, seed=58)
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), 0, q_len, start)
    out = ops.attention(q, kc, vc, 0, q_len, start, pos)
    assert _rel(out, ref) < 1e-2


def test_prefill_attention_long_sequence():
    """A 2048-token causal prefill (16 key tiles per query tile)."""
    nq, nkv, D, S, q_len = 32, 4, 128, 2048, 2048
    kc = _randn(1, nkv, S, D, seed=90)
    vc = _randn(1, nkv, S, D, seed=91)
    q = _randn(q_len, nq, D, seed=92)
    pos = torch.zeros(1, device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), 0, q_len, 0)
    out = ops.attention(q, kc, vc, 0, q_len, 0, pos)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("D,q_len,start,off", [(128, 100, 0, 0), (128, 130, 0, 1), (64, 77, 0, 0),
                                             (128, 40, 24, 0)])
def test_prefill_attention_padding_mask(D, q_len, start, off):
    """Key ranges (padding masks): rows fully visible, right-padded,
    left-padded, and a left-padded row whose first queries see no key
    (output zeros, as the fp32 statement defines)."""
    B, nkv, S = 4, 2, 256
    nq = 8
    kc = _randn(B + off, nkv, S, D, seed=95)
    vc = _randn(B + off, nkv, S, D, seed=96)
    q = _randn(B * q_len, nq, D, seed=97)
    end = start + q_len
    lo = torch.tensor([0] * off + [0, 0, end // 2, 3], dtype=torch.int32, device=DEV)
    hi = torch.tensor([0] * off + [end, end - 9, end, end - 1], dtype=torch.int32, device=DEV)
    pos = torch.tensor([start], device=DEV, dtype=torch.int32)
    ref = torch_ref.attention(q.float(), kc.float(), vc.float(), off, q_len, start, (lo, hi))
    out = ops.attention(q, kc, vc, off, q_len, start, pos, (lo, hi))
    assert _rel(out, ref) < 1e-2
    # rows with no visible key are exactly zero
    o = out.view(B, q_len, nq * D)
    assert torch.all(o[2, : max(0, end // 2 - start)] == 0)


def test_gemm_sm_budget_same_result():
    """Capping the persistent grid changes the schedule, not the result."""
    x = _randn(200, 2048, seed=93)
    w = _randn(1024, 2048, scale=0.02, seed=94)
    full = ops.linear(x, w)
    with ops.sm_budget(40):
        capped = ops.linear(x, w)
    assert torch.equal(full, capped)


@pytest.mark.parametrize("T", [1, 16, 100])
def test_moe_gate_alone(T):
    """The fused gate's ids / weights equal the router top-k of the fp32
    reference (as expert -> weight maps; near-ties may swap order)."""
    H, E = 2048, 128
    h = _randn(T, H, seed=95)
    pw = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    wr = _randn(E, H, scale=0.02, seed=96)
    xn_r, ids_r, w_r = torch_ref.router_topk(h, pw, wr, 8, 1e-6)
    xn, ws = ops.moe_gate(h, pw, wr, 8, 1e-6)
    assert _rel(xn, xn_r) < 1e-2
    dense = torch.zeros(T, E, device=DEV).scatter_(1, ws.ids.long(), ws.weights)
    dense_r = torch.zeros(T, E, device=DEV).scatter_(1, ids_r.long(), w_r)
    assert (dense - dense_r).abs().max() < 2e-2
    assert int(ws.num_rows) == T * 8
