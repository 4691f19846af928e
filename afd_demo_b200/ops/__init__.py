"""Op layer: each function runs the sm_100a kernel on CUDA tensors and the
PyTorch statement (``torch_ref``) on CPU tensors.

There is no silent fallback on the GPU: a CUDA tensor with the extension
missing raises. The extension is ``afd_demo_b200/_C*.so`` built in place by
``python setup.py build_ext --inplace`` (or the build entry point at the repository root).
"""

from __future__ import annotations

import math
import os
from typing import List, NamedTuple, Optional, Sequence, Tuple

import torch

from . import torch_ref

_C = None

# Kernel-launching entry points of the extension and how many kernels each
# call launches (decode attention adds a merge kernel when split).
_KERNEL_CALLS = {"gemm", "sum_rmsnorm", "qk_norm_rope_cache", "decode_attention",
                 "prefill_attention", "router_topk", "moe_align", "moe_gather", "moe_combine",
                 "argmax", "signal_flags", "wait_flags", "add_i32", "peer_copy",
                 "decode_attention_fused", "moe_route", "moe_gate", "gemm_down_combine",
                 "moe_align_mt", "decode_attention_tc"}


class LaunchCounter:
    """Counts this package's kernel launches issued from Python (a CUDA graph
    replays what was counted while it was captured)."""

    def __init__(self):
        self.count = 0

    def reset(self) -> int:
        n, self.count = self.count, 0
        return n


LAUNCHES = LaunchCounter()


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if name not in _KERNEL_CALLS:
            return fn

        def call(*a):
            LAUNCHES.count += 2 if (name == "decode_attention" and a[6] > 1) else 1
            return fn(*a)

        return call


def ext():
    """The compiled extension (raises if it was not built)."""
    global _C
    if _C is None:
        try:
            from .. import _C as mod  # type: ignore
        except ImportError as e:  # pragma: no cover - exercised where the extension is not built
            raise RuntimeError(
                "afd_demo_b200._C is not built: run `python setup.py build_ext --inplace`") from e
        _C = _Counted(mod)
    return _C


def ext_available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


_NUM_SMS: Optional[int] = None


def num_sms() -> int:
    global _NUM_SMS
    if _NUM_SMS is None:
        _NUM_SMS = int(ext().num_sms())
    return _NUM_SMS


class sm_budget:
    """Caps the grid of the persistent GEMMs launched inside the block at `n`
    SMs (None or 0: no cap), leaving the rest to kernels of a concurrent
    stream. Launch parameters are fixed at launch, so a captured CUDA graph
    keeps the cap that was active during capture."""

    def __init__(self, n: Optional[int]):
        self.n = int(n or 0)

    def __enter__(self):
        if self.n:
            ext().set_gemm_sm_cap(self.n)
        return self

    def __exit__(self, *exc):
        if self.n:
            ext().set_gemm_sm_cap(0)
        return False


class no_pdl:
    """Launches inside the block go without programmatic dependent launch.
    With two streams on one GPU, a kernel launched early by PDL parks its
    persistent CTAs on SMs while it waits for its predecessor, and the other
    stream's kernels cannot use them: one-GPU prefill DBO measured 70-72 ms
    without PDL against 80-83 ms with it (serial: 67-69 ms either way). A
    captured CUDA graph keeps the setting of its capture."""

    def __enter__(self):
        ext().set_pdl_override(0)
        return self

    def __exit__(self, *exc):
        ext().set_pdl_override(-1)
        return False


# ------------------------------------------------------------------ norms --
class FlagWait(NamedTuple):
    """A receive folded into the consuming kernel: the kernel waits (bounded
    by `timeout_ns`) until every flag reaches *epoch + value before reading
    its input; a timeout is recorded in `status`."""
    flags: Sequence[int]
    value: int
    status: torch.Tensor
    timeout_ns: int
    epoch: Optional[torch.Tensor]


def _wait_args(wait: Optional[FlagWait]) -> tuple:
    if wait is None:
        return [], 0, None, 0, None
    return list(wait.flags), int(wait.value), wait.status, int(wait.timeout_ns), wait.epoch


def wait_flags(wait: Optional[FlagWait]) -> None:
    """Stand-alone form of a folded wait (a one-CTA kernel)."""
    if wait is not None:
        ext().wait_flags(list(wait.flags), int(wait.value), wait.status, int(wait.timeout_ns),
                         wait.epoch)


def sum_rmsnorm(parts: Sequence[torch.Tensor], w: torch.Tensor, eps: float,
                want_sum: bool = True, out: Optional[torch.Tensor] = None,
                wait: Optional[FlagWait] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """x = sum(parts), y = RMSNorm(x). Returns (x, y); x is parts[0] itself
    when there is a single part. `wait`: the parts arrive from peers; the
    kernel waits for their flags first."""
    if not _cuda(parts[0]):
        return torch_ref.sum_rmsnorm(parts, w, eps)
    p0 = parts[0]
    H = p0.shape[-1]
    rows = p0.numel() // H
    y = out if out is not None else torch.empty(rows, H, device=p0.device, dtype=p0.dtype)
    x = None
    if len(parts) > 1 and want_sum:
        x = torch.empty(rows, H, device=p0.device, dtype=p0.dtype)
    ext().sum_rmsnorm([p.reshape(rows, H) for p in parts], w, x, y, float(eps),
                      *_wait_args(wait))
    return (x if x is not None else p0.reshape(rows, H)), y


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return sum_rmsnorm([x], w, eps)[1]


# ------------------------------------------------------------------- GEMM --
def _block_n(rows: int) -> int:
    """Token rows per GEMM tile: the smallest of 64/128/256 that covers the
    rows (decode), 256 for large dense GEMMs (prefill)."""
    return 64 if rows <= 64 else (128 if rows <= 128 else 256)


# row-block size of prefill-sized grouped GEMMs (AFD_MOE_BN_LARGE=256 for A/B)
_MOE_BN_LARGE = int(os.environ.get("AFD_MOE_BN_LARGE", "128"))
# prefill-sized expert GEMMs (at least this many routed rows per local expert on
# average, 128-row blocks) run on the token-major kernel; AFD_MOE_TM=0 keeps
# them on the swap-AB kernel (A/B measurements)
_MOE_TM = os.environ.get("AFD_MOE_TM", "1") != "0"
_MOE_TM_MIN_ROWS = 96
# prefill-sized dense GEMMs (more than 256 rows, output features a multiple of
# 256) on the token-major kernel: "residual" (default) = those with a residual
# add (o_proj), "all", or "none" = all on the swap-AB kernel (A/B measurements)
_DENSE_TM = os.environ.get("AFD_DENSE_TM", "residual")


def _moe_block_n(rows: int) -> int:
    """Row-block size of the grouped expert GEMMs by token count: 64 for
    decode-sized batches (up to 256 tokens: with top-8 of 128 experts an
    expert sees about T/16 rows, so one 64-row block holds it, and the
    smaller token tile leaves room for one more weight stage); 128 for
    mid-sized ones (two TMEM accumulators per SwiGLU tile, double-buffered);
    `AFD_MOE_BN_LARGE` for prefill-sized ones. The MMA width follows each
    block's actual row count, so a short last block costs little."""
    return 64 if rows <= 256 else (128 if rows < 2048 else _MOE_BN_LARGE)


def _wave_splits(units: int, k_iters: int, gain: float = 1.1) -> int:
    """Split-K factor (1 or 2) for a grouped GEMM whose units fill the
    persistent grid's last wave poorly: 2 when that raises the share of busy
    CTA slots by at least `gain` (each split adds a partial-tile store and a
    reduction)."""
    n = num_sms()
    if units <= 0 or k_iters % 2 or k_iters < 4:
        return 1
    eff = lambda u: u / (((u + n - 1) // n) * n)  # noqa: E731
    return 2 if eff(2 * units) >= gain * eff(units) else 1


# upper bound of the split-K factor of the dense decode GEMMs (AFD_MAX_SPLITS for A/B)
_MAX_SPLITS = int(os.environ.get("AFD_MAX_SPLITS", "16"))


def _dense_token_major(T: int, N: int, has_residual: bool) -> bool:
    """Whether a dense GEMM runs on the token-major kernel (128 token rows x
    256 features per tile): prefill sizes (more than 256 rows) with a multiple
    of 256 output features, and by default only with a residual add. Its
    row-segment epilogue reads the residual row by row (o_proj: 0.72 of the bf16
    peak at 8192 tokens against 0.58 on the swap-AB kernel, whose transposing
    epilogue the residual slows); qkv, without a residual, is faster on the
    swap-AB kernel's 256-token tiles."""
    if T <= 256 or N % 256 != 0:
        return False
    return _DENSE_TM == "all" or (_DENSE_TM == "residual" and has_residual)


def _moe_token_major(block_n: int, gathered: bool, T: int, top_k: int, n_experts: int) -> bool:
    """Whether the grouped expert GEMMs run on the token-major kernel: 128-row
    blocks of rows already gathered into expert order, and at least
    _MOE_TM_MIN_ROWS routed rows per expert on average (fuller blocks: the
    kernel's M is fixed at 128 rows, where the swap-AB kernel's N follows each
    block's row count)."""
    return (_MOE_TM and block_n == 128 and gathered
            and T * top_k >= _MOE_TM_MIN_ROWS * n_experts)


def _decode_tiling(T: int, N: int, K: int) -> Tuple[int, int]:
    """(token block, split-K factor) of a decode-sized dense GEMM (T <= 256),
    from a sweep of every combination on B200 for the qkv and o_proj shapes:
    64-row token blocks unless that leaves more tiles than SMs (then 128).
    With fewer than 40 tiles, the split that brings the units to about 128
    with at least 8 k-steps each; with more, a split of two only when each
    half still streams 32 k-steps (a split's partial store and last-CTA
    reduction cost more than shorter streams gain)."""
    n = num_sms()
    bn = 64
    while bn < 256 and T > bn and ((T + bn - 1) // bn) * (N // 128) > n:
        bn *= 2
    tiles = ((T + bn - 1) // bn) * (N // 128)
    k_iters = K // 64
    s = 1
    if tiles < 40:
        while (s * 2 <= _MAX_SPLITS and tiles * s * 2 <= 128 and k_iters % (s * 2) == 0
               and k_iters // (s * 2) >= 8):
            s *= 2
    elif tiles * 2 <= n and k_iters % 2 == 0 and k_iters // 2 >= 32 and _MAX_SPLITS >= 2:
        s = 2
    return bn, s


class _SplitKWorkspace:
    """fp32 partial-sum slices (one per split) and zero-initialised tile
    counters for split-K GEMMs. The kernel resets the counters after every
    launch, so one pair is reused forever; it is private to one stream (two
    streams never share)."""

    _pool: dict = {}
    _retired: list = []  # outgrown buffers stay alive: captured graphs may hold them

    @classmethod
    def get(cls, device, tiles: int, block_n: int, splits: int):
        stream = torch.cuda.current_stream(device)
        key = (device.index, stream.cuda_stream)
        need = splits * tiles * block_n * 128
        ws = cls._pool.get(key)
        if ws is None or ws[0].numel() < need or ws[1].numel() < tiles:
            old = ws
            n = max(need, old[0].numel() if old else 0)
            t = max(tiles, old[1].numel() if old else 0)
            ws = (torch.empty(n, device=device, dtype=torch.float32),
                  torch.zeros(t, device=device, dtype=torch.int32))
            if old is not None:
                cls._retired.append(old)
            cls._pool[key] = ws
        return ws


def linear(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None, peers: Sequence[int] = (), peer_row_offset: int = 0,
           flags: Sequence[int] = (), signal_value: int = 0,
           done_counter: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None,
           epoch: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = x @ w^T (+ residual) on the tcgen05 GEMM. `peers` are device
    addresses of peer-GPU buffers that receive the same rows (row offset
    `peer_row_offset`); with `done_counter`, the last CTA publishes
    `*epoch + signal_value` to each address in `flags`."""
    if not _cuda(x):
        return torch_ref.linear(x, w, residual)
    T, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(T, N, device=x.device, dtype=x.dtype)
    if N % 128 != 0:
        raise ValueError(f"linear: output features {N} must be a multiple of 128")
    tm = False
    if T <= 256:
        bn, splits = _decode_tiling(T, N, K)
    elif _dense_token_major(T, N, residual is not None):
        bn, splits, tm = 128, 1, True
    else:
        bn, splits = _block_n(T), 1
    tiles = ((T + bn - 1) // bn) * (N // 128)
    if T > 256 and not tm and 2 * tiles <= num_sms():
        # few output features (e.g. the router) over many tokens: narrower
        # token tiles spread the work over more SMs than split-K would
        bn = 64
        tiles = ((T + bn - 1) // bn) * (N // 128)
    ws = cnt = None
    if splits > 1:
        ws, cnt = _SplitKWorkspace.get(x.device, tiles, bn, splits)
    ext().gemm(w, x, out, N // 128, N, 0, None, None, T, residual, None, False, bn,
               tiles * splits, list(peers), int(peer_row_offset), list(flags), int(signal_value),
               done_counter, status, epoch, splits, ws, cnt, None, tm, False)
    return out


# -------------------------------------------------------------- attention --
def qk_norm_rope_cache(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor,
                       rope: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       start_pos: int, start_pos_dev: Optional[torch.Tensor], q_len: int,
                       batch_offset: int, nq: int, nkv: int, eps: float) -> torch.Tensor:
    if not _cuda(qkv):
        return torch_ref.qk_norm_rope_cache(qkv, q_norm, k_norm, rope, k_cache, v_cache,
                                            batch_offset, q_len, start_pos, nq, nkv, eps)
    T = qkv.shape[0]
    D = k_cache.shape[-1]
    q = torch.empty(T, nq, D, device=qkv.device, dtype=qkv.dtype)
    ext().qk_norm_rope_cache(qkv, q_norm, k_norm, rope, q, k_cache, v_cache, start_pos_dev,
                             q_len, batch_offset, nq, nkv, float(eps))
    return q


# Decode attention kernel: "tc" = tcgen05/TMEM/TMA kernel (head_dim 128, 4 or 8
# query heads per kv head; other shapes use the mma.sync kernels), "mma" =
# the mma.sync fused kernel and the split-KV SIMT kernel (A/B measurements).
_DECODE_ATTN = os.environ.get("AFD_DECODE_ATTN", "tc")
# prefill attention kernel: "tc" = tcgen05, two query heads of a kv group per
# CTA (one per CTA when the group is odd), "tc1" = tcgen05 with one head per
# CTA, "mma" = the mma.sync kernel (A/B measurements; padding masks always
# take the mma.sync kernel)
_PREFILL_ATTN = os.environ.get("AFD_PREFILL_ATTN", "tc")
_PREFILL_VARIANT = {"tc": 0, "tc1": 1, "mma": 2}
_DECODE_TILE = 128  # keys per tile of the tcgen05 decode kernel

# cost model of the tcgen05 decode kernel, in units of one 128-key tile's
# softmax round on one CTA: a work item's fixed cost (Q, pipeline fill,
# output) and a split merge; the HBM time of one tile across the GPU
_DEC_ITEM_COST = 2.0
_DEC_MERGE_COST = 3.0
_DEC_TILE_HBM = 0.01


def decode_splits(B: int, nkv: int, kv_len: int, sms: Optional[int] = None) -> int:
    """Key splits per (sequence, kv head) for the tcgen05 decode kernel: the
    count with the lowest estimated time, max(the busiest CTA's tiles and
    item overheads, the whole KV read at HBM speed) plus a merge when split.
    Splitting pays only when there are fewer (sequence, kv head) pairs than
    SMs and the sequences are long."""
    n = sms or num_sms()
    tiles = max(1, (kv_len + _DECODE_TILE - 1) // _DECODE_TILE)
    hbm = B * nkv * tiles * _DEC_TILE_HBM
    best, best_cost = 1, None
    for s in range(1, min(tiles, 16) + 1):
        waves = (B * nkv * s + n - 1) // n
        per = (tiles + s - 1) // s
        cost = max(waves * (per + _DEC_ITEM_COST), hbm) + (_DEC_MERGE_COST if s > 1 else 0.0)
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    return best


class _DecodeCounters:
    """Zeroed per-(sequence, kv head) merge counters of the tcgen05 decode
    kernel (the merging CTA resets its counter), one buffer per (device,
    stream); outgrown buffers stay alive for captured graphs."""

    _pool: dict = {}
    _retired: list = []

    @classmethod
    def get(cls, device, n: int) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        c = cls._pool.get(key)
        if c is None or c.numel() < n:
            if c is not None:
                cls._retired.append(c)
            c = torch.zeros(max(n, 1024), device=device, dtype=torch.int32)
            cls._pool[key] = c
        return c


def _tc_decode_ok(nq: int, nkv: int, D: int) -> bool:
    return _DECODE_ATTN == "tc" and bool(ext().decode_tc_supported(nq, nkv, D))


def decode_attention_tc(q: Optional[torch.Tensor], k_cache: torch.Tensor, v_cache: torch.Tensor,
                        batch_offset: int, start_pos: int, start_pos_dev: torch.Tensor,
                        nsplit: Optional[int] = None, status: Optional[torch.Tensor] = None,
                        fused: Optional[tuple] = None) -> torch.Tensor:
    """tcgen05 decode attention: q [B, nq, D] (one query per sequence, at
    position *start_pos_dev) over cache rows [batch_offset, +B); returns
    [B, nq, D]. `start_pos` (host) sizes the key splits; the kernel reads the
    position from the device, so graph replays may grow it. `fused` =
    (qkv [B, (nq + 2 nkv) D], q_norm, k_norm, rope, eps, nq) replaces q: the
    same launch applies q/k RMSNorm and RoPE and appends the token's K and V."""
    nkv, D = k_cache.shape[1], k_cache.shape[3]
    if fused is not None:
        qkv, q_norm, k_norm, rope, eps, nq = fused
        B = qkv.shape[0]
        dev = qkv.device
        out = torch.empty(B, nq, D, device=dev, dtype=qkv.dtype)
    else:
        B, nq, _ = q.shape
        dev = q.device
        out = torch.empty_like(q)
    if nsplit is None:
        nsplit = decode_splits(B, nkv, start_pos + 1)
    o_part = ml_part = cnt = None
    if nsplit > 1:
        o_part = torch.empty(B * nq, nsplit, D, device=dev, dtype=torch.float32)
        ml_part = torch.empty(B * nq, nsplit, 2, device=dev, dtype=torch.float32)
        cnt = _DecodeCounters.get(dev, B * nkv)
    if fused is not None:
        ext().decode_attention_tc(None, k_cache, v_cache, out, start_pos_dev, int(batch_offset),
                                  int(nsplit), o_part, ml_part, cnt, status, num_sms(), qkv,
                                  q_norm, k_norm, rope, float(eps))
    else:
        ext().decode_attention_tc(q.contiguous(), k_cache, v_cache, out, start_pos_dev,
                                  int(batch_offset), int(nsplit), o_part, ml_part, cnt, status,
                                  num_sms(), None, None, None, None, 0.0)
    return out


def decode_attention_fused(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor,
                           rope: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           start_pos: int, start_pos_dev: Optional[torch.Tensor],
                           batch_offset: int, nq: int, nkv: int, eps: float) -> torch.Tensor:
    """One decode step of attention for B sequences: q/k RMSNorm + RoPE of the
    new token, K/V append at `start_pos`, attention over positions
    0..start_pos. qkv [B, (nq + 2 nkv) D] -> [B, nq * D]."""
    if not _cuda(qkv):
        q = torch_ref.qk_norm_rope_cache(qkv, q_norm, k_norm, rope, k_cache, v_cache,
                                         batch_offset, 1, start_pos, nq, nkv, eps)
        return torch_ref.attention(q, k_cache, v_cache, batch_offset, 1, start_pos)
    B = qkv.shape[0]
    D = k_cache.shape[-1]
    nkv = k_cache.shape[1]
    if _tc_decode_ok(nq, nkv, D):
        # q/k RMSNorm + RoPE + KV append + tcgen05 attention in one launch
        return decode_attention_tc(None, k_cache, v_cache, batch_offset, start_pos,
                                   start_pos_dev,
                                   fused=(qkv, q_norm, k_norm, rope, eps, nq)).view(B, nq * D)
    out = torch.empty(B, nq, D, device=qkv.device, dtype=qkv.dtype)
    ext().decode_attention_fused(qkv, q_norm, k_norm, rope, k_cache, v_cache, out,
                                 start_pos_dev, batch_offset, nq, float(eps))
    return out.view(B, nq * D)


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, batch_offset: int,
              q_len: int, start_pos: int, start_pos_dev: Optional[torch.Tensor],
              key_range: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
    """Causal GQA attention over the cache; returns [T, nq * D]. `key_range`
    (prefill only) = (lo, hi) int32 tensors indexed by cache row: keys outside
    [lo, hi) are hidden (padding masks)."""
    if not _cuda(q):
        return torch_ref.attention(q, k_cache, v_cache, batch_offset, q_len, start_pos,
                                   key_range)
    T, nq, D = q.shape
    out = torch.empty(T, nq, D, device=q.device, dtype=q.dtype)
    if q_len == 1:
        if key_range is not None:
            raise ValueError("padding key ranges apply to prefill (q_len > 1) only")
        nkv = k_cache.shape[1]
        if _tc_decode_ok(nq, nkv, D):
            return decode_attention_tc(q, k_cache, v_cache, batch_offset, start_pos,
                                       start_pos_dev).view(T, nq * D)
        tiles = (start_pos + 1 + 63) // 64
        nsplit = max(1, min(tiles, (2 * num_sms() + T * nkv - 1) // max(1, T * nkv)))
        o_part = ml_part = None
        if nsplit > 1:
            o_part = torch.empty(T, nq, nsplit, D, device=q.device, dtype=torch.float32)
            ml_part = torch.empty(T, nq, nsplit, 2, device=q.device, dtype=torch.float32)
        ext().decode_attention(q, k_cache, v_cache, out, start_pos_dev, batch_offset, nsplit,
                               o_part, ml_part)
    else:
        lo, hi = key_range if key_range is not None else (None, None)
        ext().prefill_attention(q, k_cache, v_cache, out, start_pos_dev, q_len, batch_offset,
                                lo, hi, _PREFILL_VARIANT[_PREFILL_ATTN])
    return out.view(T, nq * D)


# -------------------------------------------------------------------- MoE --
def router_topk(h: torch.Tensor, post_norm_w: torch.Tensor, w_router: torch.Tensor, top_k: int,
                eps: float, norm_topk_prob: bool = True
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Post-attention RMSNorm, router projection, fp32 softmax, top-k,
    renormalise: (normed x, ids int32 [T,k], weights fp32 [T,k])."""
    if not _cuda(h):
        return torch_ref.router_topk(h, post_norm_w, w_router, top_k, eps, norm_topk_prob)
    xn = rmsnorm(h, post_norm_w, eps)
    E = w_router.shape[0]
    if E % 128 == 0:
        logits = linear(xn, w_router)
    else:  # tiny test models: router narrower than one GEMM tile
        logits = torch.nn.functional.linear(xn, w_router)
    T = h.shape[0]
    ids = torch.empty(T, top_k, device=h.device, dtype=torch.int32)
    w = torch.empty(T, top_k, device=h.device, dtype=torch.float32)
    ext().router_topk(logits, ids, w, top_k, bool(norm_topk_prob))
    return xn, ids, w


_GATHER4_MAX_TOKENS = 512


class MoEWorkspace:
    """Device buffers of one MoE call (sized for T tokens)."""

    def __init__(self, T: int, top_k: int, n_local: int, H: int, I: int, block_n: int, device,
                 dtype):
        R = T * top_k
        mk = lambda *s, dt=torch.int32: torch.empty(*s, device=device, dtype=dt)  # noqa: E731
        self.inv = mk(R)
        self.row_token = mk(R)
        self.row_weight = mk(R, dt=torch.float32)
        self.expert_offsets = mk(n_local + 1)
        max_blocks = n_local + (R + block_n - 1) // block_n
        self.blocks = mk(max_blocks, 4)
        self.num_blocks = mk(1)
        self.num_rows = mk(1)
        self.act = mk(R, I, dt=dtype)
        self.y = mk(R, H, dt=dtype)
        self.ids = mk(T, top_k)
        self.weights = mk(T, top_k, dt=torch.float32)
        self.max_blocks = max_blocks
        self.block_n = block_n


# decode-sized token counts: up to here the F2A rows are stored by the combine
# itself (straight to the attention ranks), or, with AFD_FUSED_COMBINE=1, by
# the down GEMM's epilogue; above, the combine writes locally and one bulk
# peer copy per attention rank moves the rows
_FUSED_COMBINE_MAX_TOKENS = 256


def _moe_gemms_combine(xn, ws: MoEWorkspace, w_gate_up, w_down, residual, out, T, k, peers,
                       seg_offsets, peer_row_offset, flags, signal_value, done_counter, epoch,
                       n_experts=None):
    """Grouped gate_up GEMM (SwiGLU epilogue) -> grouped down GEMM
    (routing-weight epilogue) -> combine (+ residual, + peer stores). For
    decode-sized batches the gate_up producer gathers token rows straight from
    xn with TMA tile::gather4; prefill-sized batches gather once into expert
    order so the producer issues one TMA box per 32 rows (swap-AB kernel) or
    per 128 rows (token-major kernel, when the experts average at least
    _MOE_TM_MIN_ROWS rows; `n_experts` = the router's expert count, default
    the local one)."""
    C = ext()
    E_loc, I2, H = w_gate_up.shape
    I = I2 // 2
    bn = ws.block_n
    if T <= _GATHER4_MAX_TOKENS:
        x, row_ids = xn, ws.row_token
    else:
        R = T * k
        x = torch.empty(R, H, device=xn.device, dtype=xn.dtype)
        C.moe_gather(xn, ws.row_token, ws.num_rows, x, R)
        row_ids = None
    # decode sizes: about one row block per hit expert, I/128 (gate_up) or
    # H/128 (down) feature tiles each -- a few tiles per SM, so when the last
    # wave of the persistent grid would run half empty, K is split in two
    max_tiles = ws.max_blocks * (I // 128)
    decode = T <= _FUSED_COMBINE_MAX_TOKENS
    est_blocks = min(E_loc, T * k)
    gu_splits = _wave_splits(est_blocks * (I // 128), H // 64) if (decode and _GU_SPLIT) else 1
    dn_splits = _wave_splits(est_blocks * (H // 128), I // 64) if (decode and _GU_SPLIT) else 1
    # decode sizes: stream-K scheduling of the expert GEMMs (equal k-iteration
    # ranges per CTA; the few tiles a range boundary cuts are reduced in two
    # pieces), so the grid's last wave is not left half empty
    sk = _STREAM_K and decode and gu_splits == 1 and dn_splits == 1
    gws = gcnt = None
    if gu_splits > 1 or sk:
        gws, gcnt = _SplitKWorkspace.get(xn.device, 2 * max_tiles, bn, max(gu_splits, 2))
    # prefill-sized: full 128-row blocks on the token-major kernel (128 x 256 MMAs,
    # row-segment epilogue); decode-sized: the swap-AB kernel
    tm = _moe_token_major(bn, row_ids is None, T, k, n_experts or E_loc)
    C.gemm(w_gate_up.view(E_loc * I2, H), x, ws.act, I // 128, I2, I, ws.blocks, ws.num_blocks,
           0, None, None, True, bn, max_tiles * gu_splits, [], 0, [], 0, None, None, None,
           gu_splits, gws, gcnt, row_ids, tm, sk)
    if out is None and not peers:
        out = torch.empty(T, H, device=xn.device, dtype=xn.dtype)
    if _FUSED_COMBINE and T <= _FUSED_COMBINE_MAX_TOKENS:
        # combine (+ residual, + F2A stores, + flags) in the down GEMM's epilogue
        C.gemm_down_combine(w_down.view(E_loc * H, I), ws.act, ws.y, H // 128, H, ws.blocks,
                            ws.num_blocks, ws.row_weight, bn, ws.max_blocks * (H // 128), ws.inv,
                            T, k, residual, out, list(peers), list(seg_offsets),
                            int(peer_row_offset), list(flags), int(signal_value), done_counter,
                            None, epoch, _CombineCounters.get(xn.device, H // 128))
        return out
    dws = dcnt = None
    dn_tiles = ws.max_blocks * (H // 128)
    if dn_splits > 1 or sk:
        dws, dcnt = _SplitKWorkspace.get(xn.device, dn_tiles, bn, max(dn_splits, 2))
    C.gemm(w_down.view(E_loc * H, I), ws.act, ws.y, H // 128, H, 0, ws.blocks, ws.num_blocks, 0,
           None, ws.row_weight, False, bn, dn_tiles * dn_splits, [], 0, [], 0, None, None,
           None, dn_splits, dws, dcnt, None, tm, sk)
    if peers and _SPLIT_F2A and T > _FUSED_COMBINE_MAX_TOKENS:
        # prefill sizes: combine locally, then one bulk peer copy per attention
        # rank's segment (the combine kernel's scattered NVLink stores run at
        # about half the link bandwidth; the copy kernel reaches ~0.7 of it)
        local = out if out is not None else torch.empty(T, H, device=xn.device, dtype=xn.dtype)
        C.moe_combine(ws.y, ws.inv, T, k, residual, local, [], [], 0, [], 0, None, None)
        row_bytes = H * local.element_size()
        for i, (dst, flag) in enumerate(zip(peers, flags)):
            lo, hi = int(seg_offsets[i]), int(seg_offsets[i + 1])
            if hi <= lo:
                continue
            grid = max(1, min(4 * num_sms(), (hi - lo) * row_bytes // (16 * 512)))
            C.peer_copy(local[lo:hi], [int(dst) + int(peer_row_offset) * row_bytes], [int(flag)],
                        int(signal_value), done_counter, epoch, grid)
        return out
    # decode sizes: the combine stores each token's row straight into its
    # attention rank's buffer (one kernel; no local copy and second launch)
    C.moe_combine(ws.y, ws.inv, T, k, residual, out, list(peers), list(seg_offsets),
                  int(peer_row_offset), list(flags), int(signal_value), done_counter, epoch)
    return out


_ALIGN_CHUNK = 2048  # routed entries per CTA of the multi-CTA routing


# AFD_BOUNDS_CHECK=1: validate the routing tables on the host after every
# routing step (debug mode, one device sync per MoE layer; see ops/checks.py)
_BOUNDS_CHECK = os.environ.get("AFD_BOUNDS_CHECK", "0") == "1"


def _check_routing(ids: torch.Tensor, weights: torch.Tensor, expert_start: int, E_loc: int,
                   ws: "MoEWorkspace") -> None:
    if not _BOUNDS_CHECK or torch.cuda.is_current_stream_capturing():
        return
    from .checks import check_routing_tables
    torch.cuda.current_stream().synchronize()
    check_routing_tables(ids, weights, expert_start, E_loc, ws.block_n, ws.inv, ws.row_token,
                         ws.row_weight, ws.expert_offsets, ws.blocks, ws.num_blocks,
                         ws.num_rows)


def _align(ids: torch.Tensor, weights: torch.Tensor, expert_start: int, E_loc: int,
           ws: "MoEWorkspace") -> None:
    """Expert-sorted rows and row blocks from top-k ids: one CTA up to two
    chunks of entries, the two-kernel multi-CTA routing above that."""
    C = ext()
    n = ids.numel()
    if n <= 2 * _ALIGN_CHUNK:
        C.moe_align(ids, weights, expert_start, E_loc, ws.block_n, ws.inv, ws.row_token,
                    ws.row_weight, ws.expert_offsets, ws.blocks, ws.num_blocks, ws.num_rows)
        return
    chunks = (n + _ALIGN_CHUNK - 1) // _ALIGN_CHUNK
    part = torch.empty(chunks * E_loc, device=ids.device, dtype=torch.int32)
    C.moe_align_mt(ids, weights, expert_start, E_loc, ws.block_n, ws.inv, ws.row_token,
                   ws.row_weight, ws.expert_offsets, ws.blocks, ws.num_blocks, ws.num_rows, part,
                   _AlignCounters.get(ids.device, 0))


def moe_experts(xn: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                w_gate_up: torch.Tensor, w_down: torch.Tensor, expert_start: int = 0,
                residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                peers: Sequence[int] = (), seg_offsets: Sequence[int] = (),
                peer_row_offset: int = 0, flags: Sequence[int] = (), signal_value: int = 0,
                done_counter: Optional[torch.Tensor] = None, epoch: Optional[torch.Tensor] = None,
                ws: Optional[MoEWorkspace] = None) -> torch.Tensor:
    """(residual +) sum over the token's local top-k experts of
    w * down(silu(gate x) * up x); bf16 [T, H]. GPU path: routing kernel,
    grouped tcgen05 GEMMs, combine (+ residual, + peer stores)."""
    T, H = xn.shape
    if not _cuda(xn):
        y = torch_ref.moe_experts(xn, ids, weights, w_gate_up, w_down, expert_start)
        if residual is not None:
            y = y + residual.float()
        return y.to(xn.dtype)
    E_loc, I2, _ = w_gate_up.shape
    k = ids.shape[1]
    if ws is None:
        ws = MoEWorkspace(T, k, E_loc, H, I2 // 2, _moe_block_n(T), xn.device, xn.dtype)
    _align(ids, weights, expert_start, E_loc, ws)
    _check_routing(ids, weights, expert_start, E_loc, ws)
    return _moe_gemms_combine(xn, ws, w_gate_up, w_down, residual, out, T, k, peers, seg_offsets,
                              peer_row_offset, flags, signal_value, done_counter, epoch)


_GATE_MAX_ENTRIES = 2048  # routed (token, k) pairs handled by the fused gate kernel


# Switches for A/B measurements: AFD_FUSED_GATE=0 selects the unfused gate kernel
# sequence, AFD_FUSED_COMBINE=1 the combine inside the down GEMM's epilogue.
_FUSED_GATE = os.environ.get("AFD_FUSED_GATE", "1") != "0"
_SPLIT_F2A = os.environ.get("AFD_SPLIT_F2A", "1") != "0"  # prefill F2A: combine, then bulk copy
# wave-balancing split-K of the decode expert GEMMs: measured slower (a split's
# partial store and reduction cost more than the fuller last wave gains), so opt-in
_GU_SPLIT = os.environ.get("AFD_GU_SPLIT", "0") == "1"
_FUSED_COMBINE = os.environ.get("AFD_FUSED_COMBINE", "0") == "1"  # measured slower (esp. with peers)
# AFD_STREAM_K=1: stream-K ranges for the decode expert GEMMs instead of
# round-robin tiles. Measured no faster (32-128 local experts, 16-256 tokens:
# the fixed per-call costs, not the last wave, keep the expert-parallel slices
# at 0.6-0.8 of the HBM bandwidth) and 2-5 us slower per call, so opt-in
_STREAM_K = os.environ.get("AFD_STREAM_K", "0") == "1"


def _gate_fusable(T: int, H: int, E: int, top_k: int) -> bool:
    return (_FUSED_GATE and T * top_k <= _GATE_MAX_ENTRIES and H in (1024, 2048, 4096)
            and E <= 256 and E % 8 == 0 and top_k <= 16)


class _GateCounters:
    """Zeroed int32 counters of the fused gate kernel (it leaves them zeroed),
    one buffer per (device, stream); outgrown buffers stay alive for graphs."""

    _pool: dict = {}
    _retired: list = []

    @classmethod
    def get(cls, device, T: int) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        c = cls._pool.get(key)
        if c is None or c.numel() < T + 1:
            if c is not None:
                cls._retired.append(c)
            c = torch.zeros(max(T + 1, 257), device=device, dtype=torch.int32)
            cls._pool[key] = c
        return c


class _CombineCounters(_GateCounters):
    """Zeroed per-feature-tile counters of the fused combine."""

    _pool: dict = {}
    _retired: list = []


class _AlignCounters(_GateCounters):
    """Zeroed completion counter of the multi-CTA routing."""

    _pool: dict = {}
    _retired: list = []


def moe_gate(h: torch.Tensor, post_norm_w: torch.Tensor, w_router: torch.Tensor, top_k: int,
             eps: float, norm_topk_prob: bool = True, expert_start: int = 0,
             n_local: Optional[int] = None, stamps: Optional[torch.Tensor] = None
             ) -> Tuple[torch.Tensor, "MoEWorkspace"]:
    """The fused decode gate alone (RMSNorm, router, top-k, routing): returns
    the normalised input and the routing workspace (ids, weights, row blocks).
    `stamps` (int64 [8], zeroed) receives %globaltimer stamps of the kernel's
    phases (diagnostics)."""
    T, H = h.shape
    E = w_router.shape[0]
    n_local = E if n_local is None else n_local
    if not _gate_fusable(T, H, E, top_k):
        raise ValueError("moe_gate: shape outside the fused gate's limits")
    ws = MoEWorkspace(T, top_k, n_local, H, 768, _moe_block_n(T), h.device, h.dtype)
    xn = torch.empty_like(h)
    logits = torch.empty(T, E, device=h.device, dtype=h.dtype)
    ext().moe_gate(h, post_norm_w, w_router, xn, logits, ws.ids, ws.weights,
                   _GateCounters.get(h.device, T), top_k, bool(norm_topk_prob), float(eps),
                   expert_start, n_local, ws.block_n, ws.inv, ws.row_token,
                   ws.row_weight, ws.expert_offsets, ws.blocks, ws.num_blocks, ws.num_rows,
                   *_wait_args(None), stamps)
    return xn, ws


def moe_ffn(h: torch.Tensor, post_norm_w: torch.Tensor, w_router: torch.Tensor,
            w_gate_up: torch.Tensor, w_down: torch.Tensor, top_k: int, eps: float,
            norm_topk_prob: bool = True, expert_start: int = 0, add_residual: bool = True,
            out: Optional[torch.Tensor] = None, peers: Sequence[int] = (),
            seg_offsets: Sequence[int] = (), peer_row_offset: int = 0, flags: Sequence[int] = (),
            signal_value: int = 0, done_counter: Optional[torch.Tensor] = None,
            epoch: Optional[torch.Tensor] = None, tracker_marks=None,
            wait: Optional[FlagWait] = None) -> torch.Tensor:
    """The whole sparse-MoE block on h = attn_out + residual: post-attention
    RMSNorm, router GEMM, softmax/top-k/renormalise + routing (one kernel for
    up to 4096 routed pairs), grouped expert GEMMs, combine. Returns
    h + moe(norm(h)) (or the local experts' partial sum)."""
    mark = tracker_marks or (lambda *_: None)
    if not _cuda(h):
        mark(True, "router")
        xn, ids, w = torch_ref.router_topk(h, post_norm_w, w_router, top_k, eps, norm_topk_prob)
        mark(False, "router")
        mark(True, "experts")
        y = moe_experts(xn, ids, w, w_gate_up, w_down, expert_start,
                        residual=h if add_residual else None)
        mark(False, "experts")
        return y
    T, H = h.shape
    E = w_router.shape[0]
    E_loc, I2, _ = w_gate_up.shape
    mark(True, "router")
    ws = MoEWorkspace(T, top_k, E_loc, H, I2 // 2, _moe_block_n(T), h.device, h.dtype)
    C = ext()
    if _gate_fusable(T, H, E, top_k):
        # decode sizes: norm + router + top-k + routing in one launch
        xn = torch.empty_like(h)
        logits = torch.empty(T, E, device=h.device, dtype=h.dtype)
        C.moe_gate(h, post_norm_w, w_router, xn, logits, ws.ids, ws.weights,
                   _GateCounters.get(h.device, T), top_k, bool(norm_topk_prob), float(eps),
                   expert_start, E_loc, ws.block_n, ws.inv, ws.row_token,
                   ws.row_weight, ws.expert_offsets, ws.blocks, ws.num_blocks, ws.num_rows,
                   *_wait_args(wait), None)
        _check_routing(ws.ids, ws.weights, expert_start, E_loc, ws)
        mark(False, "router")
        mark(True, "experts")
        y = _moe_gemms_combine(xn, ws, w_gate_up, w_down, h if add_residual else None, out, T,
                               top_k, peers, seg_offsets, peer_row_offset, flags, signal_value,
                               done_counter, epoch, n_experts=E)
        mark(False, "experts")
        return y
    xn = sum_rmsnorm([h], post_norm_w, eps, wait=wait)[1]
    logits = linear(xn, w_router) if E % 128 == 0 else torch.nn.functional.linear(xn, w_router)
    if T * top_k <= 4096 and E <= 256:
        C.moe_route(logits, ws.ids, ws.weights, top_k, bool(norm_topk_prob), expert_start, E_loc,
                    ws.block_n, ws.inv, ws.row_token, ws.row_weight, ws.expert_offsets,
                    ws.blocks, ws.num_blocks, ws.num_rows)
    else:
        C.router_topk(logits, ws.ids, ws.weights, top_k, bool(norm_topk_prob))
        _align(ws.ids, ws.weights, expert_start, E_loc, ws)
    _check_routing(ws.ids, ws.weights, expert_start, E_loc, ws)
    mark(False, "router")
    mark(True, "experts")
    y = _moe_gemms_combine(xn, ws, w_gate_up, w_down, h if add_residual else None, out, T, top_k,
                           peers, seg_offsets, peer_row_offset, flags, signal_value,
                           done_counter, epoch, n_experts=E)
    mark(False, "experts")
    return y


def dense_mlp(xn: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
              residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not _cuda(xn):
        y = torch_ref.dense_mlp(xn, w_gate_up, w_down)
        return y if residual is None else (y.float() + residual.float()).to(xn.dtype)
    T, H = xn.shape
    I2 = w_gate_up.shape[0]
    I = I2 // 2
    if I % 128:
        raise ValueError(f"dense MLP width {I} (this rank's slice) is not a multiple of 128, "
                         "the SwiGLU GEMM's feature tile")
    act = torch.empty(T, I, device=xn.device, dtype=xn.dtype)
    bn = _block_n(T)
    units = ((T + bn - 1) // bn) * (I // 128)
    ext().gemm(w_gate_up, xn, act, I // 128, I2, I, None, None, T, None, None, True, bn, units,
               [], 0, [], 0, None, None, None, 1, None, None, None, False, False)
    return linear(act, w_down, residual=residual)


# ------------------------------------------------------------- sampling --
class _ArgmaxCounters(_GateCounters):
    """Per-row counters of the split argmax (zeroed; the kernel leaves them
    zeroed), one buffer per (device, stream). They are kept apart from the
    partials, whose layout depends on the row count: in a shared buffer a
    call with fewer rows would leave its partials where a later call with
    more rows expects zeroed counters."""

    _pool: dict = {}
    _retired: list = []


class _ArgmaxPartials:
    """Per-chunk partial maxima of the split argmax (no initial value needed),
    one buffer per (device, stream); outgrown buffers stay alive for graphs."""

    _pool: dict = {}
    _retired: list = []

    @classmethod
    def get(cls, device, n: int) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        b = cls._pool.get(key)
        if b is None or b.numel() < n:
            if b is not None:
                cls._retired.append(b)
            b = torch.empty(n, device=device, dtype=torch.int32)
            cls._pool[key] = b
        return b


def argmax(logits: torch.Tensor) -> torch.Tensor:
    """First index of the row maximum (torch.argmax semantics for finite
    values) [rows, V] bf16 -> [rows] int64. Large rows are split over several
    CTAs with a last-CTA reduction."""
    if not _cuda(logits) or logits.dtype != torch.bfloat16:
        return torch_ref.argmax(logits)
    rows = logits.shape[0]
    out = torch.empty(rows, device=logits.device, dtype=torch.int64)
    counters = _ArgmaxCounters.get(logits.device, rows)
    partials = _ArgmaxPartials.get(logits.device,
                                   ext().argmax_partial_ints(rows, logits.shape[1]))
    ext().argmax(logits, out, counters, partials)
    return out


def rope_table(max_pos: int, head_dim: int, theta: float, device) -> torch.Tensor:
    return torch_ref.rope_table(max_pos, head_dim, theta, device, torch.bfloat16)
