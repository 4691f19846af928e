"""Pure-PyTorch statements of every op the framework runs.

These are (1) the CPU execution path (the reference's ``--backend cpu`` /
gloo mode, src/utils/device.py:55-63) and (2) the oracle the CUDA kernels are
tested against. Numerics follow HF Qwen3-MoE (transformers 5.x,
``modeling_qwen3_moe``): RMSNorm in fp32 then cast, weight multiply in the
activation dtype; router softmax in fp32 over the projected logits, top-k,
renormalise; experts ``down(silu(gate(x)) * up(x)) * w``.

The kernels accumulate in fp32 and round once where HF rounds several times,
so GPU-vs-oracle comparisons are tolerance based.
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return w * (xf * torch.rsqrt(var + eps)).to(dt)


def sum_rmsnorm(parts: Sequence[torch.Tensor], w: torch.Tensor, eps: float
                ) -> Tuple[torch.Tensor, torch.Tensor]:
    """x = sum(parts) (fp32 sum, one rounding); returns (x, rmsnorm(x))."""
    if len(parts) == 1:
        x = parts[0]
    else:
        acc = parts[0].float()
        for p in parts[1:]:
            acc = acc + p.float()
        x = acc.to(parts[0].dtype)
    return x, rmsnorm(x, w, eps)


def linear(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None
           ) -> torch.Tensor:
    y = F.linear(x, w)
    if residual is not None:
        y = y + residual
    return y


def rope_table(max_pos: int, head_dim: int, theta: float, device, dtype=torch.float32
               ) -> torch.Tensor:
    """[max_pos, head_dim] table: cos in the first half, sin in the second,
    for the half-dim frequencies (HF default RoPE). Values are rounded to the
    activation dtype as HF does (``cos.to(x.dtype)``) but stored as fp32."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64, device=device)
                                .float() / head_dim))
    pos = torch.arange(max_pos, device=device, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    cos = freqs.cos().to(dtype).float()
    sin = freqs.sin().to(dtype).float()
    return torch.cat([cos, sin], dim=-1).contiguous()


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rope(x: torch.Tensor, cos_sin: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """x [T, nh, D]; pos [T] int; table from rope_table."""
    D = x.shape[-1]
    cs = cos_sin[pos.long()]  # [T, D]
    cos = torch.cat([cs[:, : D // 2], cs[:, : D // 2]], -1).to(x.dtype)[:, None, :]
    sin = torch.cat([cs[:, D // 2:], cs[:, D // 2:]], -1).to(x.dtype)[:, None, :]
    return (x * cos) + (_rotate_half(x) * sin)


def qk_norm_rope_cache(qkv: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
                       cos_sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       batch_offset: int, q_len: int, start_pos: int, n_q: int, n_kv: int,
                       eps: float) -> torch.Tensor:
    """Split qkv [T, (nq+2nkv)*D]; per-head RMSNorm of q and k; RoPE; write k,v
    into the cache at rows batch_offset + t // q_len, positions
    start_pos + t % q_len. Returns q [T, nq, D]."""
    T = qkv.shape[0]
    D = q_norm_w.shape[0]
    q = qkv[:, : n_q * D].view(T, n_q, D)
    k = qkv[:, n_q * D: (n_q + n_kv) * D].view(T, n_kv, D)
    v = qkv[:, (n_q + n_kv) * D:].view(T, n_kv, D)
    q = rmsnorm(q, q_norm_w, eps)
    k = rmsnorm(k, k_norm_w, eps)
    t = torch.arange(T, device=qkv.device)
    pos = start_pos + t % q_len
    b = batch_offset + t // q_len
    q = apply_rope(q, cos_sin, pos)
    k = apply_rope(k, cos_sin, pos)
    k_cache[b, :, pos] = k.to(k_cache.dtype)
    v_cache[b, :, pos] = v.to(v_cache.dtype)
    return q.contiguous()


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              batch_offset: int, q_len: int, start_pos: int,
              key_range: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
    """Causal GQA attention of q [B*q_len, nq, D] against cache rows
    [batch_offset, batch_offset+B) and positions [0, start_pos+q_len).
    Query i of a sequence sits at position start_pos+i and sees keys <= it.
    `key_range` = (lo, hi), int tensors indexed by cache row: only keys in
    [lo, hi) are visible (padding); a query that sees no key outputs zeros.
    Returns [B*q_len, nq*D]."""
    T, nq, D = q.shape
    B = T // q_len
    kv_len = start_pos + q_len
    k = k_cache[batch_offset:batch_offset + B, :, :kv_len].float()
    v = v_cache[batch_offset:batch_offset + B, :, :kv_len].float()
    nkv = k.shape[1]
    g = nq // nkv
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    qf = q.view(B, q_len, nq, D).transpose(1, 2).float()  # [B, nq, q_len, D]
    s = torch.matmul(qf, k.transpose(-1, -2)) / math.sqrt(D)
    qpos = start_pos + torch.arange(q_len, device=q.device)
    kpos = torch.arange(kv_len, device=q.device)
    mask = (kpos[None, :] > qpos[:, None])[None, None]  # [1, 1, q_len, kv_len]
    if key_range is not None:
        lo = key_range[0][batch_offset:batch_offset + B].to(q.device).long()
        hi = key_range[1][batch_offset:batch_offset + B].to(q.device).long()
        out_of_range = (kpos[None, :] < lo[:, None]) | (kpos[None, :] >= hi[:, None])
        mask = mask | out_of_range[:, None, None, :]
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)  # rows with no visible key -> 0
    o = torch.matmul(p, v)  # [B, nq, q_len, D]
    return o.transpose(1, 2).reshape(T, nq * D).to(q.dtype)


def router_topk(h: torch.Tensor, post_norm_w: torch.Tensor, w_router: torch.Tensor,
                top_k: int, eps: float, norm_topk_prob: bool = True
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """post-attention RMSNorm + router: returns (normed x, ids int32 [T,k],
    weights fp32 [T,k])."""
    xn = rmsnorm(h, post_norm_w, eps)
    logits = F.linear(xn, w_router)
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    w, ids = torch.topk(probs, top_k, dim=-1)
    if norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    return xn, ids.to(torch.int32), w.float()


def moe_experts(xn: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                w_gate_up: torch.Tensor, w_down: torch.Tensor, expert_start: int = 0
                ) -> torch.Tensor:
    """Sum over the token's top-k experts that live in [expert_start,
    expert_start + E_local) of w * down(silu(gate x) * up x). fp32 accumulate."""
    T, H = xn.shape
    E_loc = w_gate_up.shape[0]
    I = w_gate_up.shape[1] // 2
    out = torch.zeros(T, H, dtype=torch.float32, device=xn.device)
    local = ids.long() - expert_start
    for e in range(E_loc):
        tok, slot = torch.where(local == e)
        if tok.numel() == 0:
            continue
        x = xn[tok]
        gu = F.linear(x, w_gate_up[e])
        a = F.silu(gu[:, :I]) * gu[:, I:]
        y = F.linear(a, w_down[e]).float() * weights[tok, slot, None]
        out.index_add_(0, tok, y)
    return out


def dense_mlp(xn: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    I = w_gate_up.shape[0] // 2
    gu = F.linear(xn, w_gate_up)
    return F.linear(F.silu(gu[:, :I]) * gu[:, I:], w_down)


def ffn_layer(h: torch.Tensor, post_norm_w, w_router, w_gate_up, w_down, top_k: int,
              eps: float, expert_start: int = 0, add_residual: bool = True,
              norm_topk_prob: bool = True, dense: Optional[Tuple] = None) -> torch.Tensor:
    """Full FFN block on the pre-combined input h = attn_out + residual:
    returns h + moe(norm(h)) (or only the local-expert partial sum when
    add_residual is False)."""
    if dense is not None:
        xn = rmsnorm(h, post_norm_w, eps)
        y = dense_mlp(xn, *dense).float()
    else:
        xn, ids, w = router_topk(h, post_norm_w, w_router, top_k, eps, norm_topk_prob)
        y = moe_experts(xn, ids, w, w_gate_up, w_down, expert_start)
    if add_residual:
        y = y + h.float()
    return y.to(h.dtype)


def argmax(logits: torch.Tensor) -> torch.Tensor:
    return logits.argmax(dim=-1)


def stack_parts(parts: List[torch.Tensor]) -> torch.Tensor:
    return torch.stack(parts, 0)
