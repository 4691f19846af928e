"""Attention role: embedding, per-layer attention block, KV cache, final norm,
LM head.

Reference: ``AttentionLayer`` / ``AttentionWorker``
(src/model/attention_worker.py:24-313), which wrap HF ``Qwen3MoeAttention`` and
shard layers over the role's visible GPUs. Here one B200 holds every layer
(≈3.6 GB of attention weights in bf16), and a layer is five ops:

1. ``sum_rmsnorm``   x = sum of the F2A partials (one per FFN rank), RMSNorm
2. ``linear``        qkv = x_n @ W_qkv^T (tcgen05 GEMM)
3. ``qk_norm_rope_cache``  per-head q/k RMSNorm, RoPE, K/V append in place
4. ``attention``     flash decode (q_len 1) or causal flash prefill
5. ``linear``        h = o @ W_o^T + x  -- the A2F hand-off: with a fused
   transport the epilogue stores h straight into the FFN GPUs' receive
   buffers and raises their flags.

``attention_block`` returns h = attn_out + residual, the
"pre-combined" tensor the reference ships to the FFN
(src/model/disaggregated.py:184). ``forward_attention_layer`` and
``forward_lm_head`` keep the reference's per-layer calls.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from .. import ops
from ..config import ModelConfig
from .kv_cache import KVCache
from .weights import AttentionWeights


class AttentionWorker:
    def __init__(self, cfg: ModelConfig, weights: AttentionWeights, device, dtype=torch.bfloat16,
                 max_batch: int = 4, max_seq: int = 2048):
        self.cfg = cfg
        self.w = weights
        self.device = torch.device(device)
        self.dtype = dtype
        self.num_layers = cfg.num_hidden_layers
        self.rope = ops.rope_table(max_seq, cfg.head_dim, cfg.rope_theta, self.device)
        self.cache = KVCache(cfg.num_hidden_layers, max_batch, cfg.num_key_value_heads, max_seq,
                             cfg.head_dim, self.device, dtype)
        self.tracker = None  # optional TimingTracker for sub-stage events
        self.layers = [AttentionLayer(self, l) for l in range(self.num_layers)]
        # (lo, hi) visible key range per cache row for the current prefill
        # (padding masks), set by the model around one forward; None = causal only
        self.key_range = None

    # the reference's attribute names (src/model/attention_worker.py:158-245);
    # one GPU holds every layer, so the role's device list is this device
    @property
    def config(self) -> ModelConfig:
        return self.cfg

    @property
    def hidden_size(self) -> int:
        return self.cfg.hidden_size

    @property
    def attention_layers(self) -> list:
        return self.layers

    @property
    def role_devices(self) -> list:
        return [self.device]

    @classmethod
    def from_pretrained(cls, model_name: str, device, dtype=torch.bfloat16,
                        max_batch: int = 4, max_seq: int = 2048,
                        random_init: Optional[bool] = None, seed: int = 0) -> "AttentionWorker":
        """Reference: ``AttentionWorker.from_pretrained``
        (src/model/attention_worker.py:316-344), which loads the whole HF
        model on the CPU and keeps its attention parts. Here only the
        checkpoint's attention-side tensors (embedding, attention, norms, LM
        head) are read, straight to `device`; a preset name without a
        checkpoint directory gets random weights (`seed`)."""
        import os

        from ..config import resolve_model_config
        from .weights import load_attention_weights, random_attention_weights

        cfg = resolve_model_config(model_name)
        if random_init is None:
            random_init = not os.path.isdir(model_name)
        w = (random_attention_weights(cfg, seed, device, dtype) if random_init
             else load_attention_weights(model_name, cfg, device, dtype))
        return cls(cfg, w, device, dtype, max_batch, max_seq)

    @classmethod
    def from_hf_model(cls, model, device, dtype=torch.bfloat16, max_batch: int = 4,
                      max_seq: int = 2048) -> "AttentionWorker":
        """The counterpart of the reference's ``AttentionWorker(model, device,
        dtype)`` (src/model/attention_worker.py:170-237), which takes a loaded
        HF ``Qwen3MoeForCausalLM``: its config and attention-side tensors are
        copied to `device` (per-expert or fused expert layouts alike)."""
        from ..config import ModelConfig
        from .weights import load_attention_weights

        cfg = ModelConfig.from_dict(model.config.to_dict())
        w = load_attention_weights(model.state_dict(), cfg, device, dtype)
        return cls(cfg, w, device, dtype, max_batch, max_seq)

    # ------------------------------------------------------------------
    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        """[B, S] ids -> [B*S, H] hidden states."""
        return torch.nn.functional.embedding(input_ids.reshape(-1), self.w.embed)

    def get_position_embeddings(self, hidden_states: torch.Tensor,
                                position_ids: Optional[torch.Tensor] = None):
        """(cos, sin) [B, S, D] for `position_ids`, with the reference's
        signature (hidden_states, position_ids); `hidden_states` only gives
        the call its HF shape. Called with one tensor, that tensor is taken as
        the position ids."""
        if position_ids is None:
            position_ids = hidden_states
        D = self.cfg.head_dim
        cs = self.rope[position_ids.long()]
        cos = torch.cat([cs[..., : D // 2]] * 2, -1).to(self.dtype)
        sin = torch.cat([cs[..., D // 2:]] * 2, -1).to(self.dtype)
        return cos, sin

    def forward_attention_layer(self, layer_idx: int, hidden_states: torch.Tensor,
                                attention_mask: Optional[torch.Tensor] = None,
                                position_ids: Optional[torch.Tensor] = None,
                                position_embeddings=None, use_cache: bool = False,
                                past_key_value=None):
        """The reference's per-layer call
        (src/model/attention_worker.py:271-307): `hidden_states` [B, S, H] ->
        (attn_output, residual), plus the KV cache with `use_cache`. Same
        behaviour as ``self.layers[layer_idx]`` (``AttentionLayer``)."""
        return self.layers[layer_idx](hidden_states, attention_mask=attention_mask,
                                      position_ids=position_ids,
                                      past_key_value=past_key_value, use_cache=use_cache,
                                      position_embeddings=position_embeddings)

    def attention_block(self, layer_idx: int, x_parts: Sequence[torch.Tensor],
                        batch_offset: int, q_len: int, start_pos: Optional[int] = None,
                        sink=None, out: Optional[torch.Tensor] = None,
                        wait=None, add_residual: bool = True) -> torch.Tensor:
        """One attention block for the micro-batch whose sequences occupy cache
        rows [batch_offset, batch_offset + T // q_len). `x_parts` are the
        layer inputs (the F2A partials); returns h = x + o_proj(attn). `wait`
        (an ``ops.FlagWait``): the parts arrive from peers and the first kernel
        waits for their flags."""
        cfg = self.cfg
        lw = self.w.layers[layer_idx]
        start = self.cache.seq_len if start_pos is None else start_pos
        x, xn = ops.sum_rmsnorm(list(x_parts), lw.in_norm, cfg.rms_norm_eps, wait=wait)
        qkv = ops.linear(xn, lw.w_qkv)
        k_l, v_l = self.cache.layer(layer_idx)
        if q_len == 1:  # decode: norm + RoPE + append folded into the attention kernel
            o = ops.decode_attention_fused(qkv, lw.q_norm, lw.k_norm, self.rope, k_l, v_l, start,
                                           self.cache.pos_dev, batch_offset,
                                           cfg.num_attention_heads, cfg.num_key_value_heads,
                                           cfg.rms_norm_eps)
        else:
            q = ops.qk_norm_rope_cache(qkv, lw.q_norm, lw.k_norm, self.rope, k_l, v_l, start,
                                       self.cache.pos_dev, q_len, batch_offset,
                                       cfg.num_attention_heads, cfg.num_key_value_heads,
                                       cfg.rms_norm_eps)
            o = ops.attention(q, k_l, v_l, batch_offset, q_len, start, self.cache.pos_dev,
                              self.key_range)
        if not add_residual:  # attention output alone (per-layer view below)
            return ops.linear(o, lw.w_o, out=out)
        if sink is not None:
            return ops.linear(o, lw.w_o, residual=x, out=out, **sink.gemm_kwargs())
        return ops.linear(o, lw.w_o, residual=x, out=out)

    def forward_lm_head(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """The reference's call (src/model/attention_worker.py:309-313): final
        RMSNorm + LM head over every position, [..., H] -> [..., V]."""
        H = self.cfg.hidden_size
        x = hidden_states.reshape(-1, H).to(self.device, self.dtype)
        logits = self.lm_head_block([x], 1, last_only=False)
        return logits.view(*hidden_states.shape[:-1], logits.shape[-1])

    def lm_head_block(self, x_parts: Sequence[torch.Tensor], q_len: int = 1,
                      last_only: bool = True, wait=None) -> torch.Tensor:
        """Final RMSNorm + LM head. With `last_only`, only the last position of
        each sequence is projected (that is all sampling needs); returns
        [B, V] (or [T, V])."""
        if wait is not None:
            ops.wait_flags(wait)  # the parts are read by torch copies below
        H = self.cfg.hidden_size
        parts = [p.reshape(-1, H) for p in x_parts]
        if last_only and q_len > 1:
            parts = [p.view(-1, q_len, H)[:, -1].contiguous() for p in parts]
        _, xn = ops.sum_rmsnorm(parts, self.w.final_norm, self.cfg.rms_norm_eps)
        return ops.linear(xn, self.w.lm_head)


class AttentionLayer:
    """Per-layer view of an AttentionWorker with the reference's call
    (src/model/attention_worker.py:24-155): input RMSNorm, q/k/v projection,
    q/k RMSNorm, RoPE, KV-cache append, causal attention, o_proj. Returns
    (attn_output, residual) as [B, S, H] each, plus the KV cache when
    `use_cache` (keys/values appended at the cache's current length, which
    the caller advances, e.g. ``KVCache.advance``). Without `use_cache` the
    sequence sits at positions 0..S-1 and the layer's cache rows are scratch.
    Positions come from the cache length, so `position_ids` and
    `position_embeddings` are accepted for the signature only; an
    `attention_mask` may be a [B, S] padding mask."""

    def __init__(self, worker: "AttentionWorker", layer_idx: int):
        self.worker = worker
        self.layer_idx = layer_idx

    def forward(self, hidden_states: torch.Tensor, attention_mask=None, position_ids=None,
                past_key_value=None, output_attentions: bool = False, use_cache: bool = False,
                position_embeddings=None):
        w = self.worker
        B, S, H = hidden_states.shape
        x = hidden_states.reshape(B * S, H).to(w.device, w.dtype)
        start = w.cache.seq_len if use_cache else 0
        if not use_cache and w.cache.seq_len != 0:
            raise ValueError("use_cache=False needs an empty KV cache (its rows are scratch)")
        from ..parallel.micro_batch import key_ranges_from_mask
        w.key_range = (key_ranges_from_mask(attention_mask.to(w.device))
                       if attention_mask is not None and attention_mask.dim() == 2 and S > 1
                       else None)
        try:
            o = w.attention_block(self.layer_idx, [x], 0, S, start_pos=start,
                                  add_residual=False)
        finally:
            w.key_range = None
        out = (o.view(B, S, H), x.view(B, S, H))
        return out + (w.cache,) if use_cache else out

    __call__ = forward
