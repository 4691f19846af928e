"""FFN role: post-attention RMSNorm, router, and the (expert-parallel slice
of the) MoE experts.

Reference: ``FFNLayer`` / ``FFNWorker`` (src/model/ffn_worker.py:31-225), which
run HF ``Qwen3MoeSparseMoeBlock`` -- a Python loop over the experts hit. Here
one layer is a fixed sequence of kernels independent of routing:

1. RMSNorm + router GEMM + fp32 softmax/top-k/renormalise
2. routing: per-expert row counts, expert-sorted rows, row blocks
3. gather of the normalised tokens into expert order
4. grouped tcgen05 GEMM  gate_up, SwiGLU epilogue
5. grouped tcgen05 GEMM  down, routing-weight epilogue
6. combine: per-token sum of its expert rows (+ residual), stored locally or
   -- with a fused transport -- straight into the attention GPUs' buffers
   with a release flag (the F2A return).

Under expert parallelism every FFN rank sees all tokens of the micro-batch and
contributes the partial sum of its local experts; FFN rank 0 also adds the
residual, so the attention side's sum over FFN ranks is the layer output.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from .. import ops
from ..config import ModelConfig
from ..utils.timing import EventType, TimingTracker
from .weights import FFNWeights


class FFNWorker:
    def __init__(self, cfg: ModelConfig, weights: FFNWeights, device, dtype=torch.bfloat16):
        self.cfg = cfg
        self.w = weights
        self.device = torch.device(device)
        self.dtype = dtype
        self.num_layers = cfg.num_hidden_layers
        self.expert_range = weights.expert_range
        self.supports_moe_timing = cfg.is_moe
        self.tracker = None  # optional TimingTracker for router / experts spans
        self.layers = [FFNLayer(self, l) for l in range(self.num_layers)]

    # the reference's attribute names (src/model/ffn_worker.py:125-189); one
    # GPU holds every layer, so the role's device list is this device
    @property
    def config(self) -> ModelConfig:
        return self.cfg

    @property
    def hidden_size(self) -> int:
        return self.cfg.hidden_size

    @property
    def ffn_layers(self) -> list:
        return self.layers

    @property
    def role_devices(self) -> list:
        return [self.device]

    @classmethod
    def from_pretrained(cls, model_name: str, device, dtype=torch.bfloat16,
                        expert_range: Optional[range] = None,
                        random_init: Optional[bool] = None, seed: int = 0,
                        dense_part: Tuple[int, int] = (0, 1)) -> "FFNWorker":
        """Reference: ``FFNWorker.from_pretrained`` (src/model/ffn_worker.py:228-256),
        which loads the whole HF model on the CPU and keeps its MLP parts.
        Here only the checkpoint's FFN-side tensors (post-attention norms,
        routers, the experts in `expert_range` (default all) and dense MLPs) are read,
        straight to `device`; a preset name without a checkpoint directory
        gets random weights (`seed`). `dense_part` = (i, n): this worker is FFN
        rank i of n and keeps that slice of each dense MLP layer."""
        import os

        from ..config import resolve_model_config
        from .weights import load_ffn_weights, random_ffn_weights

        cfg = resolve_model_config(model_name)
        if random_init is None:
            random_init = not os.path.isdir(model_name)
        w = (random_ffn_weights(cfg, expert_range, seed, device, dtype, dense_part) if random_init
             else load_ffn_weights(model_name, cfg, expert_range, device, dtype, dense_part))
        return cls(cfg, w, device, dtype)

    @classmethod
    def from_hf_model(cls, model, device, dtype=torch.bfloat16,
                      expert_range: Optional[range] = None,
                      dense_part: Tuple[int, int] = (0, 1)) -> "FFNWorker":
        """The counterpart of the reference's ``FFNWorker(model, device, dtype)``
        (src/model/ffn_worker.py:135-189), which takes a loaded HF
        ``Qwen3MoeForCausalLM``: its config and FFN-side tensors (experts in
        `expert_range`, default all) are copied to `device`; experts may be
        stored per expert or fused (transformers 5)."""
        from ..config import ModelConfig
        from .weights import load_ffn_weights

        cfg = ModelConfig.from_dict(model.config.to_dict())
        w = load_ffn_weights(model.state_dict(), cfg, expert_range, device, dtype, dense_part)
        return cls(cfg, w, device, dtype)

    def _mark(self, start: bool, et: EventType, l: int, mb: int):
        if self.tracker is not None:
            (self.tracker.mark_start if start else self.tracker.mark_end)(et, l, mb)

    def forward_ffn_layer(self, layer_idx: int, hidden_states: torch.Tensor,
                          add_residual: bool = True, sink=None, out: Optional[torch.Tensor] = None,
                          mb_idx: int = 0, wait=None, return_timing: bool = False):
        """h [T, H] (= attn_out + residual) -> h + moe(norm(h)) [T, H], or only
        the local experts' partial sum when `add_residual` is False. `wait`
        (an ``ops.FlagWait``): h arrives from peers; the first kernel waits.
        `return_timing` (the reference's flag, src/model/ffn_worker.py:201-225)
        returns (output, ``FFNStageTiming``) through the layer view."""
        if return_timing:
            return self.layers[layer_idx](hidden_states, return_timing=True)
        cfg = self.cfg
        lw = self.w.layers[layer_idx]
        H = cfg.hidden_size
        h = hidden_states.reshape(-1, H)
        residual = h if add_residual else None
        kw = sink.combine_kwargs() if sink is not None else {}
        if lw.w_router is None:  # dense MLP layer (mlp_only_layers)
            if sink is not None:
                raise NotImplementedError("the fused F2A store covers MoE layers only; "
                                          "use --comm-impl nccl for models with dense layers")
            self._mark(True, EventType.MOE_SHARED_OR_DENSE, layer_idx, mb_idx)
            xn = ops.sum_rmsnorm([h], lw.post_norm, cfg.rms_norm_eps, wait=wait)[1]
            y = ops.dense_mlp(xn, lw.w_dense_gate_up, lw.w_dense_down, residual=residual)
            self._mark(False, EventType.MOE_SHARED_OR_DENSE, layer_idx, mb_idx)
            return y
        stage = {"router": EventType.MOE_ROUTER, "experts": EventType.MOE_EXPERTS}
        return ops.moe_ffn(h, lw.post_norm, lw.w_router, lw.w_gate_up, lw.w_down,
                           cfg.num_experts_per_tok, cfg.rms_norm_eps, cfg.norm_topk_prob,
                           lw.expert_start, add_residual=residual is not None, out=out,
                           tracker_marks=lambda start, name: self._mark(start, stage[name],
                                                                        layer_idx, mb_idx),
                           wait=wait, **kw)


@dataclass
class FFNStageTiming:
    """Host-observed FFN stage times in seconds (the reference's
    src/model/ffn_worker.py:23-28)."""
    router_s: float = 0.0
    experts_s: float = 0.0
    shared_or_dense_s: float = 0.0


class FFNLayer:
    """Per-layer view of an FFNWorker with the reference's call
    (src/model/ffn_worker.py:31-122): h (+ residual, when given separately)
    -> h + moe(post_attention_norm(h)), [B, S, H] or [T, H]. With
    `return_timing`, the router and expert stages are timed on the host with
    a device synchronisation around each (a debugging aid, as in the
    reference)."""

    def __init__(self, worker: "FFNWorker", layer_idx: int):
        self.worker = worker
        self.layer_idx = layer_idx

    @property
    def is_sparse_moe(self) -> bool:
        return self.worker.w.layers[self.layer_idx].w_router is not None

    def forward(self, hidden_states: torch.Tensor, residual: Optional[torch.Tensor] = None,
                output_device=None, return_timing: bool = False):
        w = self.worker
        shape = hidden_states.shape
        h = hidden_states if residual is None else residual + hidden_states
        h = h.reshape(-1, shape[-1]).to(w.device, w.dtype)
        saved = w.tracker
        tr = TimingTracker("ffn", w.num_layers, 1, mode="sync") if return_timing else saved
        w.tracker = tr
        try:
            out = w.forward_ffn_layer(self.layer_idx, h, add_residual=True).view(shape)
        finally:
            w.tracker = saved
        if output_device is not None:
            out = out.to(output_device)
        if not return_timing:
            return out
        st = FFNStageTiming()
        for ev in tr.finish().events:
            if ev.event_type == EventType.MOE_ROUTER.value:
                st.router_s += ev.duration_ms / 1e3
            elif ev.event_type == EventType.MOE_EXPERTS.value:
                st.experts_s += ev.duration_ms / 1e3
            elif ev.event_type == EventType.MOE_SHARED_OR_DENSE.value:
                st.shared_or_dense_s += ev.duration_ms / 1e3
        return out, st

    __call__ = forward
