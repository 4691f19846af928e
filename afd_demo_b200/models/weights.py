"""Qwen3-MoE weights: seeded random init, safetensors writer and a role/expert
sharded loader.

The reference loads the *full* HF model on the CPU of every role and keeps only
its role's submodules (src/model/disaggregated.py:76-117). Here each rank reads
only the tensors it owns, straight from the safetensors shards:

* attention ranks: embedding, per-layer input norm, q/k/v/o projections,
  q/k norms, final norm, LM head;
* FFN ranks: per-layer post-attention norm, router, and the experts in their
  expert-parallel slice; a dense MLP layer (``mlp_only_layers``, or every
  layer of a dense Qwen3 model) is split over the FFN ranks along its
  intermediate dimension (``dense_slice``).

On-disk layout (HF Qwen3-MoE, per-expert keys)::

    model.embed_tokens.weight                                   [V, H]
    model.layers.{l}.input_layernorm.weight                     [H]
    model.layers.{l}.self_attn.{q,k,v,o}_proj.weight            [Q|KV|KV, H], [H, Q]
    model.layers.{l}.self_attn.{q,k}_norm.weight                [D]
    model.layers.{l}.post_attention_layernorm.weight            [H]
    model.layers.{l}.mlp.gate.weight                            [E, H]
    model.layers.{l}.mlp.experts.{e}.{gate,up,down}_proj.weight [I,H],[I,H],[H,I]
    model.norm.weight                                           [H]
    lm_head.weight                                              [V, H]

In-memory layout (what the kernels consume):

* ``w_qkv``  [Q+2KV, H]  q, k, v rows concatenated (one GEMM);
* ``w_gate_up`` [E_local, 2I, H]  gate rows then up rows per expert (same
  as HF's fused ``gate_up_proj``);
* ``w_down`` [E_local, H, I].

Random init draws every tensor from its own generator seeded by
(seed, tensor name), so any shard of any topology sees the same values as the
unsharded model on the same device type.
"""

from __future__ import annotations

import hashlib
import json
import os
import re
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Tuple

import torch

from ..config import ModelConfig


def _name_seed(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def _randn(shape, name: str, seed: int, std: float, device, dtype) -> torch.Tensor:
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(_name_seed(seed, name))
    t = torch.randn(*shape, generator=g, device=dev, dtype=torch.float32)
    t.mul_(std)
    return t.to(dtype)


@dataclass
class AttentionLayerWeights:
    in_norm: torch.Tensor
    w_qkv: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    w_o: torch.Tensor


@dataclass
class FFNLayerWeights:
    post_norm: torch.Tensor
    # sparse MoE layer
    w_router: Optional[torch.Tensor] = None
    w_gate_up: Optional[torch.Tensor] = None  # [E_local, 2I, H]
    w_down: Optional[torch.Tensor] = None     # [E_local, H, I]
    expert_start: int = 0
    # dense MLP layer (mlp_only_layers)
    w_dense_gate_up: Optional[torch.Tensor] = None  # [2I, H]
    w_dense_down: Optional[torch.Tensor] = None     # [H, I]


@dataclass
class AttentionWeights:
    embed: torch.Tensor
    final_norm: torch.Tensor
    lm_head: torch.Tensor
    layers: List[AttentionLayerWeights] = field(default_factory=list)


@dataclass
class FFNWeights:
    layers: List[FFNLayerWeights] = field(default_factory=list)
    expert_range: range = range(0)


# --------------------------------------------------------------------------
# random init
# --------------------------------------------------------------------------

def _norm_init(n: int, name: str, seed: int, device, dtype) -> torch.Tensor:
    # HF initialises RMSNorm weights to 1; a small seeded jitter keeps the
    # oracle comparison sensitive to a norm weight being applied wrongly.
    return (1.0 + _randn((n,), name, seed, 0.05, device, torch.float32)).to(dtype)


def random_attention_weights(cfg: ModelConfig, seed: int = 0, device="cpu",
                             dtype=torch.bfloat16) -> AttentionWeights:
    std = cfg.initializer_range
    H = cfg.hidden_size
    aw = AttentionWeights(
        embed=_randn((cfg.vocab_size, H), "embed", seed, 1.0, device, dtype),
        final_norm=_norm_init(H, "final_norm", seed, device, dtype),
        lm_head=_randn((cfg.vocab_size, H), "lm_head", seed, std, device, dtype),
    )
    for l in range(cfg.num_hidden_layers):
        aw.layers.append(_layer_only_attention(cfg, l, seed, dtype, device))
    return aw


def random_ffn_weights(cfg: ModelConfig, expert_range: Optional[range] = None, seed: int = 0,
                       device="cpu", dtype=torch.bfloat16,
                       dense_part: Tuple[int, int] = (0, 1)) -> FFNWeights:
    if expert_range is None:
        expert_range = range(cfg.num_experts)
    fw = FFNWeights(expert_range=expert_range)
    for l in range(cfg.num_hidden_layers):
        fw.layers.append(_layer_only_ffn(cfg, l, seed, dtype, device, expert_range, dense_part))
    return fw


# --------------------------------------------------------------------------
# safetensors writer / loader
# --------------------------------------------------------------------------

def _attn_layer_tensors(cfg: ModelConfig, l: int, lw: AttentionLayerWeights) -> Dict[str, torch.Tensor]:
    Q, KV = cfg.q_size, cfg.kv_size
    p = f"model.layers.{l}."
    return {
        p + "input_layernorm.weight": lw.in_norm,
        p + "self_attn.q_proj.weight": lw.w_qkv[:Q],
        p + "self_attn.k_proj.weight": lw.w_qkv[Q:Q + KV],
        p + "self_attn.v_proj.weight": lw.w_qkv[Q + KV:],
        p + "self_attn.o_proj.weight": lw.w_o,
        p + "self_attn.q_norm.weight": lw.q_norm,
        p + "self_attn.k_norm.weight": lw.k_norm,
    }


def _ffn_layer_tensors(cfg: ModelConfig, l: int, lw: FFNLayerWeights) -> Dict[str, torch.Tensor]:
    p = f"model.layers.{l}."
    out = {p + "post_attention_layernorm.weight": lw.post_norm}
    if lw.w_router is not None:
        I = cfg.moe_intermediate_size
        out[p + "mlp.gate.weight"] = lw.w_router
        for i in range(lw.w_gate_up.shape[0]):
            e = lw.expert_start + i
            out[p + f"mlp.experts.{e}.gate_proj.weight"] = lw.w_gate_up[i, :I]
            out[p + f"mlp.experts.{e}.up_proj.weight"] = lw.w_gate_up[i, I:]
            out[p + f"mlp.experts.{e}.down_proj.weight"] = lw.w_down[i]
    else:
        DI = cfg.intermediate_size
        out[p + "mlp.gate_proj.weight"] = lw.w_dense_gate_up[:DI]
        out[p + "mlp.up_proj.weight"] = lw.w_dense_gate_up[DI:]
        out[p + "mlp.down_proj.weight"] = lw.w_dense_down
    return out


def save_checkpoint(path: str, cfg: ModelConfig, attn: AttentionWeights, ffn: FFNWeights) -> None:
    """Write an HF-layout checkpoint: config.json, one safetensors shard per
    layer plus one for the embedding/head, and model.safetensors.index.json."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    cfg.save(path)
    weight_map: Dict[str, str] = {}

    def _write(fname: str, tensors: Dict[str, torch.Tensor]):
        tensors = {k: v.detach().contiguous().cpu() for k, v in tensors.items()}
        save_file(tensors, os.path.join(path, fname), metadata={"format": "pt"})
        for k in tensors:
            weight_map[k] = fname

    _write("model-embed-head.safetensors", {
        "model.embed_tokens.weight": attn.embed,
        "model.norm.weight": attn.final_norm,
        "lm_head.weight": attn.lm_head,
    })
    for l in range(cfg.num_hidden_layers):
        t = _attn_layer_tensors(cfg, l, attn.layers[l])
        t.update(_ffn_layer_tensors(cfg, l, ffn.layers[l]))
        _write(f"model-layer-{l:05d}.safetensors", t)
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f, indent=1)


def write_random_checkpoint(path: str, cfg: ModelConfig, seed: int = 0,
                            dtype=torch.bfloat16, device="cpu") -> None:
    """Random-init checkpoint written layer by layer (bounded host memory).
    `device` is where the random tensors are drawn (a GPU draws the 30B
    parameters of Qwen3-30B-A3B in seconds); the values depend on it."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    cfg.save(path)
    weight_map: Dict[str, str] = {}
    one = ModelConfig(**{**cfg.__dict__, "num_hidden_layers": 1})
    aw0 = random_attention_weights(one, seed=seed, device=device, dtype=dtype)
    head = {"model.embed_tokens.weight": aw0.embed, "model.norm.weight": aw0.final_norm,
            "lm_head.weight": aw0.lm_head}
    save_file({k: v.contiguous().cpu() for k, v in head.items()},
              os.path.join(path, "model-embed-head.safetensors"), metadata={"format": "pt"})
    weight_map.update({k: "model-embed-head.safetensors" for k in head})
    for l in range(cfg.num_hidden_layers):
        aw = _layer_only_attention(cfg, l, seed, dtype, device)
        fw = _layer_only_ffn(cfg, l, seed, dtype, device)
        t = _attn_layer_tensors(cfg, l, aw)
        t.update(_ffn_layer_tensors(cfg, l, fw))
        fname = f"model-layer-{l:05d}.safetensors"
        save_file({k: v.contiguous().cpu() for k, v in t.items()}, os.path.join(path, fname),
                  metadata={"format": "pt"})
        weight_map.update({k: fname for k in t})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f, indent=1)


def _layer_only_attention(cfg: ModelConfig, l: int, seed: int, dtype,
                          device="cpu") -> AttentionLayerWeights:
    """One layer's attention weights; each tensor is one seeded draw (q, k and
    v projections together), so initialisation takes a few launches per
    layer."""
    std = cfg.initializer_range
    H, Q, KV, D = cfg.hidden_size, cfg.q_size, cfg.kv_size, cfg.head_dim
    p = f"layers.{l}."
    return AttentionLayerWeights(
        in_norm=_norm_init(H, p + "in_norm", seed, device, dtype),
        w_qkv=_randn((Q + 2 * KV, H), p + "qkv", seed, std, device, dtype),
        q_norm=_norm_init(D, p + "q_norm", seed, device, dtype),
        k_norm=_norm_init(D, p + "k_norm", seed, device, dtype),
        w_o=_randn((H, Q), p + "o", seed, std, device, dtype),
    )


def dense_slice(gate_up: torch.Tensor, down: torch.Tensor,
                part: Tuple[int, int] = (0, 1)) -> Tuple[torch.Tensor, torch.Tensor]:
    """FFN rank i of n (`part` = (i, n)) keeps rows [i*DI/n, (i+1)*DI/n) of a
    dense MLP's gate and of its up projection (`gate_up` is [2*DI, H], gate
    rows first) and the same columns of `down` [H, DI]. Its output is then
    that slice's share of the down projection, and the attention side's sum
    of the FFN ranks' outputs (the same sum that adds up the experts'
    partials) is the whole MLP."""
    i, n = part
    if n == 1:
        return gate_up, down
    DI = down.shape[1]
    if DI % n:
        raise ValueError(f"dense intermediate size {DI} does not split over {n} FFN ranks")
    w = DI // n
    lo, hi = i * w, (i + 1) * w
    return (torch.cat([gate_up[lo:hi], gate_up[DI + lo:DI + hi]]).contiguous(),
            down[:, lo:hi].contiguous())


def _layer_only_ffn(cfg: ModelConfig, l: int, seed: int, dtype, device="cpu",
                    expert_range: Optional[range] = None,
                    dense_part: Tuple[int, int] = (0, 1)) -> FFNLayerWeights:
    """One layer's FFN weights. The experts' gate/up and down projections are
    one seeded draw each over all experts of the layer, of which this rank
    keeps `expert_range`: every expert-parallel split therefore holds the
    same values as one GPU holding all experts. A dense layer is drawn whole
    and this rank keeps its `dense_part` slice (``dense_slice``)."""
    std = cfg.initializer_range
    H, I, E = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts
    er = range(E) if expert_range is None else expert_range
    p = f"layers.{l}."
    lw = FFNLayerWeights(post_norm=_norm_init(H, p + "post_norm", seed, device, dtype))
    if cfg.is_sparse_layer(l):
        lw.w_router = _randn((E, H), p + "router", seed, std, device, dtype)
        gu = _randn((E, 2 * I, H), p + "experts.gate_up", seed, std, device, dtype)
        dn = _randn((E, H, I), p + "experts.down", seed, std, device, dtype)
        if len(er) != E:  # keep only this rank's experts (no view of the full draw)
            gu = gu[er.start:er.stop].clone()
            dn = dn[er.start:er.stop].clone()
        lw.w_gate_up, lw.w_down, lw.expert_start = gu, dn, er.start
    else:
        DI = cfg.intermediate_size
        lw.w_dense_gate_up, lw.w_dense_down = dense_slice(
            _randn((2 * DI, H), p + "dense.gate_up", seed, std, device, dtype),
            _randn((H, DI), p + "dense.down", seed, std, device, dtype), dense_part)
    return lw


class _ShardReader:
    """Lazily opens the safetensors shards listed in the index and reads single
    tensors (no full-model materialisation)."""

    def __init__(self, path: str):
        from safetensors import safe_open

        self.path = path
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                self.weight_map = json.load(f)["weight_map"]
        else:
            single = os.path.join(path, "model.safetensors")
            with safe_open(single, "pt") as h:
                self.weight_map = {k: "model.safetensors" for k in h.keys()}
        self._handles: Dict[str, object] = {}
        self._safe_open = safe_open

    def get(self, key: str) -> torch.Tensor:
        fname = self.weight_map[key]
        h = self._handles.get(fname)
        if h is None:
            h = self._safe_open(os.path.join(self.path, fname), "pt")
            self._handles[fname] = h
        return h.get_tensor(key)

    def __contains__(self, key: str) -> bool:
        return key in self.weight_map


class _StateDictReader:
    """Reads tensors from an in-memory state dict under the checkpoint's key
    names. Experts may be stored per expert (``mlp.experts.{e}.gate_proj.weight``
    and so on: transformers 4, and every saved checkpoint) or fused
    (``mlp.experts.gate_up_proj`` [E, 2I, H], gate rows first, and
    ``mlp.experts.down_proj`` [E, H, I]: a transformers 5 model in memory);
    fused ones are sliced per expert."""

    _PER_EXPERT = re.compile(r"^(.*\.mlp\.experts\.)(\d+)\.(gate_proj|up_proj|down_proj)\.weight$")

    def __init__(self, state_dict):
        self.sd = state_dict

    def get(self, key: str) -> torch.Tensor:
        t = self.sd.get(key)
        if t is not None:
            return t
        m = self._PER_EXPERT.match(key)
        if m is not None:
            base, e, proj = m.group(1), int(m.group(2)), m.group(3)
            if proj == "down_proj":
                fused = self.sd.get(base + "down_proj")
                if fused is not None:
                    return fused[e]
            else:
                fused = self.sd.get(base + "gate_up_proj")
                if fused is not None:
                    half = fused.shape[1] // 2
                    return fused[e, :half] if proj == "gate_proj" else fused[e, half:]
        raise KeyError(key)

    def __contains__(self, key: str) -> bool:
        try:
            self.get(key)
        except KeyError:
            return False
        return True


def _reader(source):
    """A checkpoint directory, or a state dict (see ``_StateDictReader``)."""
    if isinstance(source, (str, os.PathLike)):
        return _ShardReader(os.fspath(source))
    return _StateDictReader(source)


def load_attention_weights(path, cfg: ModelConfig, device="cpu",
                           dtype=torch.bfloat16) -> AttentionWeights:
    """The attention-side tensors of `path`: a checkpoint directory or a
    state dict with the checkpoint's key names."""
    r = _reader(path)
    cv = lambda t: t.to(device=device, dtype=dtype)  # noqa: E731
    lm_key = "lm_head.weight" if "lm_head.weight" in r else "model.embed_tokens.weight"
    aw = AttentionWeights(embed=cv(r.get("model.embed_tokens.weight")),
                          final_norm=cv(r.get("model.norm.weight")),
                          lm_head=cv(r.get(lm_key)))
    for l in range(cfg.num_hidden_layers):
        p = f"model.layers.{l}."
        aw.layers.append(AttentionLayerWeights(
            in_norm=cv(r.get(p + "input_layernorm.weight")),
            w_qkv=cv(torch.cat([r.get(p + "self_attn.q_proj.weight"),
                                r.get(p + "self_attn.k_proj.weight"),
                                r.get(p + "self_attn.v_proj.weight")])),
            q_norm=cv(r.get(p + "self_attn.q_norm.weight")),
            k_norm=cv(r.get(p + "self_attn.k_norm.weight")),
            w_o=cv(r.get(p + "self_attn.o_proj.weight")),
        ))
    return aw


def load_ffn_weights(path, cfg: ModelConfig, expert_range: Optional[range] = None,
                     device="cpu", dtype=torch.bfloat16,
                     dense_part: Tuple[int, int] = (0, 1)) -> FFNWeights:
    """The FFN-side tensors of `path` (experts in `expert_range`, the
    `dense_part` slice of dense layers): a checkpoint directory or a state
    dict with the checkpoint's key names."""
    r = _reader(path)
    cv = lambda t: t.to(device=device, dtype=dtype)  # noqa: E731
    if expert_range is None:
        expert_range = range(cfg.num_experts)
    I = cfg.moe_intermediate_size
    H = cfg.hidden_size
    fw = FFNWeights(expert_range=expert_range)
    for l in range(cfg.num_hidden_layers):
        p = f"model.layers.{l}."
        lw = FFNLayerWeights(post_norm=cv(r.get(p + "post_attention_layernorm.weight")))
        if cfg.is_sparse_layer(l):
            lw.w_router = cv(r.get(p + "mlp.gate.weight"))
            gu = torch.empty(len(expert_range), 2 * I, H, device=device, dtype=dtype)
            dn = torch.empty(len(expert_range), H, I, device=device, dtype=dtype)
            for i, e in enumerate(expert_range):
                q = p + f"mlp.experts.{e}."
                gu[i, :I] = cv(r.get(q + "gate_proj.weight"))
                gu[i, I:] = cv(r.get(q + "up_proj.weight"))
                dn[i] = cv(r.get(q + "down_proj.weight"))
            lw.w_gate_up, lw.w_down, lw.expert_start = gu, dn, expert_range.start
        else:
            lw.w_dense_gate_up, lw.w_dense_down = dense_slice(
                cv(torch.cat([r.get(p + "mlp.gate_proj.weight"), r.get(p + "mlp.up_proj.weight")])),
                cv(r.get(p + "mlp.down_proj.weight")), dense_part)
        fw.layers.append(lw)
    return fw


def iter_tensors(w) -> Iterable[torch.Tensor]:
    if isinstance(w, AttentionWeights):
        yield from (w.embed, w.final_norm, w.lm_head)
        for lw in w.layers:
            yield from (lw.in_norm, lw.w_qkv, lw.q_norm, lw.k_norm, lw.w_o)
    else:
        for lw in w.layers:
            for t in (lw.post_norm, lw.w_router, lw.w_gate_up, lw.w_down,
                      lw.w_dense_gate_up, lw.w_dense_down):
                if t is not None:
                    yield t
