"""Model and run configuration.

`ModelConfig` carries the Qwen3-MoE hyper-parameters the framework needs. The
reference reads them through `AutoConfig.from_pretrained`
(src/model/disaggregated.py:815); here they are a plain dataclass that can be
read from / written to a HuggingFace-style `config.json`, so a checkpoint
directory written by `afd_demo_b200.models.weights` is also loadable by
`transformers` (model_type ``qwen3_moe``).

`Topology` describes how the GPUs of one node are split into attention ranks
(data-parallel over the batch) and FFN ranks (expert-parallel over the
experts). The reference only has the fixed 1 attention + 1 FFN rank split
(src/distributed/__init__.py:156-165).
"""

from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional


@dataclass
class ModelConfig:
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_hidden_layers: int = 48
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    num_experts: int = 128
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 768
    intermediate_size: int = 6144  # dense-MLP width (only for non-MoE layers)
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    norm_topk_prob: bool = True
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False
    decoder_sparse_step: int = 1
    mlp_only_layers: List[int] = field(default_factory=list)
    initializer_range: float = 0.02
    model_type: str = "qwen3_moe"

    # ---- derived sizes -------------------------------------------------
    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def gqa_group(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def is_sparse_layer(self, layer_idx: int) -> bool:
        """Same rule as HF Qwen3MoeDecoderLayer: MoE unless listed in mlp_only_layers."""
        return (
            self.num_experts > 0
            and layer_idx not in self.mlp_only_layers
            and (layer_idx + 1) % self.decoder_sparse_step == 0
        )

    # ---- (de)serialisation --------------------------------------------
    def to_hf_dict(self) -> Dict:
        d = dataclasses.asdict(self)
        d.update(
            {
                "architectures": ["Qwen3ForCausalLM" if self.model_type == "qwen3"
                                  else "Qwen3MoeForCausalLM"],
                "hidden_act": "silu",
                "attention_bias": False,
                "attention_dropout": 0.0,
                "use_sliding_window": False,
                "sliding_window": None,
                "output_router_logits": False,
                "router_aux_loss_coef": 0.001,
                "torch_dtype": "bfloat16",
                "bos_token_id": 151643,
                "eos_token_id": 151645,
                "use_cache": True,
                "rope_parameters": {"rope_type": "default", "rope_theta": self.rope_theta},
            }
        )
        return d

    @classmethod
    def from_dict(cls, d: Dict) -> "ModelConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        kw = {k: v for k, v in d.items() if k in names}
        # transformers 5 writes the expert count as num_local_experts; a dense
        # model's config (model_type "qwen3") has no expert count at all
        if "num_experts" not in d:
            kw["num_experts"] = d.get("num_local_experts", 0)
        if "rope_theta" not in d and isinstance(d.get("rope_parameters"), dict):
            kw["rope_theta"] = d["rope_parameters"].get("rope_theta", cls.rope_theta)
        if "head_dim" not in d and "hidden_size" in d and "num_attention_heads" in d:
            kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
        return cls(**kw)

    @classmethod
    def from_pretrained(cls, path: str) -> "ModelConfig":
        cfg_path = os.path.join(path, "config.json") if os.path.isdir(path) else path
        with open(cfg_path) as f:
            return cls.from_dict(json.load(f))

    def save(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(self.to_hf_dict(), f, indent=2)


def qwen3_30b_a3b() -> ModelConfig:
    """Qwen3-30B-A3B shapes: 48 layers, hidden 2048, 32q/4kv heads x 128,
    128 experts top-8, moe_intermediate 768, vocab 151936, RoPE theta 1e6."""
    return ModelConfig()


def tiny_qwen3_moe() -> ModelConfig:
    """The 2-layer CPU/gloo oracle model: hidden 256, 4q/2kv heads x 64,
    8 experts top-2, moe_intermediate 128, vocab 1024, RoPE theta 1e6."""
    return ModelConfig(
        vocab_size=1024,
        hidden_size=256,
        num_hidden_layers=2,
        num_attention_heads=4,
        num_key_value_heads=2,
        head_dim=64,
        num_experts=8,
        num_experts_per_tok=2,
        moe_intermediate_size=128,
        intermediate_size=512,
        max_position_embeddings=4096,
    )


def small_qwen3_moe() -> ModelConfig:
    """A GPU-test model with the real per-layer shapes of Qwen3-30B-A3B
    (hidden 2048, 32q/4kv x 128, 128 experts top-8, moe_intermediate 768)
    but only 2 layers and a 4096-token vocabulary."""
    return ModelConfig(num_hidden_layers=2, vocab_size=4096)


def mini_qwen3_moe() -> ModelConfig:
    """A fast GPU-test model that exercises every sm_100a kernel path:
    hidden 1024, 2 layers, 16q/2kv heads x 64, 128 experts top-8,
    moe_intermediate 256, vocab 2048."""
    return ModelConfig(vocab_size=2048, hidden_size=1024, num_hidden_layers=2,
                       num_attention_heads=16, num_key_value_heads=2, head_dim=64,
                       moe_intermediate_size=256, intermediate_size=2048)


PRESETS = {
    "qwen3-30b-a3b": qwen3_30b_a3b,
    "Qwen/Qwen3-30B-A3B": qwen3_30b_a3b,
    "tiny": tiny_qwen3_moe,
    "small": small_qwen3_moe,
    "mini": mini_qwen3_moe,
}


def resolve_model_config(name_or_path: str) -> ModelConfig:
    """A preset name, a checkpoint directory, or a config.json path."""
    if name_or_path in PRESETS:
        return PRESETS[name_or_path]()
    if os.path.exists(name_or_path):
        return ModelConfig.from_pretrained(name_or_path)
    base = os.path.basename(os.path.normpath(name_or_path))
    for k, fn in PRESETS.items():
        if base.lower() == os.path.basename(k).lower():
            return fn()
    raise FileNotFoundError(f"no preset or checkpoint named {name_or_path!r}")


@dataclass
class Topology:
    """Attention ranks 0..n_attn-1, FFN ranks n_attn..n_attn+n_ffn-1.

    world_size 1 co-locates both roles in one process on one GPU.
    """

    n_attn: int = 1
    n_ffn: int = 1
    colocated: bool = False

    @property
    def world_size(self) -> int:
        return 1 if self.colocated else self.n_attn + self.n_ffn

    @classmethod
    def for_world(cls, world_size: int, n_attn: Optional[int] = None,
                  n_ffn: Optional[int] = None) -> "Topology":
        if world_size == 1:
            return cls(1, 1, colocated=True)
        if n_attn is None and n_ffn is None:
            n_attn = world_size // 2
        if n_attn is None:
            n_attn = world_size - n_ffn
        if n_ffn is None:
            n_ffn = world_size - n_attn
        if n_attn < 1 or n_ffn < 1 or n_attn + n_ffn != world_size:
            raise ValueError(f"bad topology {n_attn}A+{n_ffn}F for world {world_size}")
        return cls(n_attn, n_ffn)

    def role_of(self, rank: int) -> str:
        if self.colocated:
            return "both"
        return "attention" if rank < self.n_attn else "ffn"

    def attn_ranks(self) -> List[int]:
        return [0] if self.colocated else list(range(self.n_attn))

    def ffn_ranks(self) -> List[int]:
        return [0] if self.colocated else list(range(self.n_attn, self.n_attn + self.n_ffn))

    def ffn_index(self, rank: int) -> int:
        return 0 if self.colocated else rank - self.n_attn

    def experts_of(self, ffn_index: int, num_experts: int) -> range:
        per = num_experts // self.n_ffn
        if per * self.n_ffn != num_experts:
            raise ValueError(f"{num_experts} experts do not split over {self.n_ffn} FFN ranks")
        return range(ffn_index * per, (ffn_index + 1) * per)

    def batch_slice(self, attn_index: int, batch: int) -> range:
        """Data-parallel split of the global batch over attention ranks."""
        base, rem = divmod(batch, self.n_attn)
        start = attn_index * base + min(attn_index, rem)
        return range(start, start + base + (1 if attn_index < rem else 0))

    def tag(self) -> str:
        return "1G" if self.colocated else f"{self.n_attn}A{self.n_ffn}F"
