"""Model layer: the attention and FFN workers (one role each), the preallocated
KV cache, checkpoint reading and random initialisation, and
``DisaggregatedQwenModel``, which holds this process's roles and runs forwards
and generation (reference: src/model/)."""

from .attention import AttentionWorker
from .disaggregated import DisaggregatedQwenModel
from .ffn import FFNWorker
from .kv_cache import KVCache
from .weights import (AttentionWeights, FFNWeights, load_attention_weights, load_ffn_weights,
                      random_attention_weights, random_ffn_weights, save_checkpoint,
                      write_random_checkpoint)

__all__ = [
    "AttentionWorker", "DisaggregatedQwenModel", "FFNWorker", "KVCache", "AttentionWeights",
    "FFNWeights", "load_attention_weights", "load_ffn_weights", "random_attention_weights",
    "random_ffn_weights", "save_checkpoint", "write_random_checkpoint",
]
