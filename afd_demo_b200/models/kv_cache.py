"""Preallocated KV cache with a DynamicCache-compatible surface.

The reference keeps an HF ``DynamicCache`` that grows by ``torch.cat`` and,
in decode DBO, slices the batch dimension per micro-batch and concatenates
the slices back on every layer of every step
(src/pipeline/decode_scheduler.py:242-283,334-335). Here the cache is one
buffer per K and V, ``[L, B_max, n_kv, S_max, D]``, written in place by the
fused q/k-norm + RoPE + append kernel; a micro-batch is just a batch offset,
so nothing is copied per step.

The current length lives both on the host (``seq_len``) and in device memory
(``pos_dev``, int32) so captured CUDA graphs read the position at replay.
``layers[l].keys / .values`` return views ``[B, n_kv, seq_len, D]`` and
``update`` appends like ``DynamicCache.update`` for code written against
the HF API.
"""

from __future__ import annotations

from typing import List, Tuple

import torch


class _LayerView:
    def __init__(self, cache: "KVCache", idx: int):
        self._c = cache
        self._i = idx

    @property
    def keys(self) -> torch.Tensor:
        c = self._c
        return c.k[self._i, : c.batch, :, : c.seq_len]

    @property
    def values(self) -> torch.Tensor:
        c = self._c
        return c.v[self._i, : c.batch, :, : c.seq_len]


class KVCache:
    def __init__(self, num_layers: int, max_batch: int, num_kv_heads: int, max_seq: int,
                 head_dim: int, device, dtype=torch.bfloat16):
        self.num_layers = num_layers
        self.max_batch = max_batch
        self.max_seq = max_seq
        shape = (num_layers, max_batch, num_kv_heads, max_seq, head_dim)
        self.k = torch.zeros(shape, device=device, dtype=dtype)
        self.v = torch.zeros(shape, device=device, dtype=dtype)
        self.seq_len = 0
        self.batch = max_batch
        self.pos_dev = torch.zeros(1, device=device, dtype=torch.int32)
        self._pending = [0] * num_layers
        self.layers: List[_LayerView] = [_LayerView(self, l) for l in range(num_layers)]

    # -------- DynamicCache-compatible surface --------------------------------
    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.seq_len

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append [B, n_kv, q, D] at the current length of layer `layer_idx`
        and return the layer's keys / values so far, as
        ``DynamicCache.update(key, value, layer_idx, cache_kwargs)`` does
        (`cache_kwargs`, RoPE metadata in HF, is not needed here); the length
        advances once every layer has appended the same count."""
        B, _, q, _ = key_states.shape
        s = self.seq_len
        self.k[layer_idx, :B, :, s:s + q] = key_states
        self.v[layer_idx, :B, :, s:s + q] = value_states
        self._pending[layer_idx] = q
        if layer_idx == self.num_layers - 1 and all(p == q for p in self._pending):
            self.advance(q)
            self._pending = [0] * self.num_layers
        return self.k[layer_idx, :B, :, : s + q], self.v[layer_idx, :B, :, : s + q]

    # -------- framework surface ---------------------------------------------
    def layer(self, l: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Full per-layer buffers [B_max, n_kv, S_max, D] for the kernels."""
        return self.k[l], self.v[l]

    def reset(self, batch: int = None) -> None:
        self.seq_len = 0
        if batch is not None:
            if batch > self.max_batch:
                raise ValueError(f"batch {batch} exceeds cache capacity {self.max_batch}")
            self.batch = batch
        self.pos_dev.zero_()

    def advance(self, n: int) -> None:
        if self.seq_len + n > self.max_seq:
            raise ValueError(f"KV cache overflow: {self.seq_len}+{n} > {self.max_seq}")
        self.seq_len += n
        self.pos_dev.add_(n)

    def nbytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()
