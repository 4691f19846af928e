"""Micro-batch splitting and the per-forward layout shared by all ranks.

Reference: ``MicroBatch`` / ``MicroBatchManager`` (src/pipeline/micro_batch.py:
17-214). The split rule is the same: ``num_micro_batches`` parts, the
remainder going to the first parts, and a batch smaller than the part count
uses one part per sequence.

``ForwardPlan`` extends that to the data-parallel attention ranks: every rank
derives, from (global batch, topology, micro-batch count, q_len), the same
table of which sequences each attention rank holds in each micro-batch and
where those tokens sit in the FFN ranks' receive buffers. No metadata needs
to travel per layer.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import List, Optional, Tuple

import torch

from ..config import Topology


def split_sizes(batch: int, num_micro_batches: int) -> List[int]:
    n = min(num_micro_batches, batch) if batch > 0 else 0
    if n == 0:
        return []
    base, rem = divmod(batch, n)
    return [base + (1 if i < rem else 0) for i in range(n)]


class MicroBatchState(Enum):
    WAITING = 0
    IN_ATTENTION = 1
    IN_TRANSIT_AF = 2
    IN_FFN = 3
    IN_TRANSIT_FA = 4
    COMPLETED = 5


@dataclass
class MicroBatch:
    id: int
    input_ids: torch.Tensor
    attention_mask: Optional[torch.Tensor] = None
    position_ids: Optional[torch.Tensor] = None
    hidden_states: Optional[torch.Tensor] = None
    state: MicroBatchState = MicroBatchState.WAITING
    current_layer: int = 0
    # the reference's remaining fields, in its order: position embeddings
    # computed once per micro-batch, and host timestamps for profiling
    position_embeddings: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
    start_time: Optional[float] = None
    end_time: Optional[float] = None
    batch_offset: int = 0  # first sequence of this micro-batch in the batch

    def advance_layer(self) -> None:
        self.current_layer += 1

    def reset_for_layer(self, layer_idx: int) -> None:
        self.current_layer = layer_idx
        self.state = MicroBatchState.WAITING

    @property
    def batch_size(self) -> int:
        return self.input_ids.shape[0]

    @property
    def seq_len(self) -> int:
        return self.input_ids.shape[1]


class MicroBatchManager:
    def __init__(self, num_micro_batches: int = 2, device=None):
        self.num_micro_batches = num_micro_batches
        self.device = device
        self.micro_batches: List[MicroBatch] = []

    def split_batch(self, input_ids: torch.Tensor,
                    attention_mask: Optional[torch.Tensor] = None) -> List[MicroBatch]:
        sizes = split_sizes(input_ids.shape[0], self.num_micro_batches)
        self.micro_batches = []
        start = 0
        for i, s in enumerate(sizes):
            ids = input_ids[start:start + s]
            am = attention_mask[start:start + s] if attention_mask is not None else None
            if self.device is not None:
                ids = ids.to(self.device)
                am = am.to(self.device) if am is not None else None
            self.micro_batches.append(MicroBatch(id=i, input_ids=ids, attention_mask=am,
                                                 batch_offset=start))
            start += s
        return self.micro_batches

    def merge_results(self, results: List[torch.Tensor]) -> torch.Tensor:
        return torch.cat(results, dim=0)

    def get_micro_batch(self, idx: int) -> MicroBatch:
        return self.micro_batches[idx]

    def all_completed(self) -> bool:
        return all(mb.state == MicroBatchState.COMPLETED for mb in self.micro_batches)

    def reset(self) -> None:
        for mb in self.micro_batches:
            mb.state = MicroBatchState.WAITING
            mb.current_layer = 0
            mb.hidden_states = None


def create_position_ids(batch_size: int, seq_len: int, device, start: int = 0) -> torch.Tensor:
    return (start + torch.arange(seq_len, device=device)).unsqueeze(0).expand(batch_size, -1)


def create_causal_mask(batch_size: int, seq_len: int, device, dtype=torch.float32) -> torch.Tensor:
    """[B, 1, S, S] lower-triangular (1 = attend)."""
    m = torch.tril(torch.ones(seq_len, seq_len, device=device, dtype=dtype))
    return m.unsqueeze(0).unsqueeze(0).expand(batch_size, 1, -1, -1)


def additive_causal_mask(batch_size: int, query_len: int, key_len: int, device,
                         dtype=torch.float32) -> torch.Tensor:
    """The reference's `_make_causal_mask` (src/model/disaggregated.py:508-535):
    [B, 1, Q, K], 0 where attended, finfo.min elsewhere."""
    if query_len == key_len:
        m = torch.tril(torch.ones(query_len, key_len, device=device, dtype=dtype))
    else:
        m = torch.ones(query_len, key_len, device=device, dtype=dtype)
    m = m.unsqueeze(0).unsqueeze(0).expand(batch_size, 1, -1, -1)
    return (1.0 - m) * torch.finfo(dtype).min


@dataclass
class MBSlot:
    """One micro-batch as seen by one attention rank."""
    idx: int
    batch_offset: int   # first cache row (local to the attention rank)
    batch_size: int
    q_len: int

    @property
    def tokens(self) -> int:
        return self.batch_size * self.q_len


@dataclass
class FFNSlot:
    """One micro-batch as seen by the FFN ranks: tokens of every attention
    rank, concatenated in attention-rank order."""
    idx: int
    seg_tokens: List[int]
    seg_offsets: List[int]

    @property
    def tokens(self) -> int:
        return sum(self.seg_tokens)


@dataclass
class ForwardPlan:
    topology: Topology
    global_batch: int
    q_len: int
    num_mb: int
    attn_batches: List[range]            # global sequence range per attention rank
    attn_slots: List[List[MBSlot]]       # [attn rank][mb]
    ffn_slots: List[FFNSlot] = field(default_factory=list)

    def slots_of(self, attn_index: int) -> List[MBSlot]:
        return self.attn_slots[attn_index]


def make_plan(topology: Topology, global_batch: int, num_micro_batches: int, q_len: int
              ) -> ForwardPlan:
    n_attn = 1 if topology.colocated else topology.n_attn
    batches = [topology.batch_slice(a, global_batch) for a in range(n_attn)]
    min_b = min(len(r) for r in batches)
    if min_b == 0:
        raise ValueError(f"global batch {global_batch} leaves an attention rank empty")
    num_mb = min(num_micro_batches, min_b)
    attn_slots: List[List[MBSlot]] = []
    for r in batches:
        sizes = split_sizes(len(r), num_mb)
        off, row = 0, []
        for m, s in enumerate(sizes):
            row.append(MBSlot(m, off, s, q_len))
            off += s
        attn_slots.append(row)
    ffn_slots = []
    for m in range(num_mb):
        seg = [attn_slots[a][m].tokens for a in range(n_attn)]
        offs = [sum(seg[:a]) for a in range(n_attn)]
        ffn_slots.append(FFNSlot(m, seg, offs))
    return ForwardPlan(topology, global_batch, q_len, num_mb, batches, attn_slots, ffn_slots)


def key_ranges_from_mask(attention_mask: Optional[torch.Tensor]
                         ) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    """Per-sequence visible key range [lo, hi) from a [B, S] 0/1 padding mask,
    as the prefill schedulers combine it with the causal mask (reference
    src/pipeline/async_scheduler.py:177-198, src/pipeline/scheduler.py:169-199).
    Each row must be one run of ones (left or right padding); an all-ones mask
    gives None (nothing to hide). Returns int32 tensors on the mask's device."""
    if attention_mask is None:
        return None
    m = attention_mask.to(torch.bool)
    if bool(m.all()):
        return None
    B, S = m.shape
    pos = torch.arange(S, device=m.device)
    n = m.sum(1)
    if bool((n == 0).any()):
        raise ValueError("attention_mask has a row with no token")
    lo = torch.where(m, pos, S).min(1).values
    hi = torch.where(m, pos + 1, 0).max(1).values
    if bool(((hi - lo) != n).any()):
        raise ValueError("attention_mask rows must be one contiguous run of ones "
                         "(left or right padding)")
    return lo.to(torch.int32), hi.to(torch.int32)
