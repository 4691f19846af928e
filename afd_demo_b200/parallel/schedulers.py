"""The reference's three schedulers as thin front ends over ``PipelineEngine``.

* ``SimplePipelineScheduler``  -- serial prefill, one blocking A->F->A round
  trip per layer and micro-batch (src/pipeline/scheduler.py:20-250).
* ``AsyncPipelineScheduler``   -- prefill DBO: two micro-batches ping-pong
  between the roles (src/pipeline/async_scheduler.py:60-796).
* ``DecodeDBOScheduler``       -- one decode step with micro-batch overlap,
  optionally cross-layer (src/pipeline/decode_scheduler.py:64-579). Timing is
  recorded on 0-based decode step 1, as in the reference.

Stats objects (``DBOStats``, ``DecodeDBOStats``) carry the same fields. With
timing enabled the events come from the device (CUDA events on the streams
that ran the work) and are written in the reference's JSON schema.
"""

from __future__ import annotations

import logging
import time
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from ..utils import device as devmod
from ..utils.timing import PipelineTiming, TimingTracker
from .micro_batch import MicroBatchManager

logger = logging.getLogger(__name__)


@dataclass
class DBOStats:
    total_time: float = 0.0
    compute_time: float = 0.0
    recv_wait_time: float = 0.0
    num_layers: int = 0
    num_micro_batches: int = 0

    @property
    def compute_ratio(self) -> float:
        return self.compute_time / self.total_time if self.total_time else 0.0

    def __str__(self) -> str:
        return (f"e2e: {self.total_time * 1000:.2f}ms | compute: {self.compute_time * 1000:.2f}ms "
                f"({self.compute_ratio:.1%}) | wait: {self.recv_wait_time * 1000:.2f}ms")


@dataclass
class DecodeDBOStats:
    total_time: float = 0.0
    compute_time: float = 0.0
    comm_time: float = 0.0
    num_tokens: int = 0
    num_layers: int = 0
    attn_compute_time: float = 0.0
    ffn_compute_time: float = 0.0
    a2f_comm_time: float = 0.0
    f2a_comm_time: float = 0.0

    @property
    def tokens_per_second(self) -> float:
        return self.num_tokens / self.total_time if self.total_time else 0.0

    def __str__(self) -> str:
        s = (f"Decode DBO: {self.total_time * 1000:.2f}ms | compute: {self.compute_time * 1000:.2f}ms"
             f" | comm: {self.comm_time * 1000:.2f}ms | {self.tokens_per_second:.1f} tok/s")
        if self.attn_compute_time or self.ffn_compute_time:
            s += (f"\n  attn={self.attn_compute_time * 1000:.2f}ms ffn="
                  f"{self.ffn_compute_time * 1000:.2f}ms a2f={self.a2f_comm_time * 1000:.2f}ms "
                  f"f2a={self.f2a_comm_time * 1000:.2f}ms")
        return s


def _trackers(model, enable: bool, num_mb: int, mode: str, comm_mode: str
              ) -> Dict[str, TimingTracker]:
    if not enable:
        return {}
    ctx = model.ctx
    roles = ["attention", "ffn"] if ctx.is_colocated else [ctx.role]
    out = {}
    for r in roles:
        t = TimingTracker(r, model.num_layers, num_mb, mode=mode, comm_timing_mode=comm_mode)
        t.timing.gpus = ctx.world_size
        t.timing.topology = ctx.topology.tag()
        out[r] = t
    return out


def _finish(trackers: Dict[str, TimingTracker], ctx) -> Optional[PipelineTiming]:
    if not trackers:
        return None
    res = {r: t.finish() for r, t in trackers.items()}
    if ctx.is_colocated:
        a = res["attention"]
        a.ffn_timing = res["ffn"]
        return a
    return res[ctx.role]


class SimplePipelineScheduler:
    """Serial schedule (reference: src/pipeline/scheduler.py:20-57, 132-...):
    the micro-batches of each layer run one after another, with the same
    constructor, ``run`` and ``get_timing_data`` as the reference's. With
    `enable_timing` the per-layer events go to a ``TimingTracker`` in
    `timing_mode` ("cuda_events", "sync" or "device")."""

    def __init__(self, model, num_micro_batches: int = 2, enable_timing: bool = False,
                 timing_mode: str = "cuda_events"):
        self.model = model
        self.ctx = model.ctx
        self.num_micro_batches = num_micro_batches
        self.enable_timing = enable_timing
        self.timing_mode = timing_mode
        self.mb_manager = MicroBatchManager(num_micro_batches, model.device)
        self._timing_data: Optional[PipelineTiming] = None

    @torch.no_grad()
    def run(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None):
        m = self.model
        nmb = min(self.num_micro_batches, input_ids.shape[0])
        tr = _trackers(m, self.enable_timing, nmb, self.timing_mode, "enqueue")
        out = m.run_forward(input_ids, "serial", self.num_micro_batches, trackers=tr,
                            reset_cache=True, attention_mask=attention_mask)
        if self.enable_timing:
            devmod.synchronize()
        self._timing_data = _finish(tr, m.ctx)
        if m.transport is not None and devmod.is_cuda():
            m.transport.check()
        return out

    def get_timing_data(self) -> Optional[PipelineTiming]:
        """The last run's timing (None unless `enable_timing`)."""
        return self._timing_data


class AsyncPipelineScheduler:
    def __init__(self, model, num_micro_batches: int = 2, use_cuda_streams: bool = True,
                 enable_timing: bool = False, timing_mode: str = "device",
                 comm_timing_mode: str = "enqueue", crosslayer: bool = True):
        self.model = model
        self.ctx = model.ctx
        self.num_micro_batches = num_micro_batches
        self.use_cuda_streams = use_cuda_streams
        self.enable_timing = enable_timing
        self.timing_mode = timing_mode
        self.comm_timing_mode = comm_timing_mode
        self.crosslayer = crosslayer
        self.mb_manager = MicroBatchManager(num_micro_batches, model.device)
        self.stats = DBOStats()
        self._timing_data: Optional[PipelineTiming] = None

    @torch.no_grad()
    def run(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None):
        m = self.model
        t0 = time.perf_counter()
        if self.enable_timing:
            m.ctx.barrier()
        nmb = min(self.num_micro_batches, input_ids.shape[0])
        tr = _trackers(m, self.enable_timing, nmb, self.timing_mode, self.comm_timing_mode)
        out = m.run_forward(input_ids, "dbo", self.num_micro_batches, self.crosslayer,
                            trackers=tr, reset_cache=True, attention_mask=attention_mask)
        if self.enable_timing:
            devmod.synchronize()
        self._timing_data = _finish(tr, m.ctx)
        self.stats = DBOStats(total_time=time.perf_counter() - t0, num_layers=m.num_layers,
                              num_micro_batches=nmb)
        if self._timing_data is not None:
            self.stats.total_time = self._timing_data.total_time_ms / 1000
            self.stats.compute_time = self._timing_data.total_compute_ms / 1000
            self.stats.recv_wait_time = self._timing_data.total_recv_wait_ms / 1000
        if m.transport is not None and devmod.is_cuda():
            m.transport.check()
        return out

    def get_stats(self) -> DBOStats:
        return self.stats

    def get_timing_data(self) -> Optional[PipelineTiming]:
        return self._timing_data


class DecodeDBOScheduler:
    def __init__(self, model, num_micro_batches: int = 2, enable_timing: bool = False,
                 timing_mode: str = "device", comm_timing_mode: str = "enqueue",
                 use_crosslayer: bool = False):
        self.model = model
        self.ctx = model.ctx
        self.num_micro_batches = num_micro_batches
        self.enable_timing = enable_timing
        self.timing_mode = timing_mode
        self.comm_timing_mode = comm_timing_mode
        self.use_crosslayer = use_crosslayer
        self.timing_step = 1  # 0-based step 1: skips the cold first step
        self._current_step = 0
        self.stats = DecodeDBOStats()
        self._timing_data: Optional[PipelineTiming] = None

    def _compute_mb_sizes(self, batch_size: int) -> List[int]:
        from .micro_batch import split_sizes
        return split_sizes(batch_size, self.num_micro_batches)

    @torch.no_grad()
    def forward_decode_dbo(self, input_ids: torch.Tensor, position_ids=None, kv_cache=None):
        m = self.model
        B = input_ids.shape[0]
        track = self.enable_timing and self._current_step == self.timing_step
        t0 = time.perf_counter()
        tr = {}
        if track:
            m.ctx.barrier()
            tr = _trackers(m, True, min(self.num_micro_batches, B), self.timing_mode,
                           self.comm_timing_mode)
        out = m.run_forward(input_ids, "dbo", self.num_micro_batches, self.use_crosslayer,
                            trackers=tr)
        if track:
            devmod.synchronize()
            self._timing_data = _finish(tr, m.ctx)
            for td in (self._timing_data, getattr(self._timing_data, "ffn_timing", None)):
                if td is not None:
                    td.timed_decode_step = self.timing_step
                    td.timed_decode_step_base = "0-based"
                    td.timed_decode_step_note = "step 0 skipped to avoid warmup/cold-start timing"
        self.stats = DecodeDBOStats(num_tokens=B, num_layers=m.num_layers,
                                    total_time=time.perf_counter() - t0)
        if self._timing_data is not None and track:
            td = self._timing_data
            self.stats.total_time = td.total_time_ms / 1000
            self.stats.compute_time = td.total_compute_ms / 1000
            self.stats.comm_time = td.total_recv_wait_ms / 1000
        self._current_step += 1
        return out

    def get_stats(self) -> DecodeDBOStats:
        return self.stats

    def get_timing_data(self) -> Optional[PipelineTiming]:
        return self._timing_data
