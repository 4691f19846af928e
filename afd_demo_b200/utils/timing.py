"""Pipeline timing: per-(layer, micro-batch) events written in the reference's
timing-JSON schema (src/utils/timing.py:31-447), so its report, audit and plot
scripts read our files unchanged.

Two recording modes:

* ``device`` (default on CUDA): CUDA events recorded on the stream that runs
  the work, with no host synchronisation inside the loop. ``finish()``
  resolves every event against a base event recorded when the tracker was
  created, so ``start``/``end`` are seconds on the device clock relative to
  the run start. This does not serialise host and device the way the
  reference's ``current_stream().synchronize()`` spans do.
* ``cuda_events`` / ``sync``: the reference's host-clock modes (a stream or
  device synchronise, then ``perf_counter``); also the CPU fallback.

Additive keys (ignored by the reference's consumers): ``device_timed``,
``gpus``, ``topology``, ``rank_max_ms``, ``roofline_frac``.
"""

from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional

import torch


class EventType(Enum):
    ATTN_COMPUTE = "attn_compute"
    FFN_COMPUTE = "ffn_compute"
    MOE_ROUTER = "moe_router"
    MOE_EXPERTS = "moe_experts"
    MOE_SHARED_OR_DENSE = "moe_shared_or_dense"
    SEND_START = "send_start"
    SEND_TRANSFER = "send_transfer"
    RECV_POST = "recv_post"
    RECV_WAIT = "recv_wait"


@dataclass
class TimingEvent:
    event_type: str
    layer_idx: int
    mb_idx: int
    start_time: float
    end_time: float
    node: str
    tensor_bytes: Optional[int] = None
    completion_source: Optional[str] = None

    @property
    def duration_ms(self) -> float:
        return (self.end_time - self.start_time) * 1000

    def to_dict(self) -> Dict[str, Any]:
        d = {
            "type": self.event_type,
            "layer": self.layer_idx,
            "mb": self.mb_idx,
            "start": self.start_time,
            "end": self.end_time,
            "duration_ms": self.duration_ms,
            "node": self.node,
        }
        if self.tensor_bytes is not None:
            d["tensor_bytes"] = self.tensor_bytes
            d["tensor_mib"] = self.tensor_bytes / (1024 * 1024)
        if self.completion_source is not None:
            d["completion_source"] = self.completion_source
        return d


@dataclass
class LayerTiming:
    """Per-micro-batch times of one layer in ms (the reference's container,
    src/utils/timing.py:81-89)."""
    layer_idx: int
    attn_compute: List[float] = field(default_factory=list)
    ffn_compute: List[float] = field(default_factory=list)
    send_time: List[float] = field(default_factory=list)
    recv_wait: List[float] = field(default_factory=list)


_OPTIONAL_KEYS = (
    "prefill_seq_len", "actual_prompt_len", "prefill_ms", "decode_loop_ms", "decode_steps",
    "decode_tpot_ms", "timed_decode_step", "timed_decode_step_base", "timed_decode_step_note",
    "device_timed", "gpus", "topology", "rank_max_ms", "roofline_frac",
)


@dataclass
class PipelineTiming:
    node: str
    num_layers: int = 0
    num_micro_batches: int = 0
    total_time_ms: float = 0.0
    comm_timing_mode: str = "enqueue"
    prefill_seq_len: Optional[int] = None
    actual_prompt_len: Optional[int] = None
    prefill_ms: Optional[float] = None
    decode_loop_ms: Optional[float] = None
    decode_steps: Optional[int] = None
    decode_tpot_ms: Optional[float] = None
    timed_decode_step: Optional[int] = None
    timed_decode_step_base: Optional[str] = None
    timed_decode_step_note: Optional[str] = None
    device_timed: Optional[bool] = None
    gpus: Optional[int] = None
    topology: Optional[str] = None
    rank_max_ms: Optional[float] = None
    roofline_frac: Optional[Dict[str, float]] = None
    events: List[TimingEvent] = field(default_factory=list)
    total_compute_ms: float = 0.0
    total_recv_wait_ms: float = 0.0
    total_send_wait_ms: float = 0.0
    total_moe_router_ms: float = 0.0
    total_moe_experts_ms: float = 0.0
    total_moe_shared_or_dense_ms: float = 0.0

    def add_event(self, event: TimingEvent) -> None:
        self.events.append(event)
        t = event.event_type
        if t in (EventType.ATTN_COMPUTE.value, EventType.FFN_COMPUTE.value):
            self.total_compute_ms += event.duration_ms
        elif t == EventType.MOE_ROUTER.value:
            self.total_moe_router_ms += event.duration_ms
        elif t == EventType.MOE_EXPERTS.value:
            self.total_moe_experts_ms += event.duration_ms
        elif t == EventType.MOE_SHARED_OR_DENSE.value:
            self.total_moe_shared_or_dense_ms += event.duration_ms
        elif t == EventType.RECV_WAIT.value:
            self.total_recv_wait_ms += event.duration_ms
        elif t == EventType.SEND_TRANSFER.value:
            self.total_send_wait_ms += event.duration_ms

    @property
    def compute_ratio(self) -> float:
        return self.total_compute_ms / self.total_time_ms if self.total_time_ms else 0.0

    def to_dict(self) -> Dict[str, Any]:
        d: Dict[str, Any] = {
            "node": self.node,
            "num_layers": self.num_layers,
            "num_micro_batches": self.num_micro_batches,
            "total_time_ms": self.total_time_ms,
            "comm_timing_mode": self.comm_timing_mode,
            "total_compute_ms": self.total_compute_ms,
            "total_recv_wait_ms": self.total_recv_wait_ms,
            "total_moe_router_ms": self.total_moe_router_ms,
            "total_moe_experts_ms": self.total_moe_experts_ms,
            "total_moe_shared_or_dense_ms": self.total_moe_shared_or_dense_ms,
            "compute_ratio": self.compute_ratio,
            "events": [e.to_dict() for e in self.events],
        }
        for k in _OPTIONAL_KEYS:
            v = getattr(self, k)
            if v is not None:
                d[k] = v
        return d

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "PipelineTiming":
        pt = cls(node=d["node"], num_layers=d.get("num_layers", 0),
                 num_micro_batches=d.get("num_micro_batches", 0),
                 total_time_ms=d.get("total_time_ms", 0.0),
                 comm_timing_mode=d.get("comm_timing_mode", "enqueue"))
        for k in _OPTIONAL_KEYS:
            if k in d:
                setattr(pt, k, d[k])
        for e in d.get("events", []):
            pt.add_event(TimingEvent(e["type"], e["layer"], e["mb"], e["start"], e["end"],
                                     e.get("node", pt.node), e.get("tensor_bytes"),
                                     e.get("completion_source")))
        return pt

    def to_json(self, indent: int = 2) -> str:
        return json.dumps(self.to_dict(), indent=indent)

    def save(self, path: str) -> None:
        with open(path, "w") as f:
            f.write(self.to_json())

    def summary(self) -> str:
        lines = [
            f"=== {self.node.upper()} ===",
            f"e2e: {self.total_time_ms:.2f}ms",
            f"compute: {self.total_compute_ms:.2f}ms ({self.compute_ratio:.1%})",
            f"recv wait: {self.total_recv_wait_ms:.2f}ms",
        ]
        if self.total_moe_router_ms > 0 or self.total_moe_experts_ms > 0:
            lines.append(f"MoE: router={self.total_moe_router_ms:.2f}ms, "
                         f"experts={self.total_moe_experts_ms:.2f}ms, "
                         f"shared/dense={self.total_moe_shared_or_dense_ms:.2f}ms")
        return "\n".join(lines)


class TimingTracker:
    """Records events for one role. See the module docstring for the modes.

    ``mark_start``/``mark_end`` bracket device work on the current stream;
    ``record_send`` records a send span (``enqueue``: isend return time;
    ``completion``: the Work future's callback, else the observed wait, else
    ``finish``), the two comm timing modes of the reference
    (src/utils/timing.py:313-394)."""

    def __init__(self, node: str, num_layers: int, num_micro_batches: int,
                 mode: str = "device", comm_timing_mode: str = "enqueue"):
        if comm_timing_mode not in ("enqueue", "completion"):
            raise ValueError(f"Unsupported comm_timing_mode: {comm_timing_mode}")
        if mode not in ("device", "cuda_events", "sync"):
            raise ValueError(f"Unsupported timing mode: {mode}")
        cuda = torch.cuda.is_available() and torch.cuda.is_initialized()
        if not cuda:
            mode = "sync"
        self.mode = mode
        self.cuda = cuda
        self.comm_timing_mode = comm_timing_mode
        self.timing = PipelineTiming(node=node, num_layers=num_layers,
                                     num_micro_batches=num_micro_batches,
                                     comm_timing_mode=comm_timing_mode,
                                     device_timed=(mode == "device"))
        self._lock = threading.Lock()
        self._open: Dict[tuple, Any] = {}
        self._device_spans: List[tuple] = []
        self._pending_send: Dict[int, Dict[str, Any]] = {}
        self._futures: List[Any] = []
        self.start_time = time.perf_counter()
        if mode == "device":
            self._base = torch.cuda.Event(enable_timing=True)
            self._base.record()

    # -- host helpers ------------------------------------------------------
    def _host_sync(self) -> None:
        if not self.cuda:
            return
        if self.mode == "cuda_events":
            torch.cuda.current_stream().synchronize()
        else:
            torch.cuda.synchronize()

    def track(self, event_type: EventType, layer_idx: int, mb_idx: int):
        """Context manager around one span: host perf_counter start and end,
        recorded as an event (the reference's sync-mode helper)."""
        return _TimingContext(self, event_type, layer_idx, mb_idx)

    def mark_start(self, event_type: EventType, layer_idx: int, mb_idx: int,
                   stream: Optional["torch.cuda.Stream"] = None) -> None:
        key = (event_type, layer_idx, mb_idx)
        if self.mode == "device":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream) if stream is not None else ev.record()
            self._open[key] = ev
        else:
            self._host_sync()
            self._open[key] = time.perf_counter()

    def mark_end(self, event_type: EventType, layer_idx: int, mb_idx: int,
                 stream: Optional["torch.cuda.Stream"] = None, tensor_bytes: Optional[int] = None,
                 completion_source: Optional[str] = None) -> None:
        key = (event_type, layer_idx, mb_idx)
        start = self._open.pop(key, None)
        if start is None:
            return
        if self.mode == "device":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream) if stream is not None else ev.record()
            self._device_spans.append((event_type, layer_idx, mb_idx, start, ev, tensor_bytes,
                                       completion_source))
        else:
            self._host_sync()
            self.record_event(event_type, layer_idx, mb_idx, start, time.perf_counter(),
                              tensor_bytes, completion_source)

    @staticmethod
    def tensor_nbytes(tensor: Optional[torch.Tensor]) -> Optional[int]:
        return None if tensor is None else int(tensor.numel() * tensor.element_size())

    def record_event(self, event_type: EventType, layer_idx: int, mb_idx: int,
                     start_time: float, end_time: float, tensor_bytes: Optional[int] = None,
                     completion_source: Optional[str] = None) -> None:
        ev = TimingEvent(event_type.value, layer_idx, mb_idx, start_time - self.start_time,
                         end_time - self.start_time, self.timing.node, tensor_bytes,
                         completion_source)
        with self._lock:
            self.timing.add_event(ev)

    def record_send(self, handle: Any, layer_idx: int, mb_idx: int, start_time: float,
                    tensor: Optional[torch.Tensor] = None) -> None:
        nbytes = self.tensor_nbytes(tensor)
        if self.comm_timing_mode == "enqueue":
            self.record_event(EventType.SEND_TRANSFER, layer_idx, mb_idx, start_time,
                              time.perf_counter(), nbytes, "enqueue")
            return
        key = id(handle)
        with self._lock:
            self._pending_send[key] = dict(layer=layer_idx, mb=mb_idx, start=start_time,
                                           nbytes=nbytes, done=False)
        try:
            fut = handle.get_future()
        except Exception:
            return
        try:
            cb = fut.then(lambda f: (self._complete_send(key, time.perf_counter(),
                                                         "future_callback"), f)[1])
            self._futures.extend([fut, cb])
        except Exception:
            self._futures.append(fut)

    def observe_send_completion(self, handle: Any) -> None:
        if self.comm_timing_mode == "completion":
            self._complete_send(id(handle), time.perf_counter(), "observed_wait")

    def _complete_send(self, key: int, end: float, source: str) -> None:
        with self._lock:
            p = self._pending_send.get(key)
            if p is None or p["done"]:
                return
            p["done"] = True
        self.record_event(EventType.SEND_TRANSFER, p["layer"], p["mb"], p["start"], end,
                          p["nbytes"], source)

    def finish(self) -> PipelineTiming:
        for key in list(self._pending_send):
            self._complete_send(key, time.perf_counter(), "tracker_finish")
        if self.mode == "device":
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            torch.cuda.synchronize()
            for (et, l, mb, s, e, nb, src) in self._device_spans:
                t0 = self._base.elapsed_time(s) / 1000.0
                t1 = self._base.elapsed_time(e) / 1000.0
                self.timing.add_event(TimingEvent(et.value, l, mb, t0, t1, self.timing.node,
                                                  nb, src or ("device" if nb else None)))
            self.timing.events.sort(key=lambda ev: (ev.start_time, ev.layer_idx, ev.mb_idx))
            self.timing.total_time_ms = self._base.elapsed_time(end)
        else:
            self.timing.total_time_ms = (time.perf_counter() - self.start_time) * 1000
        return self.timing


class _TimingContext:
    def __init__(self, tracker: "TimingTracker", event_type: EventType, layer_idx: int,
                 mb_idx: int):
        self.tracker = tracker
        self.event_type = event_type
        self.layer_idx = layer_idx
        self.mb_idx = mb_idx

    def __enter__(self):
        self.start_time = time.perf_counter()
        return self

    def __exit__(self, *exc) -> bool:
        self.tracker.record_event(self.event_type, self.layer_idx, self.mb_idx,
                                  self.start_time, time.perf_counter())
        return False


def merge_timings(attn: PipelineTiming, ffn: PipelineTiming) -> Dict[str, Any]:
    return {
        "attention": attn.to_dict(),
        "ffn": ffn.to_dict(),
        "combined": {
            "num_layers": attn.num_layers,
            "num_micro_batches": attn.num_micro_batches,
            "attn_e2e_ms": attn.total_time_ms,
            "ffn_e2e_ms": ffn.total_time_ms,
            "attn_compute_ms": attn.total_compute_ms,
            "ffn_compute_ms": ffn.total_compute_ms,
            "attn_recv_wait_ms": attn.total_recv_wait_ms,
            "ffn_recv_wait_ms": ffn.total_recv_wait_ms,
            "attn_moe_router_ms": attn.total_moe_router_ms,
            "attn_moe_experts_ms": attn.total_moe_experts_ms,
            "attn_moe_shared_or_dense_ms": attn.total_moe_shared_or_dense_ms,
            "ffn_moe_router_ms": ffn.total_moe_router_ms,
            "ffn_moe_experts_ms": ffn.total_moe_experts_ms,
            "ffn_moe_shared_or_dense_ms": ffn.total_moe_shared_or_dense_ms,
            "attn_compute_ratio": attn.compute_ratio,
            "ffn_compute_ratio": ffn.compute_ratio,
        },
    }
