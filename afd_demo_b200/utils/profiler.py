"""Small profiling helpers with the reference's interface
(src/utils/profiler.py:20-221): ``TimingResult``, a host ``Timer``, a device
``CUDATimer`` (CUDA events), an aggregating ``Profiler`` (``timer``,
``record``, ``get_stats``, ``report``, ``reset``), the ``profile_function``
decorator and ``print_memory_stats``. Every elapsed time is in ms."""

from __future__ import annotations

import contextlib
import functools
import logging
import time
from collections import defaultdict
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional

import torch

logger = logging.getLogger(__name__)


@dataclass
class TimingResult:
    name: str
    elapsed_ms: float
    count: int = 1

    @property
    def avg_ms(self) -> float:
        return self.elapsed_ms / self.count if self.count > 0 else 0.0


class Timer:
    """Host wall time of the enclosed block."""

    def __init__(self, name: str = ""):
        self.name = name
        self.elapsed = 0.0

    def __enter__(self) -> "Timer":
        self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc) -> bool:
        self.elapsed = (time.perf_counter() - self._t0) * 1000
        if self.name:
            logger.debug(f"{self.name}: {self.elapsed:.3f} ms")
        return False

    @property
    def elapsed_ms(self) -> float:
        return self.elapsed


class CUDATimer:
    """Device time of the work enqueued inside the block on `stream` (the
    current stream by default): CUDA events on both sides, the end event
    synchronised at exit. `sync` also drains the device before the start
    event, as the reference's timer does. Falls back to host time without
    CUDA."""

    def __init__(self, name: str = "", sync: bool = True,
                 stream: Optional[torch.cuda.Stream] = None):
        self.name = name
        self.sync = sync
        self.stream = stream
        self.elapsed = 0.0
        self._cuda = torch.cuda.is_available()

    def __enter__(self) -> "CUDATimer":
        if self._cuda:
            if self.sync:
                torch.cuda.synchronize()
            self._s = torch.cuda.Event(enable_timing=True)
            self._e = torch.cuda.Event(enable_timing=True)
            self._s.record(self.stream)
        else:
            self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc) -> bool:
        if self._cuda:
            self._e.record(self.stream)
            self._e.synchronize()
            self.elapsed = self._s.elapsed_time(self._e)
        else:
            self.elapsed = (time.perf_counter() - self._t0) * 1000
        if self.name:
            logger.debug(f"{self.name}: {self.elapsed:.3f} ms")
        return False

    @property
    def elapsed_ms(self) -> float:
        return self.elapsed


class Profiler:
    """Named lists of timings with count / total / avg / min / max."""

    def __init__(self):
        self.timings: Dict[str, List[float]] = defaultdict(list)

    @contextlib.contextmanager
    def timer(self, name: str, use_cuda: bool = True):
        t = CUDATimer(name) if (use_cuda and torch.cuda.is_available()) else Timer(name)
        with t:
            yield t
        self.timings[name].append(t.elapsed_ms)

    def record(self, name: str, elapsed_ms: float) -> None:
        self.timings[name].append(elapsed_ms)

    def get_stats(self, name: str) -> Dict[str, float]:
        v = self.timings.get(name, [])
        if not v:
            return {"count": 0, "total_ms": 0.0, "avg_ms": 0.0, "min_ms": 0.0, "max_ms": 0.0}
        return {"count": len(v), "total_ms": sum(v), "avg_ms": sum(v) / len(v),
                "min_ms": min(v), "max_ms": max(v)}

    def result(self, name: str) -> TimingResult:
        st = self.get_stats(name)
        return TimingResult(name, st["total_ms"], st["count"])

    def report(self) -> str:
        rule = "=" * 60
        lines = [rule, "Profiling Report", rule]
        for name in sorted(self.timings):
            st = self.get_stats(name)
            lines.append(f"{name:30s} | count: {st['count']:4d} | total: {st['total_ms']:8.2f}ms"
                         f" | avg: {st['avg_ms']:8.2f}ms")
        lines.append(rule)
        return "\n".join(lines)

    def reset(self) -> None:
        self.timings.clear()


_PROFILER: Optional[Profiler] = None


def get_profiler() -> Profiler:
    global _PROFILER
    if _PROFILER is None:
        _PROFILER = Profiler()
    return _PROFILER


def profile_function(name: Optional[str] = None, use_cuda: bool = True) -> Callable:
    """Record each call of the decorated function in the global profiler."""
    def decorator(fn: Callable) -> Callable:
        label = name or fn.__name__

        @functools.wraps(fn)
        def wrapper(*a, **kw) -> Any:
            with get_profiler().timer(label, use_cuda=use_cuda):
                return fn(*a, **kw)

        return wrapper

    return decorator


def print_memory_stats(device: Optional[torch.device] = None) -> None:
    """Log allocated / reserved / peak device memory (GB)."""
    if not torch.cuda.is_available():
        logger.info("CUDA not available")
        return
    if device is None:
        device = torch.cuda.current_device()
    gb = 2**30
    logger.info(f"GPU memory: allocated={torch.cuda.memory_allocated(device) / gb:.2f}GB "
                f"reserved={torch.cuda.memory_reserved(device) / gb:.2f}GB "
                f"peak={torch.cuda.max_memory_allocated(device) / gb:.2f}GB")
