"""Small profiling helpers (reference: src/utils/profiler.py:32-221):
a host ``Timer``, a device ``CUDATimer`` (CUDA events), an aggregating
``Profiler`` with a ``profile_function`` decorator, and ``print_memory_stats``."""

from __future__ import annotations

import functools
import logging
import time
from collections import defaultdict
from typing import Callable, Dict, List, Optional

import torch

logger = logging.getLogger(__name__)


class Timer:
    def __init__(self, name: str = ""):
        self.name = name
        self.elapsed_ms = 0.0

    def __enter__(self):
        self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        self.elapsed_ms = (time.perf_counter() - self._t0) * 1000
        return False


class CUDATimer:
    """Device time of the enclosed work on the current stream (events +
    synchronize of the end event)."""

    def __init__(self, name: str = "", stream: Optional[torch.cuda.Stream] = None):
        self.name = name
        self.stream = stream
        self.elapsed_ms = 0.0

    def __enter__(self):
        if torch.cuda.is_available():
            self._s = torch.cuda.Event(enable_timing=True)
            self._e = torch.cuda.Event(enable_timing=True)
            self._s.record(self.stream)
        else:
            self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if torch.cuda.is_available():
            self._e.record(self.stream)
            self._e.synchronize()
            self.elapsed_ms = self._s.elapsed_time(self._e)
        else:
            self.elapsed_ms = (time.perf_counter() - self._t0) * 1000
        return False


class Profiler:
    def __init__(self):
        self.records: Dict[str, List[float]] = defaultdict(list)

    def record(self, name: str, ms: float) -> None:
        self.records[name].append(ms)

    def timer(self, name: str, device: bool = False):
        prof = self

        class _Ctx:
            def __enter__(self_inner):
                self_inner.t = CUDATimer(name) if device else Timer(name)
                self_inner.t.__enter__()
                return self_inner.t

            def __exit__(self_inner, *exc):
                self_inner.t.__exit__(*exc)
                prof.record(name, self_inner.t.elapsed_ms)
                return False

        return _Ctx()

    def summary(self) -> Dict[str, Dict[str, float]]:
        out = {}
        for k, v in self.records.items():
            out[k] = {"count": len(v), "total_ms": sum(v), "mean_ms": sum(v) / len(v),
                      "min_ms": min(v), "max_ms": max(v)}
        return out

    def reset(self) -> None:
        self.records.clear()


_PROFILER = Profiler()


def get_profiler() -> Profiler:
    return _PROFILER


def profile_function(name: Optional[str] = None, device: bool = False) -> Callable:
    def deco(fn):
        label = name or fn.__qualname__

        @functools.wraps(fn)
        def wrapper(*a, **kw):
            with _PROFILER.timer(label, device=device):
                return fn(*a, **kw)

        return wrapper

    return deco


def print_memory_stats(prefix: str = "") -> None:
    if not torch.cuda.is_available():
        return
    gb = 2**30
    logger.info(f"{prefix}GPU memory: allocated={torch.cuda.memory_allocated() / gb:.2f}GB "
                f"reserved={torch.cuda.memory_reserved() / gb:.2f}GB "
                f"peak={torch.cuda.max_memory_allocated() / gb:.2f}GB")
