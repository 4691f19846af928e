"""Device backend selection: ``cuda`` (NCCL) or ``cpu`` (gloo).

Same contract as the reference's src/utils/device.py:37-173 (``init_backend``,
``DEVICE_TYPE``, ``DIST_BACKEND``, ``synchronize``, ``Event``, ``Stream``,
``apply_backend_envs``). There is no NPU variant: the CUDA path is sm_100a only.
"""

from __future__ import annotations

import contextlib
import logging
import os
from typing import Optional

import torch

logger = logging.getLogger(__name__)

DEVICE_TYPE: str = "cpu"
DIST_BACKEND: str = "gloo"
_INITIALIZED = False


def init_backend(backend: str = "auto") -> str:
    global DEVICE_TYPE, DIST_BACKEND, _INITIALIZED
    if _INITIALIZED:
        return DEVICE_TYPE
    backend = backend.lower()
    if backend == "auto":
        backend = "cuda" if torch.cuda.is_available() else "cpu"
    if backend == "cuda":
        if not torch.cuda.is_available():
            raise RuntimeError("backend=cuda requested but no CUDA device is visible")
        DEVICE_TYPE, DIST_BACKEND = "cuda", "nccl"
    elif backend == "cpu":
        DEVICE_TYPE, DIST_BACKEND = "cpu", "gloo"
    else:
        raise ValueError(f"unknown backend {backend!r}")
    _INITIALIZED = True
    return DEVICE_TYPE


def reset_backend() -> None:
    """Forget the selection (tests switch backends within one process)."""
    global _INITIALIZED, DEVICE_TYPE, DIST_BACKEND
    _INITIALIZED = False
    DEVICE_TYPE, DIST_BACKEND = "cpu", "gloo"


def is_cuda() -> bool:
    return DEVICE_TYPE == "cuda"


is_available = is_cuda  # the reference's name


def device_module():
    """torch.cuda, or None on the CPU backend."""
    return torch.cuda if is_cuda() else None


def current_device_str(local_rank: int = 0) -> str:
    return f"cuda:{local_rank}" if is_cuda() else "cpu"


def device_count() -> int:
    return torch.cuda.device_count() if is_cuda() else 0


def device_for(local_rank: int = 0) -> torch.device:
    return torch.device(f"cuda:{local_rank}") if is_cuda() else torch.device("cpu")


def set_device(local_rank: int) -> None:
    if is_cuda():
        torch.cuda.set_device(local_rank)


def synchronize(device: Optional[int] = None) -> None:
    if is_cuda():
        torch.cuda.synchronize(device)


def current_stream_synchronize() -> None:
    if is_cuda():
        torch.cuda.current_stream().synchronize()


def Event(enable_timing: bool = True):
    return torch.cuda.Event(enable_timing=enable_timing) if is_cuda() else None


def Stream():
    return torch.cuda.Stream() if is_cuda() else None


def stream_context(stream):
    if stream is None or not is_cuda():
        return contextlib.nullcontext()
    return torch.cuda.stream(stream)


def empty_cache() -> None:
    if is_cuda():
        torch.cuda.empty_cache()


def memory_allocated(device=None) -> int:
    """Bytes held by tensors (0 on the CPU backend)."""
    return torch.cuda.memory_allocated(device) if is_cuda() else 0


def max_memory_allocated(device=None) -> int:
    return torch.cuda.max_memory_allocated(device) if is_cuda() else 0


def memory_reserved(device=None) -> int:
    """Bytes held by the caching allocator (0 on the CPU backend)."""
    return torch.cuda.memory_reserved(device) if is_cuda() else 0


def memory_allocated_gb() -> float:
    return torch.cuda.memory_allocated() / 2**30 if is_cuda() else 0.0


def max_memory_allocated_gb() -> float:
    return torch.cuda.max_memory_allocated() / 2**30 if is_cuda() else 0.0


def apply_backend_envs() -> None:
    """NCCL settings the reference exports for its p2p path
    (src/utils/device.py:168-173): a 32 MiB buffer so that A2F sends do not
    block on flow control, one channel per net peer."""
    if is_cuda():
        os.environ.setdefault("NCCL_BUFFSIZE", "33554432")
        os.environ.setdefault("NCCL_NCHANNELS_PER_NET_PEER", "1")
