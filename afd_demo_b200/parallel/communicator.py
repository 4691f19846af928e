"""Buffered point-to-point communicator with the reference's interface.

Reference: ``AFDCommunicator`` (src/distributed/communicator.py:20-300): a
ring of ``num_buffers`` send and receive buffers with a state each,
``send_async`` / ``recv_async`` returning a buffer index, ``wait_send`` /
``wait_recv`` / ``wait_all_recvs``, blocking ``send_sync`` / ``recv_sync``
and ``synchronize``, over torch.distributed p2p (NCCL on CUDA, gloo on CPU).

This framework's own schedules do not use it: their A2F/F2A hand-offs are the
transports in ``transport.py`` (fused peer-memory stores, or NCCL p2p for the
baseline). The class serves code written against the reference's API.
Differences that keep it correct: each buffer is one flat allocation and a
message uses its first ``numel`` elements, so the view handed to NCCL/gloo is
always contiguous (a slice of a [B, S, H] buffer is not, and a contiguous copy
would receive the data instead of the buffer); the copy into a send buffer
runs on the communication stream after it waits for the producing stream.
"""

from __future__ import annotations

import logging
import math
from dataclasses import dataclass
from enum import Enum
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from .dist import get_distributed_context

logger = logging.getLogger(__name__)


class BufferState(Enum):
    FREE = 0
    SENDING = 1
    RECEIVING = 2
    READY = 3


@dataclass
class CommBuffer:
    tensor: torch.Tensor                      # flat storage of max_batch * max_seq * hidden
    state: BufferState = BufferState.FREE
    handle: Optional[object] = None           # pending dist.Work
    requested_shape: Optional[Tuple[int, ...]] = None


class AFDCommunicator:
    def __init__(self, hidden_size: int, max_seq_len: int, max_batch_size: int,
                 num_buffers: int = 2, dtype: torch.dtype = torch.bfloat16,
                 peer: Optional[int] = None):
        """`peer` defaults to the context's peer rank (the other role in a
        two-rank job)."""
        self.ctx = get_distributed_context()
        self.hidden_size = hidden_size
        self.max_seq_len = max_seq_len
        self.max_batch_size = max_batch_size
        self.num_buffers = num_buffers
        self.dtype = dtype
        self.peer = self.ctx.peer_rank if peer is None else peer
        self.device = self.ctx.device
        self.comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self.send_buffers: List[CommBuffer] = []
        self.recv_buffers: List[CommBuffer] = []
        self._init_buffers()
        self._send_idx = 0
        self._recv_idx = 0
        self._pending_sends: List[object] = []
        self._pending_recvs: List[object] = []

    # -------------------------------------------------------------- buffers
    def _init_buffers(self) -> None:
        n = self.max_batch_size * self.max_seq_len * self.hidden_size
        for _ in range(self.num_buffers):
            self.send_buffers.append(CommBuffer(torch.empty(n, dtype=self.dtype,
                                                            device=self.device)))
            self.recv_buffers.append(CommBuffer(torch.empty(n, dtype=self.dtype,
                                                            device=self.device)))

    @staticmethod
    def _finish(buf: CommBuffer, pending: List[object]) -> None:
        """Wait for the buffer's outstanding operation once and forget it (a
        completed gloo Work must not be waited on again)."""
        h = buf.handle
        if h is not None:
            h.wait()
            buf.handle = None
            for i, p in enumerate(pending):
                if p is h:
                    del pending[i]
                    break

    def _get_send_buffer(self) -> Tuple[int, CommBuffer]:
        idx = self._send_idx
        self._send_idx = (idx + 1) % self.num_buffers
        return idx, self.send_buffers[idx]

    def _get_recv_buffer(self) -> Tuple[int, CommBuffer]:
        idx = self._recv_idx
        self._recv_idx = (idx + 1) % self.num_buffers
        return idx, self.recv_buffers[idx]

    def _shape(self, shape: Tuple[int, ...]) -> Tuple[int, ...]:
        shape = tuple(int(s) for s in shape)
        return shape + (self.hidden_size,) if len(shape) == 2 else shape

    def _view(self, buf: CommBuffer, shape: Tuple[int, ...]) -> torch.Tensor:
        shape = self._shape(shape)
        n = math.prod(shape)
        if n > buf.tensor.numel():
            raise ValueError(f"message of shape {shape} exceeds the buffer "
                             f"({self.max_batch_size} x {self.max_seq_len} x {self.hidden_size})")
        return buf.tensor[:n].view(shape)

    # ---------------------------------------------------------------- async
    def send_async(self, tensor: torch.Tensor, tag: int = 0) -> int:
        """Copy `tensor` into the next send buffer and start sending it;
        returns the buffer index."""
        idx, buf = self._get_send_buffer()
        self._finish(buf, self._pending_sends)
        view = self._view(buf, tuple(tensor.shape))
        if self.comm_stream is not None:
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                view.copy_(tensor)
            self.comm_stream.synchronize()
        else:
            view.copy_(tensor)
        buf.handle = dist.isend(view, dst=self.peer, tag=tag)
        buf.state = BufferState.SENDING
        self._pending_sends.append(buf.handle)
        return idx

    def recv_async(self, shape: Tuple[int, ...], tag: int = 0) -> int:
        """Post a receive of `shape` ([B, S] means [B, S, hidden]) into the
        next receive buffer; returns the buffer index."""
        idx, buf = self._get_recv_buffer()
        self._finish(buf, self._pending_recvs)
        buf.requested_shape = self._shape(shape)
        buf.handle = dist.irecv(self._view(buf, buf.requested_shape), src=self.peer, tag=tag)
        buf.state = BufferState.RECEIVING
        self._pending_recvs.append(buf.handle)
        return idx

    def wait_send(self, buffer_idx: Optional[int] = None) -> None:
        """Wait for one send buffer (or all) to be free again."""
        bufs = self.send_buffers if buffer_idx is None else [self.send_buffers[buffer_idx]]
        for buf in bufs:
            self._finish(buf, self._pending_sends)
            buf.state = BufferState.FREE

    def wait_recv(self, buffer_idx: int) -> torch.Tensor:
        """Wait for one receive; returns a view of the buffer with the
        requested shape (valid until the buffer is reused)."""
        buf = self.recv_buffers[buffer_idx]
        self._finish(buf, self._pending_recvs)
        buf.state = BufferState.READY
        if buf.requested_shape is None:
            return buf.tensor
        return self._view(buf, buf.requested_shape)

    def wait_all_recvs(self) -> List[torch.Tensor]:
        out = []
        for buf in self.recv_buffers:
            if buf.state == BufferState.RECEIVING:
                self._finish(buf, self._pending_recvs)
                buf.state = BufferState.READY
                out.append(self._view(buf, buf.requested_shape) if buf.requested_shape
                           else buf.tensor)
        return out

    # ----------------------------------------------------------------- sync
    def send_sync(self, tensor: torch.Tensor, tag: int = 0) -> None:
        dist.send(tensor.contiguous(), dst=self.peer, tag=tag)

    def recv_sync(self, shape: Tuple[int, ...], tag: int = 0) -> torch.Tensor:
        t = torch.empty(self._shape(shape), dtype=self.dtype, device=self.device)
        dist.recv(t, src=self.peer, tag=tag)
        return t

    def synchronize(self) -> None:
        self.wait_send()
        for buf in self.recv_buffers:
            self._finish(buf, self._pending_recvs)
        if self.comm_stream is not None:
            self.comm_stream.synchronize()
