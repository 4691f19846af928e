"""A2F / F2A transports: how a micro-batch's hidden states move between the
attention role and the FFN role for one layer.

Reference: ``AFDCommunicator`` (src/distributed/communicator.py:37-300) and the
per-scheduler isend/irecv calls (§ NCCL call sites: src/pipeline/
async_scheduler.py:147-154, src/pipeline/decode_scheduler.py:301-552).

Every transport keeps the host asynchronous: sends and receives are
enqueued, and a receive makes the *consuming stream* wait (CUDA event, NCCL
work, or a bounded device-side flag wait), so one host loop can enqueue a
whole forward and a captured CUDA graph can replay it.

* ``LocalTransport``  -- both roles in one process on one GPU: the tensor is
  handed over by reference, ordered by CUDA events between the attention and
  FFN streams.
* ``NcclTransport``   -- the reference's mechanism: NCCL isend/irecv on two
  directional communicators (attention->FFN, FFN->attention). This is the
  comparison baseline (``--comm-impl nccl``).
* ``PeerTransport``   -- the fused path: receive buffers and flags live in
  peer-mapped memory (CUDA IPC over NVLink). The attention o_proj GEMM's
  epilogue stores h into every FFN rank's buffer and its last CTA raises the
  flags; the FFN combine kernel stores the layer output (residual included)
  into the attention ranks' buffers and raises theirs. Receives are bounded
  device-side waits whose timeouts land in a status word that ``check()``
  turns into ``AFDCommTimeout``.
"""

from __future__ import annotations

import datetime
import logging
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .. import ops
from . import faults
from .micro_batch import ForwardPlan

logger = logging.getLogger(__name__)


class AFDCommTimeout(RuntimeError):
    """A device-side wait for a peer's flag expired."""


class Transport:
    fused = False

    def begin(self, plan: ForwardPlan) -> None:
        self.plan = plan

    def end(self) -> None:
        pass

    # attention side
    def a2f_sink(self, l: int, m: int):
        return None

    def a2f_send(self, l: int, m: int, h: torch.Tensor) -> None:
        raise NotImplementedError

    def f2a_recv(self, l: int, m: int) -> List[torch.Tensor]:
        raise NotImplementedError

    # FFN side
    def a2f_recv(self, l: int, m: int) -> torch.Tensor:
        raise NotImplementedError

    def f2a_sink(self, l: int, m: int):
        return None

    def f2a_send(self, l: int, m: int, out: torch.Tensor) -> None:
        raise NotImplementedError

    # A transport may leave the receive's wait to the consuming kernel: after
    # a2f_recv / f2a_recv, take_wait() hands over the pending wait (or None).
    defer_waits = False

    def take_wait(self):
        return None

    def check(self) -> None:
        pass


# ---------------------------------------------------------------- local ---
class LocalTransport(Transport):
    """Co-located roles: hand tensors over through CUDA events."""

    def __init__(self, attn_stream=None, ffn_stream=None):
        self.attn_stream = attn_stream
        self.ffn_stream = ffn_stream
        self._a2f: Dict[Tuple[int, int], Tuple[torch.Tensor, object]] = {}
        self._f2a: Dict[Tuple[int, int], Tuple[torch.Tensor, object]] = {}

    @staticmethod
    def _mark(t: torch.Tensor):
        if t.is_cuda:
            ev = torch.cuda.Event()
            ev.record()
            return ev
        return None

    @staticmethod
    def _take(t: torch.Tensor, ev) -> torch.Tensor:
        if ev is not None:
            cur = torch.cuda.current_stream()
            cur.wait_event(ev)
            t.record_stream(cur)
        return t

    def a2f_send(self, l, m, h):
        self._a2f[(l, m)] = (h, self._mark(h))

    def a2f_recv(self, l, m):
        return self._take(*self._a2f.pop((l, m)))

    def f2a_send(self, l, m, out):
        self._f2a[(l, m)] = (out, self._mark(out))

    def f2a_recv(self, l, m):
        return [self._take(*self._f2a.pop((l, m)))]


# ----------------------------------------------------------------- NCCL ---
class NcclTransport(Transport):
    """isend/irecv between every attention rank and every FFN rank on the
    two directional groups of the distributed context. Tag semantics follow
    the reference (NCCL ignores tags; order per communicator is what
    matches sends to receives)."""

    def __init__(self, ctx, hidden: int, dtype, device, crosslayer: bool = True):
        self.ctx = ctx
        self.H = hidden
        self.dtype = dtype
        self.device = device
        self.crosslayer = crosslayer
        self._a2f_group = ctx.a2f_group
        self._f2a_group = ctx.f2a_group
        self._pending_send: Dict[Tuple[int, int], List] = {}
        self._posted_recv: Dict[Tuple[int, int], Tuple[List, List[torch.Tensor]]] = {}

    @staticmethod
    def tag(l: int, m: int, num_mb: int, direction: str) -> int:
        """Decode-DBO tag formula of the reference
        (src/pipeline/decode_scheduler.py:122-125)."""
        return 10000 + l * (num_mb * 2) + m * 2 + (0 if direction == "a2f" else 1)

    def _wait(self, w) -> None:
        """Wait for a p2p work item, bounded by the process-group timeout so
        that a peer that is gone or a message that never comes ends as an
        error. gloo p2p work items wait forever unless given a timeout (and
        cannot be polled); an NCCL wait only orders streams on the host, and
        NCCL's watchdog aborts the communicator when the timeout expires."""
        try:
            if self.device.type == "cpu":
                w.wait(timeout=datetime.timedelta(seconds=self.ctx.config.timeout_s))
            else:
                w.wait()
        except RuntimeError as e:
            if "Timed out" in str(e) or "timeout" in str(e).lower():
                raise AFDCommTimeout(f"p2p wait timed out: {e}") from e
            raise

    def _retire_sends(self, l: int, m: int) -> None:
        for w, _t in self._pending_send.pop((l, m), []):
            self._wait(w)

    # attention side ---------------------------------------------------
    def a2f_send(self, l, m, h):
        if l > 0:
            self._retire_sends(l - 1, m)
        h = h.contiguous()
        works = [] if faults.plan().drop("a2f", l, m) else \
            [(dist.isend(h, dst=f, group=self._a2f_group), h) for f in self.ctx.ffn_ranks()]
        self._pending_send[(l, m)] = works
        if self.crosslayer:
            self.post_f2a_recv(l, m)

    def post_f2a_recv(self, l, m):
        if (l, m) in self._posted_recv:
            return
        slot = self.plan.slots_of(self.ctx.attn_index)[m]
        bufs, works = [], []
        for f in self.ctx.ffn_ranks():
            b = torch.empty(slot.tokens, self.H, device=self.device, dtype=self.dtype)
            works.append(dist.irecv(b, src=f, group=self._f2a_group))
            bufs.append(b)
        self._posted_recv[(l, m)] = (works, bufs)

    def f2a_recv(self, l, m):
        self.post_f2a_recv(l, m)
        works, bufs = self._posted_recv.pop((l, m))
        for w in works:
            self._wait(w)
        return bufs

    # FFN side ------------------------------------------------------------
    def a2f_recv(self, l, m):
        slot = self.plan.ffn_slots[m]
        buf = torch.empty(slot.tokens, self.H, device=self.device, dtype=self.dtype)
        works = []
        for a, r in enumerate(self.ctx.attn_ranks()):
            o, n = slot.seg_offsets[a], slot.seg_tokens[a]
            works.append(dist.irecv(buf[o:o + n], src=r, group=self._a2f_group))
        for w in works:
            self._wait(w)
        return buf

    def f2a_send(self, l, m, out):
        if l > 0:
            self._retire_sends(l - 1, m)
        slot = self.plan.ffn_slots[m]
        works = []
        if not faults.plan().drop("f2a", l, m):
            for a, r in enumerate(self.ctx.attn_ranks()):
                o, n = slot.seg_offsets[a], slot.seg_tokens[a]
                part = out[o:o + n].contiguous()
                works.append((dist.isend(part, dst=r, group=self._f2a_group), part))
        self._pending_send[(l, m)] = works

    def end(self) -> None:
        for key in list(self._pending_send):
            self._retire_sends(*key)
        for works, _ in self._posted_recv.values():
            for w in works:
                self._wait(w)
        self._posted_recv.clear()


# ----------------------------------------------------------------- peer ---
@dataclass
class _Layout:
    """Byte layout of one rank's peer-visible region (identical on all ranks
    of a role, so a peer computes addresses from the base pointer)."""
    flags_bytes: int
    data_offset: int
    mb_stride: int
    slot_stride: int
    total: int


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class GemmSink:
    def __init__(self, **kw):
        self.kw = kw

    def gemm_kwargs(self):
        return self.kw

    def combine_kwargs(self):
        return self.kw


class PeerTransport(Transport):
    """Fused A2F/F2A over CUDA-IPC peer memory (one node, NVLink/NVSwitch).

    Region of an FFN rank:       flags [num_mb][n_attn] int32 | data [num_mb][max_tokens_all, H]
    Region of an attention rank: flags [num_mb][n_ffn]  int32 | data [num_mb][n_ffn][max_tokens_a, H]

    A flag for layer l of one forward holds ``epoch + l + 1 - L``; the local
    epoch advances by L at ``begin`` (a device kernel, so graph replays
    advance it too). Waits are bounded (``timeout_ms``)."""

    fused = True

    def __init__(self, ctx, hidden: int, num_layers: int, max_tokens_per_mb: int,
                 max_tokens_per_mb_attn: int, num_mb: int, device, dtype=torch.bfloat16,
                 timeout_ms: float = 10000.0):
        from .. import ops

        self.C = ops.ext()
        self.ctx = ctx
        self.H = hidden
        self.L = num_layers
        self.num_mb = num_mb
        self.device = device
        self.dtype = dtype
        self.timeout_ns = int(timeout_ms * 1e6)
        self.n_attn = len(ctx.attn_ranks())
        self.n_ffn = len(ctx.ffn_ranks())
        esz = torch.tensor([], dtype=dtype).element_size()
        self.Ta = max_tokens_per_mb_attn
        self.Tall = max_tokens_per_mb
        self.ffn_layout, self.attn_layout = self.make_layouts(
            self.n_attn, self.n_ffn, num_mb, self.Ta, self.Tall, hidden, esz)
        my_layout = self.attn_layout if ctx.role == "attention" else self.ffn_layout
        self.region = self.C.ipc_alloc(my_layout.total, device.index if device.index is not None
                                       else torch.cuda.current_device())
        self.base = self.region.data_ptr()
        self.epoch = torch.zeros(1, device=device, dtype=torch.int32)
        self.status = torch.zeros(2, device=device, dtype=torch.int32)
        self.counters = torch.zeros(num_mb, device=device, dtype=torch.int32)
        self._dropbox = torch.zeros(16, device=device, dtype=torch.int32)  # injected drops
        self._pending = None
        self.defer_waits = True
        # exchange IPC handles (collective over all ranks)
        handle = bytes(self.C.ipc_handle(self.region))
        allh: List[Optional[bytes]] = [None] * ctx.world_size
        dist.all_gather_object(allh, handle)
        self.peer_base: Dict[int, int] = {}
        others = ctx.ffn_ranks() if ctx.role == "attention" else ctx.attn_ranks()
        for r in others:
            self.peer_base[r] = int(self.C.ipc_open(allh[r]))
        torch.cuda.synchronize()
        dist.barrier(device_ids=[ctx.local_rank])

    @staticmethod
    def make_layouts(n_attn: int, n_ffn: int, num_mb: int, tokens_attn: int, tokens_all: int,
                     hidden: int, esz: int):
        """(FFN region, attention region) layouts: flags first (one int32 per
        micro-batch and peer, 4 KiB aligned), then the data slots (256-byte
        aligned): an FFN rank holds one slot per micro-batch for every
        attention rank's rows, an attention rank one slot per micro-batch and
        FFN rank."""
        fa = _align(4 * num_mb * max(n_attn, n_ffn), 4096)
        ffn_slot = _align(tokens_all * hidden * esz)
        attn_slot = _align(tokens_attn * hidden * esz)
        return (_Layout(fa, fa, ffn_slot, 0, fa + num_mb * ffn_slot),
                _Layout(fa, fa, n_ffn * attn_slot, attn_slot, fa + num_mb * n_ffn * attn_slot))

    # address helpers ----------------------------------------------------
    def _ffn_data(self, base: int, m: int) -> int:
        lay = self.ffn_layout
        return base + lay.data_offset + m * lay.mb_stride

    def _ffn_flag(self, base: int, m: int, a: int) -> int:
        return base + 4 * (m * self.n_attn + a)

    def _attn_data(self, base: int, m: int, f: int) -> int:
        lay = self.attn_layout
        return base + lay.data_offset + m * lay.mb_stride + f * lay.slot_stride

    def _attn_flag(self, base: int, m: int, f: int) -> int:
        return base + 4 * (m * self.n_ffn + f)

    def _view(self, addr: int, rows: int) -> torch.Tensor:
        off = addr - self.base
        esz = torch.tensor([], dtype=self.dtype).element_size()
        return self.region[off: off + rows * self.H * esz].view(self.dtype).view(rows, self.H)

    # lifecycle -------------------------------------------------------------
    def begin(self, plan: ForwardPlan) -> None:
        self.plan = plan
        for s in plan.ffn_slots:
            if s.tokens > self.Tall:
                raise ValueError(f"micro-batch of {s.tokens} tokens exceeds peer buffer {self.Tall}")
        for row in plan.attn_slots:
            for s in row:
                if s.tokens > self.Ta:
                    raise ValueError(f"{s.tokens} tokens exceed attention buffer {self.Ta}")
        self.C.add_i32(self.epoch, self.L)

    def _recv_wait(self, flags: List[int], value: int) -> None:
        w = ops.FlagWait(flags, value, self.status, self.timeout_ns, self.epoch)
        if self.defer_waits:
            self._pending = w
        else:
            ops.wait_flags(w)

    def take_wait(self):
        w, self._pending = self._pending, None
        return w

    def check(self) -> None:
        st = self.status.cpu()
        if int(st[0]) != 0:
            raise AFDCommTimeout(f"device wait failed: code={int(st[0])} site={int(st[1])}")

    def _common(self, l: int, m: int, flags: List[int]) -> dict:
        return dict(flags=flags, signal_value=l + 1 - self.L, done_counter=self.counters[m:m + 1],
                    epoch=self.epoch)

    # attention side --------------------------------------------------------
    def a2f_sink(self, l, m):
        a = self.ctx.attn_index
        off = self.plan.ffn_slots[m].seg_offsets[a]
        fr = self.ctx.ffn_ranks()
        flags = [self._ffn_flag(self.peer_base[f], m, a) for f in fr]
        if faults.plan().drop("a2f", l, m):
            flags = [self._dropbox.data_ptr()] * len(flags)  # raised here, seen by nobody
        kw = self._common(l, m, flags)
        kw.update(peers=[self._ffn_data(self.peer_base[f], m) for f in fr], peer_row_offset=off,
                  status=self.status)
        return GemmSink(**kw)

    def a2f_send(self, l, m, h):
        pass  # the o_proj epilogue already stored h and raised the flags

    def f2a_recv(self, l, m):
        flags = [self._attn_flag(self.base, m, f) for f in range(self.n_ffn)]
        self._recv_wait(flags, l + 1 - self.L)
        T = self.plan.slots_of(self.ctx.attn_index)[m].tokens
        return [self._view(self._attn_data(self.base, m, f), T) for f in range(self.n_ffn)]

    # FFN side ----------------------------------------------------------------
    def a2f_recv(self, l, m):
        flags = [self._ffn_flag(self.base, m, a) for a in range(self.n_attn)]
        self._recv_wait(flags, l + 1 - self.L)
        return self._view(self._ffn_data(self.base, m), self.plan.ffn_slots[m].tokens)

    def f2a_sink(self, l, m):
        f = self.ctx.ffn_index
        slot = self.plan.ffn_slots[m]
        ar = self.ctx.attn_ranks()
        flags = [self._attn_flag(self.peer_base[a], m, f) for a in ar]
        if faults.plan().drop("f2a", l, m):
            flags = [self._dropbox.data_ptr()] * len(flags)
        kw = self._common(l, m, flags)
        kw.update(peers=[self._attn_data(self.peer_base[a], m, f) for a in ar],
                  seg_offsets=list(slot.seg_offsets) + [slot.tokens], peer_row_offset=0)
        return GemmSink(**kw)

    def f2a_send(self, l, m, out):
        pass  # the combine kernel already stored the rows and raised the flags

    def close(self) -> None:
        for p in self.peer_base.values():
            self.C.ipc_close(p)
        self.peer_base.clear()
