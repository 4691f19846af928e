"""One forward pass (a prefill or one decode step) of the disaggregated model
for the roles this process holds, over micro-batches, through a transport.

The host loop only *enqueues* work: per (layer, micro-batch) the attention
block runs on the attention stream, the FFN block on the FFN stream, and every
receive makes the consuming stream wait. The schedule decides the order and
the waits:

* ``serial``   -- per layer and micro-batch a full A->F->A round trip before
  the next micro-batch starts (reference ``SimplePipelineScheduler`` /
  ``forward_layer_sync``, src/pipeline/scheduler.py:221-236).
* ``dbo``      -- dual-batch overlap: the attention block of micro-batch m+1
  runs while the FFN works on micro-batch m. Layer-synchronous by default:
  layer l+1 starts only after every micro-batch's layer-l result is back
  (reference decode DBO without ``--crosslayer``).
* ``dbo`` + ``crosslayer`` -- micro-batch m enters layer l+1 as soon as its
  own layer-l result is back (reference ``--crosslayer``,
  src/pipeline/decode_scheduler.py:304-332).

Streams: one GPU holding both roles runs the attention blocks on one stream
and the FFN blocks on another. With the roles on separate GPUs and the fused
peer-memory transport, cross-layer DBO gives each micro-batch its own stream
on every rank (the receives are device-side flag waits, so nothing orders
the two micro-batches but the data): one micro-batch's latency-bound kernels
then run beside the other's weight-streaming GEMMs, whose grid leaves a few
SMs free for them.
"""

from __future__ import annotations

import os
import time
from typing import Dict, List, Optional

import torch

from .. import ops
from ..utils.timing import EventType, TimingTracker
from .micro_batch import ForwardPlan


# AFD_DEFER_WAITS=0: a stand-alone wait kernel per receive (A/B measurements)
_DEFER_WAITS = os.environ.get("AFD_DEFER_WAITS", "1") != "0"


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _on(stream):
    return torch.cuda.stream(stream) if stream is not None else _Null()


class PipelineEngine:
    def __init__(self, model):
        self.model = model

    def forward(self, plan: ForwardPlan, input_ids: Optional[torch.Tensor], mode: str = "dbo",
                crosslayer: bool = False, trackers: Optional[Dict[str, TimingTracker]] = None,
                last_only: bool = True, advance_cache: bool = True) -> Optional[torch.Tensor]:
        """Runs all layers. `input_ids` are this attention rank's sequences
        [B_local, q_len] (ignored on an FFN-only rank). Returns logits on
        attention ranks ([B_local, V] with `last_only`, else [B_local*q_len, V])."""
        if mode not in ("serial", "dbo"):
            raise ValueError(f"unknown schedule {mode!r}")
        m_ = self.model
        colocated = m_.ctx.is_attention_node and m_.ctx.is_ffn_node
        serial = mode == "serial"
        s_main = m_.attn_stream
        s_ffn = m_.ffn_stream if (colocated and not serial) else s_main
        mb_streams = None
        if (not serial and crosslayer and not colocated and s_main is not None
                and plan.num_mb > 1 and getattr(m_, "mb_streams_enabled", False)
                and m_.transport.fused):
            mb_streams = m_.mb_streams(plan.num_mb)
        caller = torch.cuda.current_stream() if s_main is not None else None
        every = {s_main, s_ffn} | set(mb_streams or ())
        for s in every - {None}:
            s.wait_stream(caller)
        # two streams sharing one GPU: no programmatic dependent launch (see ops.no_pdl)
        two_streams_one_gpu = colocated and not serial and s_main is not None
        try:
            with (ops.no_pdl() if two_streams_one_gpu else _Null()):
                return self._forward(plan, input_ids, serial, crosslayer, trackers or {},
                                     last_only, advance_cache, s_main, s_ffn, mb_streams)
        finally:
            for s in every - {None}:
                caller.wait_stream(s)

    def _forward(self, plan, input_ids, serial, crosslayer, trackers, last_only, advance_cache,
                 s_attn, s_ffn, mb_streams=None):
        m_ = self.model
        ctx = m_.ctx
        tr = m_.transport
        L = m_.num_layers
        ta = trackers.get("attention")
        tf = trackers.get("ffn")
        has_attn, has_ffn = ctx.is_attention_node, ctx.is_ffn_node
        colocated = has_attn and has_ffn
        with _on(s_attn):
            tr.begin(plan)
        # fold each receive's wait into the consuming kernel, except when
        # timing: then the receive wait is its own (measured) span
        # With one stream per micro-batch a receive is never folded: a folded
        # wait spins inside a kernel whose CTAs can fill the GPU, starving the
        # other micro-batch's stream -- on both ranks at once, a cycle. The
        # stand-alone wait is one CTA and releases its dependents only once
        # the flags arrive.
        if tr.fused:
            tr.defer_waits = _DEFER_WAITS and not (ta or tf) and mb_streams is None
        if has_ffn:
            m_.ffn_worker.tracker = tf

        # co-located DBO: the FFN's persistent GEMMs leave SMs to the attention
        # stream so the two micro-batches really run side by side; likewise
        # with one stream per micro-batch on separate-GPU roles
        ffn_sms = m_.colocated_ffn_sms if (colocated and not serial) else 0
        if mb_streams is not None and m_.mb_gemm_free_sms > 0:
            ffn_sms = max(1, ops.num_sms() - m_.mb_gemm_free_sms)

        def st_attn(m: int):
            return mb_streams[m] if mb_streams is not None else s_attn

        def st_ffn(m: int):
            return mb_streams[m] if mb_streams is not None else s_ffn

        def fork():
            # the per-micro-batch streams start after the role stream's work so far
            if mb_streams is not None:
                for s in mb_streams:
                    s.wait_stream(s_attn)

        def ffn_block(l: int, m: int):
            with _on(st_ffn(m)), ops.sm_budget(ffn_sms):
                if tf:
                    tf.mark_start(EventType.RECV_WAIT, l, m)
                h = tr.a2f_recv(l, m)
                wait = tr.take_wait()
                if tf:
                    tf.mark_end(EventType.RECV_WAIT, l, m)
                    tf.mark_start(EventType.FFN_COMPUTE, l, m)
                out = m_.ffn_worker.forward_ffn_layer(
                    l, h, add_residual=(ctx.ffn_index == 0), sink=tr.f2a_sink(l, m), mb_idx=m,
                    wait=wait)
                if tf:
                    tf.mark_end(EventType.FFN_COMPUTE, l, m)
                t0 = time.perf_counter()
                tr.f2a_send(l, m, out)
                if tf and not tr.fused:
                    tf.record_send(None, l, m, t0, out)

        if not has_attn:
            fork()
            for l in range(L):
                for m in range(plan.num_mb):
                    ffn_block(l, m)
            with _on(s_ffn):
                if mb_streams is not None:
                    for s in mb_streams:
                        s_ffn.wait_stream(s)
                tr.end()
            return None

        attn = m_.attention_worker
        slots = plan.slots_of(ctx.attn_index)
        cache = attn.cache
        start = cache.seq_len
        xs: Dict[int, List[torch.Tensor]] = {}
        with _on(s_attn):
            x0 = attn.embed(input_ids)
            for s in slots:
                r0 = s.batch_offset * s.q_len
                xs[s.idx] = [x0[r0:r0 + s.tokens]]
        fork()
        if mb_streams is not None:
            for s in mb_streams:
                x0.record_stream(s)
        have = {(s.idx, -1) for s in slots}  # (m, l): layer-l output of m received
        waits: Dict[int, object] = {}  # m -> wait left to the consumer of xs[m]

        def recv(l: int, m: int):
            if (m, l) in have:
                return
            if ta:
                ta.mark_start(EventType.RECV_WAIT, l, m)
            xs[m] = tr.f2a_recv(l, m)
            w = tr.take_wait()
            if w is not None:
                waits[m] = w
            if ta:
                ta.mark_end(EventType.RECV_WAIT, l, m)
            have.add((m, l))

        for l in range(L):
            if not serial and not crosslayer and l > 0:
                with _on(s_attn):
                    for s in slots:
                        recv(l - 1, s.idx)
            for s in slots:
                m = s.idx
                with _on(st_attn(m)):
                    recv(l - 1, m)
                    if ta:
                        ta.mark_start(EventType.ATTN_COMPUTE, l, m)
                    h = attn.attention_block(l, xs[m], s.batch_offset, s.q_len,
                                                     start_pos=start, sink=tr.a2f_sink(l, m),
                                                     wait=waits.pop(m, None))
                    if ta:
                        ta.mark_end(EventType.ATTN_COMPUTE, l, m)
                    t0 = time.perf_counter()
                    tr.a2f_send(l, m, h)
                    if ta and not tr.fused:
                        ta.record_send(None, l, m, t0, h)
                if colocated:
                    ffn_block(l, m)
                if serial:
                    with _on(s_attn):
                        recv(l, m)
        logits = []
        for s in slots:
            with _on(st_attn(s.idx)):
                recv(L - 1, s.idx)
                logits.append(attn.lm_head_block(xs[s.idx], s.q_len, last_only=last_only,
                                                   wait=waits.pop(s.idx, None)))
        with _on(s_attn):
            if mb_streams is not None:
                for s in mb_streams:
                    s_attn.wait_stream(s)
                for t in logits:
                    t.record_stream(s_attn)
            out = torch.cat(logits, 0) if len(logits) > 1 else logits[0]
            if advance_cache:
                cache.advance(plan.q_len)
            tr.end()
        return out
