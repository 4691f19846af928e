"""DisaggregatedQwenModel: the roles of this process, their transport, the
forward passes and autoregressive generation.

Reference: ``DisaggregatedQwenModel`` (src/model/disaggregated.py:27-829):
``from_pretrained``, ``forward``, ``forward_prefill``, ``forward_decode``,
``generate``, ``forward_layer_sync``, ``forward_layer_with_cache``,
``_make_causal_mask``. Differences by design:

* weights are read per role / per expert shard (or random-initialised on the
  device) instead of loading the full model on every rank's CPU;
* the KV cache is preallocated (``KVCache``) and written in place;
* a forward is enqueued asynchronously through ``PipelineEngine``; decode
  steps can be captured into a CUDA graph (``use_cuda_graph``) and replayed;
* ``generate`` can stream every step's tokens to pinned host memory and feed
  the next step's input back from it (``host_io``), the path a serving front
  end uses.

All attention ranks receive the *global* ``input_ids`` [B, S] and each runs
its data-parallel slice; FFN ranks only need the shape.
"""

from __future__ import annotations

import gc
import logging
import time
from typing import Any, Dict, Optional

import torch

from .. import ops
from ..config import ModelConfig, Topology, resolve_model_config
from ..parallel.dist import DistributedContext, get_distributed_context
from ..parallel import faults
from ..parallel.engine import PipelineEngine
from ..parallel.health import AFDPeerFailure
from ..parallel.micro_batch import ForwardPlan, additive_causal_mask, key_ranges_from_mask, make_plan
from ..parallel.transport import LocalTransport, NcclTransport, PeerTransport, Transport
from ..utils import device as devmod
from ..utils.sampling import sample_next_token
from .attention import AttentionWorker
from .ffn import FFNWorker
from .weights import (load_attention_weights, load_ffn_weights, random_attention_weights,
                      random_ffn_weights)

logger = logging.getLogger(__name__)


class DisaggregatedQwenModel:
    def __init__(self, config: ModelConfig, device, dtype=torch.bfloat16,
                 ctx: Optional[DistributedContext] = None):
        self.config = config
        self.device = torch.device(device)
        self.dtype = dtype
        self.ctx = ctx or get_distributed_context()
        if not self.ctx.initialized:
            from ..parallel.dist import DistributedConfig
            self.ctx.initialize(DistributedConfig(world_size=1, backend=devmod.DIST_BACKEND))
        if self.device.type == "cuda":
            # streams, CUDA graphs and the peer-memory mappings are made on the
            # current device: make it this model's (one process drives one GPU)
            if self.device.index is None:
                self.device = torch.device("cuda", torch.cuda.current_device())
            elif torch.cuda.current_device() != self.device.index:
                logger.info(f"current CUDA device set to {self.device}")
                torch.cuda.set_device(self.device)
        self.hidden_size = config.hidden_size
        self.num_layers = config.num_hidden_layers
        self.model_type = config.model_type
        self.is_moe = config.is_moe
        self.has_router = config.is_moe
        self.supports_moe_timing = config.is_moe
        self.attention_worker: Optional[AttentionWorker] = None
        self.ffn_worker: Optional[FFNWorker] = None
        self.transport: Optional[Transport] = None
        self.communicator = None  # the reference's AFDCommunicator (setup_communicator)
        self.engine = PipelineEngine(self)
        self.attn_stream = None
        self.ffn_stream = None
        self.max_batch_size = 0
        self.max_seq_len = 0
        self.num_micro_batches = 2
        self.comm_impl = "local"
        self._last_generation_metrics: Dict[str, Any] = {}
        self._last_decode_timing = None
        self._graphs: Dict[Any, Any] = {}
        # SMs left to the FFN's persistent GEMMs when both roles share a GPU
        # in a DBO schedule (0: all); AFD_COLOCATED_FFN_SMS overrides
        import os
        self.colocated_ffn_sms = int(os.environ.get("AFD_COLOCATED_FFN_SMS", "0"))
        # Separate-GPU roles under cross-layer DBO with the fused transport:
        # one stream per micro-batch on each rank, so that one micro-batch's
        # latency-bound kernels (norms, attention, MoE gate, combine, hand-offs)
        # run beside the other's weight-streaming GEMMs. The FFN GEMMs then
        # leave `mb_gemm_free_sms` SMs to the other stream's kernels.
        # AFD_MB_STREAMS=0 keeps one stream per rank (A/B measurements).
        self.mb_streams_enabled = os.environ.get("AFD_MB_STREAMS", "1") != "0"
        self.mb_gemm_free_sms = int(os.environ.get("AFD_MB_GEMM_FREE_SMS", "20"))
        self._mb_streams: list = []

    # ------------------------------------------------------------ set-up
    @property
    def kv_cache(self):
        return self.attention_worker.cache if self.attention_worker is not None else None

    @property
    def topology(self) -> Topology:
        return self.ctx.topology

    def local_batch(self, global_batch: int) -> range:
        if not self.ctx.is_attention_node or self.ctx.is_colocated:
            return range(global_batch)
        return self.topology.batch_slice(self.ctx.attn_index, global_batch)

    def load_weights(self, model_name: Optional[str], random_init: bool = False, seed: int = 0,
                     max_batch_size: int = 4, max_seq_len: int = 2048) -> None:
        cfg = self.config
        ctx = self.ctx
        dev, dt = self.device, self.dtype
        local_max_batch = len(self.local_batch(max_batch_size)) if ctx.is_attention_node else 0
        if ctx.is_attention_node:
            aw = (random_attention_weights(cfg, seed, dev, dt) if random_init
                  else load_attention_weights(model_name, cfg, dev, dt))
            self.attention_worker = AttentionWorker(cfg, aw, dev, dt, max(1, local_max_batch),
                                                    max_seq_len)
        if ctx.is_ffn_node:
            er = range(cfg.num_experts) if ctx.is_colocated else \
                self.topology.experts_of(ctx.ffn_index, cfg.num_experts)
            # dense layers: this FFN rank's slice of the intermediate dimension
            dp = (0, 1) if ctx.is_colocated else (ctx.ffn_index, self.topology.n_ffn)
            fw = (random_ffn_weights(cfg, er, seed, dev, dt, dense_part=dp) if random_init
                  else load_ffn_weights(model_name, cfg, er, dev, dt, dense_part=dp))
            self.ffn_worker = FFNWorker(cfg, fw, dev, dt)
        logger.info(f"weights ready for role {ctx.role} (experts "
                    f"{self.ffn_worker.expert_range if self.ffn_worker else '-'})")

    def setup_transport(self, comm_impl: str = "auto", max_batch_size: int = 4,
                        max_seq_len: int = 2048, num_micro_batches: int = 2,
                        crosslayer: bool = True, timeout_ms: float = 10000.0) -> None:
        """Streams and the A2F/F2A transport. ``auto`` = local when
        co-located, fused peer memory on CUDA for MoE models, NCCL otherwise
        (gloo on CPU; also on CUDA when some layer is a dense MLP)."""
        ctx = self.ctx
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.num_micro_batches = num_micro_batches
        if self.device.type == "cuda":
            self.attn_stream = torch.cuda.Stream(self.device)
            self.ffn_stream = torch.cuda.Stream(self.device) if ctx.is_colocated else self.attn_stream
        # the fused F2A store is the MoE combine's epilogue: models with dense
        # MLP layers hand off over NCCL
        dense = any(not self.config.is_sparse_layer(l) for l in range(self.num_layers))
        if ctx.is_colocated:
            comm_impl = "local"
        elif comm_impl == "auto":
            comm_impl = "fused" if self.device.type == "cuda" and not dense else "nccl"
        elif comm_impl == "fused" and dense:
            raise ValueError("the fused transport covers MoE layers only; this model has dense "
                             "MLP layers: use comm_impl 'nccl' (or 'auto')")
        self.comm_impl = comm_impl
        if comm_impl == "local":
            self.transport = LocalTransport(self.attn_stream, self.ffn_stream)
        elif comm_impl == "nccl":
            self.transport = NcclTransport(ctx, self.hidden_size, self.dtype, self.device,
                                           crosslayer=crosslayer)
        elif comm_impl == "fused":
            topo = self.topology
            per_attn = max(len(topo.batch_slice(a, max_batch_size)) for a in range(topo.n_attn))
            # largest micro-batch: a single micro-batch of the whole prefill
            max_tok_attn = per_attn * max_seq_len
            max_tok_all = max_batch_size * max_seq_len
            self.transport = PeerTransport(ctx, self.hidden_size, self.num_layers, max_tok_all,
                                           max_tok_attn, max(num_micro_batches, 1), self.device,
                                           self.dtype, timeout_ms=timeout_ms)
        else:
            raise ValueError(f"unknown comm impl {comm_impl!r}")

    def mb_streams(self, n: int) -> list:
        """One CUDA stream per micro-batch (created once, reused)."""
        while len(self._mb_streams) < n:
            self._mb_streams.append(torch.cuda.Stream(self.device))
        return self._mb_streams[:n]

    def setup_communicator(self, max_seq_len: int = 2048, max_batch_size: int = 4,
                           num_buffers: int = 2) -> None:
        """Transport set-up under the reference's name
        (src/model/disaggregated.py:117-143). With the roles on separate ranks
        it also builds ``self.communicator``: the reference's buffered
        point-to-point ``AFDCommunicator`` to the other role's first rank, for
        code that sends through it directly (this framework's forwards use the
        transport). Every rank calls it."""
        self.setup_transport("auto", max_batch_size, max_seq_len, num_buffers)
        if not self.ctx.is_colocated and self.ctx.world_size > 1:
            from ..parallel.communicator import AFDCommunicator

            self.communicator = AFDCommunicator(self.hidden_size, max_seq_len, max_batch_size,
                                                num_buffers, self.dtype)

    @classmethod
    def from_pretrained(cls, model_name: str, device=None, dtype=torch.bfloat16,
                        max_seq_len: int = 2048, max_batch_size: int = 4,
                        comm_impl: str = "auto", random_init: Optional[bool] = None,
                        seed: int = 0, num_micro_batches: int = 2,
                        timeout_ms: float = 10000.0) -> "DisaggregatedQwenModel":
        """`model_name` is a checkpoint directory or a preset name
        (``qwen3-30b-a3b``, ``tiny``, ``small``); presets without a checkpoint
        are random-initialised."""
        import os

        cfg = resolve_model_config(model_name)
        if random_init is None:
            random_init = not os.path.isdir(model_name)
        ctx = get_distributed_context()
        if not ctx.initialized:
            from ..parallel.dist import DistributedConfig
            ctx.initialize(DistributedConfig(world_size=1, backend=devmod.DIST_BACKEND))
        device = device if device is not None else ctx.device
        faults.plan().on_load()
        m = cls(cfg, device, dtype, ctx)
        m.load_weights(model_name, random_init=random_init, seed=seed,
                       max_batch_size=max_batch_size, max_seq_len=max_seq_len)
        m.setup_transport(comm_impl, max_batch_size, max_seq_len, num_micro_batches,
                          timeout_ms=timeout_ms)
        return m

    # ----------------------------------------------------------- forwards
    def plan(self, global_batch: int, q_len: int, num_micro_batches: int) -> ForwardPlan:
        return make_plan(self.topology, global_batch, num_micro_batches, q_len)

    def _local_ids(self, input_ids: torch.Tensor) -> Optional[torch.Tensor]:
        if not self.ctx.is_attention_node:
            return None
        r = self.local_batch(input_ids.shape[0])
        return input_ids[r.start:r.stop].to(self.device)

    def run_forward(self, input_ids: torch.Tensor, mode: str = "serial", num_micro_batches: int = 1,
                    crosslayer: bool = False, trackers=None, last_only: bool = True,
                    reset_cache: bool = False, attention_mask: Optional[torch.Tensor] = None
                    ) -> Optional[torch.Tensor]:
        """One forward of every layer. `attention_mask` [B, S] (1 = token, 0 =
        padding; prefill only) hides padded keys as the reference's prefill
        schedulers do; positions stay 0..S-1."""
        B, S = input_ids.shape
        plan = self.plan(B, S, num_micro_batches)
        if reset_cache and self.kv_cache is not None:
            self.kv_cache.reset(len(self.local_batch(B)))
        aw = self.attention_worker
        if attention_mask is not None and aw is not None:
            if S == 1:
                raise ValueError("attention_mask applies to prefill (seq_len > 1) only")
            r = self.local_batch(B)
            aw.key_range = key_ranges_from_mask(attention_mask[r.start:r.stop].to(self.device))
        try:
            return self.engine.forward(plan, self._local_ids(input_ids), mode=mode,
                                       crosslayer=crosslayer, trackers=trackers,
                                       last_only=last_only)
        finally:
            if aw is not None:
                aw.key_range = None

    def run_prefill_chunked(self, input_ids: torch.Tensor, chunk: int, mode: str = "serial",
                            num_micro_batches: int = 1, crosslayer: bool = False,
                            last_only: bool = True) -> Optional[torch.Tensor]:
        """Prefill in sequence chunks of `chunk` tokens, one forward per chunk
        over the same preallocated KV cache: chunk c's queries sit at positions
        c*chunk .. and attend to every key of the chunks before it (the prefill
        kernels take a cached prefix). The activations of one forward then
        scale with the chunk, not the prompt. Each chunk runs the schedule
        `mode` over the batch's micro-batches. Returns the last position's
        logits ([B_local, V], `last_only`) or every position's
        ([B_local * S, V], chunks concatenated per sequence) on attention ranks.
        Padding masks are not supported here (they apply to one-shot prefill)."""
        B, S = input_ids.shape
        if chunk <= 0:
            raise ValueError("chunk must be positive")
        outs = []
        for c0 in range(0, S, chunk):
            out = self.run_forward(input_ids[:, c0:c0 + chunk], mode, num_micro_batches,
                                   crosslayer, last_only=last_only, reset_cache=(c0 == 0))
            outs.append(out)
        if outs[-1] is None or last_only:
            return outs[-1]
        # per chunk [B_local * len, V] -> [B_local, S, V] -> [B_local * S, V]
        Bl = len(self.local_batch(B))
        parts = [o.view(Bl, -1, o.shape[-1]) for o in outs]
        return torch.cat(parts, 1).reshape(Bl * S, -1)

    def check_token_ids(self, input_ids: torch.Tensor) -> None:
        """Raises ValueError unless every id is in [0, vocab_size). The public
        entry points (generate, forward, forward_prefill) check their prompt
        once, so that a bad id fails on the host instead of in the GPU's
        embedding lookup (a device-side assert that poisons the context)."""
        if input_ids.numel() == 0:
            return
        lo, hi = int(input_ids.min()), int(input_ids.max())
        V = self.config.vocab_size
        if lo < 0 or hi >= V:
            raise ValueError(f"token ids must lie in [0, {V}); got [{lo}, {hi}]")

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None
                ) -> Optional[torch.Tensor]:
        """Full-sequence serial forward (validation path); logits for every
        position [B_local, S, V] on attention ranks."""
        B, S = input_ids.shape
        self.check_token_ids(input_ids)
        out = self.run_forward(input_ids, "serial", 1, last_only=False, reset_cache=True,
                               attention_mask=attention_mask)
        if out is None:
            return None
        return out.view(-1, S, out.shape[-1])

    @torch.no_grad()
    def forward_prefill(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                        mode: str = "serial", num_micro_batches: int = 1,
                        crosslayer: bool = False, last_only: bool = False,
                        chunk_size: Optional[int] = None) -> Optional[torch.Tensor]:
        """Prefill (resets and fills the KV cache). Logits [B_local, S, V] on
        attention ranks, as the reference's forward_prefill returns them
        (src/model/disaggregated.py:377-443); `last_only` projects only the
        last position ([B_local, V]), which is all sampling needs. The
        reference's generate always prefills serially and unsplit;
        `mode="dbo"` runs the micro-batched overlap instead. `chunk_size`
        prefills the prompt in sequence chunks (``run_prefill_chunked``)."""
        S = input_ids.shape[1]
        self.check_token_ids(input_ids)
        if chunk_size and chunk_size < S:
            if attention_mask is not None:
                raise ValueError("chunked prefill takes no padding mask")
            out = self.run_prefill_chunked(input_ids, chunk_size, mode, num_micro_batches,
                                           crosslayer, last_only=last_only)
        else:
            out = self.run_forward(input_ids, mode, num_micro_batches, crosslayer,
                                   reset_cache=True, attention_mask=attention_mask,
                                   last_only=last_only)
        if out is None or last_only:
            return out
        return out.view(-1, S, out.shape[-1])

    @torch.no_grad()
    def forward_decode(self, input_ids: torch.Tensor) -> Optional[torch.Tensor]:
        """One serial decode step for tokens [B, 1]; logits [B_local, 1, V] on
        attention ranks (the reference's shape, src/model/disaggregated.py:445-506)."""
        out = self.run_forward(input_ids, "serial", 1)
        return None if out is None else out.unsqueeze(1)

    # ------------------------------------------------ per-layer entry points
    def _one_layer(self, layer_idx: int, hidden_states: torch.Tensor, start: int,
                   attention_mask: Optional[torch.Tensor]) -> torch.Tensor:
        if not (self.ctx.is_attention_node and self.ctx.is_ffn_node):
            raise NotImplementedError(
                "per-layer calls run where both roles live (one process); across ranks the "
                "layers run inside forward / forward_prefill / generate")
        aw, fw = self.attention_worker, self.ffn_worker
        B, S, H = hidden_states.shape
        x = hidden_states.reshape(B * S, H).to(self.device, self.dtype)
        aw.key_range = (key_ranges_from_mask(attention_mask.to(self.device))
                        if attention_mask is not None and attention_mask.dim() == 2 and S > 1
                        else None)
        try:
            h = aw.attention_block(layer_idx, [x], 0, S, start_pos=start)
        finally:
            aw.key_range = None
        return fw.forward_ffn_layer(layer_idx, h, add_residual=True).view(B, S, H)

    @torch.no_grad()
    def forward_layer_sync(self, layer_idx: int, hidden_states: torch.Tensor,
                           attention_mask: Optional[torch.Tensor] = None,
                           position_ids: Optional[torch.Tensor] = None,
                           position_embeddings=None) -> torch.Tensor:
        """One layer (attention + FFN) of a whole sequence, positions 0..S-1,
        without a KV cache to continue: hidden [B, S, H] -> [B, S, H], as the
        reference's validation path (src/model/disaggregated.py:142-224). The
        layer's KV-cache rows serve as scratch; layer 0 resets the cache.
        `attention_mask` may be a [B, S] padding mask; positions are always
        0..S-1 and `position_embeddings` are computed inside the kernels, so
        both position arguments are accepted for the reference's signature
        and not needed."""
        if layer_idx == 0 or self.kv_cache.seq_len != 0:
            self.kv_cache.reset(hidden_states.shape[0])
        return self._one_layer(layer_idx, hidden_states, 0, attention_mask)

    @torch.no_grad()
    def forward_layer_with_cache(self, layer_idx: int, hidden_states: torch.Tensor,
                                 attention_mask: Optional[torch.Tensor] = None,
                                 position_ids: Optional[torch.Tensor] = None,
                                 position_embeddings=None, use_cache: bool = True
                                 ) -> torch.Tensor:
        """One layer for tokens that continue the KV cache: S prompt tokens
        (prefill; call reset_kv_cache() first) or S = 1 (decode), as the
        reference's src/model/disaggregated.py:307-375. The cache length
        advances by S after the last layer, so calling every layer in order
        is one forward step."""
        S = hidden_states.shape[1]
        out = self._one_layer(layer_idx, hidden_states, self.kv_cache.seq_len,
                              attention_mask if S > 1 else None)
        if use_cache and layer_idx == self.num_layers - 1:
            self.kv_cache.advance(S)
        return out

    def _make_causal_mask(self, batch_size: int, query_len: int, key_len: int) -> torch.Tensor:
        return additive_causal_mask(batch_size, query_len, key_len, self.device, self.dtype)

    def setup_kv_cache(self, max_batch_size: Optional[int] = None,
                       max_seq_len: Optional[int] = None) -> None:
        if self.kv_cache is not None:
            self.kv_cache.reset()

    def reset_kv_cache(self) -> None:
        self.setup_kv_cache()

    # -------------------------------------------------------- CUDA graphs
    def decode_step(self, tokens: torch.Tensor, mode: str, num_mb: int, crosslayer: bool,
                    use_cuda_graph: bool) -> Optional[torch.Tensor]:
        """One decode step; with `use_cuda_graph` the step (all layers, both
        streams, transport waits and signals, cache position update) is
        captured once per (batch, schedule) and replayed."""
        B = tokens.shape[0]
        # the NCCL baseline keeps host-side work handles: it runs eagerly
        if not use_cuda_graph or self.device.type != "cuda" or self.comm_impl == "nccl":
            return self.run_forward(tokens, mode, num_mb, crosslayer)
        key = (B, mode, num_mb, crosslayer)
        g = self._graphs.get(key)
        if g is None:
            g = _StepGraph(self, B, mode, num_mb, crosslayer)
            self._graphs[key] = g
        return g.run(tokens)

    def release_graphs(self) -> None:
        self._graphs.clear()

    def warm_up(self, input_ids: torch.Tensor, max_rounds: int = 8, **generate_kwargs) -> int:
        """Runs `generate(input_ids, **generate_kwargs)` until the CUDA caching
        allocator stops adding device segments (at most `max_rounds` calls;
        every rank runs the same number). Until then, a forward can stall on
        cudaMalloc for up to hundreds of ms; with both roles on one GPU the two
        streams hand tensors to each other, and the pool keeps growing for
        several forwards. Call it at the largest batch and prompt that will be
        served, after starting the process with
        ``PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True`` on one GPU.
        Returns the number of calls made (1 without CUDA)."""
        import torch.distributed as dist

        last = -1
        for i in range(max(1, max_rounds)):
            self.generate(input_ids, **generate_kwargs)
            if self.device.type != "cuda":
                return i + 1
            torch.cuda.synchronize(self.device)
            n = int(torch.cuda.memory_stats(self.device).get("num_device_alloc", 0))
            grew = torch.tensor([1.0 if (i < 1 or n != last) else 0.0], device=self.device)
            if self.ctx.world_size > 1 and dist.is_initialized():
                dist.all_reduce(grew, op=dist.ReduceOp.MAX)
            last = n
            if float(grew.item()) == 0.0:
                return i + 1
        return max(1, max_rounds)

    @torch.no_grad()
    def transport_agreement(self, input_ids: torch.Tensor, mode: str = "dbo",
                            num_micro_batches: int = 2, crosslayer: bool = True
                            ) -> Dict[str, float]:
        """Self-check of the A2F/F2A transport in use against NCCL
        point-to-point (the reference's mechanism; gloo on CPU): one prefill
        forward of `input_ids` from an empty cache over each, with the same
        kernels otherwise. Returns ``max_abs_diff``, the largest |difference|
        of the last-position logits, and ``argmax_agree``, the fraction of
        sequences whose greedy next token is the same, agreed over every
        rank (max and min). Every rank calls it with the same arguments; the
        cache holds the second forward's keys and values afterwards."""
        import torch.distributed as dist

        if self.ctx.is_colocated:
            raise ValueError("one process holds both roles: there is no transport to compare")
        cuda = self.device.type == "cuda"
        first = self.run_forward(input_ids, mode, num_micro_batches, crosslayer, reset_cache=True)
        if cuda:
            torch.cuda.synchronize(self.device)
        saved = (self.transport, self.comm_impl)
        self.transport = NcclTransport(self.ctx, self.hidden_size, self.dtype, self.device,
                                       crosslayer=crosslayer)
        self.comm_impl = "nccl"
        try:
            second = self.run_forward(input_ids, mode, num_micro_batches, crosslayer,
                                      reset_cache=True)
            if cuda:
                torch.cuda.synchronize(self.device)
        finally:
            self.transport, self.comm_impl = saved
        diff, agree = 0.0, 1.0
        if first is not None and first.shape[0] > 0:
            a, b = first.float(), second.float()
            diff = float((a - b).abs().max())
            agree = float((a.argmax(-1) == b.argmax(-1)).float().mean())
        t = torch.tensor([diff, -agree], dtype=torch.float64, device=self.device)
        if self.ctx.world_size > 1 and dist.is_initialized():
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return {"max_abs_diff": float(t[0]), "argmax_agree": -float(t[1])}

    # --------------------------------------------------------- generation
    def generate(self, *args, **kwargs) -> torch.Tensor:
        """See ``_generate``. A failure on this rank is published to the
        others (when failure detection is on) before it propagates.

        Python's cyclic garbage collector is paused for the call (and
        restored after): the prefill is enqueued from Python, and a full
        collection over the process's objects in the middle of it leaves the
        GPU idle for tens of milliseconds."""
        gc_on = gc.isenabled()
        gc.disable()
        try:
            return self._generate(*args, **kwargs)
        except AFDPeerFailure:
            raise
        except BaseException as e:
            self.ctx.report_failure(f"{type(e).__name__}: {e}")
            raise
        finally:
            if gc_on:
                gc.enable()

    @torch.no_grad()
    def _generate(self, input_ids: torch.Tensor, max_new_tokens: int = 50, temperature: float = 1.0,
                 top_k: int = 50, top_p: float = 0.9, do_sample: bool = True,
                 eos_token_id: Optional[int] = None, pad_token_id: Optional[int] = None,
                 use_decode_dbo: bool = True, num_decode_micro_batches: int = 2,
                 enable_timing: bool = False, timing_mode: str = "device",
                 comm_timing_mode: str = "enqueue", decode_use_crosslayer: bool = False,
                 prefill_mode: str = "serial", num_prefill_micro_batches: int = 1,
                 use_cuda_graph: bool = False, host_io: bool = False,
                 generator: Optional[torch.Generator] = None,
                 prefill_chunk_size: Optional[int] = None) -> torch.Tensor:
        """Prefill, then `max_new_tokens - 1` decode steps (the first token
        comes from the prefill logits), like the reference's generate
        (src/model/disaggregated.py:537-701). EOS does not stop the loop so
        all ranks stay in lock step.

        Returns this attention rank's sequences [B_local, S + max_new_tokens]
        (FFN-only ranks return the input). Metrics land in
        ``_last_generation_metrics``: prefill_ms, decode_loop_ms, decode_steps,
        decode_tpot_ms (device time between events on the main stream).
        `prefill_chunk_size` prefills in sequence chunks of that many tokens
        (``run_prefill_chunked``); prefill_ms then covers every chunk."""
        from ..parallel.schedulers import DecodeDBOScheduler

        B, S = input_ids.shape
        self.check_token_ids(input_ids)
        ctx = self.ctx
        is_attn = ctx.is_attention_node
        cuda = self.device.type == "cuda"
        use_dbo = use_decode_dbo and B >= num_decode_micro_batches
        dec_mode = "dbo" if use_dbo else "serial"
        dec_mb = num_decode_micro_batches if use_dbo else 1
        local = self._local_ids(input_ids) if is_attn else None
        ev = (lambda: _stamp(cuda))  # noqa: E731

        devmod.synchronize()
        ctx.barrier()
        t_pf0 = ev()
        # prefill DBO pipelines micro-batches across layers, as the reference's
        # AsyncPipelineScheduler does (src/pipeline/async_scheduler.py:281-456)
        if prefill_chunk_size and prefill_chunk_size < S:
            logits = self.run_prefill_chunked(input_ids, prefill_chunk_size, prefill_mode,
                                              num_prefill_micro_batches,
                                              crosslayer=(prefill_mode == "dbo"))
        else:
            logits = self.run_forward(input_ids, prefill_mode, num_prefill_micro_batches,
                                      crosslayer=(prefill_mode == "dbo"), reset_cache=True)
        t_pf1 = ev()
        generated = [local] if is_attn else []
        next_tok = None
        pinned = None
        if is_attn:
            next_tok = sample_next_token(logits, temperature, top_k, top_p, do_sample, generator)
            generated.append(next_tok)
            if host_io and cuda:
                pinned = torch.empty(next_tok.shape, dtype=torch.int64, pin_memory=True)
        step_in = torch.zeros(B, 1, dtype=torch.long, device=self.device)
        sched = None
        if use_dbo and enable_timing:
            sched = DecodeDBOScheduler(self, dec_mb, enable_timing=True, timing_mode=timing_mode,
                                       comm_timing_mode=comm_timing_mode,
                                       use_crosslayer=decode_use_crosslayer)
        devmod.synchronize()
        ctx.barrier()
        steps = max(max_new_tokens - 1, 0)
        t_d0 = ev()
        fault_plan = faults.plan()
        for step in range(steps):
            if fault_plan.active:
                fault_plan.before_step(ctx.rank, step)
            ctx.check_health()
            if is_attn:
                if host_io and cuda:
                    pinned.copy_(next_tok, non_blocking=True)     # D2H: the step's result
                    torch.cuda.current_stream().synchronize()
                    next_tok = pinned.to(self.device, non_blocking=True)  # H2D: next input
                r = self.local_batch(B)
                step_in[r.start:r.stop] = next_tok
            if sched is not None:  # timed runs stay eager; step 1 records events
                logits = sched.forward_decode_dbo(step_in)
            else:
                logits = self.decode_step(step_in, dec_mode, dec_mb, decode_use_crosslayer,
                                          use_cuda_graph)
            if is_attn:
                next_tok = sample_next_token(logits, temperature, top_k, top_p, do_sample,
                                             generator)
                generated.append(next_tok)
        if host_io and cuda and is_attn and steps > 0:
            pinned.copy_(next_tok, non_blocking=True)
        t_d1 = ev()
        devmod.synchronize()
        if self.transport is not None:
            self.transport.check()
        ctx.barrier()
        prefill_ms = _elapsed(t_pf0, t_pf1)
        decode_ms = _elapsed(t_d0, t_d1)
        self._last_generation_metrics = {
            "prefill_ms": prefill_ms,
            "decode_loop_ms": decode_ms,
            "decode_steps": steps,
            "decode_tpot_ms": decode_ms / steps if steps else None,
        }
        if sched is not None:
            self._last_decode_timing = sched.get_timing_data()
            if self._last_decode_timing is not None:
                for k, v in self._last_generation_metrics.items():
                    setattr(self._last_decode_timing, k, v)
        if not is_attn:
            return input_ids
        return torch.cat(generated, dim=1)


def _stamp(cuda: bool):
    if cuda:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e
    return time.perf_counter()


def _elapsed(a, b) -> float:
    if isinstance(a, float):
        return (b - a) * 1000.0
    b.synchronize()
    return a.elapsed_time(b)


class _StepGraph:
    """A captured decode step for a fixed (batch, schedule). Inputs are copied
    into a static token buffer; the cache position lives in device memory, so
    the same graph serves every step."""

    def __init__(self, model: DisaggregatedQwenModel, B: int, mode: str, num_mb: int,
                 crosslayer: bool):
        self.m = model
        self.tokens = torch.zeros(B, 1, dtype=torch.long, device=model.device)
        self.args = (mode, num_mb, crosslayer)
        cache = model.kv_cache
        # warm-up outside capture (lazy inits, kernel attributes), then rewind
        pos0 = cache.seq_len if cache is not None else 0
        s = torch.cuda.Stream(model.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            model.run_forward(self.tokens, mode, num_mb, crosslayer)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        if cache is not None:
            cache.seq_len = pos0
            cache.pos_dev.fill_(pos0)
        self.graph = torch.cuda.CUDAGraph()
        before = ops.LAUNCHES.count
        # capture_begin/end on a side stream instead of the torch.cuda.graph
        # context manager, which empties the allocator cache: the next prefill
        # would then cudaMalloc all of its buffers again
        cs = torch.cuda.Stream(model.device)
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cs):
            self.graph.capture_begin()
            try:
                self.out = model.engine.forward(model.plan(B, 1, num_mb),
                                                model._local_ids(self.tokens), mode=mode,
                                                crosslayer=crosslayer, advance_cache=False)
                if cache is not None:
                    cache.pos_dev.add_(1)
            finally:
                self.graph.capture_end()
        torch.cuda.current_stream().wait_stream(cs)
        # this package's kernels inside one replay
        self.launches = ops.LAUNCHES.count - before

    def run(self, tokens: torch.Tensor) -> Optional[torch.Tensor]:
        self.tokens.copy_(tokens)
        self.graph.replay()
        cache = self.m.kv_cache
        if cache is not None:
            cache.seq_len += 1
        return self.out
