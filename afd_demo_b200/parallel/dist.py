"""Process bootstrap: rendezvous, role map, directional groups, barrier.

Reference: ``DistributedConfig`` / ``DistributedContext``
(src/distributed/__init__.py:18-294). The reference has exactly two ranks
(attention = rank 0, FFN = rank 1). Here the role map covers one node of
1, 2, 4 or 8 GPUs:

* world 1: both roles in one process on one GPU ("colocated");
* world N > 1: ranks [0, n_attn) are attention ranks (data parallel over the
  batch), ranks [n_attn, N) are FFN ranks (expert parallel), n_attn = N // 2
  unless given.

``peer_rank`` keeps the reference's 2-rank meaning (the other role's first
rank). The process group gets a finite timeout so that a rank that died
turns the survivors' next collective into an error instead of a hang.
"""

from __future__ import annotations

import datetime
import logging
import os
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from ..config import Topology
from ..utils import device as devmod

logger = logging.getLogger(__name__)


@dataclass
class DistributedConfig:
    world_size: int = 2
    rank: int = 0
    local_rank: int = 0
    backend: str = "nccl"
    init_method: Optional[str] = None
    master_addr: str = "127.0.0.1"
    master_port: str = "29500"
    attn_node_rank: int = 0
    ffn_node_rank: int = 1
    n_attn: Optional[int] = None
    n_ffn: Optional[int] = None
    timeout_s: float = 600.0
    # host-side failure detection (heartbeats + failure key in the store)
    detect_failures: bool = False
    heartbeat_s: float = 0.2
    dead_after_s: float = 5.0


class DistributedContext:
    """Process-wide singleton (same access pattern as the reference)."""

    _instance = None

    def __new__(cls):
        if cls._instance is None:
            cls._instance = super().__new__(cls)
            cls._instance._ready = False
        return cls._instance

    def __init__(self):
        if getattr(self, "_constructed", False):
            return
        self._constructed = True
        self.config: Optional[DistributedConfig] = None
        self.topology: Optional[Topology] = None
        self._ready = False
        self._a2f_group = None
        self._f2a_group = None
        self._warmup_result = None
        self.monitor = None

    # ------------------------------------------------------------------
    def initialize(self, config: Optional[DistributedConfig] = None) -> None:
        if self._ready:
            logger.warning("distributed context already initialised")
            return
        if config is None:
            config = config_from_env()
        self.config = config
        self.topology = Topology.for_world(config.world_size, config.n_attn, config.n_ffn)
        if config.world_size == 2 and config.attn_node_rank == 1:
            # reference's swapped 2-rank layout (--attn-node-rank 1 --ffn-node-rank 0)
            self._swap = True
        else:
            self._swap = False
        devmod.set_device(config.local_rank)
        if config.world_size > 1 and not dist.is_initialized():
            os.environ["MASTER_ADDR"] = str(config.master_addr)
            os.environ["MASTER_PORT"] = str(config.master_port)
            os.environ["RANK"] = str(config.rank)
            os.environ["WORLD_SIZE"] = str(config.world_size)
            kwargs = dict(backend=config.backend, world_size=config.world_size, rank=config.rank,
                          timeout=datetime.timedelta(seconds=config.timeout_s))
            kwargs["init_method"] = config.init_method or "env://"
            if config.backend == "nccl":
                kwargs["device_id"] = torch.device(f"cuda:{config.local_rank}")
            dist.init_process_group(**kwargs)
        if config.world_size > 1 and config.detect_failures:
            from .health import PeerMonitor
            store = dist.distributed_c10d._get_default_store()
            self.monitor = PeerMonitor(store, config.rank, config.world_size,
                                       config.heartbeat_s, config.dead_after_s)
        self._ready = True
        logger.info(f"distributed ready: rank={config.rank}/{config.world_size} role={self.role} "
                    f"topology={self.topology.tag()}")

    @property
    def initialized(self) -> bool:
        return self._ready

    is_initialized = initialized  # the reference's name

    def _config_from_env(self) -> DistributedConfig:
        return config_from_env()

    # ------------------------------------------------------------------
    @property
    def rank(self) -> int:
        return self.config.rank if self.config else 0

    @property
    def world_size(self) -> int:
        return self.config.world_size if self.config else 1

    @property
    def local_rank(self) -> int:
        return self.config.local_rank if self.config else 0

    @property
    def device(self) -> torch.device:
        return devmod.device_for(self.local_rank)

    def _logical_rank(self, rank: Optional[int] = None) -> int:
        r = self.rank if rank is None else rank
        if getattr(self, "_swap", False):
            return 1 - r
        return r

    def physical_rank(self, logical: int) -> int:
        return 1 - logical if getattr(self, "_swap", False) else logical

    @property
    def role(self) -> str:
        return self.topology.role_of(self._logical_rank())

    @property
    def is_attention_node(self) -> bool:
        return self.role in ("attention", "both")

    @property
    def is_ffn_node(self) -> bool:
        return self.role in ("ffn", "both")

    @property
    def is_colocated(self) -> bool:
        return self.role == "both"

    @property
    def attn_index(self) -> int:
        return self._logical_rank() if self.role == "attention" else 0

    @property
    def ffn_index(self) -> int:
        return self.topology.ffn_index(self._logical_rank()) if self.role == "ffn" else 0

    def attn_ranks(self) -> List[int]:
        return [self.physical_rank(r) for r in self.topology.attn_ranks()]

    def ffn_ranks(self) -> List[int]:
        return [self.physical_rank(r) for r in self.topology.ffn_ranks()]

    @property
    def peer_rank(self) -> int:
        """The other role's first rank (2-rank meaning of the reference)."""
        if self.is_colocated:
            return self.rank
        return self.ffn_ranks()[0] if self.role == "attention" else self.attn_ranks()[0]

    # ------------------------------------------------------------------
    @property
    def a2f_group(self):
        if self._a2f_group is None:
            self._init_directional_groups()
        return self._a2f_group

    @property
    def f2a_group(self):
        if self._f2a_group is None:
            self._init_directional_groups()
        return self._f2a_group

    def _init_directional_groups(self) -> None:
        """Two extra communicators over all ranks: attention->FFN and
        FFN->attention traffic each keep their own FIFO, so a posted F2A
        receive never blocks an A2F send (reference
        src/distributed/__init__.py:198-215). Collective: every rank calls it."""
        if self.world_size == 1:
            return
        ranks = list(range(self.world_size))
        self._a2f_group = dist.new_group(ranks=ranks)
        self._f2a_group = dist.new_group(ranks=ranks)
        from .warmup import warmup_p2p
        warmup_p2p(self, num_rounds=2, groups=[self._a2f_group, self._f2a_group])

    def warmup(self, num_rounds: int = 3) -> dict:
        from .warmup import warmup_p2p
        extra = [g for g in (self._a2f_group, self._f2a_group) if g is not None]
        self._warmup_result = warmup_p2p(self, num_rounds=num_rounds, groups=[None] + extra)
        return self._warmup_result

    def barrier(self) -> None:
        if dist.is_initialized():
            if self.config.backend == "nccl":
                dist.barrier(device_ids=[self.local_rank])
            else:
                dist.barrier()

    def check_health(self) -> None:
        """Raise ``AFDPeerFailure`` if another rank failed (between steps)."""
        if self.monitor is not None:
            self.monitor.check()

    def report_failure(self, reason: str) -> None:
        """Tell the other ranks that this one is failing."""
        if self.monitor is not None:
            self.monitor.report(reason)

    def cleanup(self) -> None:
        """Destroy the process group (NCCL 2.28 tears down cleanly; the
        reference skips this for an NCCL 2.26 teardown crash)."""
        if self.monitor is not None:
            self.monitor.stop()
            self.monitor = None
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception as e:  # pragma: no cover
                logger.warning(f"destroy_process_group: {e}")
        self._a2f_group = self._f2a_group = None
        self._ready = False

    @classmethod
    def reset(cls) -> None:
        """Forget the singleton (tests)."""
        cls._instance = None


def config_from_env(backend: Optional[str] = None) -> DistributedConfig:
    ws = int(os.environ.get("WORLD_SIZE", 1))
    return DistributedConfig(
        world_size=ws,
        rank=int(os.environ.get("RANK", 0)),
        local_rank=int(os.environ.get("LOCAL_RANK", 0)),
        backend=backend or devmod.DIST_BACKEND,
        master_addr=os.environ.get("MASTER_ADDR", "127.0.0.1"),
        master_port=os.environ.get("MASTER_PORT", "29500"),
    )


def get_distributed_context() -> DistributedContext:
    return DistributedContext()


def init_distributed(rank: int, world_size: int, master_addr: str = "127.0.0.1",
                     master_port: str = "29500", backend: str = "nccl",
                     local_rank: Optional[int] = None, **kw) -> DistributedContext:
    cfg = DistributedConfig(world_size=world_size, rank=rank,
                            local_rank=rank if local_rank is None else local_rank,
                            backend=backend, master_addr=master_addr, master_port=master_port,
                            init_method=f"tcp://{master_addr}:{master_port}", **kw)
    ctx = get_distributed_context()
    ctx.initialize(cfg)
    return ctx
