"""Distribution and scheduling: the distributed context (roles per rank), the
pipeline engine and the reference's scheduler classes over it, micro-batch
planning, the A2F/F2A transports (fused peer memory, NCCL, local), the
reference's buffered communicator, P2P warm-up, and host-side failure
detection and fault injection (reference: src/distributed/, src/pipeline/)."""

from .dist import (DistributedConfig, DistributedContext, config_from_env,
                   get_distributed_context, init_distributed)
from .engine import PipelineEngine
from .micro_batch import (ForwardPlan, MicroBatch, MicroBatchManager, MicroBatchState,
                          create_causal_mask, create_position_ids, make_plan, split_sizes)
from .schedulers import (AsyncPipelineScheduler, DBOStats, DecodeDBOScheduler, DecodeDBOStats,
                         SimplePipelineScheduler)
from .transport import AFDCommTimeout, LocalTransport, NcclTransport, PeerTransport

__all__ = [
    "DistributedConfig", "DistributedContext", "config_from_env", "get_distributed_context",
    "init_distributed", "PipelineEngine", "ForwardPlan", "MicroBatch", "MicroBatchManager",
    "MicroBatchState", "create_causal_mask", "create_position_ids", "make_plan", "split_sizes",
    "AsyncPipelineScheduler", "DBOStats", "DecodeDBOScheduler", "DecodeDBOStats",
    "SimplePipelineScheduler", "AFDCommTimeout", "LocalTransport", "NcclTransport",
    "PeerTransport",
]
