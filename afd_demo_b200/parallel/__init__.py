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
