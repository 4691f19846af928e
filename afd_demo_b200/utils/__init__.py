from . import device
from .sampling import StoppingCriteria, repetition_penalty, sample_next_token, top_k_filtering, top_p_filtering
from .timing import EventType, PipelineTiming, TimingEvent, TimingTracker, merge_timings
from .validation import compare_tensors, rel_err, validate_output

__all__ = [
    "device", "StoppingCriteria", "repetition_penalty", "sample_next_token", "top_k_filtering",
    "top_p_filtering", "EventType", "PipelineTiming", "TimingEvent", "TimingTracker",
    "merge_timings", "compare_tensors", "rel_err", "validate_output",
]
