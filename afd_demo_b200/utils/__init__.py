"""Helpers with the reference's names: device selection, timers and the
profiler, sampling, the timing tracker and its JSON schema, and output
validation (reference: src/utils/)."""

from . import device
from .profiler import CUDATimer, Timer, profile_function
from .sampling import StoppingCriteria, repetition_penalty, sample_next_token, top_k_filtering, top_p_filtering
from .timing import EventType, PipelineTiming, TimingEvent, TimingTracker, merge_timings
from .validation import compare_tensors, rel_err, validate_output

__all__ = [
    "device", "CUDATimer", "Timer", "profile_function", "StoppingCriteria", "repetition_penalty", "sample_next_token", "top_k_filtering",
    "top_p_filtering", "EventType", "PipelineTiming", "TimingEvent", "TimingTracker",
    "merge_timings", "compare_tensors", "rel_err", "validate_output",
]
