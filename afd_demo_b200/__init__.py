"""afd_demo_b200: attention/FFN-disaggregated Qwen3-MoE inference with
dual-batch overlap, built for NVIDIA B200 (sm_100a).

Layers (bottom up): ``utils`` (device backend, timing, sampling), ``ops``
(sm_100a kernels with PyTorch statements for the CPU path), ``models``
(weights, KV cache, attention and FFN roles, the disaggregated model),
``parallel`` (bootstrap, micro-batches, transports, engine, schedulers),
``main`` (CLI) and ``scripts`` (experiment drivers and reports).
"""

__version__ = "0.1.0"
