"""Command-line entry point: ``python -m afd_demo_b200.main [flags]``.

Same flags and defaults as the reference's ``src/main.py`` (src/main.py:74-158),
the same two programs (prefill-only ``--no-generate`` and autoregressive
generation), and the same timing-JSON files under
``results/prefill_dbo/timing_{role}_{suffix}.json``. Additions:

* topology: ``--world-size`` 1 (both roles on one GPU), 2, 4 or 8 with
  ``--attn-gpus/--ffn-gpus`` (attention data-parallel, FFN expert-parallel);
  torchrun launches read RANK/LOCAL_RANK/WORLD_SIZE with ``--local-test``;
* ``--comm-impl {auto,fused,nccl}``: fused peer-memory kernels or the NCCL
  isend/irecv baseline; ``--comm-timeout-ms`` bounds every device-side wait;
* ``--synthetic`` / ``--random-init --seed``: uniform random token ids and
  random weights of the named architecture (no checkpoint or tokenizer);
* ``--cuda-graph``: capture decode steps;
* timing mode ``device`` (default): CUDA events on the streams that ran the
  work, no host synchronisation inside the loop.

On any exception the process logs it and exits 1 (OOM exits 2, the status the
experiment matrix keys on).
"""

from __future__ import annotations

import argparse
import json
import logging
import os
import sys
import time
import warnings
from typing import Optional

import torch

DEFAULT_MODEL_PATH = os.environ.get("MODEL_PATH", "qwen3-30b-a3b")

# Quiet third-party libraries as the reference's CLI does (src/main.py:27-38).
# Its default HF_ENDPOINT mirror is not set: checkpoints are read from local
# directories only, nothing is downloaded.
for _k, _v in (("TRANSFORMERS_VERBOSITY", "error"), ("HF_HUB_DISABLE_PROGRESS_BARS", "1"),
               ("HF_HUB_VERBOSITY", "error"), ("TOKENIZERS_PARALLELISM", "false")):
    os.environ.setdefault(_k, _v)
warnings.filterwarnings("ignore", category=FutureWarning)
warnings.filterwarnings("ignore", category=DeprecationWarning)


def setup_logging(verbose: bool = False) -> logging.Logger:
    level = logging.DEBUG if verbose else logging.INFO
    for name in ("transformers", "torch.distributed", "huggingface_hub", "urllib3",
                 "afd_demo_b200.parallel.warmup"):
        logging.getLogger(name).setLevel(logging.WARNING if verbose else logging.ERROR)
    logging.basicConfig(level=level,
                        format="%(asctime)s [%(levelname)s] %(message)s" if verbose else "%(message)s",
                        handlers=[logging.StreamHandler(sys.stdout)], force=True)
    return logging.getLogger("afd_demo_b200")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="AFD on B200 - attention/FFN disaggregation")
    p.add_argument("--model-name", type=str, default=DEFAULT_MODEL_PATH,
                   help="checkpoint directory or preset (qwen3-30b-a3b, small, mini, tiny)")
    p.add_argument("--role", choices=["attention", "ffn", "auto"], default="auto")
    p.add_argument("--world-size", type=int, default=int(os.environ.get("WORLD_SIZE", 2)))
    p.add_argument("--rank", type=int, default=None)
    p.add_argument("--local-rank", type=int, default=None)
    p.add_argument("--attn-node-rank", type=int, default=0)
    p.add_argument("--ffn-node-rank", type=int, default=1)
    p.add_argument("--attn-gpus", type=int, default=None, help="attention ranks (data parallel)")
    p.add_argument("--ffn-gpus", type=int, default=None, help="FFN ranks (expert parallel)")
    p.add_argument("--master-addr", type=str, default="127.0.0.1")
    p.add_argument("--master-port", type=str, default="29500")
    p.add_argument("--local-test", action="store_true",
                   help="take rank / world size from the launcher environment (torchrun)")
    p.add_argument("--batch-size", type=int, default=2)
    p.add_argument("--max-seq-len", type=int, default=128)
    p.add_argument("--prefill-seq-len", type=int, default=None)
    p.add_argument("--prefill-chunk-size", type=int, default=None,
                   help="prefill in sequence chunks of this many tokens (one forward per "
                        "chunk over the same KV cache)")
    p.add_argument("--dtype", choices=["float16", "bfloat16", "float32"], default="bfloat16")
    p.add_argument("--prompt", type=str, default="Hello, how are you today?")
    p.add_argument("--timing", action="store_true")
    p.add_argument("--timing-mode", choices=["device", "cuda_events", "sync"], default="device")
    p.add_argument("--timing-suffix", type=str, default="")
    p.add_argument("--results-dir", type=str, default="results")
    p.add_argument("--verbose", "-v", action="store_true")
    p.add_argument("--no-dbo", action="store_true")
    p.add_argument("--num-micro-batches", type=int, default=2)
    p.add_argument("--crosslayer", action="store_true")
    p.add_argument("--comm-timing-mode", choices=["enqueue", "completion"], default="enqueue")
    p.add_argument("--no-generate", action="store_true")
    p.add_argument("--max-new-tokens", type=int, default=50)
    p.add_argument("--temperature", type=float, default=0.7)
    p.add_argument("--top-k", type=int, default=50)
    p.add_argument("--top-p", type=float, default=0.9)
    p.add_argument("--greedy", action="store_true")
    p.add_argument("--warmup-p2p", action="store_true")
    p.add_argument("--warmup-rounds", type=int, default=3)
    p.add_argument("--prefill-warmup-rounds", type=int, default=None)
    p.add_argument("--backend", choices=["auto", "cuda", "cpu"], default="auto")
    p.add_argument("--comm-impl", choices=["auto", "fused", "nccl"], default="auto")
    p.add_argument("--comm-timeout-ms", type=float, default=10000.0,
                   help="bound of every device-side flag wait of the fused transport")
    p.add_argument("--pg-timeout-s", type=float, default=None,
                   help="process-group timeout (default max(60, 6 x comm timeout))")
    p.add_argument("--detect-failures", action="store_true",
                   help="heartbeats and a failure key in the rendezvous store; ranks stop "
                        "before their next step when another rank failed")
    p.add_argument("--synthetic", action="store_true",
                   help="uniform random token ids instead of a tokenised prompt")
    p.add_argument("--random-init", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--cuda-graph", action="store_true", help="capture decode steps")
    p.add_argument("--config", type=str, default=None,
                   help="YAML run configuration (flag defaults; the command line overrides)")
    return p


def load_yaml_defaults(path: str, parser: argparse.ArgumentParser) -> dict:
    """Flag defaults from a YAML run configuration: every leaf key (at any
    nesting depth) that names a CLI flag (``-`` written as ``_``) becomes
    that flag's default. Unknown keys are an error."""
    import yaml

    with open(path) as f:
        tree = yaml.safe_load(f) or {}
    known = {a.dest for a in parser._actions}
    out = {}

    def walk(node, where):
        for k, v in node.items():
            if isinstance(v, dict):
                walk(v, f"{where}{k}.")
            elif k in known:
                out[k] = v
            else:
                raise ValueError(f"{path}: unknown key {where}{k}")

    walk(tree, "")
    return out


def parse_args(argv=None):
    p = build_parser()
    pre = argparse.ArgumentParser(add_help=False)
    pre.add_argument("--config", default=None)
    known, _ = pre.parse_known_args(argv)
    if known.config:
        p.set_defaults(**load_yaml_defaults(known.config, p))
    return p.parse_args(argv)


def get_dtype(name: str) -> torch.dtype:
    return {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[name]


def get_effective_prefill_seq_len(prefill_seq_len: Optional[int], max_seq_len: int) -> int:
    return prefill_seq_len if prefill_seq_len is not None else max_seq_len


def tokenize_batch_prompts(tokenizer, prompts, prefill_seq_len: Optional[int], max_seq_len: int):
    """Fixed-length padding/truncation when an experiment seq is given, else
    dynamic padding (reference src/main.py:170-189)."""
    target = get_effective_prefill_seq_len(prefill_seq_len, max_seq_len)
    if prefill_seq_len is not None:
        inputs = tokenizer(prompts, return_tensors="pt", padding="max_length", truncation=True,
                           max_length=target)
    else:
        inputs = tokenizer(prompts, return_tensors="pt", padding=True, truncation=True,
                           max_length=target)
    return inputs, target


def build_distributed_config(args):
    from .parallel.dist import DistributedConfig
    from .utils import device as devmod

    if args.local_test:
        rank = int(os.environ.get("RANK", 0))
        local_rank = int(os.environ.get("LOCAL_RANK", 0))
        world = int(os.environ.get("WORLD_SIZE", args.world_size))
        addr = os.environ.get("MASTER_ADDR", args.master_addr)
        port = os.environ.get("MASTER_PORT", args.master_port)
    else:
        if args.role == "attention":
            rank = args.attn_node_rank
        elif args.role == "ffn":
            rank = args.ffn_node_rank
        else:
            rank = args.rank if args.rank is not None else int(os.environ.get("RANK",
                                                                              args.attn_node_rank))
        local_rank = args.local_rank if args.local_rank is not None else \
            int(os.environ.get("LOCAL_RANK", 0))
        world = args.world_size
        addr, port = args.master_addr, args.master_port
    if args.rank is not None:
        rank = args.rank
    if args.local_rank is not None:
        local_rank = args.local_rank
    return DistributedConfig(world_size=world, rank=rank, local_rank=local_rank,
                             backend=devmod.DIST_BACKEND, master_addr=addr, master_port=str(port),
                             attn_node_rank=args.attn_node_rank,
                             ffn_node_rank=args.ffn_node_rank, n_attn=args.attn_gpus,
                             n_ffn=args.ffn_gpus,
                             timeout_s=(args.pg_timeout_s if args.pg_timeout_s else
                                        max(60.0, args.comm_timeout_ms / 1000 * 6)),
                             detect_failures=args.detect_failures)


def _load_tokenizer(model_name: str, logger):
    if not os.path.isdir(model_name):
        return None
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(model_name, trust_remote_code=True)
        if tok.pad_token is None:
            tok.pad_token = tok.eos_token
        return tok
    except Exception as e:  # no tokenizer files next to the weights
        logger.info(f"no tokenizer in {model_name} ({type(e).__name__}); using synthetic ids")
        return None


def prepare_inputs(args, model, tokenizer, seq_len: int):
    """Global [B, S] ids on every rank: tokenised prompt (attention ranks
    broadcast nothing: every rank builds the same ids) or synthetic ids."""
    B = args.batch_size
    if tokenizer is not None and not args.synthetic:
        inputs, _ = tokenize_batch_prompts(tokenizer, [args.prompt] * B, args.prefill_seq_len,
                                           args.max_seq_len)
        return inputs["input_ids"], inputs.get("attention_mask")
    g = torch.Generator().manual_seed(args.seed + 1)
    return torch.randint(0, model.config.vocab_size, (B, seq_len), generator=g), None


def _timing_path(args, ctx, suffix: str) -> str:
    d = os.path.join(args.results_dir, "prefill_dbo")
    os.makedirs(d, exist_ok=True)
    role = ctx.role if not ctx.is_colocated else "attention"
    idx = ctx.attn_index if role == "attention" else ctx.ffn_index
    tag = role if idx == 0 else f"{role}{idx}"
    return os.path.join(d, f"timing_{tag}_{suffix}.json")


def _write_json(path: str, data: dict) -> None:
    with open(path, "w") as f:
        json.dump(data, f, indent=2)


def _save_pipeline_timing(args, ctx, timing, suffix, logger, **extra):
    for k, v in extra.items():
        setattr(timing, k, v)
    path = _timing_path(args, ctx, suffix)
    timing.save(path)
    logger.info(f"Timing saved: {path}")
    ffn = getattr(timing, "ffn_timing", None)
    if ctx.is_colocated and ffn is not None:
        for k, v in extra.items():
            setattr(ffn, k, v)
        fpath = path.replace("timing_attention_", "timing_ffn_")
        ffn.save(fpath)
        logger.info(f"Timing saved: {fpath}")


def _save_serial(args, ctx, data, suffix, logger):
    path = _timing_path(args, ctx, suffix)
    _write_json(path, data)
    if ctx.is_colocated:
        _write_json(path.replace("timing_attention_", "timing_ffn_"), {**data, "role": "ffn"})
    logger.info(f"Timing saved: {path}")


def _rank_max(ctx, value: float) -> float:
    import torch.distributed as dist

    if ctx.world_size == 1 or not dist.is_initialized():
        return value
    dev = ctx.device
    t = torch.tensor([value], device=dev, dtype=torch.float64 if dev.type == "cpu"
                     else torch.float32)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _setup(args):
    from .models import DisaggregatedQwenModel
    from .parallel.dist import get_distributed_context

    logger = setup_logging(args.verbose)
    ctx = get_distributed_context()
    ctx.initialize(build_distributed_config(args))
    dtype = get_dtype(args.dtype)
    logger.info(f"[{ctx.role.upper()}] rank={ctx.rank}, device={ctx.device}, dtype={dtype}, "
                f"topology={ctx.topology.tag()}")
    return logger, ctx, dtype, DisaggregatedQwenModel


def run_inference_demo(args) -> None:
    """Prefill only: serial (SimplePipelineScheduler) or DBO
    (AsyncPipelineScheduler); timing JSON as the reference writes it."""
    from .parallel.schedulers import AsyncPipelineScheduler, SimplePipelineScheduler
    from .utils import device as devmod

    logger, ctx, dtype, Model = _setup(args)
    seq = get_effective_prefill_seq_len(args.prefill_seq_len, args.max_seq_len)
    model = Model.from_pretrained(args.model_name, device=ctx.device, dtype=dtype,
                                  max_seq_len=seq, max_batch_size=args.batch_size,
                                  comm_impl=args.comm_impl, random_init=args.random_init or None,
                                  seed=args.seed, num_micro_batches=args.num_micro_batches,
                                  timeout_ms=args.comm_timeout_ms)
    logger.info(f"[{ctx.role.upper()}] model_type={model.model_type}, moe={model.is_moe}, "
                f"router={model.has_router}, comm={model.comm_impl}")
    if args.verbose:
        from .utils.profiler import print_memory_stats
        print_memory_stats()
    ctx.barrier()
    if args.warmup_p2p:
        w = ctx.warmup(num_rounds=args.warmup_rounds)
        logger.info(f"P2P warmup: cold={w['cold_latency_ms']:.3f}ms, warm={w['warm_latency_ms']:.3f}ms")
    tokenizer = _load_tokenizer(args.model_name, logger) if ctx.is_attention_node else None
    input_ids, attention_mask = prepare_inputs(args, model, tokenizer, seq)
    logger.info(f"Input shape: {tuple(input_ids.shape)}")
    use_dbo = not args.no_dbo
    if use_dbo:
        sched = AsyncPipelineScheduler(model, args.num_micro_batches, enable_timing=args.timing,
                                       timing_mode=args.timing_mode,
                                       comm_timing_mode=args.comm_timing_mode,
                                       crosslayer=True)
        name = "DBO"
    else:
        sched = SimplePipelineScheduler(model, args.num_micro_batches)
        name = "SYNC"

    def run_once():
        ctx.barrier()
        devmod.synchronize()
        t0 = time.perf_counter()
        out = sched.run(input_ids, attention_mask)
        devmod.synchronize()
        return out, time.perf_counter() - t0

    rounds = args.prefill_warmup_rounds or 0
    if rounds:
        saved = getattr(sched, "enable_timing", False)
        if hasattr(sched, "enable_timing"):
            sched.enable_timing = False
        for i in range(rounds):
            _, el = run_once()
            logger.info(f"  warmup {i + 1}/{rounds}: {el * 1000:.1f} ms")
        if hasattr(sched, "enable_timing"):
            sched.enable_timing = saved
    output, elapsed = run_once()
    elapsed_max = _rank_max(ctx, elapsed * 1000)
    if ctx.is_attention_node:
        logger.info(f"[{name}] prefill_time={elapsed * 1000:.2f}ms (max over ranks "
                    f"{elapsed_max:.2f}ms)")
        if use_dbo:
            logger.info(f"[DBO] {sched.get_stats()}")
    suffix = args.timing_suffix or (f"b{args.batch_size}_t{args.max_new_tokens}" if use_dbo else
                                    f"serial_b{args.batch_size}_t{args.max_new_tokens}")
    if args.timing and use_dbo:
        td = sched.get_timing_data()
        if td is not None:
            _save_pipeline_timing(args, ctx, td, suffix, logger, prefill_seq_len=seq,
                                  actual_prompt_len=int(input_ids.shape[1]),
                                  rank_max_ms=elapsed_max)
            if ctx.is_attention_node:
                logger.info(td.summary())
    elif args.timing:
        _save_serial(args, ctx, {
            "mode": "serial", "role": ctx.role if not ctx.is_colocated else "attention",
            "total_time_ms": elapsed * 1000, "batch_size": args.batch_size,
            "prefill_seq_len": seq, "actual_prompt_len": int(input_ids.shape[1]),
            "max_new_tokens": args.max_new_tokens, "device_timed": False,
            "rank_max_ms": elapsed_max, "gpus": ctx.world_size,
            "topology": ctx.topology.tag()}, suffix, logger)
    if ctx.is_attention_node and output is not None:
        pred = output.argmax(-1)
        for i in range(min(len(pred), 2)):
            tok = tokenizer.decode(pred[i]) if tokenizer is not None else int(pred[i])
            logger.info(f"Output[{i}]: next token -> {tok!r}")
    ctx.barrier()
    ctx.cleanup()


def run_generation_demo(args) -> None:
    """Prefill + decode loop; serial or decode DBO (optionally cross-layer)."""
    from .utils import device as devmod

    logger, ctx, dtype, Model = _setup(args)
    seq = get_effective_prefill_seq_len(args.prefill_seq_len, args.max_seq_len)
    model = Model.from_pretrained(args.model_name, device=ctx.device, dtype=dtype,
                                  max_seq_len=seq + args.max_new_tokens,
                                  max_batch_size=args.batch_size, comm_impl=args.comm_impl,
                                  random_init=args.random_init or None, seed=args.seed,
                                  num_micro_batches=args.num_micro_batches,
                                  timeout_ms=args.comm_timeout_ms)
    if args.verbose:
        from .utils.profiler import print_memory_stats
        print_memory_stats()
    ctx.barrier()
    if args.warmup_p2p:
        w = ctx.warmup(num_rounds=args.warmup_rounds)
        logger.info(f"P2P warmup: cold={w['cold_latency_ms']:.3f}ms, warm={w['warm_latency_ms']:.3f}ms")
    tokenizer = _load_tokenizer(args.model_name, logger) if ctx.is_attention_node else None
    input_ids, _ = prepare_inputs(args, model, tokenizer, seq)
    B, prompt_len = input_ids.shape
    use_dbo = not args.no_dbo
    logger.info(f"Starting generation... (DBO: {use_dbo}, crosslayer: {args.crosslayer})")
    devmod.synchronize()
    t0 = time.perf_counter()
    out = model.generate(input_ids, max_new_tokens=args.max_new_tokens,
                         temperature=args.temperature, top_k=args.top_k, top_p=args.top_p,
                         do_sample=not args.greedy,
                         eos_token_id=tokenizer.eos_token_id if tokenizer else None,
                         pad_token_id=tokenizer.pad_token_id if tokenizer else None,
                         use_decode_dbo=use_dbo, num_decode_micro_batches=args.num_micro_batches,
                         enable_timing=args.timing, timing_mode=args.timing_mode,
                         comm_timing_mode=args.comm_timing_mode,
                         decode_use_crosslayer=args.crosslayer, use_cuda_graph=args.cuda_graph,
                         prefill_chunk_size=args.prefill_chunk_size)
    devmod.synchronize()
    gen_time = time.perf_counter() - t0
    met = dict(model._last_generation_metrics)
    tpot_max = _rank_max(ctx, met.get("decode_tpot_ms") or 0.0)
    num_generated = out.shape[1] - prompt_len if ctx.is_attention_node else 0
    if ctx.is_attention_node:
        logger.info(f"Generated {num_generated} tokens in {gen_time * 1000:.2f}ms")
        if tokenizer is not None:
            logger.info(f"\n=== Generated Text ===\n{tokenizer.decode(out[0], skip_special_tokens=True)}")
        else:
            logger.info(f"Generated ids[0]: {out[0, prompt_len:].tolist()}")
        fmt = lambda v: "N/A" if v is None else f"{v:.3f}ms"  # noqa: E731
        logger.info(f"Generation timing: prefill={fmt(met.get('prefill_ms'))}, "
                    f"decode_loop={fmt(met.get('decode_loop_ms'))}, "
                    f"decode_steps={met.get('decode_steps')}, "
                    f"decode_tpot={fmt(met.get('decode_tpot_ms'))} (max over ranks "
                    f"{tpot_max:.3f}ms, {1000 * B / tpot_max if tpot_max else 0:.1f} tok/s)")
    td = model._last_decode_timing
    if args.timing and td is not None:
        suffix = args.timing_suffix or f"decode_b{args.batch_size}_t{args.max_new_tokens}"
        _save_pipeline_timing(args, ctx, td, suffix, logger, prefill_seq_len=seq,
                              actual_prompt_len=prompt_len, rank_max_ms=tpot_max,
                              **{k: met.get(k) for k in ("prefill_ms", "decode_loop_ms",
                                                         "decode_steps", "decode_tpot_ms")})
    elif args.timing:
        suffix = args.timing_suffix or f"decode_serial_b{args.batch_size}_t{args.max_new_tokens}"
        _save_serial(args, ctx, {
            "mode": "serial", "role": ctx.role if not ctx.is_colocated else "attention",
            "total_time_ms": gen_time * 1000, "prefill_ms": met.get("prefill_ms"),
            "decode_loop_ms": met.get("decode_loop_ms"), "decode_steps": met.get("decode_steps"),
            "decode_tpot_ms": met.get("decode_tpot_ms"), "batch_size": args.batch_size,
            "prefill_seq_len": seq, "actual_prompt_len": prompt_len,
            "max_new_tokens": args.max_new_tokens,
            "tokens_per_sec": (num_generated / gen_time) if num_generated else 0,
            "device_timed": True, "rank_max_ms": tpot_max, "gpus": ctx.world_size,
            "topology": ctx.topology.tag()}, suffix, logger)
    model.release_graphs()
    ctx.barrier()
    ctx.cleanup()


def main(argv=None) -> int:
    warnings.filterwarnings("ignore", category=UserWarning)
    args = parse_args(argv)
    from .utils import device as devmod

    devmod.init_backend(args.backend)
    devmod.apply_backend_envs()
    try:
        if args.no_generate:
            run_inference_demo(args)
        else:
            run_generation_demo(args)
    except torch.cuda.OutOfMemoryError as e:
        logging.error(f"OutOfMemoryError: {e}")
        _report(f"OutOfMemoryError: {e}")
        return 2
    except Exception as e:
        logging.error(f"Error: {e}", exc_info=True)
        _report(f"{type(e).__name__}: {e}")
        return 1
    return 0


def _report(reason: str) -> None:
    from .parallel.dist import get_distributed_context

    ctx = get_distributed_context()
    if ctx.initialized:
        ctx.report_failure(reason)


if __name__ == "__main__":
    sys.exit(main())
