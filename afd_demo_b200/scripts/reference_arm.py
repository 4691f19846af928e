"""Reference arm of ``bench.py``: the unmodified reference (afd_demo's ``src``
package, copied verbatim into ``baseline/_ref``) run through its own public
API on the same machine, metric and config as our arm.

What runs is the reference's stock code path and nothing of this package:

* ``src.distributed.DistributedContext.initialize`` (src/distributed/__init__.py:60-115)
* ``src.model.DisaggregatedQwenModel.from_pretrained`` (src/model/disaggregated.py:793-829),
  which loads the HF checkpoint with ``AutoModelForCausalLM`` on the host and
  keeps the attention or FFN half per role
* ``DisaggregatedQwenModel.generate`` with greedy decoding, prefill DBO and
  cross-layer decode DBO (src/model/disaggregated.py:540-700), whose
  ``_last_generation_metrics`` give prefill ms and decode TPOT.

The only shared piece is the input data: a random-init Qwen3-30B-A3B
checkpoint in the HF safetensors layout, written once per machine by this
package's checkpoint writer (data preparation, outside every timed region)
and reused by later runs.

Topology: the reference has exactly two ranks, one attention GPU and one FFN
GPU (src/distributed/__init__.py role map; scripts/run_single.sh:224-270).
With N = 1 GPU it cannot run (two NCCL ranks on one GPU are rejected and there
is no single-process path). With N >= 2 ranks 0 and 1 run it on their GPUs and
the other ranks stay idle; the global batch is the same as our arm's.

Timing: the reference's decode loop is bracketed by a device synchronize and a
barrier on both sides (src/model/disaggregated.py:639-682), so its host
``decode_tpot_ms`` is the synchronized wall time per step; the arm reports
the max over the two ranks.
"""

from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile
import time
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_ROOT = os.path.join(REPO, "baseline", "_ref")

METRIC = "Qwen3-30B-A3B decode TPOT ms & prefill TTFT ms, DBO vs serial, at 1/2/4/8 B200"

_CKPT_VERSION = 1


def unavailable(why: str) -> dict:
    return {"impl": "reference", "unavailable": why}


def _ref_importable() -> Optional[str]:
    """Why the reference cannot run in this environment, or None."""
    import importlib.util

    if not os.path.isdir(os.path.join(REF_ROOT, "src", "model")):
        return ("reference sources missing at baseline/_ref/src (copy the reference's src/ "
                "tree there; pip cannot install it: no setup.py or pyproject.toml)")
    for mod in ("transformers", "accelerate"):
        if importlib.util.find_spec(mod) is None:
            # src/model/disaggregated.py:88 loads with
            # AutoModelForCausalLM.from_pretrained(device_map="cpu"), which
            # transformers only allows with accelerate installed
            return (f"the reference's weight loader (src/model/disaggregated.py:88, "
                    f"AutoModelForCausalLM.from_pretrained(device_map='cpu')) needs the "
                    f"'{mod}' package, which is not installed and has no offline wheel")
    return None


def checkpoint_bytes(cfg) -> int:
    H, I, E, L = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts, cfg.num_hidden_layers
    attn = H * (cfg.q_size + 2 * cfg.kv_size) + cfg.q_size * H + 2 * cfg.head_dim + H
    ffn = E * 3 * I * H + E * H + H
    return 2 * (L * (attn + ffn) + 2 * cfg.vocab_size * H + H)


def prepare_checkpoint(path: str, cfg, seed: int, device: str, is_writer: bool,
                       timeout_s: float = 3600.0) -> Optional[str]:
    """Rank 0 writes the random checkpoint (unless a complete one is already
    there); the other participant polls for the READY marker. Returns an
    error string, or None when the checkpoint is ready."""
    marker = os.path.join(path, "READY")
    tag = json.dumps({"v": _CKPT_VERSION, "cfg": cfg.to_hf_dict(), "seed": seed}, sort_keys=True)
    if is_writer:
        if os.path.exists(marker) and open(marker).read() == tag:
            return None
        parent = os.path.dirname(os.path.abspath(path)) or "."
        os.makedirs(parent, exist_ok=True)
        need = checkpoint_bytes(cfg)
        free = shutil.disk_usage(parent).free
        if free < need * 1.05 + (1 << 30):
            return (f"no room for the {need / 1e9:.1f} GB random-init checkpoint the reference "
                    f"loads ({free / 1e9:.1f} GB free under {parent}; set AFD_REF_CKPT)")
        if os.path.exists(path):
            shutil.rmtree(path)
        from ..models.weights import write_random_checkpoint

        write_random_checkpoint(path, cfg, seed=seed, device=device)
        with open(marker, "w") as f:
            f.write(tag)
        return None
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        if os.path.exists(marker) and open(marker).read() == tag:
            return None
        time.sleep(1.0)
    return "timed out waiting for the checkpoint writer"


def _default_ckpt_dir(model: str, seed: int) -> str:
    root = os.environ.get("AFD_REF_CKPT_ROOT", tempfile.gettempdir())
    return os.environ.get("AFD_REF_CKPT", os.path.join(root, f"afd_ref_ckpt_{model}_seed{seed}"))


def run_reference(args, backend: str = "cuda") -> Optional[dict]:
    """Run the reference for bench.py's metric and config. Returns the JSON
    line on rank 0 and None elsewhere (the caller prints it)."""
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    gpus = getattr(args, "gpus", world)
    if gpus < 2 and backend == "cuda":
        return unavailable("the reference needs two ranks (1 attention GPU + 1 FFN GPU) and "
                           "has no single-GPU path; NCCL rejects two ranks on one GPU")
    err = _ref_importable()
    if err:
        return unavailable(err) if rank == 0 else None
    if rank >= 2:
        return None  # the reference's world is ranks 0 (attention) and 1 (FFN)

    import torch

    from ..config import PRESETS

    cfg = PRESETS[args.model]()
    if getattr(args, "layers", None):
        cfg.num_hidden_layers = args.layers
    seed = 0
    B = args.batch or args.batch_per_gpu * gpus
    S, T = args.seq, args.tokens
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = f"cuda:{local}" if backend == "cuda" else "cpu"
    ckpt = _default_ckpt_dir(args.model if not getattr(args, "layers", None)
                             else f"{args.model}_L{args.layers}", seed)
    err = prepare_checkpoint(ckpt, cfg, seed, dev if backend == "cuda" else "cpu",
                             is_writer=(rank == 0))
    if err:
        # the other participant learns of it by timing out on the marker
        return unavailable(err) if rank == 0 else None

    sys.path.insert(0, REF_ROOT)
    from src.distributed import DistributedConfig, get_distributed_context  # noqa: E402
    from src.model import DisaggregatedQwenModel  # noqa: E402
    from src.utils import device as refdev  # noqa: E402

    refdev.init_backend(backend)
    os.environ.pop("TORCHELASTIC_USE_AGENT_STORE", None)
    port = int(os.environ.get("MASTER_PORT", "29500")) + 17
    dcfg = DistributedConfig(rank=rank, local_rank=local if backend == "cuda" else 0,
                             world_size=2, backend=refdev.DIST_BACKEND,
                             init_method=f"tcp://127.0.0.1:{port}", master_addr="127.0.0.1",
                             master_port=str(port), attn_node_rank=0, ffn_node_rank=1)
    ctx = get_distributed_context()
    ctx.initialize(dcfg)
    device = ctx.device
    dtype = torch.bfloat16 if backend == "cuda" else torch.float32
    t_load = time.time()
    model = DisaggregatedQwenModel.from_pretrained(ckpt, device=device, dtype=dtype,
                                                   max_seq_len=S + T + args.warmup + 8,
                                                   max_batch_size=B)
    load_s = time.time() - t_load
    g = torch.Generator().manual_seed(1234)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g).to(device)

    def gen(new_tokens: int, dbo: bool, crosslayer: bool) -> dict:
        model.kv_cache = None  # a fresh cache sized for this call
        model.generate(input_ids=ids, max_new_tokens=new_tokens, do_sample=False,
                       use_decode_dbo=dbo, num_decode_micro_batches=2,
                       decode_use_crosslayer=crosslayer)
        return dict(model._last_generation_metrics)

    gen(max(args.warmup, 2) + 1, True, True)  # untimed warm-up (prefill + W decode steps)
    met_xl = gen(args.steps + 1, True, True)
    met_serial = None
    if not getattr(args, "no_serial", False):
        met_serial = gen(max(3, min(args.steps, 10)) + 1, False, False)

    vals = [met_xl["decode_tpot_ms"], met_xl["prefill_ms"],
            met_serial["decode_tpot_ms"] if met_serial else 0.0,
            met_serial["prefill_ms"] if met_serial else 0.0]
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tpot_xl, ttft_dbo, tpot_serial, ttft_serial = (float(x) for x in t.tolist())
    ctx.barrier()
    if rank != 0:
        return None
    value = 1000.0 * B / tpot_xl
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tok/s (decode, 1000*batch/TPOT)",
        "n_gpus": gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tpot_xl,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if backend == "cuda" else "fp32",
        "data": "synthetic token ids uniform in [0, vocab), random-init weights",
        "config": {"model": "Qwen3-30B-A3B" if args.model == "qwen3-30b-a3b" else args.model,
                   "global_batch": B, "seq_len": S, "decode_tokens": args.steps + 1,
                   "parallelism": "reference 1A1F (ranks 0-1; other ranks idle)",
                   "mode": "decode DBO, cross-layer, 2 micro-batches (reference generate)",
                   "l2": "inputs larger than L2 (all expert weights read every step)",
                   "timing": "reference generate metrics: synchronized host time, max over ranks"},
        "decode_tpot_ms": {"dbo_crosslayer": tpot_xl, "serial": tpot_serial or None},
        "prefill_ttft_ms": {"dbo": ttft_dbo, "serial": ttft_serial or None},
        "load_s": load_s,
    }
