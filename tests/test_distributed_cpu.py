"""Multi-process runs on CPU with gloo: 1 attention + 1 FFN rank,
2 attention (data parallel) + 2 FFN (expert parallel) ranks, and the uneven
splits 1 attention + 2 FFN and 2 attention + 1 FFN must generate the same greedy
tokens as the single-process model, in serial, DBO and cross-layer DBO schedules
(the tiny Qwen3-MoE oracle configuration)."""

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from afd_demo_b200.config import tiny_qwen3_moe
from afd_demo_b200.models.weights import (random_attention_weights, random_ffn_weights,
                                          save_checkpoint)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def ckpt():
    d = tempfile.mkdtemp(prefix="afd_tiny_")
    cfg = tiny_qwen3_moe()
    save_checkpoint(d, cfg, random_attention_weights(cfg, 0, "cpu", torch.float32),
                    random_ffn_weights(cfg, None, 0, "cpu", torch.float32))
    return d


def _ids():
    return torch.randint(0, 1024, (4, 24), generator=torch.Generator().manual_seed(3))


def _mask():
    # right, left and no padding across the batch (each attention rank gets a slice)
    m = torch.ones(4, 24, dtype=torch.long)
    m[1, 20:] = 0
    m[2, :6] = 0
    m[3, 15:] = 0
    return m


def _worker(rank, world, port, ckpt, modes, out_dir, n_attn=None):
    import torch

    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cpu")
    ctx = get_distributed_context()
    ctx.initialize(DistributedConfig(world_size=world, rank=rank, backend="gloo",
                                     master_addr="127.0.0.1", master_port=str(port),
                                     n_attn=n_attn, timeout_s=120))
    m = DisaggregatedQwenModel.from_pretrained(ckpt, device="cpu", dtype=torch.float32,
                                               max_seq_len=64, max_batch_size=4,
                                               comm_impl="nccl")
    res = {}
    for name, kw in modes.items():
        res[name] = m.generate(_ids(), max_new_tokens=5, do_sample=False, **kw)
    res["padded_prefill"] = m.run_forward(_ids(), "dbo", 2, reset_cache=True,
                                          attention_mask=_mask())
    # every rank gets the same agreed figures
    res["agreement"] = m.transport_agreement(_ids())
    if world == 2:
        # the reference's model.communicator, between the two roles
        m.setup_communicator(max_seq_len=8, max_batch_size=2)
        if ctx.is_attention_node:
            m.communicator.send_sync(torch.full((2, 8, m.hidden_size), 3.0), tag=5)
        else:
            got = m.communicator.recv_sync((2, 8), tag=5)
            assert got.shape == (2, 8, m.hidden_size) and bool((got == 3.0).all())
        res["generate_after_setup"] = m.generate(_ids(), max_new_tokens=5, do_sample=False,
                                                 use_decode_dbo=False)
    if ctx.is_attention_node:
        torch.save(res, os.path.join(out_dir, f"attn{ctx.attn_index}.pt"))
    ctx.barrier()
    ctx.cleanup()


MODES = {
    "serial": dict(use_decode_dbo=False),
    "dbo": dict(use_decode_dbo=True, prefill_mode="dbo", num_prefill_micro_batches=2),
    "xl": dict(use_decode_dbo=True, decode_use_crosslayer=True),
}


def _reference(ckpt):
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cpu")
    m = DisaggregatedQwenModel.from_pretrained(ckpt, device="cpu", dtype=torch.float32,
                                               max_seq_len=64, max_batch_size=4)
    toks = m.generate(_ids(), max_new_tokens=5, do_sample=False, use_decode_dbo=False)
    return toks, m.run_forward(_ids(), "serial", 1, reset_cache=True, attention_mask=_mask())


@pytest.mark.parametrize("world,n_attn", [(2, 1), (4, 2), (3, 1), (3, 2)],
                         ids=["1A1F", "2A2F", "1A2F", "2A1F"])
def test_multi_rank_matches_single_process(ckpt, world, n_attn):
    want, want_logits = _reference(ckpt)
    out = tempfile.mkdtemp(prefix="afd_out_")
    mp.start_processes(_worker, args=(world, _free_port(), ckpt, MODES, out, n_attn),
                       nprocs=world, join=True, start_method="spawn")
    for name in MODES:
        got = torch.cat([torch.load(os.path.join(out, f"attn{a}.pt"))[name]
                         for a in range(n_attn)])
        assert torch.equal(got, want), (world, name)
    # padded prefill: each attention rank applies its slice of the mask
    got = torch.cat([torch.load(os.path.join(out, f"attn{a}.pt"))["padded_prefill"]
                     for a in range(n_attn)])
    torch.testing.assert_close(got, want_logits, rtol=1e-4, atol=1e-4)
    if world == 2:  # the transport rebuilt by setup_communicator still generates the same
        got = torch.load(os.path.join(out, "attn0.pt"))["generate_after_setup"]
        assert torch.equal(got, want)
    # the transport self-check: the same transport twice is the same computation
    for a in range(n_attn):
        agreement = torch.load(os.path.join(out, f"attn{a}.pt"))["agreement"]
        assert agreement == {"max_abs_diff": 0.0, "argmax_agree": 1.0}, agreement


def test_single_process_schedules_agree(ckpt):
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cpu")
    m = DisaggregatedQwenModel.from_pretrained(ckpt, device="cpu", dtype=torch.float32,
                                               max_seq_len=64, max_batch_size=4)
    outs = {k: m.generate(_ids(), max_new_tokens=5, do_sample=False, **kw)
            for k, kw in MODES.items()}
    assert torch.equal(outs["serial"], outs["dbo"])
    assert torch.equal(outs["serial"], outs["xl"])
    with pytest.raises(ValueError, match="no transport"):
        m.transport_agreement(_ids())


def _dense_ckpt(kind: str) -> str:
    d = tempfile.mkdtemp(prefix=f"afd_{kind}_")
    cfg = tiny_qwen3_moe()
    if kind == "mixed":
        cfg.mlp_only_layers = [1]  # layer 1 is a dense MLP, layer 0 MoE
    else:  # a dense Qwen3 model: no experts at all
        cfg.num_experts, cfg.model_type = 0, "qwen3"
    save_checkpoint(d, cfg, random_attention_weights(cfg, 0, "cpu", torch.float32),
                    random_ffn_weights(cfg, None, 0, "cpu", torch.float32))
    return d


@pytest.mark.parametrize("kind", ["mixed", "dense"])
@pytest.mark.parametrize("world,n_attn", [(3, 1), (4, 2)], ids=["1A2F", "2A2F"])
def test_dense_layers_split_over_ffn_ranks(kind, world, n_attn):
    """Dense MLP layers on several FFN ranks: each rank holds a slice of the
    intermediate dimension and the attention side's sum of the partials is the
    whole MLP, so tokens equal the single-process model's."""
    d = _dense_ckpt(kind)
    want, want_logits = _reference(d)
    out = tempfile.mkdtemp(prefix="afd_out_")
    mp.start_processes(_worker, args=(world, _free_port(), d, MODES, out, n_attn),
                       nprocs=world, join=True, start_method="spawn")
    for name in MODES:
        got = torch.cat([torch.load(os.path.join(out, f"attn{a}.pt"))[name]
                         for a in range(n_attn)])
        assert torch.equal(got, want), (kind, world, name)
    got = torch.cat([torch.load(os.path.join(out, f"attn{a}.pt"))["padded_prefill"]
                     for a in range(n_attn)])
    torch.testing.assert_close(got, want_logits, rtol=1e-4, atol=1e-4)
