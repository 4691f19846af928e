"""Multi-GPU runs (one process per GPU) of the fused peer-memory transport
and the NCCL baseline against the single-GPU model, and the fused transport
against NCCL on the same ranks (``transport_agreement``). Skipped with fewer
than two GPUs. NVLS stays off (plain peer loads/stores only)."""

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ids(B=8, S=40):
    return torch.randint(0, 2048, (B, S), generator=torch.Generator().manual_seed(5))


def _run(rank, world, port, impl, out_dir):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cuda")
    torch.cuda.set_device(rank)
    ctx = get_distributed_context()
    ctx.initialize(DistributedConfig(world_size=world, rank=rank, local_rank=rank,
                                     backend="nccl", master_addr="127.0.0.1",
                                     master_port=str(port), timeout_s=120))
    m = DisaggregatedQwenModel.from_pretrained("mini", device=f"cuda:{rank}", max_seq_len=96,
                                               max_batch_size=8, comm_impl=impl,
                                               timeout_ms=20000)
    res = {}
    ids = _ids()
    # 320 tokens per micro-batch: the prefill-sized F2A path (combine, then bulk copy)
    res["prefill_long"] = m.run_forward(_ids(S=80), "dbo", 2, True, reset_cache=True)
    res["prefill_logits"] = m.run_forward(ids, "dbo", 2, True, reset_cache=True)
    for name, kw in {"serial": dict(use_decode_dbo=False),
                     "xl": dict(use_decode_dbo=True, decode_use_crosslayer=True,
                                prefill_mode="dbo", num_prefill_micro_batches=2),
                     "graph": dict(use_decode_dbo=True, decode_use_crosslayer=True,
                                   prefill_mode="dbo", num_prefill_micro_batches=2,
                                   use_cuda_graph=True, host_io=True)}.items():
        res[name] = m.generate(ids, max_new_tokens=6, do_sample=False, **kw)
    torch.cuda.synchronize()
    m.transport.check()
    # the fused transport against NCCL point-to-point on one prefill
    agreement = m.transport_agreement(ids) if impl == "fused" else None
    if ctx.is_attention_node:
        out = {k: v.cpu() for k, v in res.items() if v is not None}
        out["agreement"] = agreement
        torch.save(out, os.path.join(out_dir, f"{impl}_w{world}_a{ctx.attn_index}.pt"))
    m.release_graphs()
    ctx.barrier()
    ctx.cleanup()


def _single(out_dir):
    import torch

    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cuda")
    m = DisaggregatedQwenModel.from_pretrained("mini", device="cuda:0", max_seq_len=96,
                                               max_batch_size=8)
    ids = _ids()
    res = {"prefill_long": m.run_forward(_ids(S=80), "dbo", 2, True, reset_cache=True),
           "prefill_logits": m.run_forward(ids, "dbo", 2, True, reset_cache=True),
           "serial": m.generate(ids, max_new_tokens=6, do_sample=False, use_decode_dbo=False)}
    torch.save({k: v.cpu() for k, v in res.items()}, os.path.join(out_dir, "single.pt"))


def _spawn(fn, nprocs, *args):
    mp.start_processes(fn, args=args, nprocs=nprocs, join=True, start_method="spawn")


@pytest.fixture(scope="module")
def single():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs >= 2 GPUs")
    d = tempfile.mkdtemp(prefix="afd_mg_")
    _spawn(_single_entry, 1, d)
    return d, torch.load(os.path.join(d, "single.pt"))


def _single_entry(i, d):
    _single(d)


@pytest.mark.parametrize("impl", ["fused", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_matches_single(single, impl, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    d, want = single
    _spawn(_run, world, world, _free_port(), impl, d)
    n_attn = world // 2
    got = [torch.load(os.path.join(d, f"{impl}_w{world}_a{a}.pt")) for a in range(n_attn)]
    logits = torch.cat([g["prefill_logits"] for g in got]).float()
    ref = want["prefill_logits"].float()
    rel = float((logits - ref).norm() / ref.norm())
    assert rel < 2e-2, rel
    long = torch.cat([g["prefill_long"] for g in got]).float()
    ref_long = want["prefill_long"].float()
    assert float((long - ref_long).norm() / ref_long.norm()) < 2e-2
    if world == 2:  # no expert split: bitwise the single-GPU computation
        assert torch.equal(torch.cat([g["serial"] for g in got]), want["serial"])
    if impl == "fused":
        a = got[0]["agreement"]
        print(f"fused vs NCCL transport, world {world}: {a}")
        assert all(g["agreement"] == a for g in got)  # agreed over every rank
        assert a["argmax_agree"] == 1.0 and a["max_abs_diff"] < 0.25, a
    for g in got:
        # same schedule eager vs captured graph: identical kernels, identical tokens
        assert torch.equal(g["xl"], g["graph"])
        # serial vs DBO split the batch differently (attention split-KV counts
        # differ), so near-tied random-model logits may flip a rare token
        assert (g["serial"] == g["xl"]).float().mean() > 0.9
