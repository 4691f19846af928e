"""Failure detection with host-side fault injection, on CPU ranks (gloo).

Every fault is made on the host (an exception, an exit, a send that is not
made); the test checks that each surviving rank stops with an error within a
bounded time instead of hanging."""

import json
import os
import socket
import tempfile
import time

import pytest
import torch
import torch.multiprocessing as mp

from afd_demo_b200.parallel.faults import FaultPlan


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_fault_spec_parsing():
    p = FaultPlan.parse("oom, raise_rank:1:3, exit_rank:0, drop:a2f:1, drop:f2a:0:1, "
                        "delay_ms:5:1")
    assert p.oom and p.raise_at == {1: 3} and p.exit_at == {0: 0}
    assert p.drops == {("a2f", 1, 0), ("f2a", 0, 1)}
    assert p.delay_ms == 5 and p.delay_rank == 1 and p.active
    assert p.drop("a2f", 1, 0) and not p.drop("a2f", 1, 0)  # one-shot
    assert not FaultPlan.parse("").active and not FaultPlan.parse(None).active
    for bad in ("boom", "drop:x:1", "raise_rank", "delay_ms:abc"):
        with pytest.raises(ValueError):
            FaultPlan.parse(bad)
    with pytest.raises(torch.OutOfMemoryError):
        FaultPlan.parse("oom").on_load()


def _rank(rank, world, port, fault, out_dir, pg_timeout):
    import faulthandler

    # a rank still running after 60 s writes its stacks and exits
    faulthandler.dump_traceback_later(60, exit=True,
                                      file=open(os.path.join(out_dir, f"stack{rank}.txt"), "w"))
    os.environ["AFD_FAULT"] = fault
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cpu")
    ctx = get_distributed_context()
    ctx.initialize(DistributedConfig(world_size=world, rank=rank, backend="gloo",
                                     master_addr="127.0.0.1", master_port=str(port),
                                     timeout_s=pg_timeout, detect_failures=True,
                                     heartbeat_s=0.1, dead_after_s=3.0))
    m = DisaggregatedQwenModel.from_pretrained("tiny", device="cpu", dtype=torch.float32,
                                               max_seq_len=48, max_batch_size=4,
                                               comm_impl="nccl")
    ids = torch.randint(0, 1024, (4, 16), generator=torch.Generator().manual_seed(0))
    t0 = time.monotonic()
    res = {"rank": rank, "error": None}
    try:
        m.generate(ids, max_new_tokens=8, do_sample=False, use_decode_dbo=True,
                   decode_use_crosslayer=True)
    except BaseException as e:  # recorded for the test
        res["error"] = type(e).__name__
        res["message"] = str(e)[:300]
    res["seconds"] = time.monotonic() - t0
    with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
        json.dump(res, f)
    if ctx.monitor is not None:
        ctx.monitor.stop()
    os._exit(0)  # skip the process-group teardown: a peer may be gone


def _launch(world, fault, pg_timeout=20.0):
    """One spawned process per rank; each may exit on its own (no process
    is killed when another one exits)."""
    out = tempfile.mkdtemp(prefix="afd_fault_")
    port = _free_port()
    mpc = mp.get_context("spawn")
    procs = [mpc.Process(target=_rank, args=(r, world, port, fault, out, pg_timeout))
             for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + 120
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.monotonic()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "ranks did not stop"
    for r in range(world):
        path = os.path.join(out, f"stack{r}.txt")
        if os.path.getsize(path):
            raise AssertionError(f"rank {r} hung:\n" + open(path).read()[-3000:])
    res = {}
    for r in range(world):
        path = os.path.join(out, f"r{r}.json")
        res[r] = json.load(open(path)) if os.path.exists(path) else None
    return res


def test_raising_rank_stops_the_others():
    res = _launch(2, "raise_rank:1:2")
    assert res[1]["error"] == "InjectedFault"
    assert res[0]["error"] in ("AFDPeerFailure", "AFDCommTimeout", "RuntimeError"), res
    assert res[0]["seconds"] < 20, res


def test_raising_rank_stops_the_others_4_ranks():
    res = _launch(4, "raise_rank:2:1")
    assert res[2]["error"] == "InjectedFault"
    for r in (0, 1, 3):
        assert res[r]["error"] is not None, res
        assert res[r]["seconds"] < 20, res


def test_silently_exiting_rank_is_detected():
    res = _launch(2, "exit_rank:1:1")
    assert res[1] is None  # left without writing anything
    assert res[0]["error"] is not None and res[0]["seconds"] < 20, res


def test_dropped_message_times_out_instead_of_hanging():
    res = _launch(2, "drop:a2f:1:0", pg_timeout=4.0)
    assert all(res[r]["error"] is not None for r in (0, 1)), res
    assert "AFDCommTimeout" in (res[0]["error"], res[1]["error"]), res
    assert max(res[r]["seconds"] for r in (0, 1)) < 30, res


def _lonely_rank(port, out_dir, timeout_s):
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cpu")
    t0 = time.monotonic()
    res = {"error": None}
    try:
        get_distributed_context().initialize(DistributedConfig(
            world_size=2, rank=0, backend="gloo", master_addr="127.0.0.1",
            master_port=str(port), timeout_s=timeout_s))
    except BaseException as e:  # recorded for the test
        res["error"] = type(e).__name__
    res["seconds"] = time.monotonic() - t0
    with open(os.path.join(out_dir, "r0.json"), "w") as f:
        json.dump(res, f)
    os._exit(0)


def test_rank_that_never_joins_fails_the_rendezvous():
    """A peer that never starts: the lone rank's rendezvous ends with an
    error within the process-group timeout instead of waiting forever."""
    out = tempfile.mkdtemp(prefix="afd_fault_")
    p = mp.get_context("spawn").Process(target=_lonely_rank, args=(_free_port(), out, 5.0))
    p.start()
    p.join(timeout=90)
    alive = p.is_alive()
    if alive:
        p.kill()
    assert not alive, "the lone rank waited for its peer forever"
    res = json.load(open(os.path.join(out, "r0.json")))
    assert res["error"] is not None and res["seconds"] < 60, res


def test_slow_rank_is_not_reported_as_failed():
    """A rank delayed by 200 ms per step (well inside the failure bounds):
    both ranks finish without an error."""
    res = _launch(2, "delay_ms:200:1")
    assert res[0]["error"] is None and res[1]["error"] is None, res
