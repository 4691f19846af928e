"""The buffered p2p communicator with the reference's interface (C4,
src/distributed/communicator.py) on two gloo ranks: async sends through a
two-buffer ring (the third send waits for the first buffer), receives of 2-D
and 3-D shapes, wait_all_recvs, blocking send/recv, and buffer-size checks.
The reference's own tests of this class (tests/test_communicator.py) need
CUDA; these run on CPU."""

import os
import socket
import tempfile

import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, out_dir):
    from afd_demo_b200.parallel.communicator import AFDCommunicator, BufferState
    from afd_demo_b200.parallel.dist import DistributedConfig, get_distributed_context
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cpu")
    ctx = get_distributed_context()
    ctx.initialize(DistributedConfig(world_size=2, rank=rank, backend="gloo",
                                     master_addr="127.0.0.1", master_port=str(port), timeout_s=60))
    H = 8
    c = AFDCommunicator(hidden_size=H, max_seq_len=4, max_batch_size=3, num_buffers=2,
                        dtype=torch.float32)
    msgs = [torch.full((2, 3, H), float(i + 1)) for i in range(3)]
    res = {}
    if rank == 0:
        idx = [c.send_async(m, tag=100 + i) for i, m in enumerate(msgs)]
        res["send_idx"] = idx
        c.wait_send()
        res["free"] = all(b.state == BufferState.FREE for b in c.send_buffers)
        c.send_sync(torch.arange(3 * 4 * H, dtype=torch.float32).view(3, 4, H), tag=7)
        try:
            c.send_async(torch.zeros(4, 4, H))
            res["too_big"] = False
        except ValueError:
            res["too_big"] = True
    else:
        got = []
        for i in range(3):
            b = c.recv_async((2, 3) if i % 2 == 0 else (2, 3, H), tag=100 + i)
            got.append(c.wait_recv(b).clone())
        res["got"] = got
        res["sync"] = c.recv_sync((3, 4), tag=7)
    c.synchronize()
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    ctx.barrier()
    ctx.cleanup()


def test_communicator_two_gloo_ranks():
    out = tempfile.mkdtemp(prefix="afd_comm_")
    mp.start_processes(_worker, args=(_free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    r0 = torch.load(os.path.join(out, "r0.pt"))
    r1 = torch.load(os.path.join(out, "r1.pt"))
    assert r0["send_idx"] == [0, 1, 0] and r0["free"] and r0["too_big"]
    for i, g in enumerate(r1["got"]):
        assert g.shape == (2, 3, 8) and torch.equal(g, torch.full((2, 3, 8), float(i + 1)))
    assert torch.equal(r1["sync"], torch.arange(3 * 4 * 8, dtype=torch.float32).view(3, 4, 8))
