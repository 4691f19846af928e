"""Debug-mode bounds checks (AFD_BOUNDS_CHECK=1): the routing-table validator
accepts every valid table (any row order inside an expert, as the routing
kernels' atomics produce) and names each kind of corruption."""

import pytest
import torch

from afd_demo_b200.ops.checks import AFDBoundsError, check_routing_tables


def _tables(T=13, k=4, E=16, start=4, n_local=8, block_n=3, seed=0):
    """A valid routing result built the slow way, rows shuffled inside each
    expert."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    w = w / w.sum(-1, keepdim=True)
    flat = ids.reshape(-1).long()
    local = flat - start
    counts = torch.zeros(n_local, dtype=torch.int64)
    for e in local:
        if 0 <= e < n_local:
            counts[e] += 1
    offs = torch.cat([torch.zeros(1, dtype=torch.int64), counts.cumsum(0)])
    n_rows = int(offs[-1])
    inv = torch.full((T * k,), -1, dtype=torch.int32)
    row_token = torch.zeros(T * k, dtype=torch.int32)
    row_weight = torch.zeros(T * k)
    for e in range(n_local):
        members = (local == e).nonzero().reshape(-1)
        perm = members[torch.randperm(members.numel(), generator=g)]
        for slot, i in enumerate(perm.tolist()):
            r = int(offs[e]) + slot
            inv[i] = r
            row_token[r] = i // k
            row_weight[r] = w.reshape(-1)[i]
    blocks = []
    for e in range(n_local):
        for r in range(int(offs[e]), int(offs[e + 1]), block_n):
            blocks.append([r, min(block_n, int(offs[e + 1]) - r), e, 0])
    blk = torch.zeros(n_local + (T * k + block_n - 1) // block_n, 4, dtype=torch.int32)
    if blocks:
        blk[:len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
    return dict(ids=ids, weights=w, expert_start=start, n_local=n_local, block_n=block_n,
                inv=inv, row_token=row_token, row_weight=row_weight,
                expert_offsets=offs.to(torch.int32), blocks=blk,
                num_blocks=torch.tensor([len(blocks)], dtype=torch.int32),
                num_rows=torch.tensor([n_rows], dtype=torch.int32))


@pytest.mark.parametrize("seed", range(4))
def test_valid_tables_pass(seed):
    check_routing_tables(**_tables(seed=seed))
    check_routing_tables(**_tables(T=1, k=8, E=128, start=0, n_local=128, block_n=64, seed=seed))


def _corrupt(name, fn, match):
    t = _tables(seed=7)
    fn(t)
    with pytest.raises(AFDBoundsError, match=match):
        check_routing_tables(**t)


def test_each_corruption_is_named():
    def first_local(t):
        return int((t["inv"] >= 0).nonzero()[0])

    _corrupt("rows", lambda t: t["num_rows"].add_(1), "num_rows")
    _corrupt("offsets", lambda t: t["expert_offsets"].__setitem__(2, t["expert_offsets"][2] + 1),
             "expert_offsets")

    def inv_nonlocal(t):
        j = int((t["inv"] < 0).nonzero()[0])
        t["inv"][j] = 0
    _corrupt("inv -1", inv_nonlocal, "non-local")

    def inv_range(t):
        t["inv"][first_local(t)] = 10_000
    _corrupt("inv range", inv_range, "outside expert")

    def dup(t):
        li = (t["inv"] >= 0).nonzero().reshape(-1)
        # two entries of the same expert share a row
        e = (t["ids"].reshape(-1)[li] - t["expert_start"])
        for a in range(len(li)):
            for b in range(a + 1, len(li)):
                if e[a] == e[b]:
                    t["inv"][li[b]] = t["inv"][li[a]]
                    return
    _corrupt("dup", dup, "share a row")

    def tok(t):
        r = int(t["inv"][first_local(t)])
        t["row_token"][r] += 1
    _corrupt("token", tok, "row_token")

    def wgt(t):
        r = int(t["inv"][first_local(t)])
        t["row_weight"][r] += 0.5
    _corrupt("weight", wgt, "row_weight")

    _corrupt("blk rows", lambda t: t["blocks"].__setitem__((0, 1), t["block_n"] + 1), "rows")
    _corrupt("blk expert", lambda t: t["blocks"].__setitem__((0, 2), 99), "expert 99")
    _corrupt("blk count", lambda t: t["num_blocks"].sub_(1), "cover")
    _corrupt("blk overflow", lambda t: t["num_blocks"].fill_(10_000), "exceeds")
