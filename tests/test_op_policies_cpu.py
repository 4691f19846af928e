"""Kernel-choice rules of the op layer (no GPU): which GEMM kernel, token
block and split each call gets, and the decode attention's key splits."""

import pytest

from afd_demo_b200 import ops


@pytest.fixture
def sms(monkeypatch):
    monkeypatch.setattr(ops, "_NUM_SMS", 148)
    return 148


@pytest.mark.parametrize("T", [1, 16, 32, 64, 128, 200, 256])
@pytest.mark.parametrize("N,K", [(5120, 2048), (2048, 4096), (128, 2048)])
def test_decode_tiling_is_valid(sms, T, N, K):
    bn, s = ops._decode_tiling(T, N, K)
    assert bn in (64, 128, 256)
    k_iters = K // 64
    assert s >= 1 and k_iters % s == 0 and k_iters // s >= 8
    tiles = ((T + bn - 1) // bn) * (N // 128)
    if tiles >= 40:
        assert s <= 2  # many tiles: at most one halving of K


def test_decode_tiling_matches_the_sweep(sms):
    # the starred choices of the qkv / o_proj sweep on B200
    assert ops._decode_tiling(16, 5120, 2048) == (64, 1)
    assert ops._decode_tiling(256, 5120, 2048) == (128, 1)
    assert ops._decode_tiling(16, 2048, 4096) == (64, 8)
    assert ops._decode_tiling(128, 2048, 4096) == (64, 4)
    assert ops._decode_tiling(256, 2048, 4096) == (64, 2)


def test_dense_token_major_rule(monkeypatch):
    monkeypatch.setattr(ops, "_DENSE_TM", "residual")
    assert ops._dense_token_major(8192, 2048, True)        # o_proj
    assert not ops._dense_token_major(8192, 5120, False)   # qkv stays swap-AB
    assert not ops._dense_token_major(256, 2048, True)     # decode sizes
    assert not ops._dense_token_major(8192, 128, True)     # router width
    monkeypatch.setattr(ops, "_DENSE_TM", "all")
    assert ops._dense_token_major(8192, 5120, False)
    monkeypatch.setattr(ops, "_DENSE_TM", "none")
    assert not ops._dense_token_major(8192, 2048, True)


def test_moe_token_major_rule(monkeypatch):
    monkeypatch.setattr(ops, "_MOE_TM", True)
    # 8192 tokens x top-8 over 128 experts = 512 rows per expert
    assert ops._moe_token_major(128, True, 8192, 8, 128)
    assert ops._moe_token_major(128, True, 1536, 8, 128)       # exactly 96 per expert
    assert not ops._moe_token_major(128, True, 1024, 8, 128)   # 64 per expert
    assert not ops._moe_token_major(64, True, 8192, 8, 128)    # decode blocks
    assert not ops._moe_token_major(128, False, 8192, 8, 128)  # gather4 rows
    monkeypatch.setattr(ops, "_MOE_TM", False)
    assert not ops._moe_token_major(128, True, 8192, 8, 128)


@pytest.mark.parametrize("rows,want", [(1, 64), (256, 64), (257, 128), (2047, 128)])
def test_moe_block_n(rows, want):
    assert ops._moe_block_n(rows) == want


@pytest.mark.parametrize("B", [1, 16, 64, 256])
@pytest.mark.parametrize("kv", [1, 128, 276, 2048, 4096])
def test_decode_splits_bounds(B, kv):
    s = ops.decode_splits(B, 4, kv, sms=148)
    tiles = max(1, (kv + 127) // 128)
    assert 1 <= s <= min(tiles, 16)
    if B * 4 >= 148:
        assert s == 1  # every SM already has a (sequence, kv head) pair
