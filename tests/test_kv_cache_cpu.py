"""KV cache: the DynamicCache-compatible surface against HF's DynamicCache,
and micro-batch writes at batch offsets against one full-batch write (the
reference's per-micro-batch slice + update + cat test, tests/test_pipeline.py:264-411,
including its uneven 3/2 split)."""

import pytest
import torch

from afd_demo_b200.models.kv_cache import KVCache
from afd_demo_b200.ops import torch_ref

transformers = pytest.importorskip("transformers")


def test_update_matches_dynamic_cache():
    L, B, H, D = 3, 5, 2, 8
    ours = KVCache(L, B, H, 32, D, "cpu", torch.float32)
    ref = transformers.DynamicCache()
    g = torch.Generator().manual_seed(0)
    for q in (7, 1, 1, 3):  # prefill, two decode steps, a 3-token chunk
        for l in range(L):
            k = torch.randn(B, H, q, D, generator=g)
            v = torch.randn(B, H, q, D, generator=g)
            ko, vo = ours.update(k, v, l, {"unused": True})
            kr, vr = ref.update(k, v, l)
            assert torch.equal(ko, kr) and torch.equal(vo, vr)
        assert ours.get_seq_length() == ref.get_seq_length()
        for l in range(L):
            assert torch.equal(ours.layers[l].keys, ref.layers[l].keys)
            assert torch.equal(ours.layers[l].values, ref.layers[l].values)


@pytest.mark.parametrize("split", [(5,), (3, 2), (1, 4), (2, 2, 1)])
def test_micro_batch_writes_equal_full_batch(split):
    """Micro-batches write their rows in place at their batch offset; the
    cache equals the one a single full-batch write produces, prefill and
    decode alike, with no slice or concatenation."""
    L, B, nq, nkv, D, S = 2, 5, 4, 2, 16, 12
    cs = torch_ref.rope_table(64, D, 1e6, "cpu")
    qn, kn = torch.ones(D), torch.ones(D)
    full = KVCache(L, B, nkv, 64, D, "cpu", torch.float32)
    mb = KVCache(L, B, nkv, 64, D, "cpu", torch.float32)
    g = torch.Generator().manual_seed(1)
    for q_len in (S, 1, 1):
        start = full.seq_len
        for l in range(L):
            qkv = torch.randn(B * q_len, (nq + 2 * nkv) * D, generator=g)
            kf, vf = full.layer(l)
            torch_ref.qk_norm_rope_cache(qkv, qn, kn, cs, kf, vf, 0, q_len, start, nq, nkv, 1e-6)
            km, vm = mb.layer(l)
            off = 0
            for n in split:
                rows = qkv[off * q_len:(off + n) * q_len]
                torch_ref.qk_norm_rope_cache(rows, qn, kn, cs, km, vm, off, q_len, start, nq, nkv,
                                             1e-6)
                off += n
        full.advance(q_len)
        mb.advance(q_len)
        for l in range(L):
            assert torch.equal(full.layers[l].keys, mb.layers[l].keys)
            assert torch.equal(full.layers[l].values, mb.layers[l].values)
    assert full.get_seq_length() == mb.get_seq_length() == S + 2


def test_overflow_and_capacity_checks():
    c = KVCache(1, 2, 1, 8, 4, "cpu", torch.float32)
    c.advance(8)
    with pytest.raises(ValueError):
        c.advance(1)
    with pytest.raises(ValueError):
        c.reset(3)
    c.reset(1)
    assert c.get_seq_length() == 0 and int(c.pos_dev) == 0 and c.layers[0].keys.shape[0] == 1
