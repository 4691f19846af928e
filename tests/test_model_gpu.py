"""Whole-model runs on one GPU (2-layer model of the Qwen3-30B-A3B shapes,
random weights): chunked prefill against one-shot prefill."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def model():
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cuda")
    torch.cuda.set_device(0)
    return DisaggregatedQwenModel.from_pretrained("small", device=DEV, dtype=torch.bfloat16,
                                                  max_seq_len=352, max_batch_size=4)


def _ids(B, S, seed):
    return torch.randint(0, 4096, (B, S), generator=torch.Generator().manual_seed(seed)).to(DEV)


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("chunk", [64, 100, 256])
def test_chunked_prefill_matches_one_shot(model, chunk):
    """Prompts of 300 tokens: one-shot prefill takes the prefill-sized kernels
    (600 rows: token-major o_proj), chunks of 64-256 rows the decode-sized
    ones, each chunk attending to the cached prefix."""
    ids = _ids(2, 300, 41)
    full = model.forward_prefill(ids)
    got = model.forward_prefill(ids, chunk_size=chunk)
    assert got.shape == full.shape
    assert _rel(got, full) < 3e-2
    assert _rel(got[:, -1], full[:, -1]) < 3e-2


def test_warm_up_settles_the_allocator(model):
    """warm_up repeats generate until a call adds no CUDA segment (bounded)."""
    ids = _ids(4, 64, 43)
    kw = dict(max_new_tokens=3, do_sample=False, use_decode_dbo=True,
              decode_use_crosslayer=True, prefill_mode="dbo", num_prefill_micro_batches=2)
    n = model.warm_up(ids, max_rounds=6, **kw)
    assert 1 <= n <= 6
    out = model.generate(ids, **kw)
    assert out.shape == (4, 67)
