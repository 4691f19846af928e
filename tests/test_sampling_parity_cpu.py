"""Sampling parity with the reference's own sampling module
(src/utils/sampling.py, loaded unmodified from the reference install in
baseline/_ref): top-k and top-p filtering, repetition penalty, greedy choice,
and seeded multinomial draws give the same results."""

import importlib.util
from pathlib import Path

import pytest
import torch

from afd_demo_b200.utils import sampling as ours

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "src" / "utils" / "sampling.py"


@pytest.fixture(scope="module")
def ref():
    if not REF.exists():
        pytest.skip("the reference install (baseline/_ref) is absent")
    spec = importlib.util.spec_from_file_location("_ref_sampling", REF)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _logits(seed=0, B=4, V=1000):
    return torch.randn(B, V, generator=torch.Generator().manual_seed(seed)) * 3


@pytest.mark.parametrize("k", [1, 5, 50, 2000])
def test_top_k(ref, k):
    x = _logits(1)
    assert torch.equal(ours.top_k_filtering(x.clone(), k), ref.top_k_filtering(x.clone(), k))


@pytest.mark.parametrize("p,keep", [(0.9, 1), (0.5, 1), (0.01, 3), (0.999, 1)])
def test_top_p(ref, p, keep):
    x = _logits(2)
    assert torch.equal(ours.top_p_filtering(x.clone(), p, keep),
                       ref.top_p_filtering(x.clone(), p, keep))


def test_repetition_penalty(ref):
    x = _logits(3)
    ids = torch.randint(0, 1000, (4, 12), generator=torch.Generator().manual_seed(4))
    ids[:, 5] = ids[:, 0]  # repeated tokens are penalised once
    assert torch.allclose(ours.repetition_penalty(x.clone(), ids, 1.3),
                          ref.repetition_penalty(x.clone(), ids, 1.3))


@pytest.mark.parametrize("temperature,top_k,top_p", [(0.7, 50, 0.9), (1.0, 0, 1.0), (1.3, 10, 0.8)])
def test_seeded_sampling_and_greedy(ref, temperature, top_k, top_p):
    x = _logits(5)
    torch.manual_seed(123)
    a = ours.sample_next_token(x.clone(), temperature, top_k, top_p, do_sample=True)
    torch.manual_seed(123)
    b = ref.sample_next_token(x.clone(), temperature, top_k, top_p, do_sample=True)
    assert torch.equal(a, b)
    assert torch.equal(ours.sample_next_token(x, do_sample=False),
                       ref.sample_next_token(x, do_sample=False))


def test_stopping_criteria(ref):
    ids = torch.tensor([[5, 9, 2], [5, 9, 7], [1, 1, 2]])
    for eos in (None, 2, 7):
        for cur in (3, 9, 10, 11):
            a = ours.StoppingCriteria(10, eos).should_stop(ids, cur)
            b = ref.StoppingCriteria(10, eos).should_stop(ids, cur)
            assert torch.equal(a, b), (eos, cur)
            assert ours.StoppingCriteria(10, eos).all_stopped(ids, cur) == \
                ref.StoppingCriteria(10, eos).all_stopped(ids, cur)
