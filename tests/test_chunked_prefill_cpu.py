"""Chunked prefill (one forward per sequence chunk over the same KV cache)
against one-shot prefill, on CPU with the tiny Qwen3-MoE in fp32."""

import tempfile

import pytest
import torch

from afd_demo_b200.config import tiny_qwen3_moe
from afd_demo_b200.models.weights import (random_attention_weights, random_ffn_weights,
                                          save_checkpoint)


@pytest.fixture(scope="module")
def model():
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.utils import device as devmod

    d = tempfile.mkdtemp(prefix="afd_chunk_")
    cfg = tiny_qwen3_moe()
    save_checkpoint(d, cfg, random_attention_weights(cfg, 0, "cpu", torch.float32),
                    random_ffn_weights(cfg, None, 0, "cpu", torch.float32))
    devmod.init_backend("cpu")
    return DisaggregatedQwenModel.from_pretrained(d, device="cpu", dtype=torch.float32,
                                                  max_seq_len=96, max_batch_size=4)


def _ids(S=37):
    return torch.randint(0, 1024, (4, S), generator=torch.Generator().manual_seed(11))


@pytest.mark.parametrize("chunk", [1, 8, 16, 36])
def test_chunked_prefill_logits_match(model, chunk):
    ids = _ids()
    full = model.forward_prefill(ids)                       # [B, S, V]
    got = model.forward_prefill(ids, chunk_size=chunk)
    torch.testing.assert_close(got, full, rtol=1e-4, atol=1e-4)
    last = model.forward_prefill(ids, chunk_size=chunk, last_only=True)
    torch.testing.assert_close(last, full[:, -1], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("mode,nmb", [("serial", 1), ("dbo", 2)])
def test_chunked_prefill_generate_same_tokens(model, mode, nmb):
    ids = _ids(29)
    kw = dict(max_new_tokens=6, do_sample=False, use_decode_dbo=True,
              decode_use_crosslayer=True, prefill_mode=mode, num_prefill_micro_batches=nmb)
    want = model.generate(ids, **kw)
    got = model.generate(ids, prefill_chunk_size=10, **kw)
    assert torch.equal(got, want)


def test_chunked_prefill_rejects_mask(model):
    ids = _ids(20)
    with pytest.raises(ValueError):
        model.forward_prefill(ids, attention_mask=torch.ones_like(ids), chunk_size=8)


def test_cli_flag():
    from afd_demo_b200.main import parse_args

    assert parse_args(["--prefill-chunk-size", "64"]).prefill_chunk_size == 64
    assert parse_args([]).prefill_chunk_size is None


def test_out_of_range_ids_fail_on_the_host(model):
    bad = _ids(8).clone()
    bad[1, 3] = 1024  # vocab of the tiny model is 1024
    for call in (lambda: model.generate(bad, max_new_tokens=2, do_sample=False),
                 lambda: model.forward_prefill(bad),
                 lambda: model.forward(bad)):
        with pytest.raises(ValueError, match="token ids"):
            call()
    neg = _ids(8).clone()
    neg[0, 0] = -1
    with pytest.raises(ValueError, match="token ids"):
        model.forward_prefill(neg)


def test_generate_restores_the_garbage_collector(model):
    import gc

    ids = _ids(12)
    assert gc.isenabled()
    model.generate(ids, max_new_tokens=2, do_sample=False)
    assert gc.isenabled()
    gc.disable()
    try:
        model.generate(ids, max_new_tokens=2, do_sample=False)
        assert not gc.isenabled()
    finally:
        gc.enable()


def test_warm_up_runs_generate(model):
    """On CPU there is no caching allocator to watch: one call."""
    assert model.warm_up(_ids(10), max_new_tokens=2, do_sample=False) == 1


def test_model_makes_its_cuda_device_current(monkeypatch):
    """A model on cuda:k makes device k current (its streams, graphs and
    peer mappings are made on the current device); a bare "cuda" takes the
    current device's index. CUDA calls are faked: no GPU is needed."""
    from afd_demo_b200.models import DisaggregatedQwenModel
    from afd_demo_b200.utils import device as devmod

    devmod.init_backend("cpu")
    current = {"dev": 0}
    calls = []
    monkeypatch.setattr(torch.cuda, "current_device", lambda: current["dev"])

    def set_device(d):
        calls.append(torch.device(d).index)
        current["dev"] = torch.device(d).index

    monkeypatch.setattr(torch.cuda, "set_device", set_device)
    m = DisaggregatedQwenModel(tiny_qwen3_moe(), "cuda:1")
    assert m.device == torch.device("cuda:1") and calls == [1]
    m = DisaggregatedQwenModel(tiny_qwen3_moe(), "cuda:1")  # already current: no call
    assert calls == [1]
    current["dev"] = 3
    m = DisaggregatedQwenModel(tiny_qwen3_moe(), "cuda")
    assert m.device == torch.device("cuda:3") and calls == [1]
