"""Schedule order of the real pipeline engine (the reference simulates its
schedulers' ordering with a fake clock, tests/test_pipeline.py:114-257; here
the engine itself runs on CPU and every transport call is recorded).

Attention side, per layer l and micro-batch m (a2f = send of layer l's
attention output, f2a = receive of layer l's FFN output):
* serial: a2f(l, m) then f2a(l, m) before the next micro-batch starts;
* DBO: all f2a(l-1, *) are received before any a2f(l, *) is sent;
* cross-layer DBO: f2a(l-1, m) is received right before a2f(l, m), so
  micro-batch 0 of layer l runs while micro-batch 1 of layer l-1 is still in
  the FFN.
The FFN side consumes a2f(l, m) in send order and answers each with f2a(l, m)."""

import pytest
import torch

from afd_demo_b200.config import tiny_qwen3_moe
from afd_demo_b200.models import DisaggregatedQwenModel
from afd_demo_b200.models.weights import (random_attention_weights, random_ffn_weights,
                                          save_checkpoint)


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("ckpt"))
    cfg = tiny_qwen3_moe()
    save_checkpoint(d, cfg, random_attention_weights(cfg, 0, "cpu", torch.float32),
                    random_ffn_weights(cfg, None, 0, "cpu", torch.float32))
    return DisaggregatedQwenModel.from_pretrained(d, device="cpu", dtype=torch.float32,
                                                  max_seq_len=64, max_batch_size=4)


def _record(model, fn):
    tr = model.transport
    log = []
    orig = {k: getattr(tr, k) for k in ("a2f_send", "f2a_recv", "a2f_recv", "f2a_send")}

    def wrap(name):
        def call(l, m, *a):
            log.append((name, l, m))
            return orig[name](l, m, *a)
        return call

    for k in orig:
        setattr(tr, k, wrap(k))
    try:
        fn()
    finally:
        for k in orig:
            delattr(tr, k)
    return log


def _attn(log):
    return [(n, l, m) for n, l, m in log if n in ("a2f_send", "f2a_recv")]


@pytest.mark.parametrize("mode,nmb,xl", [("serial", 2, False), ("dbo", 2, False),
                                         ("dbo", 2, True)])
def test_engine_order(model, mode, nmb, xl):
    L = model.num_layers
    ids = torch.randint(0, 1024, (4, 9), generator=torch.Generator().manual_seed(0))
    log = _record(model, lambda: model.run_forward(ids, mode, nmb, crosslayer=xl,
                                                   reset_cache=True))
    att = _attn(log)
    want = []
    for l in range(L):
        if mode == "serial":
            for m in range(nmb):
                want += [("a2f_send", l, m), ("f2a_recv", l, m)]
        elif not xl:
            if l > 0:
                want += [("f2a_recv", l - 1, m) for m in range(nmb)]
            want += [("a2f_send", l, m) for m in range(nmb)]
        else:
            for m in range(nmb):
                if l > 0:
                    want.append(("f2a_recv", l - 1, m))
                want.append(("a2f_send", l, m))
    if mode != "serial":
        want += [("f2a_recv", L - 1, m) for m in range(nmb)]
    assert att == want
    # FFN side: every A2F is consumed once, in send order, and answered
    ffn = [(n, l, m) for n, l, m in log if n in ("a2f_recv", "f2a_send")]
    sends = [(l, m) for n, l, m in att if n == "a2f_send"]
    assert [(l, m) for n, l, m in ffn if n == "a2f_recv"] == sends
    for i in range(0, len(ffn), 2):
        assert ffn[i][0] == "a2f_recv" and ffn[i + 1] == ("f2a_send",) + ffn[i][1:]
    # every send precedes its receive
    pos = {e: i for i, e in enumerate(log)}
    for l, m in sends:
        assert pos[("a2f_send", l, m)] < pos[("a2f_recv", l, m)] < pos[("f2a_send", l, m)] \
            < pos[("f2a_recv", l, m)]


def test_schedules_agree_numerically(model):
    ids = torch.randint(0, 1024, (4, 9), generator=torch.Generator().manual_seed(1))
    outs = [model.run_forward(ids, mode, nmb, crosslayer=xl, reset_cache=True)
            for mode, nmb, xl in (("serial", 1, False), ("serial", 2, False), ("dbo", 2, False),
                                  ("dbo", 2, True), ("dbo", 3, True))]
    for o in outs[1:]:
        torch.testing.assert_close(o, outs[0], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("timing_mode", ["cuda_events", "sync"])
def test_serial_scheduler_timing(model, timing_mode):
    """The reference's serial-scheduler interface: ``enable_timing`` fills
    ``get_timing_data`` with per-layer, per-micro-batch events; without it the
    timing stays None; the logits equal the engine's serial forward."""
    from afd_demo_b200.parallel.schedulers import SimplePipelineScheduler

    ids = torch.randint(0, 1024, (4, 9), generator=torch.Generator().manual_seed(2))
    plain = SimplePipelineScheduler(model, 2)
    out = plain.run(ids)
    assert plain.get_timing_data() is None
    timed = SimplePipelineScheduler(model, num_micro_batches=2, enable_timing=True,
                                    timing_mode=timing_mode)
    torch.testing.assert_close(timed.run(ids), out)
    t = timed.get_timing_data()
    assert t is not None and t.num_layers == model.num_layers and t.num_micro_batches == 2
    assert t.total_time_ms > 0
    d = t.to_dict()
    layers = {e["layer"] for e in d["events"]}
    assert layers == set(range(model.num_layers)), layers
    assert {e["mb"] for e in d["events"]} == {0, 1}
