"""Host-side parity with the reference's own modules, loaded unmodified from
the reference install in baseline/_ref: micro-batch splitting and merging
(src/pipeline/micro_batch.py), position ids and causal masks, the timing JSON
(src/utils/timing.py) and tensor
comparison (src/utils/validation.py). Same inputs, same outputs."""

import importlib.util
import sys
from pathlib import Path

import pytest
import torch

from afd_demo_b200.parallel import micro_batch as ours_mb
from afd_demo_b200.utils import validation as ours_val

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "src"


def _load(rel: str, name: str):
    path = REF / rel
    if not path.exists():
        pytest.skip("the reference install (baseline/_ref) is absent")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses look their module up while being built
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def ref_mb():
    return _load("pipeline/micro_batch.py", "_ref_micro_batch")


@pytest.fixture(scope="module")
def ref_val():
    return _load("utils/validation.py", "_ref_validation")


@pytest.mark.parametrize("B", [1, 2, 3, 5, 8, 9])
@pytest.mark.parametrize("nmb", [1, 2, 3, 4])
def test_split_and_merge(ref_mb, B, nmb):
    cpu = torch.device("cpu")
    ids = torch.arange(B * 6).view(B, 6)
    mask = (torch.rand(B, 6, generator=torch.Generator().manual_seed(B)) > 0.3).long()
    mine = ours_mb.MicroBatchManager(nmb, cpu).split_batch(ids, mask)
    theirs = ref_mb.MicroBatchManager(nmb, cpu).split_batch(ids, mask)
    assert [m.batch_size for m in mine] == [m.batch_size for m in theirs]
    assert [m.id for m in mine] == [m.id for m in theirs]
    for a, b in zip(mine, theirs):
        assert torch.equal(a.input_ids, b.input_ids)
        assert torch.equal(a.attention_mask, b.attention_mask)
        assert a.seq_len == b.seq_len
    outs = [m.input_ids.float() * 2 for m in mine]
    assert torch.equal(ours_mb.MicroBatchManager(nmb, cpu).merge_results(outs),
                       ref_mb.MicroBatchManager(nmb, cpu).merge_results(outs))


def test_positions_and_causal_mask(ref_mb):
    cpu = torch.device("cpu")
    assert torch.equal(ours_mb.create_position_ids(3, 7, cpu),
                       ref_mb.create_position_ids(3, 7, cpu))
    assert torch.equal(ours_mb.create_causal_mask(2, 5, cpu), ref_mb.create_causal_mask(2, 5, cpu))


@pytest.mark.parametrize("scale", [0.0, 1e-5, 1e-2, 1.0])
def test_compare_tensors(ref_val, scale):
    a = torch.randn(64, 32, generator=torch.Generator().manual_seed(0))
    b = a + scale * torch.randn(64, 32, generator=torch.Generator().manual_seed(1))
    close_o, met_o = ours_val.compare_tensors(a, b)
    close_r, met_r = ref_val.compare_tensors(a, b)
    assert close_o == close_r
    for k, v in met_r.items():
        assert k in met_o
        assert met_o[k] == pytest.approx(v, rel=1e-6, abs=1e-12), k
    assert ours_val.validate_output(a, b) == ref_val.validate_output(a, b)


@pytest.fixture(scope="module")
def ref_timing():
    return _load("utils/timing.py", "_ref_timing")


def _fill(mod, node):
    pt = mod.PipelineTiming(node=node, num_layers=3, num_micro_batches=2, total_time_ms=9.5,
                            comm_timing_mode="completion")
    pt.prefill_ms = 4.25
    pt.decode_tpot_ms = 1.5
    pt.decode_steps = 3
    t = 0.0
    kinds = ["attn_compute", "send_transfer", "recv_wait", "moe_router", "moe_experts",
             "ffn_compute", "recv_post", "send_start", "moe_shared_or_dense"]
    for l in range(3):
        for m in range(2):
            for i, k in enumerate(kinds):
                ev = mod.TimingEvent(k, l, m, t, t + 0.0001 * (i + 1), node,
                                     tensor_bytes=4096 * (i + 1) if "send" in k else None,
                                     completion_source="wait" if k == "send_transfer" else None)
                pt.add_event(ev)
                t += 0.0002
    return pt


def test_timing_json_and_merge(ref_timing):
    from afd_demo_b200.utils import timing as ours

    assert {e.value for e in ours.EventType} == {e.value for e in ref_timing.EventType}
    for node in ("attention", "ffn"):
        assert _fill(ours, node).to_dict() == _fill(ref_timing, node).to_dict()
    mine = ours.merge_timings(_fill(ours, "attention"), _fill(ours, "ffn"))
    theirs = ref_timing.merge_timings(_fill(ref_timing, "attention"), _fill(ref_timing, "ffn"))
    assert mine == theirs
    # and the JSON round trip through this framework's reader
    back = ours.PipelineTiming.from_dict(_fill(ref_timing, "ffn").to_dict())
    assert back.to_dict() == _fill(ref_timing, "ffn").to_dict()


def test_serial_baseline_resolution():
    """scripts/experiment_baselines.py: mode classes and the serial baseline
    chosen for every kind of serial cache entry."""
    ref = _load("../scripts/experiment_baselines.py", "_ref_baselines")
    from afd_demo_b200.scripts import experiment_baselines as ours

    modes = [None, "", "serial", "prefill", "prefill-dbo", "prefill_dbo", "decode", "decode-dbo",
             "decode_dbo", "decode-dbo-crosslayer", "dbo_crosslayer", "crosslayer", "dbo", "weird"]
    for m in modes:
        assert ours.normalize_mode(m) == ref.normalize_mode(m), m
    for p in ["results/decode-dbo/x.json", "results/prefill-dbo/x.json", "results/serial/x.json",
              "r/decode-dbo-crosslayer/timing_attention_decode-dbo-crosslayer_b2.json", "a/b.json"]:
        assert ours.infer_mode_from_path(p) == ref.infer_mode_from_path(p), p
    caches = [{}, {"prefill_ms": 12.0}, {"decode_tpot_ms": 3.0}, {"decode_step_ms": 9.0},
              {"total_time_ms": 5.0}, {"prefill_ms": 12.0, "decode_tpot_ms": 3.0},
              {"prefill_ms": None, "decode_tpot_ms": 0.0}, {"prefill_ms": "7.5"}]
    for c in caches:
        for m in modes:
            a, b = ours.resolve_serial_baseline(c, m), ref.resolve_serial_baseline(c, m)
            assert (a.value_ms, a.unit, a.source, a.available) == \
                   (b.value_ms, b.unit, b.source, b.available), (c, m)


def test_profiler_interface():
    """utils/profiler.py against the reference's (src/utils/profiler.py):
    the same names, signatures and statistics for the same recorded times."""
    ref = _load("utils/profiler.py", "_ref_profiler")
    from afd_demo_b200.utils import profiler as ours

    a, b = ours.Profiler(), ref.Profiler()
    for P in (a, b):
        for v in (1.0, 2.5, 4.0):
            P.record("a", v)
        with P.timer("t", use_cuda=False):
            pass
    assert a.get_stats("a") == b.get_stats("a")
    assert a.get_stats("missing") == b.get_stats("missing")
    assert [ln.split("|")[:2] for ln in a.report().splitlines() if "|" in ln and "t " not in ln] == \
           [ln.split("|")[:2] for ln in b.report().splitlines() if "|" in ln and "t " not in ln]
    assert ours.TimingResult("x", 6.0, 3).avg_ms == ref.TimingResult("x", 6.0, 3).avg_ms
    for T in (ours.Timer, ref.Timer):
        with T("x") as t:
            pass
        assert t.elapsed_ms >= 0.0
    calls = []

    @ours.profile_function("f", use_cuda=False)
    def f(x):
        calls.append(x)
        return x + 1

    assert f(1) == 2 and calls == [1] and ours.get_profiler().get_stats("f")["count"] >= 1
