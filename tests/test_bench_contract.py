"""bench.py's output contract: one JSON line with the fields the benchmark
driver reads, for this framework's arm (GPU) and the reference arm (CPU here:
with one GPU the reference has no runnable topology, so it must say so)."""

import json
import os
import subprocess
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _json_lines(out: str):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def test_reference_arm_single_gpu_prints_unavailable():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference"], cwd=REPO,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    assert lines[0]["impl"] == "reference"
    assert isinstance(lines[0]["unavailable"], str) and lines[0]["unavailable"]


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_bench_json_contract_small_model():
    """A 2-layer model with the real layer shapes, so it runs in seconds; its
    line must be labelled as that model and carry no baseline ratio."""
    cmd = [sys.executable, "bench.py", "--model", "small", "--batch-per-gpu", "8", "--seq", "64",
           "--tokens", "4", "--steps", "3", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    d = lines[0]
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "clocks",
              "e2e", "gpu_launches"):
        assert k in d, k
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["value"] == pytest.approx(1000.0 * 8 / d["ms_per_step"], rel=1e-6)
    assert d["higher_is_better"] is True and d["dtype"] == "bf16"
    assert d["vs_baseline"] is None
    assert d["config"]["model"].startswith("small") and d["config"]["global_batch"] == 8
    assert d["gpu_launches"] > 0
    e2e = d["e2e"]
    assert e2e["value"] > 0 and e2e["h2d_bytes_per_step"] == 8 * 8
    assert e2e["d2h_bytes_per_step"] == 8 * 8
    assert "sm_mhz" in d["clocks"] and "reasons" in d["clocks"]


def test_clock_sampler_keeps_samples_of_the_timed_region():
    """Only nvidia-smi rows stamped inside the timed region are summarised;
    a region shorter than the interval keeps the nearest row on each side."""
    import datetime

    sys.path.insert(0, REPO)
    from bench import ClockSampler

    base = datetime.datetime(2026, 1, 1, 12, 0, 0)

    def row(ms, sm, reasons=("Not Active",) * 4):
        t = (base + datetime.timedelta(milliseconds=ms)).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        return [t, "0", str(sm), "1965", "700.0", "0x0"] + list(reasons)

    rows = [row(0, 600), row(50, 1900), row(100, 1950),
            row(150, 1960, ("Not Active", "Not Active", "Not Active", "Active")), row(200, 700)]
    t = lambda ms: (base + datetime.timedelta(milliseconds=ms)).timestamp()  # noqa: E731
    d = ClockSampler.summarise(rows, t(40), t(160))
    assert d["samples_in_region"] == 3 and d["sm_mhz"] == 1950.0
    assert d["reasons"] == ["sw_power_cap"] and d["sm_max_mhz"] == 1965.0
    near = ClockSampler.summarise(rows, t(60), t(90))  # no row inside
    assert near["samples_in_region"] == 0 and near["samples"] == 2
    assert near["sm_mhz"] == (1900.0 + 1950.0) / 2
    assert ClockSampler.summarise(rows)["samples"] == 5
