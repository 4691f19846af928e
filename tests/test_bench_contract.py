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
