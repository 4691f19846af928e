"""Orchestration and reporting scripts on CPU: the experiment matrix over two
gloo ranks with the tiny Qwen3-MoE, then the audit, report, Gantt and plot
scripts on its output (the reference's integration testing is this matrix
plus the baseline audit, scripts/run_experiment_matrix.sh and
scripts/audit_experiment_baselines.py)."""

import csv
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

from afd_demo_b200.scripts.experiment_baselines import (normalize_mode, resolve_serial_baseline,
                                                        serial_cache_path)

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_mode_normalisation_and_baselines():
    assert normalize_mode("prefill-dbo") == "prefill"
    assert normalize_mode("decode_dbo_crosslayer") == "decode"
    assert normalize_mode("serial") is None and normalize_mode(None) is None
    cache = {"prefill_ms": 12.0, "decode_tpot_ms": 3.0, "decode_step_ms": 9.0}
    assert resolve_serial_baseline(cache, "prefill-dbo").value_ms == 12.0
    assert resolve_serial_baseline(cache, "decode-dbo").value_ms == 3.0
    legacy = resolve_serial_baseline({"decode_step_ms": 9.0}, "decode")
    assert not legacy.available and legacy.source == "legacy-decode-step-ms"
    assert not resolve_serial_baseline({"total_time_ms": 5.0}, "prefill").available
    assert not resolve_serial_baseline(cache, "serial").available
    assert serial_cache_path(Path("r"), 4, 128, 20) == Path("r/serial/cache/b4_s128_t20.json")


@pytest.fixture(scope="module")
def matrix(tmp_path_factory):
    res = tmp_path_factory.mktemp("matrix")
    env = dict(os.environ, RESULTS_DIR=str(res), MODEL_PATH="tiny", GPUS="2",
               MASTER_PORT=str(_free_port()), CUDA_VISIBLE_DEVICES="")
    p = subprocess.run(["bash", "afd_demo_b200/scripts/run_experiment_matrix.sh", "--modes",
                        "serial,prefill-dbo,decode-dbo,decode-dbo-crosslayer", "--batches", "2",
                        "--seqs", "32", "--tokens", "4"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    return res


def test_matrix_summary_and_layout(matrix):
    rows = list(csv.DictReader(open(matrix / "experiment_matrix_summary.csv")))
    assert [r["mode"] for r in rows] == ["serial", "prefill-dbo", "decode-dbo",
                                         "decode-dbo-crosslayer"]
    assert all(r["status"] == "ok" for r in rows), rows
    cache = json.load(open(matrix / "serial" / "cache" / "b2_s32_t4.json"))
    assert cache["prefill_ms"] > 0 and cache["decode_tpot_ms"] > 0
    for mode in ("prefill-dbo", "decode-dbo", "decode-dbo-crosslayer"):
        for role in ("attention", "ffn"):
            d = json.load(open(matrix / mode / f"timing_{role}_{mode}_b2_s32_t4.json"))
            assert d["node"] == role and d["num_layers"] == 2 and d["events"]
            assert {e["type"] for e in d["events"]} <= {
                "attn_compute", "ffn_compute", "moe_router", "moe_experts",
                "moe_shared_or_dense", "send_start", "send_transfer", "recv_post", "recv_wait"}
        assert (matrix / mode / f"report_{mode}_b2_s32_t4.md").exists()


def test_matrix_uses_serial_cache(matrix):
    env = dict(os.environ, RESULTS_DIR=str(matrix), MODEL_PATH="tiny", GPUS="2",
               MASTER_PORT=str(_free_port()), CUDA_VISIBLE_DEVICES="")
    p = subprocess.run(["bash", "afd_demo_b200/scripts/run_experiment_matrix.sh", "--modes",
                        "serial", "--batches", "2", "--seqs", "32", "--tokens", "4"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0
    rows = list(csv.DictReader(open(matrix / "experiment_matrix_summary.csv")))
    assert rows[-1]["status"] == "cached"


def test_audit_pairs_every_dbo_row(matrix, tmp_path):
    out = tmp_path / "audit.csv"
    p = subprocess.run([sys.executable, "-m", "afd_demo_b200.scripts.audit_experiment_baselines",
                        "--root", str(matrix), "--output-csv", str(out)],
                       cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    rows = list(csv.DictReader(open(out)))
    assert list(rows[0]) == ["root", "mode", "tag", "batch", "seq", "tokens", "status",
                             "serial_cache", "serial_baseline_ms", "dbo_ms", "speedup", "note"]
    assert len(rows) == 3 and all(r["status"] == "ok" for r in rows), rows
    assert {r["mode"] for r in rows} == {"prefill", "decode"}


def test_report_gantt_and_plot_all(matrix, tmp_path):
    mode = "decode-dbo-crosslayer"
    attn = matrix / mode / f"timing_attention_{mode}_b2_s32_t4.json"
    ffn = matrix / mode / f"timing_ffn_{mode}_b2_s32_t4.json"
    rep = tmp_path / "r.md"
    p = subprocess.run([sys.executable, "-m", "afd_demo_b200.scripts.gen_experiment_report",
                        "--attn-timing", str(attn), "--ffn-timing", str(ffn), "--output", str(rep),
                        "--mode", mode, "--batch", "2", "--seq", "32", "--tokens", "4",
                        "--serial-baseline", str(matrix / "serial/cache/b2_s32_t4.json")],
                       cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    text = rep.read_text()
    assert "|" in text and "TPOT" in text
    png = tmp_path / "g.png"
    p = subprocess.run([sys.executable, "-m", "afd_demo_b200.scripts.visualize_dbo_pipeline",
                        "--attn-timing", str(attn), "--ffn-timing", str(ffn), "--output", str(png),
                        "--num-layers", "2"], cwd=ROOT, capture_output=True, text=True,
                       timeout=120)
    assert p.returncode == 0, p.stderr
    assert png.read_bytes()[:8] == b"\x89PNG\r\n\x1a\n"
    p = subprocess.run([sys.executable, "-m", "afd_demo_b200.scripts.plot_all_pipelines",
                        "--root", str(matrix)], cwd=ROOT, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stderr
    assert list(matrix.glob("*/pipelines_index.md"))


def test_run_single_oom_exit_code(tmp_path):
    """A run whose log shows an out-of-memory error exits 2 (the matrix's
    stop-escalating signal); an impossible batch on a 4-sequence cache does."""
    env = dict(os.environ, RESULTS_DIR=str(tmp_path), MODEL_PATH="tiny", GPUS="1",
               CUDA_VISIBLE_DEVICES="", AFD_FAULT="oom")
    p = subprocess.run(["bash", "afd_demo_b200/scripts/run_single.sh", "local", "2", "16",
                        "--tokens", "2"], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 2, p.stdout[-2000:]
    assert "OOM DETECTED" in p.stdout


REF_SCRIPTS = ROOT / "baseline" / "_ref" / "scripts"


def _no_pyc():
    return dict(os.environ, PYTHONDONTWRITEBYTECODE="1")  # leave the install untouched


@pytest.mark.skipif(not (REF_SCRIPTS / "gen_experiment_report.py").exists(),
                    reason="the reference install (baseline/_ref) is absent")
def test_reference_scripts_read_our_outputs(matrix, tmp_path):
    """Schema parity, checked by the reference's own tools: its report
    generator and baseline audit (scripts/gen_experiment_report.py,
    scripts/audit_experiment_baselines.py, unmodified) read this framework's
    timing JSONs and serial cache."""
    cache = matrix / "serial" / "cache" / "b2_s32_t4.json"
    for mode in ("serial", "prefill-dbo", "decode-dbo", "decode-dbo-crosslayer"):
        tag = f"{mode}_b2_s32_t4"
        out = tmp_path / f"{mode}.md"
        p = subprocess.run(
            [sys.executable, "gen_experiment_report.py",
             "--attn-timing", str(matrix / mode / f"timing_attention_{tag}.json"),
             "--ffn-timing", str(matrix / mode / f"timing_ffn_{tag}.json"),
             "--output", str(out), "--mode", mode, "--batch", "2", "--seq", "32",
             "--tokens", "4", "--serial-baseline", str(cache)],
            cwd=REF_SCRIPTS, capture_output=True, text=True, timeout=120, env=_no_pyc())
        assert p.returncode == 0, (mode, p.stderr[-2000:])
        text = out.read_text()
        assert "Layer averages" in text
        if mode != "serial":
            assert "speedup" in text
    audit = tmp_path / "audit.csv"
    p = subprocess.run([sys.executable, "audit_experiment_baselines.py", "--root", str(matrix),
                        "--output-csv", str(audit)],
                       cwd=REF_SCRIPTS, capture_output=True, text=True, timeout=120, env=_no_pyc())
    assert p.returncode == 0, p.stderr[-2000:]
    rows = list(csv.DictReader(open(audit)))
    assert len(rows) == 3 and all(r["status"] == "ok" for r in rows)
    assert {r["note"] for r in rows} == {"decode_tpot_ms", "prefill_ms"}


def test_comm_bench_host_section_reference_schema(tmp_path):
    """The comm microbenchmark on 2 gloo ranks writes the reference's JSON
    layout ({"meta", "results"}, per-span mean/median/p95/min/max) and its
    nine CSV columns."""
    out = tmp_path / "comm.json"
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    p = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port",
                        str(_free_port()), "-m", "afd_demo_b200.scripts.bench_comm_transfer",
                        "--backend", "cpu", "--sizes-mib", "0.004,1", "--iters", "4",
                        "--warmup", "1", "--blocking", "--output", str(out)],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    d = json.loads(out.read_text())
    assert set(d) == {"meta", "results"}
    assert d["meta"]["dist_backend"] == "gloo" and d["meta"]["world_size"] == 2
    assert [r["size_mib_requested"] for r in d["results"]] == [0.004, 1.0]
    for r in d["results"]:
        for span in ("sender_enqueue_ms", "sender_completion_ms", "receiver_wait_ms",
                     "blocking_send_ms", "blocking_recv_ms"):
            assert set(r[span]) == {"mean", "median", "p95", "min", "max"}
            assert r[span]["min"] <= r[span]["p95"] <= r[span]["max"]
    rows = list(csv.DictReader(open(out.with_suffix(".csv"))))
    assert list(rows[0]) == ["size_mib_requested", "tensor_mib", "tensor_bytes",
                             "sender_enqueue_mean_ms", "sender_completion_mean_ms",
                             "receiver_wait_mean_ms", "blocking_send_mean_ms",
                             "blocking_recv_mean_ms", "completion_bandwidth_mib_s"]
    assert int(rows[1]["tensor_bytes"]) == 2**20


def test_decode_cells_cli():
    """The one-load matrix script parses its options (it needs GPUs to run)."""
    p = subprocess.run([sys.executable, "-m", "afd_demo_b200.scripts.decode_cells", "--help"],
                       capture_output=True, text=True, cwd=ROOT, timeout=120)
    assert p.returncode == 0, p.stderr
    for opt in ("--batches", "--seqs", "--modes", "--attn-gpus", "--output"):
        assert opt in p.stdout


def test_run_node_reference_form_dry_run():
    """run_node.sh <role> [master_addr] [master_port] [options]: the role picks
    the rank and is passed on; options pass through; other first words fail."""
    def cmd(*a):
        p = subprocess.run(["bash", "afd_demo_b200/scripts/run_node.sh", *a], cwd=ROOT,
                           env=dict(os.environ, RUN_NODE_DRY_RUN="1"), capture_output=True,
                           text=True, timeout=60)
        return p.returncode, p.stdout.split(), p.stderr

    rc, argv, _ = cmd("ffn", "10.1.2.3", "29600", "--no-dbo")
    assert rc == 0
    flag = lambda f: argv[argv.index(f) + 1]  # noqa: E731
    assert (flag("--role"), flag("--rank"), flag("--master-addr"), flag("--master-port")) == \
        ("ffn", "1", "10.1.2.3", "29600")
    assert argv[-1] == "--no-dbo"
    rc, argv, _ = cmd("attention", "--greedy")
    assert rc == 0 and flag("--rank") == "0" and flag("--master-port") == "29500"
    rc, argv, _ = cmd("--no-dbo")  # environment form: no role
    assert rc == 0 and "--role" not in argv
    rc, _, err = cmd("worker")
    assert rc == 1 and "role must be" in err


def test_run_node_reference_form_two_ranks(tmp_path):
    """Both roles started the reference's way (role, address, port) on CPU
    over gloo with the tiny model; each rank exits 0."""
    port = str(_free_port())
    env = dict(os.environ, MODEL_PATH="tiny", BATCH_SIZE="2", MAX_SEQ_LEN="32", TOKENS="3",
               CUDA_DEVICES="")
    common = ["127.0.0.1", port, "--synthetic", "--prefill-seq-len", "8", "--greedy",
              "--no-dbo", "--results-dir", str(tmp_path)]
    procs = [subprocess.Popen(["bash", "afd_demo_b200/scripts/run_node.sh", role, *common],
                              cwd=ROOT, env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True)
             for role in ("attention", "ffn")]
    outs = []
    try:
        for p in procs:
            outs.append(p.communicate(timeout=600)[0])
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert [p.returncode for p in procs] == [0, 0], "\n".join(o[-2000:] for o in outs)


@pytest.mark.parametrize("module", ["kernel_probe", "bench_kernels", "trace_decode", "decode_cells",
                                    "bench_comm_transfer", "capture_serial_split", "gen_experiment_report",
                                    "audit_experiment_baselines", "visualize_dbo_pipeline",
                                    "plot_all_pipelines"])
def test_script_imports_and_parses_arguments(module):
    """Every script module imports without a GPU and answers --help (the GPU
    tools run only on a GPU box; an import error there would show up here)."""
    p = subprocess.run([sys.executable, "-m", f"afd_demo_b200.scripts.{module}", "--help"],
                       cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr[-2000:]
    assert "usage" in p.stdout.lower()
