"""CPU tests of the offline parts of two tools: the decode-trace summary
(`scripts/trace_decode.py`: critical-path charge per kernel, peer-wait split,
busy union) on a synthetic kernel list, and the serial-split capture
(`scripts/capture_serial_split.py`: cache selection, the prefill/decode split
merged into a cache entry, dry run)."""

import json

import pytest

from afd_demo_b200.scripts import capture_serial_split as css
from afd_demo_b200.scripts import trace_decode as td


def _trace(tmp_path, events, steps=2, layers=1, role="attention"):
    p = tmp_path / "trace.json"
    p.write_text(json.dumps({"events": events, "steps": steps, "layers": layers,
                             "role": role}))
    return str(p)


def test_summary_charges_the_last_step_and_splits_waits(tmp_path):
    step = [["gemm_kernel(a)", 0.0, 10.0], [td.WAIT_KERNEL, 10.0, 20.0],
            ["norm_kernel", 30.0, 5.0]]
    # two steps; the second starts at 100 us
    ev = step + [[n, s + 100.0, d] for n, s, d in step]
    out = td.summarize(_trace(tmp_path, ev))
    assert "last step 0.04 ms, 3 kernels" in out  # 35 us
    assert "F2A waits    20.0 us" in out and "kernels    15.0 us" in out
    assert "GPU busy 100.0%" in out
    # kernel names are cut at their argument list
    assert "gemm_kernel " in out and "(a)" not in out


def test_summary_removes_overlap_from_the_charge(tmp_path):
    # an early-launched kernel (PDL) overlaps its predecessor: it is charged
    # only from the predecessor's end
    ev = [["a", 0.0, 10.0], ["b", 4.0, 10.0]]
    out = td.summarize(_trace(tmp_path, ev, steps=1, role="ffn"))
    lines = {ln.split()[0]: ln for ln in out.splitlines()[1:] if not ln.strip().startswith("split")}
    assert " 0.010 ms" in lines["a"] and " 0.004 ms" in lines["b"]
    assert "A2F waits" in out


def test_busy_union_counts_overlaps_once():
    ev = [("a", 0.0, 10.0), ("b", 5.0, 10.0), ("c", 20.0, 5.0)]
    assert td._busy_union(ev) == pytest.approx(20.0)
    assert td._busy_union([]) == 0.0


def test_summary_of_an_empty_trace(tmp_path):
    assert "no kernels" in td.summarize(_trace(tmp_path, []))


def _cache(root, name, **fields):
    d = root / "serial" / "cache"
    d.mkdir(parents=True, exist_ok=True)
    (d / name).write_text(json.dumps(fields))
    return d / name


def test_capture_selects_cache_entries(tmp_path):
    _cache(tmp_path, "b4_s128_t20.json", total_time_ms=1.0)
    _cache(tmp_path, "b8_s128_t20.json", total_time_ms=1.0)
    _cache(tmp_path, "b8_s512_t20.json", total_time_ms=1.0)
    _cache(tmp_path, "notes.json", total_time_ms=1.0)  # not a cell: ignored
    d = tmp_path / "serial" / "cache"
    assert [(c.batch, c.seq, c.tokens) for c in css.iter_configs(d)] == \
        [(4, 128, 20), (8, 128, 20), (8, 512, 20)]
    assert [(c.batch, c.seq) for c in css.iter_configs(d, batches={8}, seqs={512})] == [(8, 512)]
    assert css.parse_list("4, 8,") == {4, 8} and css.parse_list("") is None


def test_capture_merges_the_split(tmp_path):
    cache = _cache(tmp_path, "b4_s128_t11.json", total_time_ms=1000.0, max_new_tokens=11)
    raw = tmp_path / "raw.json"
    raw.write_text(json.dumps({"total_time_ms": 200.0}))
    assert not css.has_split(cache)
    prefill, step = css.merge_split(cache, raw)
    assert (prefill, step) == (200.0, 80.0)  # (1000 - 200) / 10 decode-loop steps
    d = json.loads(cache.read_text())
    assert d["decode_tpot_ms"] == d["decode_step_ms"] == 80.0 and d["decode_steps"] == 10
    assert css.has_split(cache)


@pytest.mark.parametrize("fields,raw_ms,match", [
    ({"total_time_ms": 100.0, "max_new_tokens": 1}, 10.0, "no decode-loop steps"),
    ({"total_time_ms": 100.0, "max_new_tokens": 5}, 200.0, "< prefill"),
])
def test_capture_rejects_inconsistent_entries(tmp_path, fields, raw_ms, match):
    cache = _cache(tmp_path, "b4_s128_t5.json", **fields)
    raw = tmp_path / "raw.json"
    raw.write_text(json.dumps({"total_time_ms": raw_ms}))
    with pytest.raises(ValueError, match=match):
        css.merge_split(cache, raw)


def test_capture_dry_run_and_missing_cache(tmp_path, capsys):
    assert css.main(["--root", str(tmp_path)]) == 2  # no serial/cache directory
    _cache(tmp_path, "b4_s128_t20.json", total_time_ms=1.0)
    _cache(tmp_path, "b8_s128_t20.json", total_time_ms=1.0, prefill_ms=1.0, decode_tpot_ms=1.0)
    assert css.main(["--root", str(tmp_path), "--dry-run", "--skip-existing"]) == 0
    out = capsys.readouterr().out
    assert "[skip-existing] b8_s128_t20" in out
    assert "run_single.sh local 4 128 --tokens 20 --no-dbo" in out
