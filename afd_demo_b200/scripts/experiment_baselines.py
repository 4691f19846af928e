"""Mode-matched serial baselines for reports, audits and plots.

Reference: scripts/experiment_baselines.py:22-79. A prefill (TTFT) comparison
uses the serial run's ``prefill_ms``; a decode (TPOT) comparison uses its
``decode_tpot_ms``. Legacy fields (``decode_step_ms``, ``total_time_ms /
tokens``) are never used as a baseline.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping, Optional


@dataclass(frozen=True)
class BaselineResolution:
    value_ms: Optional[float]
    unit: Optional[str]
    source: str
    warning: Optional[str] = None

    @property
    def available(self) -> bool:
        return self.value_ms is not None and self.value_ms > 0


def normalize_mode(mode: Optional[str]) -> Optional[str]:
    """'prefill' / 'decode' comparison class of a mode or directory name."""
    if not mode:
        return None
    m = mode.lower().replace("_", "-")
    if "prefill" in m:
        return "prefill"
    if "decode" in m:
        return "decode"
    return None


def infer_mode_from_path(path) -> Optional[str]:
    return normalize_mode(str(path))


def resolve_serial_baseline(cache: Mapping[str, Any], mode: Optional[str]) -> BaselineResolution:
    mode = normalize_mode(mode)
    if mode == "prefill":
        v = cache.get("prefill_ms")
        if v is not None:
            return BaselineResolution(float(v), "TTFT", "prefill_ms")
        return BaselineResolution(None, None, "missing",
                                  "TTFT baseline missing; a TPOT-style total is not comparable")
    if mode == "decode":
        v = cache.get("decode_tpot_ms")
        if v is not None:
            return BaselineResolution(float(v), "TPOT", "decode_tpot_ms")
        if cache.get("decode_step_ms") is not None:
            return BaselineResolution(None, None, "legacy-decode-step-ms",
                                      "decode_tpot_ms missing; legacy decode_step_ms not used")
        return BaselineResolution(None, None, "missing", "exact TPOT baseline missing")
    return BaselineResolution(None, None, "unknown-mode",
                              "could not infer prefill/decode comparison mode")


def serial_cache_path(root: Path, batch, seq, tokens) -> Path:
    return Path(root) / "serial" / "cache" / f"b{batch}_s{seq}_t{tokens}.json"
