"""Mode-matched serial baselines for reports, audits and plots.

Reference: scripts/experiment_baselines.py:22-79. A prefill (TTFT) comparison
uses the serial run's ``prefill_ms``; a decode (TPOT) comparison uses its
``decode_tpot_ms``. Legacy fields (``decode_step_ms``, ``total_time_ms /
tokens``) are never used as a baseline.

The result record (``BaselineResolution``) and its ``source`` tags are the
interface the report, audit and Gantt scripts read, so they keep the
reference's names; the rule itself is the table ``_RULES`` below.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping, NamedTuple, Optional, Tuple


@dataclass(frozen=True)
class BaselineResolution:
    value_ms: Optional[float]
    unit: Optional[str]
    source: str
    warning: Optional[str] = None

    @property
    def available(self) -> bool:
        return self.value_ms is not None and self.value_ms > 0


class _Rule(NamedTuple):
    key: str                    # the serial-cache field that is the baseline
    unit: str                   # what it measures
    legacy: Tuple[str, ...]     # fields that look like a baseline but are not one
    missing: str                # warning when `key` is absent


# comparison class -> how its serial baseline is found
_RULES = {
    "prefill": _Rule("prefill_ms", "TTFT", (),
                     "TTFT baseline missing; a TPOT-style total is not comparable"),
    "decode": _Rule("decode_tpot_ms", "TPOT", ("decode_step_ms",),
                    "exact TPOT baseline missing"),
}


def normalize_mode(mode: Optional[str]) -> Optional[str]:
    """'prefill' / 'decode' comparison class of a mode or directory name
    (the first class whose name occurs in it; prefill before decode)."""
    if not mode:
        return None
    m = mode.lower().replace("_", "-")
    return next((cls for cls in _RULES if cls in m), None)


def infer_mode_from_path(path) -> Optional[str]:
    return normalize_mode(str(path))


def resolve_serial_baseline(cache: Mapping[str, Any], mode: Optional[str]) -> BaselineResolution:
    rule = _RULES.get(normalize_mode(mode))
    if rule is None:
        return BaselineResolution(None, None, "unknown-mode",
                                  "could not infer prefill/decode comparison mode")
    if cache.get(rule.key) is not None:
        return BaselineResolution(float(cache[rule.key]), rule.unit, rule.key)
    for old in rule.legacy:
        if cache.get(old) is not None:
            return BaselineResolution(None, None, "legacy-" + old.replace("_", "-"),
                                      f"{rule.key} missing; legacy {old} not used")
    return BaselineResolution(None, None, "missing", rule.missing)


def serial_cache_path(root: Path, batch, seq, tokens) -> Path:
    return Path(root) / "serial" / "cache" / f"b{batch}_s{seq}_t{tokens}.json"
