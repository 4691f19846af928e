"""Tensor comparison helpers (reference: src/utils/validation.py:11-50)."""

from __future__ import annotations

from typing import Dict, Tuple

import torch


def compare_tensors(a: torch.Tensor, b: torch.Tensor, rtol: float = 1e-3, atol: float = 1e-3,
                    name: str = "tensor") -> Tuple[bool, Dict[str, float]]:
    """allclose plus max/mean absolute and relative differences."""
    if a.shape != b.shape:
        return False, {"error": f"shape mismatch {tuple(a.shape)} vs {tuple(b.shape)}"}
    af, bf = a.detach().float().cpu(), b.detach().float().cpu()
    diff = (af - bf).abs()
    rel = diff / bf.abs().clamp_min(1e-8)
    metrics = {
        "max_abs_diff": float(diff.max()) if diff.numel() else 0.0,
        "mean_abs_diff": float(diff.mean()) if diff.numel() else 0.0,
        "max_rel_diff": float(rel.max()) if rel.numel() else 0.0,
        "mean_rel_diff": float(rel.mean()) if rel.numel() else 0.0,
    }
    return bool(torch.allclose(af, bf, rtol=rtol, atol=atol)), metrics


def validate_output(output: torch.Tensor, expected: torch.Tensor, rtol: float = 1e-2,
                    atol: float = 1e-2) -> bool:
    ok, _ = compare_tensors(output, expected, rtol, atol)
    return ok


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in fp32."""
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))
