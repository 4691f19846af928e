"""Tensor comparison helpers (reference: src/utils/validation.py:11-50)."""

from __future__ import annotations

from typing import Dict, Tuple

import torch


def compare_tensors(a: torch.Tensor, b: torch.Tensor, rtol: float = 1e-3, atol: float = 1e-5,
                    name: str = "tensor") -> Tuple[bool, Dict[str, float]]:
    """allclose(a, b) plus max/mean absolute differences and max/mean
    differences relative to |a| (+1e-10), with the reference's defaults."""
    if a.shape != b.shape:
        return False, {"error": f"shape mismatch {tuple(a.shape)} vs {tuple(b.shape)}"}
    af, bf = a.detach().float().cpu(), b.detach().float().cpu()
    diff = (af - bf).abs()
    rel = diff / (af.abs() + 1e-10)
    metrics = {
        "max_abs_diff": float(diff.max()) if diff.numel() else 0.0,
        "mean_abs_diff": float(diff.mean()) if diff.numel() else 0.0,
        "max_rel_diff": float(rel.max()) if rel.numel() else 0.0,
        "mean_rel_diff": float(rel.mean()) if rel.numel() else 0.0,
    }
    return bool(torch.allclose(af, bf, rtol=rtol, atol=atol)), metrics


def validate_output(output: torch.Tensor, reference: torch.Tensor, rtol: float = 1e-3,
                    atol: float = 1e-5) -> bool:
    """Whether `output` is within tolerance of `reference` (allclose with the
    reference as the expected side)."""
    ok, _ = compare_tensors(reference, output, rtol, atol, name="model_output")
    return ok


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in fp32."""
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))
