"""Numerics contract (API of cacheblend-hf-v7 ``tolerance.py``): four tolerance
categories and ``assert_logits_close``.  The bounds are the reference's:

  IDENTICAL_PATH  max|diff| == 0
  SAME_SHAPE      max|diff| < 1e-3
  MIXED_SHAPE     argmax identical everywhere and max|diff| < 5e-2
  RECOMPUTE_PATH  max|diff| < 1e-3
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


class Tolerance(Enum):
    IDENTICAL_PATH = "identical"
    SAME_SHAPE = "same_shape"
    MIXED_SHAPE = "mixed_shape"
    RECOMPUTE_PATH = "recompute_path"


@dataclass
class ToleranceResult:
    passed: bool
    max_diff: float
    argmax_match_ratio: float
    category: Tolerance
    detail: str


_BOUNDS = {
    Tolerance.IDENTICAL_PATH: ("max_diff == 0", lambda d, a: d == 0.0),
    Tolerance.SAME_SHAPE: ("max_diff < 1e-3", lambda d, a: d < 1e-3),
    Tolerance.MIXED_SHAPE: ("argmax == 1.0 AND max_diff < 5e-2", lambda d, a: a == 1.0 and d < 5e-2),
    Tolerance.RECOMPUTE_PATH: ("max_diff < 1e-3", lambda d, a: d < 1e-3),
}


def assert_logits_close(actual, expected, category: Tolerance, name: str = "logits") -> ToleranceResult:
    """Compare two logits tensors under a category; raise AssertionError on failure."""
    if actual.shape != expected.shape:
        raise AssertionError(f"{name} shape mismatch: {actual.shape} vs {expected.shape}")
    if category not in _BOUNDS:
        raise ValueError(f"Unknown tolerance category: {category}")
    max_diff = float((actual.float() - expected.float()).abs().max().item())
    match = float((actual.argmax(dim=-1) == expected.argmax(dim=-1)).float().mean().item())
    bound, ok = _BOUNDS[category]
    passed = bool(ok(max_diff, match))
    detail = (f"{name}: max_diff={max_diff:.3e}, argmax_match={match:.4f}, "
              f"category={category.value}, bound={bound}, passed={passed}")
    res = ToleranceResult(passed, max_diff, match, category, detail)
    if not passed:
        raise AssertionError(detail)
    return res
