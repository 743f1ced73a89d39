"""Shared test helpers: seeded inputs and bit-level comparisons."""
from __future__ import annotations

import numpy as np
import torch

GOLDEN = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden")


def golden(name: str):
    return np.load(f"{GOLDEN}/{name}")


def to_bits(t: torch.Tensor) -> np.ndarray:
    """16-bit tensor -> uint16 numpy bit patterns."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(bits: np.ndarray, dtype=torch.bfloat16, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(dtype).to(device)


def ulp_diff_bf16(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 units-in-the-last-place between two bit arrays."""
    def ordered(b):
        b = b.astype(np.int32)
        return np.where(b & 0x8000, 0x8000 - b, b)   # monotone integer line
    return np.abs(ordered(a_bits) - ordered(b_bits))


def mock_model(dtype=torch.float32, device="cpu"):
    """The CPU-mock decoder (tiny Mistral, seed 0) used by the golden fixtures."""
    from golden.make_golden import build_mock_model
    return build_mock_model(torch.float32).to(dtype).to(device)
