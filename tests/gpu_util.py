"""Helpers for the GPU parity tests (device <-> oracle conversions)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

DTYPE_NAMES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}

# North-star tolerance for attention outputs in bf16.
MAX_ABS = 2e-2
MEAN_ABS = 1e-3


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def host(t: torch.Tensor) -> np.ndarray:
    """Device tensor -> numpy; float types become float32 carriers."""

    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().numpy()
    return t.numpy()


def assert_attention_close(actual: torch.Tensor, expected: np.ndarray, *, max_abs=MAX_ABS, mean_abs=MEAN_ABS,
                           what="attention"):
    a = host(actual).astype(np.float64)
    diff = np.abs(a - expected)
    assert np.isfinite(a).all(), f"{what}: non-finite output"
    assert diff.max() <= max_abs, f"{what}: max abs err {diff.max():.3e} > {max_abs}"
    assert diff.mean() <= mean_abs, f"{what}: mean abs err {diff.mean():.3e} > {mean_abs}"
    return float(diff.max()), float(diff.mean())
