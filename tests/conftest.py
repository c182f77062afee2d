"""Shared pytest configuration: the ``gpu`` marker and golden-vector loaders."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(GOLDEN_DIR, "golden.npz")) as data:
        arrays = {name: data[name] for name in data.files}
    with open(os.path.join(GOLDEN_DIR, "golden.json")) as handle:
        meta = json.load(handle)
    return arrays, meta["cases"]


def bf16_array(bits: np.ndarray) -> np.ndarray:
    """float32 carrier of a stored bf16 bit pattern."""

    from oracle.numerics import from_bf16_bits

    return from_bf16_bits(bits)
