"""Floating-point storage types in numpy.  TEST INFRASTRUCTURE ONLY.

numpy has no bfloat16, so bf16 tensors are represented as float32 arrays whose
values are exactly representable in bf16.  ``round_to`` reproduces torch's
``Tensor.to(dtype)`` rounding (round-to-nearest-even) used throughout the
reference, e.g. unicache/storage/physical.py:173-174 and :201.
"""

from __future__ import annotations

import numpy as np

DTYPES = ("bfloat16", "float16", "float32")


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bf16 value, returned as float32 (NaN kept)."""

    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 data to a storage dtype, keeping float32 as carrier."""

    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x.copy()
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_round(x)
    raise ValueError(f"unsupported dtype {dtype}")


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit pattern of bf16-representable float32 values."""

    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


FLOAT32_EPS = np.float32(np.finfo(np.float32).eps)


def canonical_bytes(x: np.ndarray, dtype: str | None = None) -> bytes:
    """Bytes that identify an array independent of its carrier: bf16 values as
    their 16-bit patterns, fp16 as float16, everything else as-is (C order)."""

    x = np.ascontiguousarray(x)
    if dtype == "bfloat16":
        return bf16_bits(x).tobytes()
    if dtype == "float16":
        return np.ascontiguousarray(x.astype(np.float16)).tobytes()
    return x.tobytes()


def digest(x: np.ndarray, dtype: str | None = None) -> str:
    import hashlib

    x = np.ascontiguousarray(x)
    header = f"{x.shape}|{dtype or x.dtype.name}|".encode()
    return hashlib.sha256(header + canonical_bytes(x, dtype)).hexdigest()
