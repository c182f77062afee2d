"""KIVI quantizer, packer and packed-cache oracle.  TEST INFRASTRUCTURE ONLY.

Restates unicache/storage/physical.py (Superone77/UniCache) in numpy:

* ``pack_codes`` / ``unpack_codes``        physical.py:66-104
* ``quantize_grouped``                     physical.py:107-175 (loop and
                                           vectorized forms; they agree
                                           bit-for-bit, tests/test_physical.py:984-1015)
* ``dequantize_grouped``                   physical.py:178-201
* ``packed_from_dense``                    physical.py:228-332 (reference backend)
* ``packed_dequantize``                    physical.py:379-423
* ``fake_quant`` / ``fake_quant_key/value`` unicache/operators/builtin.py:23-65

Arrays hold float32 carriers of values representable in ``dtype`` (see
``oracle.numerics``).  Packed words are int32 exactly like the reference's
``torch.sum(moved << shifts, dtype=torch.int32)`` (a wrapping sum of disjoint
bit fields, i.e. a bitwise OR).
"""

from __future__ import annotations

import math

import numpy as np

from .numerics import FLOAT32_EPS, round_to


def pack_codes(codes: np.ndarray, bits: int, dim: int) -> np.ndarray:
    """physical.py:66-85: 8-bit stays uint8; 2/4-bit pack along ``dim``."""

    if bits == 8:
        return codes.astype(np.uint8)
    if bits not in (2, 4):
        raise ValueError(f"Packed KIVI storage supports 2, 4, or 8 bits, got {bits}")
    dim = dim if dim >= 0 else codes.ndim + dim
    factor = 32 // bits
    moved = np.moveaxis(codes, dim, -1).astype(np.uint32)
    length = moved.shape[-1]
    padded = int(math.ceil(length / factor) * factor)
    if padded != length:
        pad = [(0, 0)] * moved.ndim
        pad[-1] = (0, padded - length)
        moved = np.pad(moved, pad)
    moved = moved.reshape(*moved.shape[:-1], -1, factor)
    shifts = (np.arange(factor, dtype=np.uint32) * bits).astype(np.uint32)
    words = np.bitwise_or.reduce(moved << shifts, axis=-1).astype(np.uint32)
    return np.ascontiguousarray(np.moveaxis(words.view(np.int32), -1, dim))


def unpack_codes(packed: np.ndarray, bits: int, dim: int, length: int) -> np.ndarray:
    """physical.py:88-104."""

    if bits == 8:
        index = [slice(None)] * packed.ndim
        index[dim] = slice(0, length)
        return packed[tuple(index)].astype(np.uint8)
    if bits not in (2, 4):
        raise ValueError(f"Packed KIVI storage supports 2, 4, or 8 bits, got {bits}")
    dim = dim if dim >= 0 else packed.ndim + dim
    factor = 32 // bits
    moved = np.moveaxis(packed, dim, -1).astype(np.int32).view(np.uint32)
    shifts = (np.arange(factor, dtype=np.uint32) * bits).astype(np.uint32)
    mask = np.uint32((1 << bits) - 1)
    unpacked = ((moved[..., None] >> shifts) & mask).reshape(*moved.shape[:-1], -1)
    unpacked = unpacked[..., :length]
    return np.ascontiguousarray(np.moveaxis(unpacked, -1, dim).astype(np.uint8))


def _quantize_groups(grouped: np.ndarray, max_code: float):
    """One group per leading index along axis 1 (physical.py:160-171)."""

    mn = grouped.min(axis=1, keepdims=True)
    mx = grouped.max(axis=1, keepdims=True)
    scale = np.maximum((mx - mn) / np.float32(max_code), FLOAT32_EPS).astype(np.float32)
    codes = np.clip(np.rint((grouped - mn) / scale), 0, max_code).astype(np.uint8)
    return codes, scale, mn


def quantize_grouped(
    data: np.ndarray,
    dtype: str,
    *,
    bits: int,
    group_dim: int,
    group_size: int,
    pack_dim: int,
):
    """physical.py:107-175: returns (packed, scale, minimum, length).

    Complete groups are vectorized as in ``_quantize_grouped``; a partial last
    group (or empty input) follows ``_quantize_grouped_reference``'s loop.
    Scale and minimum are stored in ``dtype`` (physical.py:131-132, 173-174).
    """

    data = np.asarray(data, dtype=np.float32)
    group_dim = group_dim if group_dim >= 0 else data.ndim + group_dim
    length = int(data.shape[group_dim])
    max_code = float((1 << bits) - 1)
    moved = np.moveaxis(data, group_dim, 0)
    full = (length // group_size) * group_size
    code_parts, scale_parts, min_parts = [], [], []
    if full:
        grouped = moved[:full].reshape(full // group_size, group_size, *moved.shape[1:])
        codes, scale, mn = _quantize_groups(grouped, max_code)
        code_parts.append(codes.reshape(full, *moved.shape[1:]))
        scale_parts.append(scale[:, 0])
        min_parts.append(mn[:, 0])
    if full != length:
        chunk = moved[full:][None]
        codes, scale, mn = _quantize_groups(chunk, max_code)
        code_parts.append(codes[0])
        scale_parts.append(scale[:, 0])
        min_parts.append(mn[:, 0])
    if not code_parts:
        raise ValueError("quantize_grouped needs at least one token")
    codes = np.moveaxis(np.concatenate(code_parts, axis=0), 0, group_dim)
    scale = np.moveaxis(np.concatenate(scale_parts, axis=0), 0, group_dim)
    minimum = np.moveaxis(np.concatenate(min_parts, axis=0), 0, group_dim)
    return (
        pack_codes(np.ascontiguousarray(codes), bits, pack_dim),
        np.ascontiguousarray(round_to(scale, dtype)),
        np.ascontiguousarray(round_to(minimum, dtype)),
        length,
    )


def dequantize_grouped(
    packed: np.ndarray,
    scale: np.ndarray,
    minimum: np.ndarray,
    *,
    bits: int,
    group_dim: int,
    group_size: int,
    pack_dim: int,
    length: int,
    dtype: str,
) -> np.ndarray:
    """physical.py:178-201: code * scale + minimum in fp32 (two roundings,
    no fused multiply-add), then one rounding to ``dtype``."""

    codes = unpack_codes(packed, bits, pack_dim, length).astype(np.float32)
    moved = np.moveaxis(codes, group_dim, 0)
    s = np.moveaxis(np.asarray(scale, np.float32), group_dim, 0)
    m = np.moveaxis(np.asarray(minimum, np.float32), group_dim, 0)
    group_index = np.arange(length) // group_size
    out = moved * s[group_index] + m[group_index]
    return round_to(np.moveaxis(out, 0, group_dim), dtype)


def packed_from_dense(
    key: np.ndarray,
    value: np.ndarray,
    dtype: str,
    *,
    k_bits: int,
    v_bits: int,
    group_size: int,
    residual_length: int,
) -> dict:
    """physical.py:228-332 with ``backend="reference"`` (reference layout).

    K groups and packs along tokens ([T/f, H, D]); V groups and packs along
    head_dim ([T, H, D/f]).  The residual suffix keeps ``dtype`` values.
    """

    if key.shape != value.shape or key.ndim != 3:
        raise ValueError("KIVI physical cache expects matching [tokens, kv_heads, head_dim] tensors")
    if k_bits not in (2, 4, 8) or v_bits not in (2, 4, 8):
        raise ValueError("KIVI physical cache supports 2, 4, or 8 bit payloads")
    tokens, heads, head_dim = map(int, key.shape)
    if group_size <= 0:
        raise ValueError("KIVI physical cache group_size must be positive")
    requested = min(tokens, max(0, int(residual_length)))
    quantized = ((tokens - requested) // group_size) * group_size
    out = {
        "k_bits": k_bits,
        "v_bits": v_bits,
        "group_size": group_size,
        "quantized_tokens": quantized,
        "head_dim": head_dim,
        "num_kv_heads": heads,
        "dtype": dtype,
        "residual_key": np.array(key[quantized:], dtype=np.float32),
        "residual_value": np.array(value[quantized:], dtype=np.float32),
    }
    if quantized:
        kc, ks, km, _ = quantize_grouped(
            key[:quantized], dtype, bits=k_bits, group_dim=0, group_size=group_size, pack_dim=0
        )
        vc, vs, vm, _ = quantize_grouped(
            value[:quantized], dtype, bits=v_bits, group_dim=2, group_size=group_size, pack_dim=2
        )
    else:
        kc = ks = km = vc = vs = vm = None
    out.update(
        key_code=kc, key_scale=ks, key_minimum=km, value_code=vc, value_scale=vs, value_minimum=vm
    )
    return out


def packed_dequantize(cache: dict, dtype: str | None = None):
    """physical.py:379-423 for the reference layout."""

    dtype = dtype or cache["dtype"]
    if cache["quantized_tokens"]:
        q_key = dequantize_grouped(
            cache["key_code"], cache["key_scale"], cache["key_minimum"],
            bits=cache["k_bits"], group_dim=0, group_size=cache["group_size"],
            pack_dim=0, length=cache["quantized_tokens"], dtype=dtype,
        )
        q_value = dequantize_grouped(
            cache["value_code"], cache["value_scale"], cache["value_minimum"],
            bits=cache["v_bits"], group_dim=2, group_size=cache["group_size"],
            pack_dim=2, length=cache["head_dim"], dtype=dtype,
        )
        key = np.concatenate([q_key, round_to(cache["residual_key"], dtype)], axis=0)
        value = np.concatenate([q_value, round_to(cache["residual_value"], dtype)], axis=0)
    else:
        key = round_to(cache["residual_key"], dtype)
        value = round_to(cache["residual_value"], dtype)
    return key, value


def to_b200_layout(cache: dict) -> dict:
    """The B200 layout is the reference layout with its first two axes swapped
    (head-major): K codes [H, T/f, D], K stats [H, T/G, D], V codes [H, T, D/f],
    V stats [H, T, D/G]; words are identical."""

    out = dict(cache)
    for name in ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum"):
        if cache[name] is not None:
            out[name] = np.ascontiguousarray(np.swapaxes(cache[name], 0, 1))
    return out


def _safe_group_size(length: int, group_size: int) -> int:
    """builtin.py:23-26."""

    if length <= 0:
        return 1
    return max(1, min(int(group_size), int(length)))


def fake_quant(data: np.ndarray, dtype: str, *, bits: int, dim: int, group_size: int) -> np.ndarray:
    """builtin.py:31-53 (``asymmetric_fake_quant``).

    Unlike the packed quantizer, the scale is clamped *before* the division:
    scale = max(mx - mn, eps) / max_int; the result is code*scale + mn in fp32,
    then rounded to ``dtype``.  A partial last group is allowed.
    """

    data = np.asarray(data, dtype=np.float32)
    if data.size == 0 or bits >= 16:
        return data.copy()
    if bits not in (2, 3, 4, 8):
        raise ValueError(f"Unsupported fake quant bits: {bits}")
    dim = dim if dim >= 0 else data.ndim + dim
    length = int(data.shape[dim])
    group = _safe_group_size(length, group_size)
    max_int = np.float32((1 << bits) - 1)
    moved = np.moveaxis(data, dim, 0)
    out = np.empty_like(moved)
    for start in range(0, length, group):
        stop = min(length, start + group)
        chunk = moved[start:stop]
        mn = chunk.min(axis=0, keepdims=True)
        mx = chunk.max(axis=0, keepdims=True)
        scale = (np.maximum(mx - mn, FLOAT32_EPS) / max_int).astype(np.float32)
        code = np.clip(np.rint((chunk - mn) / scale), 0, max_int).astype(np.float32)
        out[start:stop] = code * scale + mn
    return round_to(np.moveaxis(out, 0, dim), dtype)


def fake_quant_key(k: np.ndarray, dtype: str, *, bits: int, group_size: int) -> np.ndarray:
    """builtin.py:56-59: keys grouped along tokens."""

    return fake_quant(k, dtype, bits=bits, dim=0, group_size=group_size)


def fake_quant_value(v: np.ndarray, dtype: str, *, bits: int, group_size: int) -> np.ndarray:
    """builtin.py:62-65: values grouped along head_dim."""

    return fake_quant(v, dtype, bits=bits, dim=-1, group_size=group_size)
