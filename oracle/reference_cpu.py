"""The reference's own CPU decode path, restated in torch (CPU) for the timed
baseline.  TEST INFRASTRUCTURE ONLY: ``bench.py``'s CPU legs time it; nothing
in the package imports it.

The reference (Superone77/UniCache) is Python and cannot travel to the GPU
box, so this module restates, operation for operation and dtype for dtype,
what its ``backend="reference"`` packed cache does for one decode token:

* ``unpack_codes``      unicache/storage/physical.py:86-104 (shift + mask of
                        every int32 word, then the [..., :length] slice)
* ``dequantize_grouped`` physical.py:178-201 (a Python loop over the groups,
                        code * scale + minimum in fp32, cast to the dtype)
* ``dequantize``        physical.py:379-423 (keys grouped and packed along
                        tokens, values along channels, then the residual)
* ``gqa_logits`` / ``gqa_apply`` physical.py:20-63 (fp32 logits, probabilities
                        cast to the value dtype for the AV product)
* ``decode``            attention_parts + softmax + apply_value
                        (physical.py:452-475; the adapter's softmax in fp32,
                        adapters/bagel.py:1205-1243)

Inputs are the reference layout (``PackedKIVICache.reference_layout()`` or
``oracle.kivi.packed_from_dense``): key codes [T/f, H, D] int32, key stats
[T/G, H, D], value codes [T, H, D/f], value stats [T, H, D/G], bf16 residual.
"""

from __future__ import annotations

import math

import torch


def unpack_codes(packed: torch.Tensor, bits: int, dim: int, length: int) -> torch.Tensor:
    dim = dim if dim >= 0 else packed.dim() + dim
    factor = 32 // bits
    moved = packed.movedim(dim, -1).to(torch.int32)
    shifts = torch.arange(factor, dtype=torch.int32) * bits
    unpacked = ((moved.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)).reshape(*moved.shape[:-1], -1)
    return unpacked[..., :length].movedim(-1, dim).to(torch.uint8).contiguous()


def dequantize_grouped(packed, scale, minimum, *, bits, group_dim, group_size, pack_dim, length, dtype):
    codes = unpack_codes(packed, bits, pack_dim, length).float()
    chunks = []
    for group_index, start in enumerate(range(0, length, group_size)):
        stop = min(length, start + group_size)
        index = [slice(None)] * codes.dim()
        index[group_dim] = slice(start, stop)
        stat = [slice(None)] * scale.dim()
        stat[group_dim] = group_index
        chunks.append(codes[tuple(index)] * scale[tuple(stat)].unsqueeze(group_dim).float()
                      + minimum[tuple(stat)].unsqueeze(group_dim).float())
    return torch.cat(chunks, dim=group_dim).to(dtype)


def dequantize(cache: dict, dtype=torch.bfloat16):
    q_key = dequantize_grouped(cache["key_code"], cache["key_scale"], cache["key_minimum"], bits=cache["k_bits"],
                               group_dim=0, group_size=cache["group_size"], pack_dim=0,
                               length=cache["quantized_tokens"], dtype=dtype)
    q_value = dequantize_grouped(cache["value_code"], cache["value_scale"], cache["value_minimum"],
                                 bits=cache["v_bits"], group_dim=2, group_size=cache["group_size"], pack_dim=2,
                                 length=cache["head_dim"], dtype=dtype)
    key = torch.cat([q_key, cache["residual_key"].to(dtype)], dim=0)
    value = torch.cat([q_value, cache["residual_value"].to(dtype)], dim=0)
    return key, value


def gqa_logits(query: torch.Tensor, key: torch.Tensor) -> torch.Tensor:
    hq, hkv = int(query.shape[1]), int(key.shape[1])
    groups = hq // hkv
    grouped_query = query.transpose(0, 1).reshape(hkv, groups, int(query.shape[0]), int(query.shape[-1]))
    grouped_key = key.transpose(0, 1).unsqueeze(1)
    logits = torch.matmul(grouped_query.float(), grouped_key.float().transpose(-1, -2))
    return logits.reshape(hq, int(query.shape[0]), int(key.shape[0]))


def gqa_apply(probabilities: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
    hq, hkv = int(probabilities.shape[0]), int(value.shape[1])
    groups = hq // hkv
    grouped = probabilities.reshape(hkv, groups, int(probabilities.shape[1]), int(probabilities.shape[2]))
    out = torch.matmul(grouped.to(value.dtype), value.transpose(0, 1).unsqueeze(1))
    return out.reshape(hq, int(probabilities.shape[1]), int(value.shape[-1]))


def decode(cache: dict, query: torch.Tensor) -> torch.Tensor:
    """One decode token: query [1, Hq, D] bf16 -> output [1, Hq, D]."""

    key, value = dequantize(cache, dtype=query.dtype)
    logits = gqa_logits(query, key) / math.sqrt(query.shape[-1])
    probs = torch.softmax(logits, dim=-1).to(value.dtype)
    return gqa_apply(probs, value).transpose(0, 1)


def cache_from_layout(layout: dict, *, k_bits: int, v_bits: int, group_size: int, quantized_tokens: int,
                      head_dim: int) -> dict:
    """Bundle reference-layout tensors (CPU) with the cache's parameters."""

    out = {name: t.cpu() for name, t in layout.items()}
    out.update(k_bits=k_bits, v_bits=v_bits, group_size=group_size, quantized_tokens=quantized_tokens,
               head_dim=head_dim)
    return out
