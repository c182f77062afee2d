"""B200 dispatch for packed KIVI segments: the counterpart of the reference's
``unicache/storage/kivi_cuda.py`` (Superone77/UniCache), with one backend only.

The reference picks between the external KIVI GEMV and Triton kernels by
query length and environment variables (kivi_cuda.py:26-34); here every call
goes to ``libunicache_b200.so``.
"""

from __future__ import annotations

import dataclasses
import math
from typing import TYPE_CHECKING, Callable

import torch

from .. import kernels

if TYPE_CHECKING:
    from .physical import PackedKIVICache


def _plans(cache) -> dict:
    plans = cache.__dict__.get("_decode_plans")
    if plans is None:
        plans = {}
        cache.__dict__["_decode_plans"] = plans
    return plans


def quantize_kivi_b200(key: torch.Tensor, value: torch.Tensor, *, k_bits: int, v_bits: int, group_size: int):
    """Pack K along tokens and V along channels in the b200 layout
    (the role of quantize_kivi_native, kivi_cuda.py:157-190)."""

    if key.shape != value.shape or key.dim() != 3:
        raise ValueError("KIVI packing expects matching [tokens, heads, dim] KV")
    return kernels.kivi_pack_kv(key, value, k_bits=k_bits, v_bits=v_bits, group_size=group_size)


def dequantize_kivi_chunk(
    cache: "PackedKIVICache",
    *,
    start: int,
    stop: int,
    dtype: torch.dtype,
    output_key: torch.Tensor | None = None,
    output_value: torch.Tensor | None = None,
    output_offset: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """kivi_cuda.py:58-93 / kivi_triton.py:690-770: restore quantized tokens
    [start, stop) into a bounded tile, optionally inside a caller workspace at
    ``output_offset``, bit-exact with ``cache.dequantize()``."""

    start = max(0, int(start))
    stop = min(int(stop), int(cache.quantized_tokens))
    if stop <= start:
        empty = cache.residual_key[:0].to(dtype)
        return empty, empty
    count = stop - start
    heads, head_dim = cache.num_kv_heads, cache.head_dim
    device = cache.key_code.device
    output_offset = int(output_offset)
    if output_key is None or output_value is None:
        if output_key is not None or output_value is not None:
            raise ValueError("Both KIVI output buffers must be provided together")
        output_offset = 0
        output_key = torch.empty((count, heads, head_dim), device=device, dtype=dtype)
        output_value = torch.empty_like(output_key)
    if (
        output_key.dim() != 3
        or output_value.shape != output_key.shape
        or tuple(output_key.shape[1:]) != (heads, head_dim)
        or output_key.device != device
        or output_value.device != device
        or output_key.dtype != dtype
        or output_value.dtype != dtype
        or output_offset < 0
        or output_offset + count > int(output_key.shape[0])
    ):
        raise ValueError("KIVI dequantization output workspace has an invalid layout")
    key_view = output_key[output_offset:output_offset + count]
    value_view = output_value[output_offset:output_offset + count]
    cache.dequantize_range(start, stop, dtype=dtype, output_key=key_view, output_value=value_view)
    return key_view, value_view


def decode_plan_for(segments: list, *, num_kv_heads: int, head_dim: int, cache_key=None, owner=None):
    """A decode plan over one sequence's segments, cached on ``owner``."""

    if owner is not None:
        plans = _plans(owner)
        plan = plans.get(cache_key)
        if plan is None:
            plan = kernels.build_decode_plan([segments], num_kv_heads=num_kv_heads, head_dim=head_dim)
            plans[cache_key] = plan
        return plan
    return kernels.build_decode_plan([segments], num_kv_heads=num_kv_heads, head_dim=head_dim)


def packed_kivi_quantized_attention_summary(
    cache: "PackedKIVICache", query: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    """kivi_cuda.py:96-120: normalised output [Lq, Hq, D] (query dtype) and
    natural-log LSE [Hq, Lq] over the packed quantized prefix only."""

    if not cache.quantized_tokens:
        raise ValueError("Packed KIVI summary requires a non-empty quantized prefix")
    kernels.require_cuda(query, "query")
    if query.dim() != 3:
        raise ValueError("query must be [queries, q_heads, head_dim]")
    queries = int(query.shape[0])
    if queries == 1:
        prefix = dataclasses.replace(cache, residual_key=cache.residual_key[:0],
                                     residual_value=cache.residual_value[:0])
        plan = decode_plan_for([prefix], num_kv_heads=cache.num_kv_heads, head_dim=cache.head_dim,
                               cache_key="prefix", owner=cache)
        plan.keepalive.append(prefix)
        out, lse = plan.run(query.to(torch.bfloat16).reshape(1, query.shape[1], query.shape[2]))
        return out.reshape(query.shape).to(query.dtype), lse.reshape(-1, 1)
    from ..adapters.attention import long_query_attention_summary

    return long_query_attention_summary(query, [cache], include_residual=False)


def packed_kivi_attention_parts(
    cache: "PackedKIVICache",
    query: torch.Tensor,
) -> tuple[torch.Tensor, Callable[[torch.Tensor], torch.Tensor]]:
    """kivi_cuda.py:238-329: logits [Hq, Lq, T+R] (fp32, scaled by 1/sqrt(D))
    and an AV closure.  This is the generic path used when probabilities must
    be materialised.  Both halves run on this library's kernels, restoring
    the codes tile by tile in shared memory (no dequantized copy of the
    segment, no library GEMM).  Fused paths never call it."""

    kernels.require_cuda(query, "query")
    if query.dim() != 3 or int(query.shape[-1]) != cache.head_dim or cache.head_dim != 128:
        raise ValueError("query must be [queries, q_heads, 128]")
    repeat = int(query.shape[1]) // cache.num_kv_heads
    if repeat * cache.num_kv_heads != int(query.shape[1]):
        raise ValueError("Query heads must be divisible by KIVI KV heads")
    if query.dtype != torch.bfloat16 or cache.residual_key.dtype != torch.bfloat16:
        raise ValueError("the b200 attention parts take a bfloat16 query and cache")
    if cache.quantized_tokens and cache.key_scale.dtype != torch.bfloat16:
        raise ValueError("the b200 attention parts read bfloat16 statistics")
    q = query.contiguous()
    lq, hq = int(q.shape[0]), int(q.shape[1])
    total = cache.quantized_tokens + int(cache.residual_key.shape[0])
    packed = cache.quantized_tokens > 0
    rk, rv = cache.residual_key, cache.residual_value
    logits = torch.empty((hq, lq, total), device=q.device, dtype=torch.float32)
    kernels.call("ucb_kivi_attention_logits", q.data_ptr(), lq, hq, cache.num_kv_heads,
                 cache.key_code.data_ptr() if packed else None, cache.key_scale.data_ptr() if packed else None,
                 cache.key_minimum.data_ptr() if packed else None, cache.key_code.stride(0) if packed else 0,
                 cache.key_scale.stride(0) if packed else 0, rk.data_ptr() if rk.numel() else None,
                 rk.stride(0), rk.stride(1), cache.quantized_tokens, int(rk.shape[0]), cache.k_bits,
                 cache.group_size, 1.0 / math.sqrt(cache.head_dim), logits.data_ptr(), kernels.stream_of(q))

    def apply_value(probabilities: torch.Tensor) -> torch.Tensor:
        kernels.require_cuda(probabilities, "probabilities")
        if tuple(probabilities.shape) != (hq, lq, total):
            raise ValueError("GQA AV probability key width must match value tokens")
        p = probabilities.contiguous()
        out = torch.empty((hq, lq, cache.head_dim), device=p.device, dtype=torch.bfloat16)
        kernels.call("ucb_kivi_attention_apply", p.data_ptr(), kernels.dtype_code(p.dtype), lq, hq,
                     cache.num_kv_heads, cache.value_code.data_ptr() if packed else None,
                     cache.value_scale.data_ptr() if packed else None,
                     cache.value_minimum.data_ptr() if packed else None,
                     cache.value_code.stride(0) if packed else 0, cache.value_scale.stride(0) if packed else 0,
                     rv.data_ptr() if rv.numel() else None, rv.stride(0), rv.stride(1), cache.quantized_tokens,
                     int(rv.shape[0]), cache.v_bits, cache.group_size, out.data_ptr(), kernels.stream_of(p))
        return out

    return logits, apply_value
