"""Attention fast paths over physical segments: the counterparts of the
reference adapter's physical attention helpers (Superone77/UniCache,
unicache/adapters/bagel.py):

* ``merge_attention_summaries``   bagel.py:57-72 (LSE merge kernel)
* ``fused_h2o_decode``            bagel.py:1860-1901 without the per-step
                                  ``torch.cat`` of every retained H2O row
* ``fused_mixed_decode``          bagel.py:1598-1858 for q_len == 1: dense,
                                  H2O, KIVI residual and packed KIVI tokens in
                                  one decode launch, no bf16 workspace
* ``PhysicalDecodeBatch``         batched decode over many sequences (the
                                  shape of ``apply_static_physical_attention_batch``,
                                  bagel.py:773-980, for decoding)
* ``long_query_attention_summary`` multi-query attention over the same
                                  segments (bagel.py:1598-1858 with q_len > 1)
"""

from __future__ import annotations

import math

import torch

from .. import kernels
from ..storage.physical import GQAH2OCache, PackedKIVICache


def merge_attention_summaries(
    summaries: list[tuple[torch.Tensor, torch.Tensor]],
) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge normalised segment outputs using their per-row log-sum-exp."""

    return kernels.lse_merge(summaries)


def _segments_for(dense_key, dense_value, physical_segments) -> list:
    segments: list = []
    if dense_key is not None and int(dense_key.shape[0]):
        segments.append((dense_key, dense_value))
    segments.extend(physical_segments)
    return segments


class PhysicalDecodeBatch:
    """Decode attention for a batch of sequences whose physical caches are
    frozen.  The device tables are built once; ``__call__`` launches one
    kernel per decode step."""

    def __init__(self, sequences: list[list], *, num_kv_heads: int, head_dim: int = 128,
                 target_ctas: int | None = None):
        self.plan = kernels.build_decode_plan(sequences, num_kv_heads=num_kv_heads, head_dim=head_dim,
                                              target_ctas=target_ctas)

    @property
    def bytes_per_step(self) -> int:
        return self.plan.bytes_per_step

    def __call__(self, query: torch.Tensor, *, out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
        """query [B, Hq, D] bf16 -> (out [B, Hq, D] bf16, lse [B, Hq] fp32 natural log)."""

        return self.plan.run(query, out=out, lse=lse)


def _single_sequence_decode(query, segments, num_kv_heads, head_dim, owner=None, key=None):
    if int(query.shape[0]) != 1:
        raise ValueError("decode attention takes a single query token")
    plan = None
    if owner is not None:
        plans = owner.__dict__.setdefault("_decode_plans", {})
        plan = plans.get(key)
    if plan is None:
        plan = kernels.build_decode_plan([segments], num_kv_heads=num_kv_heads, head_dim=head_dim)
        if owner is not None:
            owner.__dict__["_decode_plans"][key] = plan
    out, lse = plan.run(query.to(torch.bfloat16))
    return out.to(query.dtype), lse


def fused_h2o_decode(query: torch.Tensor, dense_key: torch.Tensor, dense_value: torch.Tensor,
                     physical_segments: list[GQAH2OCache]) -> torch.Tensor:
    """Decode over [dense ‖ H2O segments] reading the compacted rows in place."""

    if not all(isinstance(s, GQAH2OCache) for s in physical_segments):
        raise ValueError("fused H2O decode takes GQAH2OCache segments")
    kv_heads = int(dense_key.shape[1]) if dense_key is not None else physical_segments[0].num_kv_heads
    out, _ = _single_sequence_decode(query, _segments_for(dense_key, dense_value, physical_segments), kv_heads,
                                     int(query.shape[-1]))
    return out


def fused_mixed_decode(query: torch.Tensor, dense_key: torch.Tensor | None, dense_value: torch.Tensor | None,
                       physical_segments: list) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode over [dense ‖ H2O ‖ packed KIVI (+ residual)] in one launch;
    returns (out [1, Hq, D], lse [1, Hq])."""

    if not physical_segments and dense_key is None:
        raise ValueError("mixed decode needs at least one segment")
    first = physical_segments[0] if physical_segments else None
    kv_heads = int(dense_key.shape[1]) if dense_key is not None else first.num_kv_heads
    return _single_sequence_decode(query, _segments_for(dense_key, dense_value, physical_segments), kv_heads,
                                   int(query.shape[-1]))


def _dequantized_segments(segments, dtype, include_residual=True):
    keys, values = [], []
    for seg in segments:
        if isinstance(seg, PackedKIVICache):
            if seg.quantized_tokens:
                k = torch.empty((seg.quantized_tokens, seg.num_kv_heads, seg.head_dim),
                                device=seg.key_code.device, dtype=dtype)
                v = torch.empty_like(k)
                seg.dequantize_range(0, seg.quantized_tokens, dtype=dtype, output_key=k, output_value=v)
                keys.append(k)
                values.append(v)
            if include_residual and int(seg.residual_key.shape[0]):
                keys.append(seg.residual_key.to(dtype))
                values.append(seg.residual_value.to(dtype))
        elif isinstance(seg, GQAH2OCache):
            keys.append(seg.key.transpose(0, 1).to(dtype))
            values.append(seg.value.transpose(0, 1).to(dtype))
        else:
            k, v = seg
            keys.append(k.to(dtype))
            values.append(v.to(dtype))
    return torch.cat(keys, dim=0), torch.cat(values, dim=0)


def long_query_attention_summary(query: torch.Tensor, segments: list, *, dense_key=None, dense_value=None,
                                 include_residual: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """Multi-query attention over physical segments: (out [Lq, Hq, D], lse [Hq, Lq]).

    Restores packed segments with the bit-exact dequant kernel and contracts
    with the library GEMM in fp32; the tensor-core long-query kernel replaces
    this path."""

    kernels.require_cuda(query, "query")
    segs = _segments_for(dense_key, dense_value, segments)
    key, value = _dequantized_segments(segs, query.dtype, include_residual=include_residual)
    lq, hq, d = map(int, query.shape)
    hkv = int(key.shape[1])
    grp = hq // hkv
    q = query.transpose(0, 1).float().reshape(hkv, grp * lq, d)
    k = key.transpose(0, 1).float()
    v = value.transpose(0, 1).float()
    logits = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(d)
    lse = torch.logsumexp(logits, dim=-1)
    probs = torch.exp(logits - lse.unsqueeze(-1))
    out = torch.matmul(probs, v).reshape(hq, lq, d).transpose(0, 1)
    return out.to(query.dtype), lse.reshape(hq, lq)
