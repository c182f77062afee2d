"""Attention fast paths over physical segments (counterpart of unicache/adapters)."""

from .attention import (
    DecodeStepGraph,
    PhysicalDecodeBatch,
    batched_long_query_attention,
    fused_h2o_decode,
    fused_mixed_decode,
    long_query_attention_summary,
    merge_attention_summaries,
)

__all__ = [
    "DecodeStepGraph",
    "PhysicalDecodeBatch",
    "batched_long_query_attention",
    "fused_h2o_decode",
    "fused_mixed_decode",
    "long_query_attention_summary",
    "merge_attention_summaries",
]
