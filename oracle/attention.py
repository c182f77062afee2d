"""GQA attention and LSE-merge oracle.  TEST INFRASTRUCTURE ONLY.

Restates (Superone77/UniCache):

* ``gqa_query_key_logits`` / ``gqa_probability_value``
  unicache/storage/physical.py:20-63 (native GQA, no repeated KV heads)
* ``attention_summary`` -- softmax attention returning the normalised output
  and the per-row log-sum-exp, the contract of ``flash_attention_summary`` and
  ``packed_kivi_quantized_attention_summary``
  (unicache/adapters/bagel.py:75-95, unicache/storage/kivi_cuda.py:96-120)
* ``merge_attention_summaries`` unicache/adapters/bagel.py:57-72
* ``mixed_attention`` -- attention over [dense ‖ physical segments], the
  semantics of ``_run_fused_mixed_attention`` / ``_run_fused_h2o_attention``
  (bagel.py:1598-1901) and of the explicit references in
  tests/test_physical.py:1546-1615 and :1416-1497.

All arithmetic is float64 over the storage values (bf16/fp16/fp32 carriers),
i.e. the exact result of the reference's algorithm; device kernels are
compared to it with a stated tolerance.
"""

from __future__ import annotations

import math

import numpy as np


def gqa_query_key_logits(query: np.ndarray, key: np.ndarray) -> np.ndarray:
    """physical.py:20-39: query [Lq, Hq, D], key [N, Hkv, D] -> [Hq, Lq, N]."""

    if query.ndim != 3 or key.ndim != 3:
        raise ValueError("GQA QK expects [tokens, heads, head_dim] tensors")
    hq, hkv = query.shape[1], key.shape[1]
    if hq % hkv:
        raise ValueError("GQA query heads must be divisible by KV heads")
    groups = hq // hkv
    q = np.asarray(query, np.float64).transpose(1, 0, 2).reshape(hkv, groups, query.shape[0], -1)
    k = np.asarray(key, np.float64).transpose(1, 0, 2)[:, None]
    return (q @ k.transpose(0, 1, 3, 2)).reshape(hq, query.shape[0], key.shape[0])


def gqa_probability_value(probabilities: np.ndarray, value: np.ndarray) -> np.ndarray:
    """physical.py:42-63: probs [Hq, Lq, N], value [N, Hkv, D] -> [Hq, Lq, D]."""

    hq, lq, n = probabilities.shape
    hkv = value.shape[1]
    if hq % hkv:
        raise ValueError("GQA probability heads must be divisible by KV heads")
    groups = hq // hkv
    p = np.asarray(probabilities, np.float64).reshape(hkv, groups, lq, n)
    v = np.asarray(value, np.float64).transpose(1, 0, 2)[:, None]
    return (p @ v).reshape(hq, lq, value.shape[-1])


def attention_summary(query: np.ndarray, key: np.ndarray, value: np.ndarray):
    """Softmax attention with scale 1/sqrt(D): returns (o [Lq, Hq, D], lse [Hq, Lq])."""

    logits = gqa_query_key_logits(query, key) / math.sqrt(query.shape[-1])
    row_max = logits.max(axis=-1, keepdims=True)
    weights = np.exp(logits - row_max)
    denom = weights.sum(axis=-1, keepdims=True)
    probs = weights / denom
    lse = (row_max + np.log(denom))[..., 0]
    out = gqa_probability_value(probs, value).transpose(1, 0, 2)
    return out, lse


def attention_probabilities(query: np.ndarray, key: np.ndarray) -> np.ndarray:
    logits = gqa_query_key_logits(query, key) / math.sqrt(query.shape[-1])
    logits = logits - logits.max(axis=-1, keepdims=True)
    weights = np.exp(logits)
    return weights / weights.sum(axis=-1, keepdims=True)


def merge_attention_summaries(summaries):
    """bagel.py:57-72: o = sum_i exp(lse_i - logsumexp_i lse_i) * o_i."""

    if not summaries:
        raise ValueError("At least one attention summary is required")
    lses = np.stack([np.asarray(lse, np.float64) for _, lse in summaries], axis=0)
    peak = lses.max(axis=0)
    total = peak + np.log(np.exp(lses - peak).sum(axis=0))
    out = np.zeros_like(np.asarray(summaries[0][0], np.float64))
    for o, lse in summaries:
        weight = np.exp(np.asarray(lse, np.float64) - total).T[..., None]
        out = out + np.asarray(o, np.float64) * weight
    return out, total


def mixed_attention(query: np.ndarray, keys: list, values: list):
    """Attention over the concatenation of several [N_i, Hkv, D] segments."""

    key = np.concatenate([np.asarray(k, np.float32) for k in keys], axis=0)
    value = np.concatenate([np.asarray(v, np.float32) for v in values], axis=0)
    return attention_summary(query, key, value)
