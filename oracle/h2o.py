"""Physical GQA H2O oracle.  TEST INFRASTRUCTURE ONLY.

Restates unicache/storage/physical.py (Superone77/UniCache):

* ``select_indices``   physical.py:511-532 (heavy top-k over the history,
                       ascending, then the recent window)
* ``h2o_from_dense``   physical.py:493-547 (gather K/V/ids/scores per KV head)
* ``update_scores``    physical.py:598-610 and the operator reduction
                       unicache/operators/physical.py:63-65
* ``trim`` / ``request_budget`` / ``enforce_budget``  physical.py:612-654

Plus the budget arithmetic of the dense backend,
unicache/storage/tensor_backend.py:199-210 (Python ``round``, i.e. banker's
rounding, on ``n * ratio`` and ``target * recent_fraction``).

Tie order: ``torch.topk`` does not define which of several equal scores wins at
the cut.  The oracle (and the device kernel) use (score descending, index
ascending), which is what ``torch.topk`` returns on every untied input.  The
golden vectors carry no ties at the cut (checked when they are made).
"""

from __future__ import annotations

import numpy as np


def topk_desc_index_asc(scores: np.ndarray, k: int) -> np.ndarray:
    """Per row: indices of the k largest scores, ties broken by lower index,
    returned in ascending index order (the ``.indices.sort()`` of physical.py:519)."""

    scores = np.asarray(scores, np.float32)
    rows = []
    for row in scores:
        order = np.lexsort((np.arange(row.shape[0]), -row.astype(np.float64)))
        rows.append(np.sort(order[:k]))
    if not rows:
        return np.zeros((0, k), np.int64)
    return np.stack(rows).astype(np.int64)


def select_indices(scores: np.ndarray, target_tokens: int, recent_tokens: int):
    """physical.py:508-532.  Returns (indexes [Hkv, keep], heavy, recent)."""

    kv_heads, tokens = scores.shape
    target = min(tokens, max(1, int(target_tokens)))
    recent = min(target, max(0, int(recent_tokens)))
    heavy = target - recent
    history_end = tokens - recent
    heavy_k = min(heavy, history_end)
    if heavy_k:
        heavy_idx = topk_desc_index_asc(scores[:, :history_end], heavy_k)
    else:
        heavy_idx = np.zeros((kv_heads, 0), np.int64)
    recent_idx = np.broadcast_to(np.arange(tokens - recent, tokens, dtype=np.int64), (kv_heads, recent))
    return np.concatenate([heavy_idx, recent_idx], axis=1), heavy, recent


def h2o_from_dense(key, value, logical_token_ids, scores, target_tokens, recent_tokens):
    """physical.py:493-547: key/value [T, Hkv, D] -> per-head [Hkv, keep, D]."""

    key = np.asarray(key)
    value = np.asarray(value)
    if key.shape != value.shape or key.ndim != 3:
        raise ValueError("Physical H2O expects matching [tokens, kv_heads, head_dim] tensors")
    tokens, kv_heads, _ = key.shape
    if tuple(scores.shape) != (kv_heads, tokens):
        raise ValueError("Physical H2O scores must be [kv_heads, segment_tokens]")
    idx, heavy, recent = select_indices(np.asarray(scores, np.float32), target_tokens, recent_tokens)
    src_k = key.transpose(1, 0, 2)
    src_v = value.transpose(1, 0, 2)
    gathered_k = np.take_along_axis(src_k, idx[..., None], axis=1)
    gathered_v = np.take_along_axis(src_v, idx[..., None], axis=1)
    ids = np.asarray(logical_token_ids, np.int64)[idx]
    kept_scores = np.take_along_axis(np.asarray(scores, np.float32), idx, axis=1)
    return {
        "key": gathered_k,
        "value": gathered_v,
        "logical_token_ids": ids,
        "cumulative_scores": kept_scores.astype(np.float32),
        "original_tokens": tokens,
        "heavy_tokens": heavy,
        "recent_tokens": recent,
        "indexes": idx,
    }


def reduce_probabilities(probabilities: np.ndarray, kv_heads: int) -> np.ndarray:
    """operators/physical.py:63-65 and physical.py:607-609:
    probs [Hq, Lq, N] -> per-KV-head received attention [Hkv, N] (float32 sum
    over queries, then over the query heads of each group)."""

    hq, _, n = probabilities.shape
    if hq % kv_heads:
        raise ValueError("Query heads must be divisible by KV heads for GQA H2O")
    groups = hq // kv_heads
    per_head = np.asarray(probabilities, np.float64).sum(axis=1)
    return per_head.reshape(kv_heads, groups, n).sum(axis=1)


def trim(cache: dict, target_tokens: int, recent_tokens: int) -> dict:
    """physical.py:624-654 on a dict made by ``h2o_from_dense``."""

    retained = cache["key"].shape[1]
    target = min(retained, max(1, int(target_tokens)))
    if target >= retained:
        return cache
    recent = min(target, max(0, int(recent_tokens)))
    heavy = target - recent
    history_end = retained - recent
    rows = []
    for head in range(cache["key"].shape[0]):
        recent_idx = np.arange(retained - recent, retained, dtype=np.int64)
        if heavy:
            heavy_idx = topk_desc_index_asc(
                cache["cumulative_scores"][head : head + 1, :history_end], min(heavy, history_end)
            )[0]
        else:
            heavy_idx = np.zeros(0, np.int64)
        rows.append(np.concatenate([heavy_idx, recent_idx]))
    idx = np.stack(rows)
    out = dict(cache)
    out["key"] = np.take_along_axis(cache["key"], idx[..., None], axis=1)
    out["value"] = np.take_along_axis(cache["value"], idx[..., None], axis=1)
    out["logical_token_ids"] = np.take_along_axis(cache["logical_token_ids"], idx, axis=1)
    out["cumulative_scores"] = np.take_along_axis(cache["cumulative_scores"], idx, axis=1)
    return out


def request_budget(cache: dict, target_tokens: int, recent_tokens: int):
    """physical.py:615-622; returns (effective, new cache, shortfall increment)."""

    retained = cache["key"].shape[1]
    requested = max(1, int(target_tokens))
    effective = min(requested, retained)
    recent = min(effective, max(0, int(recent_tokens)))
    heavy = effective - recent
    out = dict(cache)
    out["recent_tokens"] = recent
    out["heavy_tokens"] = heavy
    return effective, trim(out, heavy + recent, recent), requested - effective


def budget_from_ratio(segment_tokens: int, ratio: float, recent_fraction: float):
    """tensor_backend.py:199-210 (Python round = round-half-even)."""

    target = max(1, int(round(int(segment_tokens) * float(ratio))))
    recent = int(round(int(target) * float(recent_fraction)))
    return target, recent
