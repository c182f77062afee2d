"""Dense-cache compaction oracle.  TEST INFRASTRUCTURE ONLY.

Restates ``TensorCacheStorageBackend.compact`` (Superone77/UniCache,
unicache/storage/tensor_backend.py:33-100): per packed sample, keep the rows
whose mask is true, preserving order, and report the compacted sample lengths.
"""

from __future__ import annotations

import numpy as np


def compact(key, value, key_type_ids, lengths, keep_masks):
    key = np.asarray(key)
    value = np.asarray(value)
    if key.shape != value.shape or key.ndim != 3:
        raise ValueError("Tensor cache backend expects matching [tokens, heads, head_dim] KV tensors")
    if sum(lengths) != key.shape[0]:
        raise ValueError("Packed sample lengths do not match the cache token count")
    if len(keep_masks) != len(lengths):
        raise ValueError("Tensor cache backend requires one keep mask per packed sample")
    rows = []
    offset = 0
    new_lengths = []
    for length, mask in zip(lengths, keep_masks):
        mask = np.asarray(mask, bool)
        if mask.ndim != 1 or mask.shape[0] != length:
            raise ValueError("Keep mask does not match its packed sample length")
        rows.append(offset + np.nonzero(mask)[0])
        new_lengths.append(int(mask.sum()))
        offset += length
    index = np.concatenate(rows) if rows else np.zeros(0, np.int64)
    types = None if key_type_ids is None else np.asarray(key_type_ids)[index]
    return key[index], value[index], types, new_lengths
