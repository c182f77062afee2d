"""Seeded synthetic KV caches with the benchmark's value distribution.

K, V ~ N(0, 1); four key channels (the same four for every KV head, chosen by
``torch.randperm(head_dim, generator=seed)[:4]``) are scaled by 10, mimicking
the outlier channels KIVI's per-channel key quantization is designed for.
Generation runs on the CPU generator so every machine produces identical
tensors for a seed; the result is moved to ``device``.
"""

from __future__ import annotations

import torch


def outlier_channels(head_dim: int, seed: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(int(seed))
    return torch.randperm(head_dim, generator=gen)[:4]


def make_kv(tokens: int, kv_heads: int, head_dim: int, *, seed: int, dtype=torch.bfloat16, device="cpu",
            outliers: bool = True):
    gen = torch.Generator().manual_seed(int(seed) + 1)
    key = torch.randn(tokens, kv_heads, head_dim, generator=gen, dtype=torch.float32)
    value = torch.randn(tokens, kv_heads, head_dim, generator=gen, dtype=torch.float32)
    if outliers:
        key[:, :, outlier_channels(head_dim, seed)] *= 10.0
    return key.to(dtype).to(device), value.to(dtype).to(device)


def make_query(batch: int, q_heads: int, head_dim: int, *, seed: int, dtype=torch.bfloat16, device="cpu"):
    gen = torch.Generator().manual_seed(int(seed) + 7919)
    return torch.randn(batch, q_heads, head_dim, generator=gen, dtype=torch.float32).to(dtype).to(device)
