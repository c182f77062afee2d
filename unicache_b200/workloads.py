"""Seeded builders of the benchmark configurations' caches, assembled through
the public API (the same calls an engine makes), shared by ``bench.py`` and
the parity tests.

Config 4 (an image-editing layer, the shape the reference's long-query patch
targets, unicache/adapters/bagel.py:1598-1858): 28 query / 4 KV heads,
head_dim 128, bf16 K, V ~ N(0, 1) with 4 outlier key channels x10.  The cache
holds 256 instruction tokens and 4900 ViT tokens, each compressed by H2O to
20% (51 and 980 per KV head, scored by the attention of the current 1024-token
latent block over the full dense cache: the reference's "full_kv_first_call"
observation, operators/physical.py:51-101), 1024 source-VAE tokens in 2-bit
KIVI, group 32, with a 32-token bf16 residual (992 packed), and 16 boundary
tokens in bf16; the latent block's own 1024 keys/values stay dense.  The
query is the latent block: Lq = 1024 positions x 28 heads.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import kernels
from .adapters.attention import long_query_attention_summary
from .storage.physical import GQAH2OCache, PackedKIVICache
from .synthetic import make_kv, make_query

CONFIG4 = {"instruction": 256, "vit": 4900, "vae": 1024, "boundary": 16, "latent": 1024, "lq": 1024,
           "q_heads": 28, "kv_heads": 4, "head_dim": 128, "ratio": 0.2, "recent_fraction": 0.25,
           "bits": 2, "group": 32, "residual": 32}


def h2o_budget(tokens: int, ratio: float, recent_fraction: float) -> tuple[int, int]:
    """(target, recent) per KV head, as the reference's storage backend
    computes them (Python rounding, tensor_backend.py:199-210)."""

    target = max(1, int(round(tokens * ratio)))
    return target, int(round(target * recent_fraction))


@dataclass
class Config4Layer:
    query: torch.Tensor            # [Lq, Hq, D] bf16
    dense: dict                    # name -> (key, value) [N, Hkv, D] bf16, the raw segments
    scores: dict                   # name -> [Hkv, N] fp32 H2O scores of the H2O segments
    first_call_lse: torch.Tensor   # [Hq, Lq] LSE of the latent block over the full dense cache
    segments: list                 # [instruction H2O, ViT H2O, VAE packed]
    dense_key: torch.Tensor        # boundary + latent rows [16 + 1024, Hkv, D]
    dense_value: torch.Tensor

    @property
    def key_tokens(self) -> int:
        n = int(self.dense_key.shape[0])
        for seg in self.segments:
            n += seg.retained_tokens if isinstance(seg, GQAH2OCache) else \
                seg.quantized_tokens + int(seg.residual_key.shape[0])
        return n


def config4_layer(device, seed: int = 1) -> Config4Layer:
    c = CONFIG4
    hkv, d = c["kv_heads"], c["head_dim"]
    names = ("instruction", "vit", "vae", "boundary", "latent")
    dense = {name: make_kv(c[name], hkv, d, seed=seed * 10 + i, device=device) for i, name in enumerate(names)}
    query = make_query(c["lq"], c["q_heads"], d, seed=seed, device=device)
    # First call: the latent block attends to the whole dense cache; its LSE
    # drives the H2O scores of the instruction and ViT segments.
    full_k = torch.cat([dense[n][0] for n in names])
    full_v = torch.cat([dense[n][1] for n in names])
    _, lse = long_query_attention_summary(query, [], dense_key=full_k, dense_value=full_v)
    scale = 1.0 / math.sqrt(d)
    scores, segments = {}, []
    for name in ("instruction", "vit"):
        k, v = dense[name]
        scores[name] = kernels.h2o_scores(query, k, lse, kv_heads=hkv, softmax_scale=scale)
        target, recent = h2o_budget(c[name], c["ratio"], c["recent_fraction"])
        segments.append(GQAH2OCache.from_dense(k, v, logical_token_ids=torch.arange(c[name], device=device),
                                               token_type_id=1, per_kv_head_scores=scores[name],
                                               target_tokens=target, recent_tokens=recent, selection_frozen=True))
    vk, vv = dense["vae"]
    segments.append(PackedKIVICache.from_dense(vk, vv, logical_token_ids=torch.arange(c["vae"], device=device),
                                               token_type_id=3, k_bits=c["bits"], v_bits=c["bits"],
                                               group_size=c["group"], residual_length=c["residual"]))
    dense_key = torch.cat([dense["boundary"][0], dense["latent"][0]])
    dense_value = torch.cat([dense["boundary"][1], dense["latent"][1]])
    return Config4Layer(query, dense, scores, lse, segments, dense_key, dense_value)
