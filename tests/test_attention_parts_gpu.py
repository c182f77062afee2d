"""PackedKIVICache.attention_parts on this library's kernels (the reference's
packed_kivi_attention_parts, unicache/storage/kivi_cuda.py:238-329; its CPU
layout computes the same from dequantize(), storage/physical.py:452-475).

* logits against the float64 oracle over the restored keys: the kernel's
  products are exact bf16 x bf16 in fp32, so within 1e-4 relative of the
  largest logit;
* apply_value against the oracle's probabilities x restored values within
  the north-star bound (max-abs 2e-2, mean-abs 1e-3), for bf16 and fp32
  probabilities (both rounded to bf16 first, as the reference casts them);
* the full generic path (logits -> softmax -> apply) against the oracle's
  attention, for 2/4/8-bit caches, groups 32/64/128, decode and multi-query
  blocks, and an appended cache whose packed tensors are capacity views."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import attention, kivi
from unicache_b200 import PackedKIVICache, kernels
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import assert_attention_close, host, need_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kb,vb,group,tokens,residual,lq", [
    (2, 2, 32, 1000, 40, 1), (4, 2, 64, 777, 64, 9), (2, 4, 128, 1500, 16, 33), (8, 8, 32, 300, 20, 5),
])
def test_attention_parts_match_oracle(kb, vb, group, tokens, residual, lq):
    need_gpu()
    key, value = make_kv(tokens, 4, 128, seed=kb + vb + group, device="cuda")
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(tokens, device="cuda"),
                                       token_type_id=3, k_bits=kb, v_bits=vb, group_size=group,
                                       residual_length=residual)
    ref = kivi.packed_from_dense(host(key), host(value), "bfloat16", k_bits=kb, v_bits=vb, group_size=group,
                                 residual_length=residual)
    rk, rv = kivi.packed_dequantize(ref)
    query = make_query(lq, 28, 128, seed=lq, device="cuda")
    logits, apply_value = cache.attention_parts(query)
    e_logits = attention.gqa_query_key_logits(host(query), rk) / math.sqrt(128)
    got = host(logits).astype(np.float64)
    assert got.shape == e_logits.shape
    assert np.abs(got - e_logits).max() <= 1e-4 * np.abs(e_logits).max()
    probs = torch.softmax(logits, dim=-1)
    for p in (probs, probs.to(torch.bfloat16)):
        out = apply_value(p)
        torch.cuda.synchronize()
        expect = attention.gqa_probability_value(host(p.to(torch.bfloat16)), rv)
        assert_attention_close(out, expect, what=f"apply_value {p.dtype}")
    e_out, _ = attention.attention_summary(host(query), rk, rv)
    assert_attention_close(apply_value(probs).transpose(0, 1), e_out, what="generic path")
    assert kernels.device_status() == 0


def test_attention_parts_on_an_appended_cache():
    need_gpu()
    key, value = make_kv(900, 4, 128, seed=3, device="cuda")
    cache = PackedKIVICache.from_dense(key[:100], value[:100], logical_token_ids=torch.arange(100, device="cuda"),
                                       token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=32)
    for t in range(100, 900, 50):
        cache.append(key[t:t + 50], value[t:t + 50], logical_token_ids=torch.arange(t, t + 50, device="cuda"))
    rebuilt = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(900, device="cuda"),
                                         token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=32)
    query = make_query(3, 28, 128, seed=4, device="cuda")
    la, aa = cache.attention_parts(query)
    lb, ab = rebuilt.attention_parts(query)
    p = torch.softmax(la, dim=-1)
    torch.cuda.synchronize()
    assert torch.equal(la, lb) and torch.equal(aa(p), ab(p))
