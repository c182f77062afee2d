"""Streaming KIVI append: a cache grown token by token (and in ragged chunks)
equals PackedKIVICache.from_dense over the whole sequence with the same
residual length, bit for bit, and decodes identically."""

from __future__ import annotations

import pytest
import torch

from unicache_b200 import PackedKIVICache, PhysicalDecodeBatch, kernels
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import need_gpu

pytestmark = pytest.mark.gpu

FIELDS = ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum",
          "residual_key", "residual_value", "logical_token_ids")


def _from_dense(key, value, stop, kb, vb, group, residual):
    return PackedKIVICache.from_dense(key[:stop], value[:stop], logical_token_ids=torch.arange(stop, device="cuda"),
                                      token_type_id=3, k_bits=kb, v_bits=vb, group_size=group,
                                      residual_length=residual)


def _assert_same(a, b):
    assert a.quantized_tokens == b.quantized_tokens
    for name in FIELDS:
        x, y = getattr(a, name), getattr(b, name)
        assert (x is None) == (y is None), name
        if x is not None:
            assert x.shape == y.shape and torch.equal(x, y), name


@pytest.mark.parametrize("kb,vb,group,residual,start,chunks", [
    (2, 2, 32, 32, 40, [1] * 70 + [5, 17, 64, 3]),
    (4, 2, 64, 128, 0, [1, 100, 200, 1, 64, 31]),
    (2, 4, 128, 16, 300, [129, 1, 1, 255]),
    (8, 8, 32, 0, 33, [31, 32, 1, 96]),
])
def test_append_equals_from_dense(kb, vb, group, residual, start, chunks):
    need_gpu()
    total = start + sum(chunks)
    key, value = make_kv(total, 4, 128, seed=kb * 100 + group, device="cuda")
    cache = _from_dense(key, value, start, kb, vb, group, residual) if start else PackedKIVICache.from_dense(
        key[:1], value[:1], logical_token_ids=torch.arange(1, device="cuda"), token_type_id=3, k_bits=kb, v_bits=vb,
        group_size=group, residual_length=residual)
    t = start if start else 1
    chunks = list(chunks)
    if not start:
        chunks[0] -= 1
    packed = 0
    for n in chunks:
        if n == 0:
            continue
        packed += cache.append(key[t:t + n], value[t:t + n], logical_token_ids=torch.arange(t, t + n, device="cuda"))
        t += n
        _assert_same(cache, _from_dense(key, value, t, kb, vb, group, residual))
    assert t == total and packed == cache.quantized_tokens - _from_dense(key, value, start or 1, kb, vb, group,
                                                                         residual).quantized_tokens


def test_appended_cache_decodes_like_the_rebuilt_one():
    need_gpu()
    key, value = make_kv(2000, 4, 128, seed=5, device="cuda")
    cache = _from_dense(key, value, 1500, 2, 2, 32, 64)
    for t in range(1500, 2000, 25):
        cache.append(key[t:t + 25], value[t:t + 25], logical_token_ids=torch.arange(t, t + 25, device="cuda"))
    query = make_query(1, 28, 128, seed=6, device="cuda")
    out_a, lse_a = PhysicalDecodeBatch([[cache]], num_kv_heads=4)(query)
    out_b, lse_b = PhysicalDecodeBatch([[_from_dense(key, value, 2000, 2, 2, 32, 64)]], num_kv_heads=4)(query)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    assert kernels.device_status() == 0


def test_append_rejects_mismatched_tokens():
    need_gpu()
    key, value = make_kv(100, 4, 128, seed=7, device="cuda")
    cache = _from_dense(key, value, 64, 2, 2, 32, 16)
    with pytest.raises(ValueError):
        cache.append(key[64:70, :2], value[64:70, :2], logical_token_ids=torch.arange(6, device="cuda"))
    with pytest.raises(ValueError):
        cache.append(key[64:70], value[64:70], logical_token_ids=torch.arange(5, device="cuda"))


def test_flushes_write_in_place_and_dequantize_exactly():
    """Flushed groups land in capacity stores: between two store growths the
    packed tensors keep their addresses (no whole-cache copy per flush), and
    the appended cache dequantizes bit-identically to the rebuilt one."""

    need_gpu()
    key, value = make_kv(3000, 4, 128, seed=8, device="cuda")
    cache = _from_dense(key, value, 256, 2, 2, 32, 32)
    cache.append(key[256:300], value[256:300], logical_token_ids=torch.arange(256, 300, device="cuda"))
    addresses, moves = cache.key_code.data_ptr(), 0
    for t in range(300, 3000, 9):
        cache.append(key[t:t + 9], value[t:t + 9], logical_token_ids=torch.arange(t, t + 9, device="cuda"))
        if cache.key_code.data_ptr() != addresses:
            moves += 1
            addresses = cache.key_code.data_ptr()
    assert cache.quantized_tokens == 2944 and moves <= 4, moves
    rebuilt = _from_dense(key, value, 3000, 2, 2, 32, 32)
    _assert_same(cache, rebuilt)
    ka, va = cache.dequantize(dtype=torch.bfloat16)
    kb, vb = rebuilt.dequantize(dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(ka, kb) and torch.equal(va, vb)
