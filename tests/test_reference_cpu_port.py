"""The torch restatement of the reference's CPU decode path (oracle/reference_cpu.py),
which ``bench.py`` times as the CPU baseline, checked on the CPU:

* against the float64 oracle (tolerance of a bf16 AV product: 2e-2 max-abs);
* when the reference project is importable in this container, against the
  reference's own ``PackedKIVICache(backend="reference").attention_parts``
  + softmax + apply_value on the same packed cache (bit for bit: same
  operations in the same order)."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from oracle import attention, kivi, reference_cpu
from unicache_b200.synthetic import make_kv, make_query

REFERENCE = "/root/reference"


def _port_cache(tokens, residual, bits, group, seed):
    key, value = make_kv(tokens + residual, 4, 128, seed=seed)
    ref = kivi.packed_from_dense(key.float().numpy(), value.float().numpy(), "bfloat16", k_bits=bits, v_bits=bits,
                                 group_size=group, residual_length=residual)
    layout = {n: torch.from_numpy(np.ascontiguousarray(ref[n]).astype(np.int32)) for n in ("key_code", "value_code")}
    for n in ("key_scale", "key_minimum", "value_scale", "value_minimum", "residual_key", "residual_value"):
        layout[n] = torch.from_numpy(np.ascontiguousarray(ref[n], dtype=np.float32)).to(torch.bfloat16)
    cache = reference_cpu.cache_from_layout(layout, k_bits=bits, v_bits=bits, group_size=group,
                                            quantized_tokens=ref["quantized_tokens"], head_dim=128)
    return key, value, ref, cache


@pytest.mark.parametrize("bits,group", [(2, 32), (4, 64)])
def test_reference_cpu_port_matches_oracle(bits, group):
    _, _, ref, cache = _port_cache(512, 64, bits, group, seed=3)
    query = make_query(1, 28, 128, seed=4)
    out = reference_cpu.decode(cache, query)
    rk, rv = kivi.packed_dequantize(ref)
    k_port, v_port = reference_cpu.dequantize(cache)
    assert np.array_equal(k_port.float().numpy(), rk) and np.array_equal(v_port.float().numpy(), rv)
    expect, _ = attention.attention_summary(query.float().numpy(), rk, rv)
    assert np.abs(out.float().numpy() - expect).max() <= 2e-2


@pytest.mark.skipif(not os.path.isdir(REFERENCE), reason="the reference project is not present")
def test_reference_cpu_port_equals_the_reference_backend():
    sys.path.insert(0, REFERENCE)
    try:
        from unicache.storage.physical import PackedKIVICache
    except Exception as exc:  # pragma: no cover - depends on the container
        pytest.skip(f"reference not importable: {exc}")
    finally:
        sys.path.remove(REFERENCE)
    key, value, _, cache = _port_cache(512, 64, 2, 32, seed=5)
    query = make_query(1, 28, 128, seed=6)
    ref_cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(576), token_type_id=3,
                                           k_bits=2, v_bits=2, group_size=32, residual_length=64,
                                           backend="reference")
    logits, apply_value = ref_cache.attention_parts(query)
    expect = apply_value(torch.softmax(logits, dim=-1).to(query.dtype)).transpose(0, 1)
    assert torch.equal(reference_cpu.decode(cache, query), expect)
