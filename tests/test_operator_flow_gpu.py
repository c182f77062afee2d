"""The reference's request -> materialise -> attend flow, driven through the
B200 operators and storage classes (unicache/operators/physical.py ->
unicache/storage/tensor_backend.py:103-239 -> the fused decode of
unicache/adapters/bagel.py:1598-1858), checked against the float64 oracle.

One sample of 600 dense tokens: 200 instruction tokens (type 1) go to H2O
(ratio 0.2, scored by the LSE-driven kernels from 64 queries over the whole
cache, the "full_kv_first_call" observation), 384 VAE tokens (type 3,
contiguous span) to 2-bit KIVI with group 32 and a 32-token residual, 16
tokens (type 4) stay dense.  The decode over the materialised cache must
match the oracle within the north-star bound."""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import attention, h2o, kivi
from unicache_b200 import (
    GQAH2OCache,
    H2OPhysicalGQAOperator,
    KIVIPackedQuantizationOperator,
    PackedKIVICache,
    TensorCacheStorageBackend,
    fused_mixed_decode,
    kernels,
)
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import assert_attention_close, host, need_gpu

pytestmark = pytest.mark.gpu


def _ctx(params, key, mask, segment, type_id, span):
    records = []
    return SimpleNamespace(
        params=params, k=key, segment_mask=mask, step=SimpleNamespace(segment_id=segment),
        runtime=SimpleNamespace(kv_metadata={"current_segment_type_id": type_id, "current_segment_span": span,
                                             "current_segment_tokens": int(mask.sum())}),
        storage_num_kv_heads=int(key.shape[1]), record=records.append, records=records, physical_request=None)


def test_operator_requests_materialise_and_decode():
    need_gpu()
    n = 600
    key, value = make_kv(n, 4, 128, seed=21, device="cuda")
    types = torch.full((n,), 4, dtype=torch.int64, device="cuda")
    types[:200] = 1
    types[200:584] = 3
    queries = make_query(64, 28, 128, seed=22, device="cuda")

    h2o_op, kivi_op = H2OPhysicalGQAOperator(), KIVIPackedQuantizationOperator()
    h2o_ctx = _ctx(h2o_op.build_params({"target_budget_ratio": 0.2, "selection_frozen": True}), key, types == 1,
                   "instruction", 1, None)
    h2o_op.update_after_attention_lse(h2o_ctx, queries, None)
    kivi_ctx = _ctx(kivi_op.build_params({"bits": 2, "group_size": 32, "residual_length": 32}), key, types == 3,
                    "source_vae", 3, (200, 584))
    kivi_op.execute(kivi_ctx)
    assert h2o_ctx.records[0]["physical_h2o_target_tokens_per_kv_head"] == 40
    assert kivi_ctx.records[0]["physical_kivi_quantized_tokens"] == 352

    result = TensorCacheStorageBackend.compact_and_materialize(
        key=key, value=value, key_type_ids=types, sample_lens=torch.tensor([n]),
        keep_masks=[torch.ones(n, dtype=torch.bool, device="cuda")],
        physical_requests=[[h2o_ctx.physical_request, kivi_ctx.physical_request]])
    selected, packed = result.physical_segments_by_sample[0]
    assert isinstance(selected, GQAH2OCache) and isinstance(packed, PackedKIVICache)
    assert int(result.key.shape[0]) == 16 and bool((result.key_type_ids == 4).all())
    assert selected.retained_tokens == 40 and packed.quantized_tokens == 352 and packed.token_type_id == 3

    # H2O scores against the oracle (probabilities of the 64 queries over the whole dense cache)
    scores = host(h2o_ctx.physical_request.per_kv_head_scores).astype(np.float64)
    expect = h2o.reduce_probabilities(attention.attention_probabilities(host(queries), host(key)), 4)
    assert np.abs(scores - expect).max() <= 1e-5 * np.abs(expect).max()
    # the selection follows the scores the request carries (tie order: score desc, index asc)
    idx, _, _ = h2o.select_indices(scores[:, :200].astype(np.float32), 40, 10)
    assert np.array_equal(host(selected.logical_token_ids), idx)

    query = make_query(1, 28, 128, seed=23, device="cuda")
    out, lse = fused_mixed_decode(query, result.key, result.value, [selected, packed])
    torch.cuda.synchronize()
    ref = kivi.packed_from_dense(host(key)[200:584], host(value)[200:584], "bfloat16", k_bits=2, v_bits=2,
                                 group_size=32, residual_length=32)
    rk, rv = kivi.packed_dequantize(ref)
    keys = [host(key)[584:], host(selected.key).transpose(1, 0, 2), rk]
    vals = [host(value)[584:], host(selected.value).transpose(1, 0, 2), rv]
    e_out, e_lse = attention.mixed_attention(host(query), keys, vals)
    assert_attention_close(out, e_out, what="operator flow decode")
    assert np.abs(host(lse).T - e_lse).max() <= 2e-2
    assert kernels.device_status() == 0
