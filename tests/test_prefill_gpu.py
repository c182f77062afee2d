"""Long-query (prefill) attention on the tcgen05 tensor cores.

The kernel is floating point, so it is checked against a plain PyTorch fp32
reference of the same non-causal attention (reference adapter
unicache/adapters/bagel.py:1796-1801 runs flash_attn_func(..., causal=False)
over the dequantized segments).  Tolerance: the north-star bf16 bound,
max-abs 2e-2 and mean-abs 1e-3 on the output, 2e-2 on the natural-log LSE.
The mixed-segment path is checked against the float64 oracle."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import attention, kivi
from unicache_b200 import GQAH2OCache, PackedKIVICache, kernels
from unicache_b200.adapters.attention import long_query_attention_summary
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import MAX_ABS, MEAN_ABS, assert_attention_close, host, need_gpu

pytestmark = pytest.mark.gpu


def _reference(q, k, v, n):
    qf, kf, vf = q.float(), k[:, :n].float(), v[:, :n].float()
    logits = torch.matmul(qf, kf.transpose(1, 2)) / math.sqrt(q.shape[-1])
    lse = torch.logsumexp(logits, dim=-1)
    return torch.matmul(torch.softmax(logits, dim=-1), vf), lse


def _operands(heads, m, n, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    n_pad = (n + 7) // 8 * 8
    q = torch.randn(heads, m, 128, generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.zeros(heads, n_pad, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    k[:, :n] = (torch.randn(heads, n, 128, generator=gen, device="cuda") * 1.5).to(torch.bfloat16)
    v[:, :n] = torch.randn(heads, n, 128, generator=gen, device="cuda").to(torch.bfloat16)
    return q, k, v, n_pad


@pytest.mark.parametrize("heads,m,n", [(1, 128, 128), (1, 128, 40), (2, 200, 300), (4, 448, 1000), (1, 64, 1)])
def test_prefill_matches_fp32_reference(heads, m, n):
    need_gpu()
    q, k, v, n_pad = _operands(heads, m, n, seed=m + n)
    out, lse = kernels.prefill_attention(q, k, v.transpose(1, 2).contiguous(), n)
    torch.cuda.synchronize()
    ref, ref_lse = _reference(q, k, v, n)
    diff = (out.float() - ref).abs()
    assert torch.isfinite(out.float()).all()
    assert float(diff.max()) <= MAX_ABS and float(diff.mean()) <= MEAN_ABS, (float(diff.max()), float(diff.mean()))
    assert float((lse - ref_lse).abs().max()) <= 2e-2
    assert kernels.device_status() == 0


def test_prefill_config4_shape_and_repeat():
    """BASELINE config 4 per layer: Lq = 1024 queries x 7 heads per KV head
    against 3095 keys, 4 KV heads; a second launch is bitwise identical."""
    need_gpu()
    q, k, v, n_pad = _operands(4, 1024 * 7, 3095, seed=4)
    vt = v.transpose(1, 2).contiguous()
    out, lse = kernels.prefill_attention(q, k, vt, 3095)
    out2, lse2 = kernels.prefill_attention(q, k, vt, 3095)
    torch.cuda.synchronize()
    ref, ref_lse = _reference(q, k, v, 3095)
    diff = (out.float() - ref).abs()
    assert float(diff.max()) <= MAX_ABS and float(diff.mean()) <= MEAN_ABS, (float(diff.max()), float(diff.mean()))
    assert float((lse - ref_lse).abs().max()) <= 2e-2
    assert torch.equal(out, out2) and torch.equal(lse, lse2)


def test_prefill_rejects_bad_arguments():
    need_gpu()
    q, k, v, n_pad = _operands(1, 128, 100, seed=1)
    with pytest.raises(ValueError):
        kernels.prefill_attention(q, k, v, 100)  # v not transposed: shape mismatch
    with pytest.raises(ValueError):
        kernels.prefill_attention(q, k[:, :100].contiguous(), v.transpose(1, 2)[:, :, :100].contiguous(), 100)


def test_long_query_over_mixed_segments_matches_oracle():
    """A 96-token query block over [dense 16 | H2O | packed KIVI + residual]."""
    need_gpu()
    heads, tokens = 4, 352
    key, value = make_kv(tokens, heads, 128, seed=31, device="cuda")
    packed = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(tokens, device="cuda"),
                                        token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=32)
    hk, hv = make_kv(200, heads, 128, seed=32, device="cuda")
    scores = torch.rand(heads, 200, generator=torch.Generator().manual_seed(5)).to("cuda")
    h2o = GQAH2OCache.from_dense(hk, hv, logical_token_ids=torch.arange(200, device="cuda"), token_type_id=1,
                                 per_kv_head_scores=scores, target_tokens=60, recent_tokens=12)
    dk, dv = make_kv(16, heads, 128, seed=33, device="cuda")
    query = make_query(96, 28, 128, seed=34, device="cuda")
    out, lse = long_query_attention_summary(query, [h2o, packed], dense_key=dk, dense_value=dv)
    torch.cuda.synchronize()
    ref = kivi.packed_from_dense(host(key), host(value), "bfloat16", k_bits=2, v_bits=2, group_size=32,
                                 residual_length=32)
    rk, rv = kivi.packed_dequantize(ref)
    keys = [host(dk), host(h2o.key).transpose(1, 0, 2), rk]
    vals = [host(dv), host(h2o.value).transpose(1, 0, 2), rv]
    e_out, e_lse = attention.mixed_attention(host(query), keys, vals)
    assert_attention_close(out, e_out, what="long-query mixed")
    assert np.abs(host(lse) - e_lse).max() <= 2e-2


def test_batched_long_query_matches_per_sample_launches():
    """bagel.py:773-980 (varlen, non-causal): three samples with different
    query lengths and segment mixes in one launch agree with three single
    launches (which may split their keys across CTAs, so within the bf16
    tolerance rather than bitwise); sample 1 is also checked against the
    oracle."""
    need_gpu()
    from unicache_b200 import batched_long_query_attention

    heads = 4
    samples, queries, dense = [], [], []
    for i, (tokens, lq, n_dense) in enumerate([(352, 40, 16), (1088, 300, 0), (200, 7, 70)]):
        key, value = make_kv(tokens, heads, 128, seed=60 + i, device="cuda")
        packed = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(tokens, device="cuda"),
                                            token_type_id=3, k_bits=2, v_bits=4, group_size=32, residual_length=32)
        segs = [packed]
        if i != 1:
            hk, hv = make_kv(150, heads, 128, seed=70 + i, device="cuda")
            sc = torch.rand(heads, 150, generator=torch.Generator().manual_seed(i)).to("cuda")
            segs.insert(0, GQAH2OCache.from_dense(hk, hv, logical_token_ids=torch.arange(150, device="cuda"),
                                                  token_type_id=1, per_kv_head_scores=sc, target_tokens=45,
                                                  recent_tokens=9))
        samples.append(segs)
        queries.append(make_query(lq, 28, 128, seed=80 + i, device="cuda"))
        dense.append(make_kv(n_dense, heads, 128, seed=90 + i, device="cuda") if n_dense else None)
    results = batched_long_query_attention(queries, samples, dense_by_sample=dense)
    for q, segs, dn, (out, lse) in zip(queries, samples, dense, results):
        single_out, single_lse = long_query_attention_summary(q, segs, dense_key=dn[0] if dn else None,
                                                              dense_value=dn[1] if dn else None)
        torch.cuda.synchronize()
        diff = (out.float() - single_out.float()).abs()
        assert float(diff.max()) <= MAX_ABS and float(diff.mean()) <= MEAN_ABS, (float(diff.max()), float(diff.mean()))
        assert float((lse - single_lse).abs().max()) <= 2e-2
    key, value = make_kv(1088, heads, 128, seed=61, device="cuda")
    ref = kivi.packed_from_dense(host(key), host(value), "bfloat16", k_bits=2, v_bits=4, group_size=32,
                                 residual_length=32)
    rk, rv = kivi.packed_dequantize(ref)
    e_out, e_lse = attention.mixed_attention(host(queries[1]), [rk], [rv])
    assert_attention_close(results[1][0], e_out, what="batched sample 1")
    assert np.abs(host(results[1][1]) - e_lse).max() <= 2e-2
    assert kernels.device_status() == 0


def test_key_split_fills_the_gpu_and_cleans_up():
    """Config 4 has 112 row blocks for 148 SMs: every row block's keys are
    split (the first 23 tiles merge the last 2 tiles' partial by LSE).  Three
    launches in a row agree bitwise with each other and with the fp32
    reference, and every flag is even (each split item adds 1 per launch)
    after each launch."""
    need_gpu()
    q, k, v, n_pad = _operands(4, 1024 * 7, 3095, seed=14)
    vt = v.transpose(1, 2).contiguous()
    first, _ = kernels.prefill_attention(q, k, vt, 3095)
    items = kernels._KEY_SPLITS[(q.device.index, 4, 7168, 3095, n_pad)]
    assert items is not None
    _, flags = kernels.prefill_split_workspace(q.device, 112, kernels.stream_of(q))
    assert int(items.shape[0]) == 2 * 112 and int(items[0, 4]) == kernels.plan_key_split(112, 25, 148) * 128
    before = flags.clone()
    results = [kernels.prefill_attention(q, k, vt, 3095) for _ in range(2)]
    torch.cuda.synchronize()
    assert int((flags % 2).abs().sum()) == 0
    assert torch.equal(flags[:112] - before[:112], torch.full_like(flags[:112], 4))
    for out, lse in results:
        assert torch.equal(out, first)
    ref, ref_lse = _reference(q, k, v, 3095)
    diff = (first.float() - ref).abs()
    assert float(diff.max()) <= MAX_ABS and float(diff.mean()) <= MEAN_ABS, (float(diff.max()), float(diff.mean()))
    assert float((results[0][1] - ref_lse).abs().max()) <= 2e-2
    assert kernels.device_status() == 0
