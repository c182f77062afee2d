"""Decode attention over packed KIVI, residual, dense and H2O spans against the
float64 oracle of the reference algorithm (dequantize, then softmax attention).

Tolerance (north star, bf16 outputs): max-abs 2e-2 and mean-abs 1e-3 on the
attention output; LSE within 2e-2 absolute (natural log)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, kivi
from unicache_b200 import (
    GQAH2OCache,
    PackedKIVICache,
    PhysicalDecodeBatch,
    fused_h2o_decode,
    fused_mixed_decode,
    kernels,
    merge_attention_summaries,
    packed_kivi_quantized_attention_summary,
)
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import assert_attention_close, host, need_gpu

pytestmark = pytest.mark.gpu

LSE_ABS = 2e-2


def test_tensor_cores_multiply_fp16_subnormal_codes_exactly():
    need_gpu()
    err = kernels.selftest_mma_subnormal()
    assert 0.0 <= err < 1e-4, err


def _packed(tokens, residual, kb, vb, group, seed, heads=4):
    key, value = make_kv(tokens, heads, 128, seed=seed, device="cuda")
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(tokens, device="cuda"),
                                       token_type_id=3, k_bits=kb, v_bits=vb, group_size=group,
                                       residual_length=residual)
    ref = kivi.packed_from_dense(host(key), host(value), "bfloat16", k_bits=kb, v_bits=vb, group_size=group,
                                 residual_length=residual)
    return cache, ref


def _oracle_decode(query_row: np.ndarray, keys: list, values: list):
    out, lse = attention.mixed_attention(query_row[None], keys, values)
    return out[0], lse[:, 0]


@pytest.mark.parametrize(
    "tokens,residual,kb,vb,group",
    [
        (320, 32, 2, 2, 32),     # 288 quantized: a half-full last stage
        (1000, 100, 4, 4, 64),   # 896 quantized, 104 residual
        (700, 32, 2, 4, 128),    # mixed bits
        (1111, 17, 4, 2, 32),
        (8320, 128, 2, 2, 32),   # config-2 sequence length
        (4224, 128, 4, 4, 64),
    ],
)
def test_single_sequence_packed_plus_residual(tokens, residual, kb, vb, group):
    need_gpu()
    cache, ref = _packed(tokens, residual, kb, vb, group, seed=tokens + kb)
    query = make_query(1, 28, 128, seed=tokens, device="cuda")
    out, lse = fused_mixed_decode(query, None, None, [cache])
    rk, rv = kivi.packed_dequantize(ref)
    eo, el = _oracle_decode(host(query)[0], [rk], [rv])
    assert_attention_close(out[0], eo, what=f"decode {tokens}/{kb}/{vb}/{group}")
    assert np.abs(host(lse)[0] - el).max() < LSE_ABS
    assert kernels.device_status() == 0


def test_quantized_prefix_summary_matches_oracle():
    need_gpu()
    cache, ref = _packed(640, 40, 2, 2, 64, seed=3)
    query = make_query(1, 28, 128, seed=5, device="cuda")[0:1]
    out, lse = packed_kivi_quantized_attention_summary(cache, query)
    q = ref["quantized_tokens"]
    rk, rv = kivi.packed_dequantize(ref)
    eo, el = attention.attention_summary(host(query), rk[:q], rv[:q])
    assert_attention_close(out, eo)
    assert np.abs(host(lse) - el).max() < LSE_ABS


def test_batch_with_dense_h2o_and_packed_segments():
    """Three sequences with different segment mixes in one launch."""

    need_gpu()
    seqs, expected = [], []
    queries = make_query(3, 28, 128, seed=77, device="cuda")
    # seq 0: dense cache + packed (2-bit, G32) with residual
    dk, dv = make_kv(37, 4, 128, seed=40, device="cuda")
    c0, r0 = _packed(600, 24, 2, 2, 32, seed=41)
    seqs.append([(dk, dv), c0])
    k0, v0 = kivi.packed_dequantize(r0)
    expected.append(([host(dk), k0], [host(dv), v0]))
    # seq 1: an H2O segment (head-major rows) + packed
    hk, hv = make_kv(500, 4, 128, seed=42, device="cuda")
    scores = torch.rand(4, 500, generator=torch.Generator().manual_seed(3)).cuda()
    hseg = GQAH2OCache.from_dense(hk, hv, logical_token_ids=torch.arange(500, device="cuda"), token_type_id=2,
                                  per_kv_head_scores=scores, target_tokens=100, recent_tokens=25,
                                  selection_frozen=True)
    c1, r1 = _packed(384, 0, 2, 2, 32, seed=43)
    seqs.append([hseg, c1])
    ho = {"key": host(hseg.key), "value": host(hseg.value)}
    k1, v1 = kivi.packed_dequantize(r1)
    expected.append((ho, k1, v1))
    # seq 2: packed only, no residual
    c2, r2 = _packed(2048, 0, 2, 2, 32, seed=44)
    seqs.append([c2])
    k2, v2 = kivi.packed_dequantize(r2)
    expected.append(([k2], [v2]))

    batch = PhysicalDecodeBatch(seqs, num_kv_heads=4)
    out, lse = batch(queries)
    qh = host(queries)
    eo, _ = _oracle_decode(qh[0], *expected[0])
    assert_attention_close(out[0], eo, what="seq0")
    # H2O keeps different tokens per KV head: evaluate the oracle head by head.
    ho, k1, v1 = expected[1]
    got = host(out[1])
    for kvh in range(4):
        keys = [ho["key"][kvh][:, None, :], k1[:, kvh:kvh + 1]]
        vals = [ho["value"][kvh][:, None, :], v1[:, kvh:kvh + 1]]
        e, _ = attention.mixed_attention(qh[1][None, kvh * 7:(kvh + 1) * 7], keys, vals)
        diff = np.abs(got[kvh * 7:(kvh + 1) * 7] - e[0])
        assert diff.max() < 2e-2 and diff.mean() < 1e-3, kvh
    eo, _ = _oracle_decode(qh[2], *expected[2])
    assert_attention_close(out[2], eo, what="seq2")
    # Static work split and a fixed merge order: a second call is bitwise identical.
    out2, lse2 = batch(queries)
    assert torch.equal(out, out2) and torch.equal(lse, lse2)


def test_fused_h2o_decode_reads_compacted_rows_in_place():
    """bagel.py:1860-1901 semantics without the per-step concat."""

    need_gpu()
    dk, dv = make_kv(3, 4, 128, seed=8, device="cuda", outliers=False)
    sk, sv = make_kv(1200, 4, 128, seed=9, device="cuda")
    scores = torch.rand(4, 1200, generator=torch.Generator().manual_seed(8)).cuda()
    seg = GQAH2OCache.from_dense(sk, sv, logical_token_ids=torch.arange(1200, device="cuda"), token_type_id=2,
                                 per_kv_head_scores=scores, target_tokens=240, recent_tokens=60,
                                 selection_frozen=True)
    query = make_query(1, 28, 128, seed=10, device="cuda")
    out = fused_h2o_decode(query, dk, dv, [seg])
    combined_k = torch.cat([dk, seg.key.transpose(0, 1)], dim=0)
    combined_v = torch.cat([dv, seg.value.transpose(0, 1)], dim=0)
    eo, _ = attention.attention_summary(host(query), host(combined_k), host(combined_v))
    assert_attention_close(out, eo)


def test_split_partials_merge_to_the_whole():
    """Summaries of two halves merged by the LSE-merge kernel equal one decode
    over the whole cache (bagel.py:57-72 linearity)."""

    need_gpu()
    key, value = make_kv(4096, 4, 128, seed=21, device="cuda")
    a = PackedKIVICache.from_dense(key[:2048], value[:2048], logical_token_ids=torch.arange(2048, device="cuda"),
                                   token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=0)
    b = PackedKIVICache.from_dense(key[2048:], value[2048:], logical_token_ids=torch.arange(2048, device="cuda"),
                                   token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=0)
    query = make_query(1, 28, 128, seed=22, device="cuda")
    oa, la = fused_mixed_decode(query, None, None, [a])
    ob, lb = fused_mixed_decode(query, None, None, [b])
    whole, lw = fused_mixed_decode(query, None, None, [a, b])
    merged, lm = merge_attention_summaries([(oa.float(), la.t().contiguous()), (ob.float(), lb.t().contiguous())])
    assert (merged - whole.float()).abs().max().item() < 1e-2
    assert (lm.t() - lw).abs().max().item() < 1e-4


def test_full_size_config2_batch_decode():
    """Config 2: 16 sequences x (8192 packed 2-bit G32 + 128 bf16 residual),
    28/4 heads.  Every sequence is checked against the oracle."""

    need_gpu()
    caches, refs = [], []
    for b in range(16):
        c, r = _packed(8320, 128, 2, 2, 32, seed=1000 + b)
        caches.append([c])
        refs.append(r)
    batch = PhysicalDecodeBatch(caches, num_kv_heads=4)
    queries = make_query(16, 28, 128, seed=99, device="cuda")
    out, lse = batch(queries)
    qh = host(queries)
    worst = 0.0
    for b in range(16):
        rk, rv = kivi.packed_dequantize(refs[b])
        eo, el = _oracle_decode(qh[b], [rk], [rv])
        mx, _ = assert_attention_close(out[b], eo, what=f"seq{b}")
        worst = max(worst, mx)
        assert np.abs(host(lse)[b] - el).max() < LSE_ABS
    assert kernels.device_status() == 0


def test_full_size_config3_per_gpu_batch_decode():
    """Config 3 per GPU (batch 64 over 8 GPUs): 8 sequences x (32768 packed
    4-bit G64 + 128 bf16 residual), 28/4 heads; sequences 0, 3 and 7 are
    checked against the oracle (the packing of all eight is checked against
    the oracle for sequence 0 bit for bit)."""

    need_gpu()
    caches, refs = [], []
    for b in range(8):
        c, r = _packed(32768 + 128, 128, 4, 4, 64, seed=2000 + b)
        caches.append([c])
        refs.append(r)
    layout = caches[0][0].reference_layout()
    assert np.array_equal(host(layout["key_code"]), refs[0]["key_code"])
    assert np.array_equal(host(layout["value_code"]), refs[0]["value_code"])
    batch = PhysicalDecodeBatch(caches, num_kv_heads=4)
    queries = make_query(8, 28, 128, seed=98, device="cuda")
    out, lse = batch(queries)
    qh = host(queries)
    for b in (0, 3, 7):
        rk, rv = kivi.packed_dequantize(refs[b])
        eo, el = _oracle_decode(qh[b], [rk], [rv])
        assert_attention_close(out[b], eo, what=f"seq{b}")
        assert np.abs(host(lse)[b] - el).max() < LSE_ABS
    assert kernels.device_status() == 0


def test_full_size_config3_long_sequence_decode():
    """Config 3, long-context half, on one GPU: ONE sequence of 131072 packed
    4-bit G64 + 128 bf16 residual tokens (4 pairs spread over every SM, so
    each pair carries hundreds of warp states and the wide state merge runs),
    checked against the oracle."""

    need_gpu()
    cache, ref = _packed(131072 + 128, 128, 4, 4, 64, seed=3100)
    query = make_query(1, 28, 128, seed=31, device="cuda")
    batch = PhysicalDecodeBatch([[cache]], num_kv_heads=4)
    assert batch.plan.num_partials > 64 * 4  # the wide merge's regime
    out, lse = batch(query)
    out2, lse2 = batch(query)
    torch.cuda.synchronize()
    assert torch.equal(out, out2) and torch.equal(lse, lse2)
    rk, rv = kivi.packed_dequantize(ref)
    eo, el = _oracle_decode(host(query)[0], [rk], [rv])
    assert_attention_close(out[0], eo, what="131072-token sequence")
    assert np.abs(host(lse)[0] - el).max() < LSE_ABS
    assert kernels.device_status() == 0


def test_decode_rejects_cpu_and_bad_query():
    need_gpu()
    cache, _ = _packed(256, 0, 2, 2, 32, seed=1)
    batch = PhysicalDecodeBatch([[cache]], num_kv_heads=4)
    with pytest.raises(RuntimeError):
        batch(torch.zeros(1, 28, 128, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        batch(torch.zeros(2, 28, 128, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        batch(torch.zeros(1, 28, 128, dtype=torch.float32, device="cuda"))


def test_decode_step_graph_matches_eager_calls_with_host_buffers():
    """DecodeStepGraph: per-step host->device query copy, decode, merge and
    device->host output/LSE copy replayed as one CUDA graph."""
    need_gpu()
    from unicache_b200 import DecodeStepGraph

    seqs = []
    for b in range(3):
        cache, _ = _packed(640 + 64 * b, 32, 2, 2, 32, seed=300 + b)
        seqs.append([cache])
    batch = PhysicalDecodeBatch(seqs, num_kv_heads=4)
    host_q = torch.empty(3, 28, 128, dtype=torch.bfloat16).pin_memory()
    host_o = torch.empty(3, 28, 128, dtype=torch.bfloat16).pin_memory()
    host_l = torch.empty(3, 28, dtype=torch.float32).pin_memory()
    step = DecodeStepGraph(batch, host_q, host_o, host_l)
    for seed in (11, 12):
        q = make_query(3, 28, 128, seed=seed)
        host_q.copy_(q)
        step()
        torch.cuda.synchronize()
        ref_o, ref_l = batch(q.cuda())
        torch.cuda.synchronize()
        assert torch.equal(host_o, ref_o.cpu()) and torch.equal(host_l, ref_l.cpu())
    with pytest.raises(ValueError):
        DecodeStepGraph(batch, torch.empty(3, 28, 128, dtype=torch.bfloat16), host_o, host_l)
