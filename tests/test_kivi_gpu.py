"""KIVI quantize/pack, dequantize and fake-quant kernels against the oracle
(bit-exact) and the reference's golden digests."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kivi
from oracle.numerics import digest
from unicache_b200 import PackedKIVICache, dequantize_kivi_chunk, kernels, kivi_fake_quant_key, kivi_fake_quant_value
from unicache_b200.synthetic import make_kv

from .conftest import bf16_array
from .gpu_util import DTYPE_NAMES, host, need_gpu

pytestmark = pytest.mark.gpu


def _to_device(arr: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(arr)).to(dtype).cuda()


def test_golden_quantizer_matrix_bit_exact(golden):
    need_gpu()
    arrays, cases = golden
    data = _to_device(bf16_array(arrays["quant_input_bf16"]), torch.bfloat16)
    for layout in ("key", "value"):
        for group in (32, 64, 128):
            for bits in (2, 4, 8):
                case = cases[f"quant/{layout}/g{group}/b{bits}"]
                pack = kernels.kivi_pack_key if layout == "key" else kernels.kivi_pack_value
                codes, scale, minimum = pack(data, bits=bits, group_size=group)
                # b200 layout -> reference layout: swap the first two axes.
                ref_codes = host(codes.transpose(0, 1).contiguous())
                assert digest(ref_codes) == case["packed"], (layout, group, bits)
                assert digest(host(scale.transpose(0, 1).contiguous()), "bfloat16") == case["scale"]
                assert digest(host(minimum.transpose(0, 1).contiguous()), "bfloat16") == case["minimum"]


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_golden_from_dense_and_dequantize(golden, bits):
    need_gpu()
    arrays, cases = golden
    case = cases[f"from_dense96/b{bits}"]
    key = _to_device(bf16_array(arrays["fd96_key"]), torch.bfloat16)
    value = _to_device(bf16_array(arrays["fd96_value"]), torch.bfloat16)
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(96, device="cuda"),
                                       token_type_id=3, k_bits=bits, v_bits=bits, group_size=32,
                                       residual_length=16)
    assert cache.quantized_tokens == case["quantized_tokens"]
    ref = cache.reference_layout()
    assert digest(host(ref["key_code"].contiguous())) == case["key_code"]
    assert digest(host(ref["value_code"].contiguous())) == case["value_code"]
    assert digest(host(ref["key_scale"].contiguous()), "bfloat16") == case["key_scale"]
    assert digest(host(ref["value_minimum"].contiguous()), "bfloat16") == case["value_minimum"]
    rk, rv = cache.dequantize()
    assert digest(host(rk), "bfloat16") == case["dequant_key"]
    assert digest(host(rv), "bfloat16") == case["dequant_value"]
    assert cache.resident_bytes == case["resident_bytes"]
    assert cache.full_precision_bytes == case["full_precision_bytes"]
    assert cache.byte_breakdown == case["byte_breakdown"]


def test_golden_residual_expansion_mixed_bits(golden):
    need_gpu()
    arrays, cases = golden
    case = cases["from_dense320/k2v4"]
    key = _to_device(bf16_array(arrays["fd320_key"]), torch.bfloat16)
    value = _to_device(bf16_array(arrays["fd320_value"]), torch.bfloat16)
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(320, device="cuda"),
                                       token_type_id=3, k_bits=2, v_bits=4, group_size=128, residual_length=32)
    assert cache.quantized_tokens == 256 and int(cache.residual_key.shape[0]) == 64
    assert cache.residual_key.numel() * cache.residual_key.element_size() == cache.residual_key.untyped_storage().nbytes()
    ref = cache.reference_layout()
    assert digest(host(ref["key_code"].contiguous())) == case["key_code"]
    assert digest(host(ref["value_code"].contiguous())) == case["value_code"]
    rk, rv = cache.dequantize()
    assert digest(host(rk), "bfloat16") == case["dequant_key"]
    assert digest(host(rv), "bfloat16") == case["dequant_value"]
    assert torch.equal(key[-64:], rk[-64:]) and torch.equal(value[-64:], rv[-64:])


def test_golden_repack_monotonic(golden):
    need_gpu()
    arrays, cases = golden
    case = cases["repack"]
    key = _to_device(bf16_array(arrays["repack_key"]), torch.bfloat16)
    value = _to_device(bf16_array(arrays["repack_value"]), torch.bfloat16)
    packed = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(64, device="cuda"),
                                        token_type_id=3, k_bits=4, v_bits=4, group_size=32, residual_length=8)
    assert packed.repack_monotonic(bits=2, group_size=32) is True
    assert packed.repack_monotonic(bits=4, group_size=32) is False
    assert packed.budget_shortfall_events == case["shortfall"] and packed.k_bits == 2
    ref = packed.reference_layout()
    assert digest(host(ref["key_code"].contiguous())) == case["key_code"]
    rk, rv = packed.dequantize()
    assert digest(host(rk), "bfloat16") == case["dequant_key"]
    assert digest(host(rv), "bfloat16") == case["dequant_value"]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("group,kb,vb", [(32, 2, 2), (64, 4, 4), (128, 2, 4), (32, 8, 8), (64, 4, 2)])
def test_pack_and_dequant_bit_exact_vs_oracle(dtype, group, kb, vb):
    need_gpu()
    key, value = make_kv(448, 4, 128, seed=group + kb, dtype=dtype, device="cuda")
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(448, device="cuda"),
                                       token_type_id=3, k_bits=kb, v_bits=vb, group_size=group, residual_length=40)
    name = DTYPE_NAMES[dtype]
    expect = kivi.packed_from_dense(host(key), host(value), name, k_bits=kb, v_bits=vb, group_size=group,
                                    residual_length=40)
    assert cache.quantized_tokens == expect["quantized_tokens"]
    ref = cache.reference_layout()
    for field in ("key_code", "value_code"):
        np.testing.assert_array_equal(host(ref[field].contiguous()), expect[field])
    for field in ("key_scale", "key_minimum", "value_scale", "value_minimum"):
        np.testing.assert_array_equal(host(ref[field].contiguous()), expect[field])
    rk, rv = cache.dequantize()
    ek, ev = kivi.packed_dequantize(expect)
    np.testing.assert_array_equal(host(rk), ek)
    np.testing.assert_array_equal(host(rv), ev)
    # dequantize(dtype=float32) rounds once, to fp32.
    fk, _ = cache.dequantize(dtype=torch.float32)
    ek32, _ = kivi.packed_dequantize(expect, "float32")
    np.testing.assert_array_equal(host(fk), ek32)


def test_chunk_dequantization_into_workspace_matches_dequantize():
    """tests/test_physical.py:650-688 semantics, with group 32 as well."""

    need_gpu()
    for bits, group in ((2, 32), (4, 64), (2, 128)):
        key, value = make_kv(384, 4, 128, seed=13, device="cuda")
        cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(384, device="cuda"),
                                           token_type_id=3, k_bits=bits, v_bits=bits, group_size=group,
                                           residual_length=0)
        ek, ev = cache.dequantize(dtype=torch.bfloat16)
        ak, av = dequantize_kivi_chunk(cache, start=128, stop=384, dtype=torch.bfloat16)
        assert torch.equal(ak, ek[128:384]) and torch.equal(av, ev[128:384])
        wk = torch.full((300, 4, 128), -7.0, device="cuda", dtype=torch.bfloat16)
        wv = torch.full_like(wk, -9.0)
        dk, dv = dequantize_kivi_chunk(cache, start=128, stop=384, dtype=torch.bfloat16, output_key=wk,
                                       output_value=wv, output_offset=16)
        assert torch.equal(dk, ek[128:384]) and torch.equal(dv, ev[128:384])
        assert torch.all(wk[:16] == -7.0) and torch.all(wv[:16] == -9.0)
        assert torch.all(wk[272:] == -7.0)
        empty_k, _ = dequantize_kivi_chunk(cache, start=400, stop=500, dtype=torch.bfloat16)
        assert empty_k.shape[0] == 0
        with pytest.raises(ValueError):
            dequantize_kivi_chunk(cache, start=0, stop=384, dtype=torch.bfloat16, output_key=wk, output_value=wv,
                                  output_offset=0)


def test_edge_cases_empty_prefix_and_all_residual():
    need_gpu()
    key, value = make_kv(20, 4, 128, seed=1, device="cuda")
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(20, device="cuda"),
                                       token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=4)
    assert cache.quantized_tokens == 0 and cache.key_code is None
    rk, rv = cache.dequantize()
    assert torch.equal(rk, key) and torch.equal(rv, value)
    with pytest.raises(ValueError):
        PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(20), token_type_id=3, k_bits=3,
                                   v_bits=2, group_size=32, residual_length=4)
    with pytest.raises(ValueError):
        PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(20), token_type_id=3, k_bits=2,
                                   v_bits=2, group_size=32, residual_length=4, backend="reference")
    with pytest.raises(RuntimeError):
        PackedKIVICache.from_dense(key.cpu(), value.cpu(), logical_token_ids=torch.arange(20), token_type_id=3,
                                   k_bits=2, v_bits=2, group_size=32, residual_length=4)


def test_constant_groups_use_epsilon_scale():
    """Degenerate groups (max == min) take scale = FLT_EPSILON and code 0."""

    need_gpu()
    key = torch.ones(64, 2, 128, device="cuda", dtype=torch.bfloat16)
    value = torch.full_like(key, -3.0)
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(64, device="cuda"),
                                       token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=0)
    expect = kivi.packed_from_dense(host(key), host(value), "bfloat16", k_bits=2, v_bits=2, group_size=32,
                                    residual_length=0)
    ref = cache.reference_layout()
    np.testing.assert_array_equal(host(ref["key_scale"].contiguous()), expect["key_scale"])
    np.testing.assert_array_equal(host(ref["key_code"].contiguous()), expect["key_code"])
    rk, rv = cache.dequantize()
    assert torch.equal(rk, key) and torch.equal(rv, value)


@pytest.mark.parametrize("bits,pattern", [
    (2, [0.0, 3.0, 0.5, 1.5, 2.5, 1.0, 2.0, 0.5]),
    (4, [0.0, 15.0, 0.5, 7.5, 14.5, 3.0, 11.5, 6.5]),
])
@pytest.mark.parametrize("gain", [1.0, 0.3, -1.7])
def test_half_integer_ties_bit_exact_vs_oracle(bits, pattern, gain):
    """Every 32-token key group and every 32-channel value group holds its
    minimum, its maximum and values whose code lies exactly on (gain 1) or
    next to (other gains, after bf16 rounding) a half-integer: those take
    the quantizer's exact-division fallback, whose round-half-even must match
    the oracle bit for bit."""

    need_gpu()
    t, c = np.meshgrid(np.arange(256), np.arange(128), indexing="ij")
    base = np.asarray(pattern, np.float32)[(t + c) % len(pattern)] * np.float32(gain)
    key = torch.from_numpy(np.stack([base, base[::-1]], axis=1)).to(torch.bfloat16).cuda()
    value = torch.from_numpy(np.stack([base[:, ::-1], base], axis=1)).to(torch.bfloat16).cuda()
    cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(256, device="cuda"),
                                       token_type_id=3, k_bits=bits, v_bits=bits, group_size=32,
                                       residual_length=0)
    expect = kivi.packed_from_dense(host(key), host(value), "bfloat16", k_bits=bits, v_bits=bits, group_size=32,
                                    residual_length=0)
    ref = cache.reference_layout()
    for field in ("key_code", "value_code", "key_scale", "key_minimum", "value_scale", "value_minimum"):
        np.testing.assert_array_equal(host(ref[field].contiguous()), expect[field], err_msg=field)
    if gain == 1.0:  # scale exactly 1: the codes are the round-half-even of the values themselves
        rk, _ = cache.dequantize(dtype=torch.float32)
        np.testing.assert_array_equal(host(rk)[:, 0], np.rint(base))


def test_full_size_config2_pack_is_bit_exact():
    """Config 2 shape (16 sequences x 8192+128 tokens, 2-bit, G32): codes and
    statistics of every sequence equal the oracle's; dequantize is idempotent
    under a second pack (codes round-trip)."""

    need_gpu()
    for b in range(16):
        key, value = make_kv(8320, 4, 128, seed=1000 + b, device="cuda")
        cache = PackedKIVICache.from_dense(key, value, logical_token_ids=torch.arange(8320, device="cuda"),
                                           token_type_id=3, k_bits=2, v_bits=2, group_size=32, residual_length=128)
        assert cache.quantized_tokens == 8192
        if b % 5 == 0:
            expect = kivi.packed_from_dense(host(key), host(value), "bfloat16", k_bits=2, v_bits=2,
                                            group_size=32, residual_length=128)
            ref = cache.reference_layout()
            for field in ("key_code", "value_code", "key_scale", "key_minimum", "value_scale", "value_minimum"):
                np.testing.assert_array_equal(host(ref[field].contiguous()), expect[field], err_msg=field)
        # Property: re-packing the dequantized cache reproduces the same codes.
        rk, rv = cache.dequantize()
        again = PackedKIVICache.from_dense(rk, rv, logical_token_ids=cache.logical_token_ids, token_type_id=3,
                                           k_bits=2, v_bits=2, group_size=32, residual_length=128)
        assert torch.equal(again.key_code, cache.key_code) and torch.equal(again.value_code, cache.value_code)


@pytest.mark.parametrize("bits", [2, 4])
def test_golden_fake_quant(golden, bits):
    need_gpu()
    arrays, cases = golden
    data = torch.from_numpy(arrays["fq_input"]).cuda()
    fk = kivi_fake_quant_key(data, bits=bits, group_size=32)
    fv = kivi_fake_quant_value(data, bits=bits, group_size=32)
    assert digest(host(fk), "float32") == cases[f"fake_quant/b{bits}"]["key"]
    assert digest(host(fv), "float32") == cases[f"fake_quant/b{bits}"]["value"]


def test_fake_quant_bf16_and_partial_groups_vs_oracle():
    need_gpu()
    key, _ = make_kv(1930, 4, 128, seed=4, device="cuda")
    for bits in (2, 3, 4, 8):
        got = kivi_fake_quant_key(key, bits=bits, group_size=32)
        np.testing.assert_array_equal(host(got), kivi.fake_quant_key(host(key), "bfloat16", bits=bits, group_size=32))
        got = kivi_fake_quant_value(key, bits=bits, group_size=48)
        np.testing.assert_array_equal(host(got), kivi.fake_quant_value(host(key), "bfloat16", bits=bits, group_size=48))


@pytest.mark.parametrize("kb,vb", [(2, 2), (2, 4), (4, 2), (4, 4), (8, 2), (2, 8), (8, 8)])
@pytest.mark.parametrize("tokens", [32, 96, 8192])
def test_fused_key_value_pack_equals_separate_kernels(kb, vb, tokens):
    """ucb_kivi_pack_kv (one launch) writes exactly what ucb_kivi_pack_key +
    ucb_kivi_pack_value write, including for a key view with a padded head
    stride and a value view with a padded token stride."""
    need_gpu()
    gen = torch.Generator(device="cuda").manual_seed(tokens + 10 * kb + vb)
    big_k = (torch.randn(tokens, 4, 136, generator=gen, device="cuda") * 3).to(torch.bfloat16)
    big_v = torch.randn(tokens, 5, 128, generator=gen, device="cuda").to(torch.bfloat16)
    key, value = big_k[:, :, :128], big_v[:, :4]
    fused = kernels.kivi_pack_kv(key, value, k_bits=kb, v_bits=vb, group_size=32)
    separate = (*kernels.kivi_pack_key(key, bits=kb, group_size=32),
                *kernels.kivi_pack_value(value, bits=vb, group_size=32))
    torch.cuda.synchronize()
    for a, b in zip(fused, separate):
        assert a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)
    assert kernels.device_status() == 0


def test_fused_pack_other_groups_use_the_separate_kernels():
    need_gpu()
    key, value = make_kv(256, 4, 128, seed=12, device="cuda")
    for g in (64, 128):
        fused = kernels.kivi_pack_kv(key, value, k_bits=4, v_bits=2, group_size=g)
        separate = (*kernels.kivi_pack_key(key, bits=4, group_size=g),
                    *kernels.kivi_pack_value(value, bits=2, group_size=g))
        for a, b in zip(fused, separate):
            assert torch.equal(a, b)


def test_from_dense_batch_equals_per_segment_packing():
    """One pack launch for a batch of segments (ragged lengths, one with no
    quantized tokens) gives the tensors from_dense gives segment by segment,
    bit for bit; a group-64 batch takes the per-segment fallback."""

    need_gpu()
    from unicache_b200 import PackedKIVICache

    lengths = [1000, 64, 2080, 20, 513]
    kv = [make_kv(n, 4, 128, seed=200 + i, device="cuda") for i, n in enumerate(lengths)]
    for kb, vb, group in ((2, 2, 32), (4, 2, 32), (2, 4, 64)):
        batch = PackedKIVICache.from_dense_batch(
            [k for k, _ in kv], [v for _, v in kv], logical_token_ids=[torch.arange(n, device="cuda") for n in lengths],
            token_type_id=3, k_bits=kb, v_bits=vb, group_size=group, residual_length=32)
        for (k, v), n, got in zip(kv, lengths, batch):
            want = PackedKIVICache.from_dense(k, v, logical_token_ids=torch.arange(n, device="cuda"), token_type_id=3,
                                              k_bits=kb, v_bits=vb, group_size=group, residual_length=32)
            assert got.quantized_tokens == want.quantized_tokens
            for name in ("key_code", "key_scale", "key_minimum", "value_code", "value_scale", "value_minimum",
                         "residual_key", "residual_value"):
                a, b = getattr(got, name), getattr(want, name)
                assert (a is None) == (b is None), name
                if a is not None:
                    assert torch.equal(a, b), (kb, vb, group, n, name)
