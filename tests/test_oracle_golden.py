"""Pin the CPU oracle to the UniCache reference through its golden vectors.

Every case in tests/golden/golden.json was produced by the reference's own
Python implementation (tests/golden/make_golden.py); here ``oracle/`` recomputes
the same case and must match bit-for-bit (digests), or, for attention outputs,
within the reference's own tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import attention, compact, h2o, kivi
from oracle.numerics import digest, from_bf16_bits

from .conftest import bf16_array


def test_quantizer_matrix_matches_reference(golden):
    arrays, cases = golden
    data = bf16_array(arrays["quant_input_bf16"])
    checked = 0
    for layout, (gdim, pdim) in {"key": (0, 0), "value": (2, 2)}.items():
        for group in (32, 64, 128):
            for bits in (2, 4, 8):
                case = cases[f"quant/{layout}/g{group}/b{bits}"]
                packed, scale, minimum, length = kivi.quantize_grouped(
                    data, "bfloat16", bits=bits, group_dim=gdim, group_size=group, pack_dim=pdim
                )
                assert length == case["length"]
                assert digest(packed) == case["packed"], (layout, group, bits)
                assert digest(scale, "bfloat16") == case["scale"], (layout, group, bits)
                assert digest(minimum, "bfloat16") == case["minimum"], (layout, group, bits)
                deq = kivi.dequantize_grouped(
                    packed, scale, minimum, bits=bits, group_dim=gdim, group_size=group,
                    pack_dim=pdim, length=length, dtype="bfloat16",
                )
                assert digest(deq, "bfloat16") == case["dequant"], (layout, group, bits)
                checked += 1
    assert checked == 18
    np.testing.assert_array_equal(
        kivi.quantize_grouped(data, "bfloat16", bits=2, group_dim=0, group_size=32, pack_dim=0)[0],
        arrays["quant/key/g32/b2/packed"],
    )


def test_partial_group_and_other_dtypes_match_reference(golden):
    arrays, cases = golden
    odd = arrays["quant_odd_fp32"]
    for layout, (gdim, pdim) in {"key": (0, 0), "value": (2, 2)}.items():
        for bits in (2, 4):
            case = cases[f"quant_odd/{layout}/b{bits}"]
            packed, scale, minimum, length = kivi.quantize_grouped(
                odd, "float32", bits=bits, group_dim=gdim, group_size=32, pack_dim=pdim
            )
            assert digest(packed) == case["packed"]
            assert digest(scale, "float32") == case["scale"]
            assert digest(minimum, "float32") == case["minimum"]
    half = arrays["quant_input_fp16"].astype(np.float32)
    for layout, (gdim, pdim) in {"key": (0, 0), "value": (2, 2)}.items():
        case = cases[f"quant_fp16/{layout}"]
        packed, scale, minimum, _ = kivi.quantize_grouped(
            half, "float16", bits=4, group_dim=gdim, group_size=64, pack_dim=pdim
        )
        assert digest(packed) == case["packed"]
        assert digest(scale, "float16") == case["scale"]
        assert digest(minimum, "float16") == case["minimum"]


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_from_dense_and_dequantize_match_reference(golden, bits):
    arrays, cases = golden
    case = cases[f"from_dense96/b{bits}"]
    key = bf16_array(arrays["fd96_key"])
    value = bf16_array(arrays["fd96_value"])
    cache = kivi.packed_from_dense(
        key, value, "bfloat16", k_bits=bits, v_bits=bits, group_size=32, residual_length=16
    )
    assert cache["quantized_tokens"] == case["quantized_tokens"]
    for name in ("key_code", "value_code"):
        assert digest(cache[name]) == case[name]
    for name in ("key_scale", "key_minimum", "value_scale", "value_minimum", "residual_key"):
        assert digest(cache[name], "bfloat16") == case[name]
    rk, rv = kivi.packed_dequantize(cache)
    assert digest(rk, "bfloat16") == case["dequant_key"]
    assert digest(rv, "bfloat16") == case["dequant_value"]


def test_residual_expansion_and_mixed_bits_match_reference(golden):
    arrays, cases = golden
    case = cases["from_dense320/k2v4"]
    cache = kivi.packed_from_dense(
        bf16_array(arrays["fd320_key"]), bf16_array(arrays["fd320_value"]), "bfloat16",
        k_bits=2, v_bits=4, group_size=128, residual_length=32,
    )
    assert cache["quantized_tokens"] == case["quantized_tokens"] == 256
    assert cache["residual_key"].shape[0] == case["residual_tokens"] == 64
    assert digest(cache["key_code"]) == case["key_code"]
    assert digest(cache["value_code"]) == case["value_code"]
    assert digest(cache["key_scale"], "bfloat16") == case["key_scale"]
    assert digest(cache["value_scale"], "bfloat16") == case["value_scale"]
    rk, rv = kivi.packed_dequantize(cache)
    assert digest(rk, "bfloat16") == case["dequant_key"]
    assert digest(rv, "bfloat16") == case["dequant_value"]


def test_monotonic_repack_matches_reference(golden):
    arrays, cases = golden
    case = cases["repack"]
    key = bf16_array(arrays["repack_key"])
    value = bf16_array(arrays["repack_value"])
    cache = kivi.packed_from_dense(key, value, "bfloat16", k_bits=4, v_bits=4, group_size=32, residual_length=8)
    # repack_monotonic (physical.py:425-450): dequantize, then pack again at 2 bits
    # keeping the residual length of the current residual.
    rk, rv = kivi.packed_dequantize(cache)
    repacked = kivi.packed_from_dense(
        rk, rv, "bfloat16", k_bits=2, v_bits=2, group_size=32,
        residual_length=cache["residual_key"].shape[0],
    )
    assert case["first"] is True and case["second"] is False and case["shortfall"] == 1
    assert repacked["quantized_tokens"] == case["quantized_tokens"]
    assert digest(repacked["key_code"]) == case["key_code"]
    assert digest(repacked["value_code"]) == case["value_code"]
    k2, v2 = kivi.packed_dequantize(repacked)
    assert digest(k2, "bfloat16") == case["dequant_key"]
    assert digest(v2, "bfloat16") == case["dequant_value"]


@pytest.mark.parametrize("bits", [2, 4])
def test_fake_quant_matches_reference(golden, bits):
    arrays, cases = golden
    data = arrays["fq_input"]
    fk = kivi.fake_quant_key(data, "float32", bits=bits, group_size=32)
    fv = kivi.fake_quant_value(data, "float32", bits=bits, group_size=32)
    assert digest(fk, "float32") == cases[f"fake_quant/b{bits}"]["key"]
    assert digest(fv, "float32") == cases[f"fake_quant/b{bits}"]["value"]


def test_h2o_known_answer(golden):
    arrays, _ = golden
    key = np.arange(8 * 2 * 4, dtype=np.float32).reshape(8, 2, 4)
    out = h2o.h2o_from_dense(key, key + 1000, np.arange(8), arrays["h2o_kat_scores"], 4, 2)
    assert out["logical_token_ids"].tolist() == [[0, 1, 6, 7], [1, 5, 6, 7]]
    np.testing.assert_array_equal(out["logical_token_ids"], arrays["h2o_kat_ids"])


def test_h2o_selection_trim_and_budget_match_reference(golden):
    arrays, cases = golden
    case = cases["h2o_random"]
    target, recent = h2o.budget_from_ratio(2048, 0.2, 0.25)
    assert (target, recent) == (case["target"], case["recent"]) == (410, 102)
    key = bf16_array(arrays["h2o_key"])
    value = bf16_array(arrays["h2o_value"])
    out = h2o.h2o_from_dense(key, value, np.arange(100, 2148), arrays["h2o_scores"], target, recent)
    np.testing.assert_array_equal(out["logical_token_ids"], arrays["h2o_ids"])
    assert out["heavy_tokens"] == case["heavy_tokens"]
    assert digest(out["key"], "bfloat16") == case["key"]
    assert digest(out["value"], "bfloat16") == case["value"]
    assert digest(out["cumulative_scores"], "float32") == case["scores"]
    assert digest(out["logical_token_ids"]) == case["ids"]

    received = h2o.reduce_probabilities(arrays["h2o_update_probs"], 4)
    updated = out["cumulative_scores"] + received.astype(np.float32)
    np.testing.assert_allclose(updated, arrays["h2o_updated_scores"], rtol=0, atol=2e-6)
    out["cumulative_scores"] = arrays["h2o_updated_scores"]
    eff1, out, short1 = h2o.request_budget(out, 300, 60)
    np.testing.assert_array_equal(out["logical_token_ids"], arrays["h2o_trim1_ids"])
    eff2, out, short2 = h2o.request_budget(out, 1000, 10)
    budget = cases["h2o_budget"]
    assert (eff1, eff2, short1 + short2) == (budget["effective1"], budget["effective2"], budget["shortfall"])
    assert out["key"].shape[1] == budget["retained"]
    assert digest(out["key"], "bfloat16") == budget["key"]
    assert digest(out["logical_token_ids"]) == budget["ids"]


def test_lse_merge_matches_reference(golden):
    arrays, _ = golden
    out, lse = attention.merge_attention_summaries(
        [(arrays["merge_oa"], arrays["merge_la"]), (arrays["merge_ob"], arrays["merge_lb"])]
    )
    np.testing.assert_allclose(out, arrays["merge_out"], atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(lse, arrays["merge_lse"], atol=1e-6, rtol=1e-6)


def test_packed_plus_dense_decode_attention_matches_reference(golden):
    arrays, _ = golden
    pk, pv = bf16_array(arrays["att_pk"]), bf16_array(arrays["att_pv"])
    dk, dv = bf16_array(arrays["att_dk"]), bf16_array(arrays["att_dv"])
    q = bf16_array(arrays["att_q"])
    cache = kivi.packed_from_dense(pk, pv, "bfloat16", k_bits=2, v_bits=2, group_size=32, residual_length=16)
    rk, rv = kivi.packed_dequantize(cache)
    out, _ = attention.mixed_attention(q, [dk, rk], [dv, rv])
    logits = attention.gqa_query_key_logits(q, np.concatenate([dk, rk])) / np.sqrt(128)
    np.testing.assert_allclose(logits, arrays["att_logits"], atol=1e-4, rtol=1e-5)
    # The reference casts probabilities to bf16 before AV (physical.py:60), so
    # its output differs from exact arithmetic by bf16 rounding.
    np.testing.assert_allclose(out, arrays["att_out"], atol=4e-3, rtol=0)
    assert np.abs(out - arrays["att_out"]).mean() < 5e-4


def test_dense_compaction_matches_reference(golden):
    arrays, cases = golden
    case = cases["compact"]
    key = bf16_array(arrays["compact_key"])
    value = bf16_array(arrays["compact_value"])
    ck, cv, ct, lens = compact.compact(
        key, value, arrays["compact_types"], [12, 18], [arrays["compact_mask0"], arrays["compact_mask1"]]
    )
    assert digest(ck, "bfloat16") == case["key"]
    assert digest(cv, "bfloat16") == case["value"]
    assert digest(ct) == case["types"]
    assert lens == case["lens"]


def test_bf16_rounding_is_nearest_even():
    from oracle.numerics import bf16_round

    x = np.array([1.0 + 2**-8, 1.0 + 3 * 2**-8, -(1.0 + 2**-8), 3.0e38], np.float32)
    assert bf16_round(x).tolist() == [1.0, 1.0 + 2**-6, -1.0, float(from_bf16_bits(np.array([0x7F62]))[0])]
