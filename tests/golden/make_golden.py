"""Write the golden vectors that pin the CPU oracle to the UniCache reference.

Run once, in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference <path to UniCache checkout>

It imports the reference's own Python implementation (``unicache.storage.physical``,
``unicache.operators.builtin``, ``unicache.adapters.bagel.merge_attention_summaries``,
``unicache.storage.tensor_backend``), runs it on seeded inputs and stores, in
``tests/golden/``:

* ``golden.npz``   the seeded inputs and the small outputs, as arrays
* ``golden.json``  sha256 digests of every output (``oracle.numerics.digest``)
                   plus scalar results

Nothing at test time reads the reference; ``tests/test_oracle_golden.py``
recomputes every case with ``oracle/`` and compares against these files.
Inputs mirror the reference's own tests (tests/test_physical.py) and the
shapes of the benchmark configurations at reduced size.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.numerics import bf16_bits, digest  # noqa: E402

def tname(t):
    import torch

    return {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}[t.dtype]


def f32(t):
    return t.detach().float().cpu().numpy()


def store_float(arrays, name, t):
    """Store a float tensor compactly: bf16 as its bit pattern."""

    dtype = tname(t)
    if dtype == "bfloat16":
        arrays[name] = bf16_bits(f32(t))
    elif dtype == "float16":
        arrays[name] = t.detach().cpu().numpy().astype(np.float16)
    else:
        arrays[name] = f32(t)
    return dtype


def dig(t):
    import torch

    if t.dtype in (torch.bfloat16, torch.float16, torch.float32):
        return digest(f32(t), tname(t))
    return digest(t.detach().cpu().numpy())


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True)
    args = parser.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))

    import torch
    from unicache.adapters.bagel import merge_attention_summaries
    from unicache.operators.builtin import kivi_fake_quant_key, kivi_fake_quant_value
    from unicache.storage.physical import (
        GQAH2OCache,
        PackedKIVICache,
        _dequantize_grouped,
        _quantize_grouped,
        _quantize_grouped_reference,
    )
    from unicache.storage.tensor_backend import TensorCacheStorageBackend

    arrays: dict[str, np.ndarray] = {}
    meta: dict = {"cases": {}}
    cases = meta["cases"]

    # 1. Quantizer matrix (tests/test_physical.py:984-1015 at [128, 4, 128]).
    torch.manual_seed(19)
    data = torch.randn(128, 4, 128, dtype=torch.bfloat16)
    store_float(arrays, "quant_input_bf16", data)
    for layout, (gdim, pdim) in {"key": (0, 0), "value": (2, 2)}.items():
        for group in (32, 64, 128):
            for bits in (2, 4, 8):
                packed, scale, minimum, length = _quantize_grouped(
                    data, bits=bits, group_dim=gdim, group_size=group, pack_dim=pdim
                )
                ref = _quantize_grouped_reference(
                    data, bits=bits, group_dim=gdim, group_size=group, pack_dim=pdim
                )
                assert torch.equal(packed, ref[0]) and torch.equal(scale, ref[1])
                deq = _dequantize_grouped(
                    packed, scale, minimum, bits=bits, group_dim=gdim, group_size=group,
                    pack_dim=pdim, length=length, dtype=torch.bfloat16,
                )
                key = f"quant/{layout}/g{group}/b{bits}"
                cases[key] = {
                    "packed": dig(packed), "scale": dig(scale), "minimum": dig(minimum),
                    "length": length, "dequant": dig(deq),
                }
                if group == 32 and bits == 2:
                    arrays[f"{key}/packed"] = packed.numpy()
                    store_float(arrays, f"{key}/scale", scale)

    # Partial last group (the loop form) and fp32 / fp16 inputs.
    torch.manual_seed(5)
    odd = torch.randn(100, 2, 96, dtype=torch.float32)
    store_float(arrays, "quant_odd_fp32", odd)
    for layout, (gdim, pdim) in {"key": (0, 0), "value": (2, 2)}.items():
        for bits in (2, 4):
            packed, scale, minimum, length = _quantize_grouped(
                odd, bits=bits, group_dim=gdim, group_size=32, pack_dim=pdim
            )
            cases[f"quant_odd/{layout}/b{bits}"] = {
                "packed": dig(packed), "scale": dig(scale), "minimum": dig(minimum), "length": length,
            }
    half = torch.randn(64, 2, 128).to(torch.float16)
    store_float(arrays, "quant_input_fp16", half)
    for layout, (gdim, pdim) in {"key": (0, 0), "value": (2, 2)}.items():
        packed, scale, minimum, length = _quantize_grouped(
            half, bits=4, group_dim=gdim, group_size=64, pack_dim=pdim
        )
        cases[f"quant_fp16/{layout}"] = {
            "packed": dig(packed), "scale": dig(scale), "minimum": dig(minimum), "length": length,
        }

    # 2. PackedKIVICache.from_dense + dequantize (tests/test_physical.py:959-982, 1070-1097).
    torch.manual_seed(0)
    key96 = torch.randn(96, 4, 128, dtype=torch.bfloat16)
    value96 = torch.randn_like(key96)
    store_float(arrays, "fd96_key", key96)
    store_float(arrays, "fd96_value", value96)
    for bits in (2, 4, 8):
        cache = PackedKIVICache.from_dense(
            key96, value96, logical_token_ids=torch.arange(96), token_type_id=3,
            k_bits=bits, v_bits=bits, group_size=32, residual_length=16, backend="reference",
        )
        rk, rv = cache.dequantize()
        cases[f"from_dense96/b{bits}"] = {
            "quantized_tokens": cache.quantized_tokens,
            "key_code": dig(cache.key_code), "key_scale": dig(cache.key_scale),
            "key_minimum": dig(cache.key_minimum), "value_code": dig(cache.value_code),
            "value_scale": dig(cache.value_scale), "value_minimum": dig(cache.value_minimum),
            "residual_key": dig(cache.residual_key), "dequant_key": dig(rk), "dequant_value": dig(rv),
            "resident_bytes": cache.resident_bytes, "full_precision_bytes": cache.full_precision_bytes,
            "byte_breakdown": cache.byte_breakdown,
        }
    torch.manual_seed(1)
    key320 = torch.randn(320, 4, 128, dtype=torch.bfloat16)
    value320 = torch.randn_like(key320)
    store_float(arrays, "fd320_key", key320)
    store_float(arrays, "fd320_value", value320)
    cache = PackedKIVICache.from_dense(
        key320, value320, logical_token_ids=torch.arange(320), token_type_id=3,
        k_bits=2, v_bits=4, group_size=128, residual_length=32, backend="reference",
    )
    rk, rv = cache.dequantize()
    cases["from_dense320/k2v4"] = {
        "quantized_tokens": cache.quantized_tokens, "residual_tokens": int(cache.residual_key.shape[0]),
        "key_code": dig(cache.key_code), "value_code": dig(cache.value_code),
        "key_scale": dig(cache.key_scale), "value_scale": dig(cache.value_scale),
        "dequant_key": dig(rk), "dequant_value": dig(rv),
    }
    # Monotonic repack (tests/test_physical.py:1099-1132).
    torch.manual_seed(2)
    key64 = torch.randn(64, 2, 128, dtype=torch.bfloat16)
    value64 = torch.randn_like(key64)
    store_float(arrays, "repack_key", key64)
    store_float(arrays, "repack_value", value64)
    packed = PackedKIVICache.from_dense(
        key64, value64, logical_token_ids=torch.arange(64), token_type_id=3,
        k_bits=4, v_bits=4, group_size=32, residual_length=8, backend="reference",
    )
    ok = packed.repack_monotonic(bits=2, group_size=32)
    refused = packed.repack_monotonic(bits=4, group_size=32)
    rk, rv = packed.dequantize()
    cases["repack"] = {
        "first": ok, "second": refused, "shortfall": packed.budget_shortfall_events,
        "k_bits": packed.k_bits, "quantized_tokens": packed.quantized_tokens,
        "key_code": dig(packed.key_code), "value_code": dig(packed.value_code),
        "dequant_key": dig(rk), "dequant_value": dig(rv),
    }

    # 3. Fake quantization (unicache/operators/builtin.py:31-65), fp32 like config 1.
    torch.manual_seed(3)
    fq = torch.randn(200, 2, 80, dtype=torch.float32)
    fq[:, :, 7] *= 10.0
    store_float(arrays, "fq_input", fq)
    for bits in (2, 4):
        fk = kivi_fake_quant_key(fq, bits=bits, group_size=32)
        fv = kivi_fake_quant_value(fq, bits=bits, group_size=32)
        cases[f"fake_quant/b{bits}"] = {"key": dig(fk), "value": dig(fv)}
        if bits == 2:
            store_float(arrays, "fq_key_b2", fk)

    # 4. H2O selection known answer (tests/test_physical.py:1195-1215).
    key8 = torch.arange(8 * 2 * 4, dtype=torch.float32).reshape(8, 2, 4)
    scores8 = torch.tensor(
        [[9.0, 8.0, 5.0, 4.0, 3.0, 2.0, 0.0, 0.0], [0.0, 8.0, 1.0, 1.0, 1.0, 9.0, 0.0, 0.0]]
    )
    h2o = GQAH2OCache.from_dense(
        key8, key8 + 1000, logical_token_ids=torch.arange(8), token_type_id=1,
        per_kv_head_scores=scores8, target_tokens=4, recent_tokens=2,
    )
    arrays["h2o_kat_scores"] = scores8.numpy()
    arrays["h2o_kat_ids"] = h2o.logical_token_ids.numpy()
    # Config-1-shaped random selection: T=2048, 4 KV heads, 20% kept.
    torch.manual_seed(7)
    scores = torch.stack([torch.randperm(2048) for _ in range(4)]).float() / 2048.0 + torch.rand(4, 2048) * 1e-4
    for row in scores:
        assert int(torch.unique(row).numel()) == row.numel(), "scores must be tie-free per head"
    k_small = torch.randn(2048, 4, 16, dtype=torch.bfloat16)
    v_small = torch.randn_like(k_small)
    ids = torch.arange(100, 2148)
    target = max(1, int(round(2048 * 0.2)))
    recent = int(round(target * 0.25))
    h2o = GQAH2OCache.from_dense(
        k_small, v_small, logical_token_ids=ids, token_type_id=2, per_kv_head_scores=scores,
        target_tokens=target, recent_tokens=recent, selection_frozen=True,
    )
    arrays["h2o_scores"] = scores.numpy()
    store_float(arrays, "h2o_key", k_small)
    store_float(arrays, "h2o_value", v_small)
    arrays["h2o_ids"] = h2o.logical_token_ids.numpy()
    cases["h2o_random"] = {
        "target": target, "recent": recent, "heavy_tokens": h2o.heavy_tokens,
        "key": dig(h2o.key), "value": dig(h2o.value), "scores": dig(h2o.cumulative_scores),
        "ids": dig(h2o.logical_token_ids),
    }
    # Score accumulation, trim and budget requests (physical.py:598-654).
    torch.manual_seed(8)
    probs = torch.softmax(torch.randn(28, 3, h2o.retained_tokens), dim=-1)
    arrays["h2o_update_probs"] = probs.numpy()
    h2o.update_scores(probs)
    arrays["h2o_updated_scores"] = h2o.cumulative_scores.numpy()
    eff1 = h2o.request_budget(300, 60)
    arrays["h2o_trim1_ids"] = h2o.logical_token_ids.numpy()
    eff2 = h2o.request_budget(1000, 10)
    cases["h2o_budget"] = {
        "effective1": eff1, "effective2": eff2, "shortfall": h2o.budget_shortfall_tokens,
        "retained": h2o.retained_tokens, "key": dig(h2o.key), "ids": dig(h2o.logical_token_ids),
    }

    # 5. LSE merge (tests/test_physical.py:181-202).
    torch.manual_seed(11)
    scores_a = torch.randn(4, 3, 7)
    scores_b = torch.randn(4, 3, 5)
    value_a = torch.randn(4, 7, 8)
    value_b = torch.randn(4, 5, 8)
    sa = (torch.matmul(torch.softmax(scores_a, -1), value_a).transpose(0, 1), torch.logsumexp(scores_a, -1))
    sb = (torch.matmul(torch.softmax(scores_b, -1), value_b).transpose(0, 1), torch.logsumexp(scores_b, -1))
    merged, lse = merge_attention_summaries([sa, sb])
    for name, t in {"merge_oa": sa[0], "merge_la": sa[1], "merge_ob": sb[0], "merge_lb": sb[1],
                    "merge_out": merged, "merge_lse": lse}.items():
        arrays[name] = f32(t)

    # 6. Attention over a packed segment plus a dense segment (decode, q_len=1)
    #    through the reference's attention_parts (physical.py:452-475).
    torch.manual_seed(4)
    pk = torch.randn(160, 4, 128, dtype=torch.bfloat16)
    pv = torch.randn_like(pk)
    pk[:, :, [3, 50, 77, 101]] *= 10
    dense_k = torch.randn(24, 4, 128, dtype=torch.bfloat16)
    dense_v = torch.randn_like(dense_k)
    query = torch.randn(1, 28, 128, dtype=torch.bfloat16)
    for name, t in {"att_pk": pk, "att_pv": pv, "att_dk": dense_k, "att_dv": dense_v, "att_q": query}.items():
        store_float(arrays, name, t)
    cache = PackedKIVICache.from_dense(
        pk, pv, logical_token_ids=torch.arange(160), token_type_id=3,
        k_bits=2, v_bits=2, group_size=32, residual_length=16, backend="reference",
    )
    logits, apply_value = cache.attention_parts(query)
    from unicache.storage.physical import gqa_probability_value, gqa_query_key_logits

    dense_logits = gqa_query_key_logits(query, dense_k) / math.sqrt(128)
    all_logits = torch.cat([dense_logits, logits], dim=-1)
    probs = torch.softmax(all_logits.float(), dim=-1)
    out = gqa_probability_value(probs[:, :, :24], dense_v).float() + apply_value(probs[:, :, 24:]).float()
    arrays["att_out"] = f32(out.transpose(0, 1))
    arrays["att_logits"] = f32(all_logits)

    # 7. Dense compaction (unicache/storage/tensor_backend.py:33-100).
    torch.manual_seed(12)
    ck = torch.randn(30, 4, 16, dtype=torch.bfloat16)
    cv = torch.randn_like(ck)
    types = torch.randint(0, 6, (30,))
    masks = [torch.rand(12) > 0.4, torch.rand(18) > 0.6]
    result = TensorCacheStorageBackend.compact(
        key=ck, value=cv, key_type_ids=types, sample_lens=torch.tensor([12, 18]), keep_masks=masks,
    )
    store_float(arrays, "compact_key", ck)
    store_float(arrays, "compact_value", cv)
    arrays["compact_types"] = types.numpy()
    arrays["compact_mask0"] = masks[0].numpy()
    arrays["compact_mask1"] = masks[1].numpy()
    cases["compact"] = {
        "key": dig(result.key), "value": dig(result.value), "types": dig(result.key_type_ids),
        "lens": result.sample_lens.tolist(), "original_bytes": result.original_bytes,
        "compacted_bytes": result.compacted_bytes,
    }

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as handle:
        json.dump(meta, handle, indent=1, sort_keys=True)
    print(f"wrote {len(arrays)} arrays and {len(cases)} digest cases")


if __name__ == "__main__":
    main()
