"""H2O selection/compaction/scoring, LSE merge and dense compaction kernels
against the oracle and the reference's golden vectors."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, compact, h2o
from oracle.numerics import digest
from unicache_b200 import (
    GQAH2OCache,
    H2OPhysicalGQAOperator,
    PhysicalCacheRequest,
    TensorCacheStorageBackend,
    kernels,
    merge_attention_summaries,
)
from unicache_b200.synthetic import make_kv

from .conftest import bf16_array
from .gpu_util import host, need_gpu

pytestmark = pytest.mark.gpu


def test_h2o_known_answer():
    """tests/test_physical.py:1195-1215."""

    need_gpu()
    key = torch.arange(8 * 2 * 4, dtype=torch.float32).reshape(8, 2, 4).cuda()
    scores = torch.tensor([[9.0, 8.0, 5.0, 4.0, 3.0, 2.0, 0.0, 0.0],
                           [0.0, 8.0, 1.0, 1.0, 1.0, 9.0, 0.0, 0.0]], device="cuda")
    cache = GQAH2OCache.from_dense(key, key + 1000, logical_token_ids=torch.arange(8, device="cuda"),
                                   token_type_id=1, per_kv_head_scores=scores, target_tokens=4, recent_tokens=2)
    assert cache.logical_token_ids.tolist() == [[0, 1, 6, 7], [1, 5, 6, 7]]
    assert torch.equal(cache.key[0, 1], key[1, 0]) and torch.equal(cache.value[1, 1], key[5, 1] + 1000)
    assert cache.resident_bytes < cache.full_precision_bytes


def test_golden_h2o_selection_trim_and_budget(golden):
    need_gpu()
    arrays, cases = golden
    case = cases["h2o_random"]
    key = torch.from_numpy(bf16_array(arrays["h2o_key"])).to(torch.bfloat16).cuda()
    value = torch.from_numpy(bf16_array(arrays["h2o_value"])).to(torch.bfloat16).cuda()
    scores = torch.from_numpy(arrays["h2o_scores"]).cuda()
    cache = GQAH2OCache.from_dense(key, value, logical_token_ids=torch.arange(100, 2148, device="cuda"),
                                   token_type_id=2, per_kv_head_scores=scores, target_tokens=case["target"],
                                   recent_tokens=case["recent"], selection_frozen=True)
    np.testing.assert_array_equal(host(cache.logical_token_ids), arrays["h2o_ids"])
    assert digest(host(cache.key), "bfloat16") == case["key"]
    assert digest(host(cache.value), "bfloat16") == case["value"]
    assert digest(host(cache.cumulative_scores), "float32") == case["scores"]
    assert cache.heavy_tokens == case["heavy_tokens"]
    probs = torch.from_numpy(arrays["h2o_update_probs"]).cuda()
    cache.update_scores(probs)
    np.testing.assert_allclose(host(cache.cumulative_scores), arrays["h2o_updated_scores"], rtol=0, atol=2e-6)
    # Continue from the reference's exact scores so the trims are comparable bit-for-bit.
    cache.cumulative_scores = torch.from_numpy(arrays["h2o_updated_scores"]).cuda()
    eff1 = cache.request_budget(300, 60)
    np.testing.assert_array_equal(host(cache.logical_token_ids), arrays["h2o_trim1_ids"])
    eff2 = cache.request_budget(1000, 10)
    budget = cases["h2o_budget"]
    assert (eff1, eff2, cache.budget_shortfall_tokens) == (budget["effective1"], budget["effective2"],
                                                          budget["shortfall"])
    assert digest(host(cache.key), "bfloat16") == budget["key"]
    assert digest(host(cache.logical_token_ids)) == budget["ids"]


@pytest.mark.parametrize("tokens,target,recent", [(2048, 410, 102), (4900, 980, 245), (16384, 3277, 819),
                                                  (256, 51, 13), (100, 100, 0), (77, 1, 0), (64, 10, 10)])
def test_selection_matches_oracle(tokens, target, recent):
    need_gpu()
    gen = torch.Generator().manual_seed(tokens)
    scores = torch.stack([torch.randperm(tokens, generator=gen) for _ in range(4)]).float()
    scores = scores / tokens + torch.rand(4, tokens, generator=gen) * 1e-5
    scores = scores.cuda()
    hist = tokens - min(target, recent)
    heavy = min(target - min(target, recent), hist)
    idx = kernels.h2o_select(scores, history_end=hist, heavy_k=heavy, recent=min(target, recent))
    expect, _, _ = h2o.select_indices(host(scores), target, recent)
    np.testing.assert_array_equal(host(idx), expect)


def test_selection_tie_order_is_lower_index_first():
    need_gpu()
    scores = torch.tensor([[1.0, 2.0, 2.0, 2.0, 0.5, 2.0, 3.0, 0.0]], device="cuda")
    idx = kernels.h2o_select(scores, history_end=8, heavy_k=3, recent=0)
    assert idx.tolist() == [[1, 2, 6]]
    neg = torch.tensor([[-1.0, -0.0, 0.0, -2.0, -1.0, 5.0]], device="cuda")
    idx = kernels.h2o_select(neg, history_end=6, heavy_k=3, recent=0)
    assert idx.tolist() == h2o.select_indices(host(neg), 3, 0)[0].tolist()


def test_probability_reduction_and_operator_request():
    need_gpu()
    probs = torch.softmax(torch.randn(28, 5, 300, generator=torch.Generator().manual_seed(2)), dim=-1).cuda()
    got = kernels.accumulate_probs(probs, 4)
    np.testing.assert_allclose(host(got), h2o.reduce_probabilities(host(probs), 4), rtol=1e-5, atol=1e-6)

    class Ctx:
        pass

    ctx = Ctx()
    ctx.storage_num_kv_heads = 4
    ctx.params = H2OPhysicalGQAOperator().build_params({"target_budget_ratio": 0.5})
    ctx.k = torch.zeros(300, 4, 128, device="cuda")
    ctx.segment_mask = torch.ones(300, dtype=torch.bool, device="cuda")

    class Step:
        segment_id = "instruction"

    class Runtime:
        kv_metadata = {"current_segment_tokens": 300}

    ctx.step, ctx.runtime = Step(), Runtime()
    records = []
    ctx.record = records.append
    H2OPhysicalGQAOperator().update_after_attention(ctx, probs)
    assert isinstance(ctx.physical_request, PhysicalCacheRequest)
    np.testing.assert_allclose(host(ctx.physical_request.per_kv_head_scores), host(got), rtol=1e-6)
    assert records[0]["physical_h2o_target_tokens_per_kv_head"] == 150


def test_scores_from_lse_match_materialised_probabilities():
    need_gpu()
    key, _ = make_kv(600, 4, 128, seed=5, device="cuda")
    query = (torch.randn(64, 28, 128, generator=torch.Generator().manual_seed(6)) * 0.5).to(torch.bfloat16).cuda()
    logits = attention.gqa_query_key_logits(host(query), host(key)) / np.sqrt(128)
    lse = np.log(np.exp(logits - logits.max(-1, keepdims=True)).sum(-1)) + logits.max(-1)
    scores = kernels.scores_from_lse(query, key, torch.from_numpy(lse.astype(np.float32)).cuda(), kv_heads=4,
                                     softmax_scale=1 / np.sqrt(128))
    probs = np.exp(logits - lse[..., None])
    np.testing.assert_allclose(host(scores), h2o.reduce_probabilities(probs, 4), rtol=2e-3, atol=1e-4)


def test_golden_lse_merge(golden):
    need_gpu()
    arrays, _ = golden
    s = [(torch.from_numpy(arrays["merge_oa"]).cuda(), torch.from_numpy(arrays["merge_la"]).cuda()),
         (torch.from_numpy(arrays["merge_ob"]).cuda(), torch.from_numpy(arrays["merge_lb"]).cuda())]
    out, lse = merge_attention_summaries(s)
    np.testing.assert_allclose(host(out), arrays["merge_out"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(host(lse), arrays["merge_lse"], atol=1e-6, rtol=1e-6)


def test_golden_dense_compaction(golden):
    need_gpu()
    arrays, cases = golden
    case = cases["compact"]
    key = torch.from_numpy(bf16_array(arrays["compact_key"])).to(torch.bfloat16).cuda()
    value = torch.from_numpy(bf16_array(arrays["compact_value"])).to(torch.bfloat16).cuda()
    types = torch.from_numpy(arrays["compact_types"]).cuda()
    masks = [torch.from_numpy(arrays["compact_mask0"]).cuda(), torch.from_numpy(arrays["compact_mask1"]).cuda()]
    result = TensorCacheStorageBackend.compact(key=key, value=value, key_type_ids=types,
                                               sample_lens=torch.tensor([12, 18]), keep_masks=masks)
    assert digest(host(result.key), "bfloat16") == case["key"]
    assert digest(host(result.value), "bfloat16") == case["value"]
    assert digest(host(result.key_type_ids)) == case["types"]
    assert result.sample_lens.tolist() == case["lens"]
    assert result.original_bytes == case["original_bytes"] and result.compacted_bytes == case["compacted_bytes"]


def test_compaction_large_and_empty_masks():
    need_gpu()
    key, value = make_kv(70000, 4, 128, seed=3, device="cuda")
    gen = torch.Generator().manual_seed(4)
    mask = torch.rand(70000, generator=gen) > 0.3
    result = TensorCacheStorageBackend.compact(key=key, value=value, key_type_ids=None,
                                               sample_lens=torch.tensor([70000]), keep_masks=[mask.cuda()])
    ek, ev, _, lens = compact.compact(host(key), host(value), None, [70000], [mask.numpy()])
    np.testing.assert_array_equal(host(result.key), ek)
    assert result.sample_lens.tolist() == lens
    none = TensorCacheStorageBackend.compact(key=key[:10], value=value[:10], key_type_ids=None,
                                             sample_lens=torch.tensor([10]),
                                             keep_masks=[torch.zeros(10, dtype=torch.bool, device="cuda")])
    assert none.key.shape[0] == 0


def test_materialize_kivi_and_h2o_requests():
    """tensor_backend.py:103-239: requests become physical segments and leave
    the dense cache."""

    need_gpu()
    key, value = make_kv(96, 4, 128, seed=12, device="cuda")
    types = torch.tensor([1] * 32 + [3] * 48 + [4] * 16, device="cuda")
    kivi_req = PhysicalCacheRequest(
        operator="kivi_packed_quantization", segment_id="source_vae", token_count=96,
        segment_mask=(types == 3), params={"bits": 2, "group_size": 32, "residual_length": 8},
        metadata={"token_type_id": 3, "token_span": (32, 80)},
    )
    h2o_req = PhysicalCacheRequest(
        operator="h2o_physical_gqa", segment_id="instruction", token_count=96, segment_mask=(types == 1),
        params={"target_budget_ratio": 0.5, "recent_budget_fraction": 0.25, "selection_frozen": True},
        per_kv_head_scores=torch.rand(4, 96, generator=torch.Generator().manual_seed(1)).cuda(),
        metadata={"token_type_id": 1},
    )
    result = TensorCacheStorageBackend.compact_and_materialize(
        key=key, value=value, key_type_ids=types, sample_lens=torch.tensor([96]),
        keep_masks=[torch.ones(96, dtype=torch.bool, device="cuda")], physical_requests=[[kivi_req, h2o_req]],
    )
    assert result.key.shape[0] == 16 and bool((result.key_type_ids == 4).all())
    packed, selected = result.physical_segments_by_sample[0]
    assert packed.quantized_tokens == 32 and packed.token_count == 48 and packed.token_type_id == 3
    assert selected.retained_tokens == 16 and selected.token_type_id == 1
    overlap = PhysicalCacheRequest(operator="kivi_packed_quantization", segment_id="x", token_count=96,
                                   segment_mask=torch.ones(96, dtype=torch.bool, device="cuda"))
    with pytest.raises(ValueError):
        TensorCacheStorageBackend.compact_and_materialize(
            key=key, value=value, key_type_ids=types, sample_lens=torch.tensor([96]),
            keep_masks=[torch.ones(96, dtype=torch.bool, device="cuda")],
            physical_requests=[[kivi_req, overlap]])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("tokens,queries,misaligned", [(97, 5, False), (64, 1, False), (1000, 37, False),
                                                       (1000, 80, False), (203, 11, True)])
def test_scores_without_lse_ragged(dtype, tokens, queries, misaligned):
    """The LSE pass (64-row x 64-token logit tiles, partials folded over the
    token blocks) at sizes that fill no tile, then the scores, against the
    float64 column sums of the materialised probabilities.  80 queries give
    560 rows per KV head: more 64-row tiles than the scoring cluster has
    blocks.  ``misaligned`` starts the keys 4 bytes past an aligned address
    (the bf16 scoring kernel's minimum), so the LSE tiles are staged element
    by element."""

    need_gpu()
    key, _ = make_kv(tokens, 4, 128, seed=tokens, dtype=dtype, device="cuda")
    if misaligned:
        shift = 4 // key.element_size()
        base = torch.empty(key.numel() + shift, dtype=dtype, device="cuda")
        base[shift:].copy_(key.reshape(-1))
        key = base[shift:].view(tokens, 4, 128)
    query = (torch.randn(queries, 28, 128, generator=torch.Generator().manual_seed(queries)) * 0.5).to(dtype).cuda()
    scores = kernels.h2o_scores(query, key, None, kv_heads=4, softmax_scale=1 / np.sqrt(128))
    logits = attention.gqa_query_key_logits(host(query).astype(np.float64), host(key).astype(np.float64)) / np.sqrt(128)
    probs = np.exp(logits - logits.max(-1, keepdims=True))
    probs /= probs.sum(-1, keepdims=True)
    expect = h2o.reduce_probabilities(probs, 4)
    np.testing.assert_allclose(host(scores), expect, rtol=1e-4 if dtype == torch.float32 else 2e-3, atol=1e-6)
    assert kernels.device_status() == 0
